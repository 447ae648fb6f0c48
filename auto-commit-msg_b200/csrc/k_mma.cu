// k_mma.cu -- tensor-core GEMM for prefill (and batched decode):
// y[m][n] (epi)= x[m][:] . W[n][:], the matmul of tensor.go:253-303 for M > 8
// tokens, on the 5th-generation tensor cores.
//
// Precision.  The reference computes in fp32.  One bf16 product (8-bit
// mantissa) gives ~1e-3 relative error on the logits, too coarse, so each
// operand is split into a bf16 pair v = hi + lo (hi = bf16(v), lo = bf16(v -
// hi)) and the product is formed as hi.hi + hi.lo + lo.hi with fp32
// accumulation (the lo.lo term is below 2^-16 of the product): three MMAs per
// K step, relative error ~1e-5.
//
// Layout.  This kernel reads weights that are already bf16 pairs: F16/F32
// weights and quantized ones whose K is not a multiple of 256 are dequantized
// (exact, tensor.go:55-226) once per tensor into two bf16 arrays (the "split
// cache", 4 bytes per weight, built on first use and kept in HBM); quantized
// weights with K % 256 == 0 take k_mma_dq.cu, which dequantizes in shared
// memory and keeps no cache.  The attention GEMMs (S = Q.K^T, O = P.V) run
// here on split operands prepared per call, as do the activations.  Both are
// stored 64x64-blocked -- element (r, c) at ((r/64)*(K/64) + c/64)*4096 +
// (r%64)*64 + c%64 -- so each TMA box is one contiguous 8 KB read (a
// row-major [n][K] box gathers 64 pieces of 128 bytes from 64 DRAM pages),
// and lands as a 128-byte-swizzled K-major tile.
//
// Kernel.  One CTA computes a tile of 128 weight rows x 64 tokens (for a
// SwiGLU pair: 64 gate rows + the same 64 up rows) over the whole K:
//   warp 0 lane 0  TMA producer: 4-stage ring of (A hi, A lo, B hi, B lo),
//                  64 K-elements per stage;
//   warp 1         allocates 64 TMEM columns; lane 0 issues
//                  tcgen05.mma (M=128, N=64, K=16, kind::f16, bf16 in, fp32
//                  accumulate) and frees stages with tcgen05.commit;
//   warps 2..5     epilogue: tcgen05.ld of their 32 TMEM lanes, bias,
//                  store / residual add / SwiGLU, coalesced over rows.
// Every wait is bounded; on a timeout the kernel records DEV_ERR_TIMEOUT,
// waits (bounded) for its copies and MMAs in flight, frees TMEM and returns.
#include <cuda.h>
#include <atomic>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <float.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "mma_dev.cuh"
#include "quant.cuh"

namespace acm {

namespace {

constexpr int MBM = 128;  // weight rows per tile (MMA M)
constexpr int MBN = 64;   // tokens per tile (MMA N)
constexpr int MBK = 64;   // K elements per stage (128 bytes of bf16: one swizzle row)
constexpr int MST = 4;    // stages
constexpr int A_BYTES = MBM * MBK * 2;  // 16 KB
constexpr int B_BYTES = MBN * MBK * 2;  // 8 KB
constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
constexpr int MMA_THREADS = 192;
constexpr int MMA_SMEM = MST * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t TMEM_COLS = 64;

constexpr uint32_t IDESC = mma::idesc_bf16(MBM, MBN);
using mma::tma_load_2d;
using mma::tc_fence_before;
using mma::tc_fence_after;
using mma::tc_commit;
using mma::tc_mma;
using mma::tc_ld16;
using mma::sw128_desc;

}  // namespace

// One weight matrix (or SwiGLU pair) of a grouped launch.
struct MmaSeg {
    CUtensorMap ahi, alo;    // W split cache, box {64, 64 rows}
    CUtensorMap ahi2, alo2;  // pair: the up-projection's cache
    int n;                   // rows
    int pair;
    int tile0;               // first tile index of this segment
    int epi;
    float *y;
    int ldy;
    const float *bias;
    const int32_t *yrow;
};
constexpr int MMA_MAX_SEG = 3;
struct MmaArgs {
    MmaSeg seg[MMA_MAX_SEG];
    int nseg;
    CUtensorMap bhi, blo;  // activations split, box {64, 64 rows}
    int m, k;
    int ttiles;            // token tiles
    // batched form (blockIdx.y = batch, one segment): operand offsets in box
    // rows, and the output row of token `tok` of batch b:
    // (rmod ? (tok % rmod) * rmul + (tok / rmod) * rdiv : tok) + b * rbatch
    int a_bstride, b_bstride, rmod, rmul, rdiv, rbatch;
    int causal, cntok, cpos0;  // MmaBatch::causal
    // split-K (blockIdx.z = K slice): partial sums to ws[slice][tok][n]
    int ksplit;
    float *ws;
};

__device__ __forceinline__ int64_t out_row(const MmaArgs &A, const MmaSeg &S, int tok, int batch) {
    if (S.yrow) return S.yrow[tok];
    const int r = A.rmod ? (tok % A.rmod) * A.rmul + (tok / A.rmod) * A.rdiv : tok;
    return (int64_t)r + (int64_t)batch * A.rbatch;
}

__global__ void __launch_bounds__(MMA_THREADS, 1) k_mma_gemm(const __grid_constant__ MmaArgs A) {
    extern __shared__ uint8_t msm_raw[];
    uint8_t *msm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(msm_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(msm + MST * STAGE_BYTES);
    uint64_t *empty = full + MST;
    uint64_t *accf = empty + MST;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // tile -> (segment, row tile, token tile); token tiles fastest so CTAs
    // sharing a weight tile run together (L2 reuse)
    int si = 0;
    while (si + 1 < A.nseg && (int)blockIdx.x >= A.seg[si + 1].tile0) si++;
    const MmaSeg &S = A.seg[si];
    const int local = blockIdx.x - S.tile0;
    const int rt = local / A.ttiles, tt = local - rt * A.ttiles;
    const int rows_per_tile = S.pair ? MBM / 2 : MBM;
    const int row0 = rt * rows_per_tile, tok0 = tt * MBN;
    const int batch = blockIdx.y;
    // this CTA's K blocks: all of them, or its slice under split-K
    const int KTA = A.k / MBK;  // K blocks of the operands (their layout)
    const int kb0 = (int)((int64_t)KTA * blockIdx.z / A.ksplit);
    int kb1 = (int)((int64_t)KTA * (blockIdx.z + 1) / A.ksplit);
    if (A.causal) {
        // the last key any query row of this token tile attends
        const int tl = min(tok0 + MBN, A.m) - 1;
        const int kmax = A.cpos0 + (tok0 / A.cntok != tl / A.cntok ? A.cntok - 1 : tl % A.cntok);
        if (A.causal == 1 && row0 > kmax) return;  // the whole CTA: every score of the tile is masked
        if (A.causal == 2) kb1 = max(kb0, min(kb1, kmax / MBK + 1));
    }
    const int KT = kb1 - kb0;

    if (tid == 0) {
        for (int i = 0; i < MST; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(accf, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    if (tid == 0) pdl_trigger();

    if (warp == 0 && lane == 0) {
        // ---- TMA producer ----
        int issued = 0;
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % MST;
            if (kt >= MST && !mbar_wait(&empty[s], ((kt / MST) & 1) ^ 1)) break;
            uint8_t *st = msm + s * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            // 64x64 block (row block rb, K block kt) starts at box row (rb*KT + kt)*64
            const int ya = ((row0 >> 6) * KTA + kb0 + kt) * 64 + batch * A.a_bstride;
            const int yb = ((tok0 >> 6) * KTA + kb0 + kt) * 64 + batch * A.b_bstride;
            if (S.pair) {
                tma_load_2d(st, &S.ahi, 0, ya, &full[s]);
                tma_load_2d(st + A_BYTES / 2, &S.ahi2, 0, ya, &full[s]);
                tma_load_2d(st + A_BYTES, &S.alo, 0, ya, &full[s]);
                tma_load_2d(st + A_BYTES + A_BYTES / 2, &S.alo2, 0, ya, &full[s]);
            } else {
                // the second 64 rows: next row block (zero-filled past the cache)
                const int ya2 = ya + KTA * 64;
                tma_load_2d(st, &S.ahi, 0, ya, &full[s]);
                tma_load_2d(st + A_BYTES / 2, &S.ahi, 0, ya2, &full[s]);
                tma_load_2d(st + A_BYTES, &S.alo, 0, ya, &full[s]);
                tma_load_2d(st + A_BYTES + A_BYTES / 2, &S.alo, 0, ya2, &full[s]);
            }
            tma_load_2d(st + 2 * A_BYTES, &A.bhi, 0, yb, &full[s]);
            tma_load_2d(st + 2 * A_BYTES + B_BYTES, &A.blo, 0, yb, &full[s]);
            issued = kt + 1;
        }
        // no copy may still be landing when the CTA exits: wait (bounded)
        // for the last fill of every stage used
        for (int s = 0; s < MST && s < issued; s++) {
            const int last = s + ((issued - 1 - s) / MST) * MST;  // last kt that used stage s
            mbar_wait_limit(&full[s], (last / MST) & 1, WAIT_LIMIT);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % MST;
            if (!mbar_wait(&full[s], (kt / MST) & 1)) break;
            tc_fence_after();
            const uint32_t st = smem_u32(msm + s * STAGE_BYTES);
            const uint32_t ahi = st, alo = st + A_BYTES, bhi = st + 2 * A_BYTES, blo = bhi + B_BYTES;
#pragma unroll
            for (int kk = 0; kk < MBK / 16; kk++) {
                const uint32_t off = kk * 32;  // 16 bf16 along K inside the swizzled row
                const uint64_t dah = sw128_desc(ahi + off), dal = sw128_desc(alo + off);
                const uint64_t dbh = sw128_desc(bhi + off), dbl = sw128_desc(blo + off);
                tc_mma(tmem, dah, dbh, IDESC, (kt | kk) != 0);
                tc_mma(tmem, dah, dbl, IDESC, 1u);
                tc_mma(tmem, dal, dbh, IDESC, 1u);
            }
            tc_commit(&empty[s]);  // stage free once these MMAs have read it
        }
        tc_commit(accf);  // all MMAs issued so far complete -> accumulator ready
    } else if (warp >= 2) {
        // ---- epilogue ----
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        // the four epilogue warps decide together: the pair exchange below
        // meets at named barriers
        const bool ok = named_and(1, 128, mbar_wait(accf, 0));
        tc_fence_after();
        if (ok) {
            const int lrow = q * 32 + lane;  // accumulator row (TMEM lane)
            float *xch = reinterpret_cast<float *>(msm);  // pair exchange [64][MBN + 1]
            for (int c0 = 0; c0 < MBN; c0 += 16) {
                float v[16];
                tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
                if (S.pair) {
                    // lanes 64..127 hold the up rows: hand them to the gate warps
                    if (q >= 2)
#pragma unroll
                        for (int j = 0; j < 16; j++) xch[(lrow - 64) * (MBN + 1) + c0 + j] = v[j];
                    named_sync(1, 128);
                    if (q < 2) {
                        const int n = row0 + lrow;
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int tok = tok0 + c0 + j;
                            if (n < S.n && tok < A.m) {
                                const float g = v[j], u = xch[lrow * (MBN + 1) + c0 + j];
                                const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_exp(-g)));
                                float *yp = S.y + out_row(A, S, tok, batch) * S.ldy + n;
                                *yp = __fmul_rn(__fmul_rn(g, sg), u);
                            }
                        }
                    }
                    named_sync(1, 128);
                } else if (A.ksplit > 1) {
                    // partial sums of this K slice (bias and epilogue in k_split_reduce)
                    const int n = row0 + lrow;
                    if (n < S.n)
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int tok = tok0 + c0 + j;
                            if (tok < A.m) A.ws[((int64_t)blockIdx.z * A.m + tok) * S.n + n] = v[j];
                        }
                } else {
                    const int n = row0 + lrow;
                    if (n < S.n) {
                        const float b = S.bias ? S.bias[n] : 0.f;
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int tok = tok0 + c0 + j;
                            if (tok < A.m) {
                                float *yp = S.y + out_row(A, S, tok, batch) * S.ldy + n;
                                const float val = S.bias ? v[j] + b : v[j];
                                if (S.epi == EPI_ADD) *yp = *yp + val;
                                else *yp = val;
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        // the accumulator must be idle before it is freed (immediate unless a
        // wait above ran out; the fixed bound, whatever the progress limit)
        mbar_wait_limit(accf, 0, WAIT_LIMIT);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// Split-K epilogue: y[tok][n] (epi)= bias[n] + sum over slices, in slice
// order (deterministic).
__global__ void k_split_reduce(const float *ws, int ks, int m, int n, float *y, int ldy, int epi, const float *bias,
                               const int32_t *yrow) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t total = (int64_t)m * n;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int tok = (int)(i / n), c = (int)(i - (int64_t)tok * n);
        float v = ws[i];
        for (int s = 1; s < ks; s++) v += ws[(int64_t)s * total + i];
        if (bias) v += bias[c];
        float *yp = y + (int64_t)(yrow ? yrow[tok] : tok) * ldy + c;
        *yp = epi == EPI_ADD ? *yp + v : v;
    }
}

// ---------------------------------------------------------------------------
// Operand preparation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16 &hi, __nv_bfloat16 &lo) {
    hi = __float2bfloat16_rn(v);
    lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}

// Offset of element (r, c) in the 64x64-blocked layout of a [rows][k] matrix.
__device__ __forceinline__ int64_t blk64(int64_t r, int c, int k) {
    return (((r >> 6) * (k >> 6) + (c >> 6)) << 12) + ((r & 63) << 6) + (c & 63);
}

// x[m][ldx] fp32 -> hi, lo bf16, 64x64-blocked
__global__ void k_split_act(const float *x, int ldx, int m, int k, __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t total = (int64_t)m * k / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e0 = i * 4;
        const int r = (int)(e0 / k), c = (int)(e0 - (int64_t)r * k);
        const int64_t e = blk64(r, c, k);
        const float4 v = *reinterpret_cast<const float4 *>(x + (int64_t)r * ldx + c);
        __nv_bfloat16 h[4], l[4];
        split_bf16(v.x, h[0], l[0]);
        split_bf16(v.y, h[1], l[1]);
        split_bf16(v.z, h[2], l[2]);
        split_bf16(v.w, h[3], l[3]);
        *reinterpret_cast<uint2 *>(hi + e) = *reinterpret_cast<uint2 *>(h);
        *reinterpret_cast<uint2 *>(lo + e) = *reinterpret_cast<uint2 *>(l);
    }
}

// RMSNorm (model.go:213-222) of row blockIdx.x fused with its split: the
// same arithmetic and reduction order as k_rmsnorm (k_misc.cu), so the split
// values are those of rmsnorm followed by k_split_act.  256 threads per row.
__global__ void __launch_bounds__(256) k_split_act_norm(const float *x, int ldx, int k, const float *w, float eps,
                                                        __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    __shared__ float red[8];
    const int r = blockIdx.x;
    const float *xr = x + (int64_t)r * ldx;
    float ss = 0.f;
    for (int i = threadIdx.x; i < k; i += 256) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += red[i];
    const float sc = rms_scale(t, k, eps);
    for (int c = threadIdx.x * 4; c < k; c += 1024) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + c);
        const float4 g = *reinterpret_cast<const float4 *>(w + c);
        __nv_bfloat16 h[4], l[4];
        split_bf16(__fmul_rn(__fmul_rn(v.x, sc), g.x), h[0], l[0]);
        split_bf16(__fmul_rn(__fmul_rn(v.y, sc), g.y), h[1], l[1]);
        split_bf16(__fmul_rn(__fmul_rn(v.z, sc), g.z), h[2], l[2]);
        split_bf16(__fmul_rn(__fmul_rn(v.w, sc), g.w), h[3], l[3]);
        const int64_t e = blk64(r, c, k);
        *reinterpret_cast<uint2 *>(hi + e) = *reinterpret_cast<uint2 *>(h);
        *reinterpret_cast<uint2 *>(lo + e) = *reinterpret_cast<uint2 *>(l);
    }
}

// A split-K GEMM's residual add (x += the ks partial sums of ws, in order, as
// k_split_reduce) fused with the RMSNorm and split of the resulting rows that
// the next GEMM reads (as k_split_act_norm): one launch instead of two, the
// same values.  Row blockIdx.x, 256 threads.
__global__ void __launch_bounds__(256) k_split_act_reduce_norm(const float *ws, int ks, int m, float *x, int k,
                                                               const float *w, float eps, __nv_bfloat16 *hi,
                                                               __nv_bfloat16 *lo) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    __shared__ float red[8];
    const int r = blockIdx.x;
    float *xr = x + (int64_t)r * k;
    const int64_t total = (int64_t)m * k;
    for (int c = threadIdx.x * 4; c < k; c += 1024) {
        const int64_t i = (int64_t)r * k + c;
        float4 v = *reinterpret_cast<const float4 *>(ws + i);
        for (int s = 1; s < ks; s++) {
            const float4 p = *reinterpret_cast<const float4 *>(ws + (int64_t)s * total + i);
            v.x += p.x;
            v.y += p.y;
            v.z += p.z;
            v.w += p.w;
        }
        float4 y = *reinterpret_cast<const float4 *>(xr + c);
        y.x = y.x + v.x;
        y.y = y.y + v.y;
        y.z = y.z + v.z;
        y.w = y.w + v.w;
        *reinterpret_cast<float4 *>(xr + c) = y;
    }
    __syncthreads();  // the row's new values, written by other threads of the CTA
    float ss = 0.f;
    for (int i = threadIdx.x; i < k; i += 256) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += red[i];
    const float sc = rms_scale(t, k, eps);
    for (int c = threadIdx.x * 4; c < k; c += 1024) {
        const float4 v = *reinterpret_cast<const float4 *>(xr + c);
        const float4 g = *reinterpret_cast<const float4 *>(w + c);
        __nv_bfloat16 h[4], l[4];
        split_bf16(__fmul_rn(__fmul_rn(v.x, sc), g.x), h[0], l[0]);
        split_bf16(__fmul_rn(__fmul_rn(v.y, sc), g.y), h[1], l[1]);
        split_bf16(__fmul_rn(__fmul_rn(v.z, sc), g.z), h[2], l[2]);
        split_bf16(__fmul_rn(__fmul_rn(v.w, sc), g.w), h[3], l[3]);
        const int64_t e = blk64(r, c, k);
        *reinterpret_cast<uint2 *>(hi + e) = *reinterpret_cast<uint2 *>(h);
        *reinterpret_cast<uint2 *>(lo + e) = *reinterpret_cast<uint2 *>(l);
    }
}

// Exact dequantization of W [n][k] (ggml blocks) -> hi, lo bf16, 64x64-blocked.
template <int T>
__global__ void k_split_weight(const uint8_t *w, int64_t n, int k, __nv_bfloat16 *hi, __nv_bfloat16 *lo) {
    const int64_t rb = row_bytes(T, k);
    const int runs = k / 32;
    const int64_t total = n * runs;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / runs;
        const int run = (int)(i - r * runs);
        float v[32];
        dequant_run32<T>(w + r * rb, run, v);
        __nv_bfloat16 h[32], l[32];
#pragma unroll
        for (int j = 0; j < 32; j++) split_bf16(v[j], h[j], l[j]);
        const int64_t e = blk64(r, run * 32, k);  // 32 consecutive elements stay contiguous
        uint4 *ph = reinterpret_cast<uint4 *>(hi + e);
        uint4 *pl = reinterpret_cast<uint4 *>(lo + e);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            ph[j] = reinterpret_cast<const uint4 *>(h)[j];
            pl[j] = reinterpret_cast<const uint4 *>(l)[j];
        }
    }
}

// ---------------------------------------------------------------------------
// Prefill attention operands (model.go:384-408 for a chunk of consecutive
// positions of one sequence), for S = Q.K^T and O = P.V on the tensor cores.
// Per kv head g (the batch index):
//   Qs [G*ntok][HD]  row h*ntok + t = query head g*G + h of token t
//   Ks [Lp][HD]      row p = cached key of position p (zero for p >= L)
//   Vt [HD][Lp]      Vt[d][p] = V[p][d] (zero for p >= L)
//   P  [G*ntok][Lp]  softmax weights
// all split to bf16 hi/lo and 64x64-blocked; Lp = L rounded up to 64.
// ---------------------------------------------------------------------------
struct AttnSplitArgs {
    const float *q;             // [ntok][nh*HD] (normed + roped)
    const float *kc, *vc;       // cache pools (fp16 elements when kv_f16)
    int kv_f16;
    const int32_t *page_row;    // page table row of the sequence
    int64_t layer_off;          // floats
    int page_size, kvd;
    int ntok, L, Lp, G, nh, hd;
    int64_t rq;                 // rows64(G*ntok)
    __nv_bfloat16 *qh, *ql, *kh, *kl, *vh, *vl;
};

// blockIdx.x < Lp/64: key block (K and V^T of 64 positions); beyond: query
// row block of Qs.  blockIdx.y = kv head.  256 threads; HD <= 128.
__global__ void __launch_bounds__(256) k_attn_split(const AttnSplitArgs a) {
    extern __shared__ float asm_[];  // [64][HD + 1] for the V transpose
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int g = blockIdx.y, hd = a.hd, tid = threadIdx.x;
    const int nkb = a.Lp / 64;
    if ((int)blockIdx.x < nkb) {
        const int p0 = blockIdx.x * 64;
        // the 64 positions lie in one page (page size a multiple of 64)
        const int64_t rowbase = a.layer_off + ((int64_t)a.page_row[p0 / a.page_size] * a.page_size +
                                               (p0 % a.page_size)) * a.kvd + (int64_t)g * hd;
        const int64_t kbase = (int64_t)g * a.Lp * hd, vbase = kbase;
        for (int i = tid; i < 64 * hd; i += 256) {
            const int pr = i / hd, d = i - pr * hd, p = p0 + pr;
            const bool ok = p < a.L;
            const int64_t e = rowbase + (int64_t)pr * a.kvd + d;
            const float kv = ok ? (a.kv_f16 ? __half2float(reinterpret_cast<const __half *>(a.kc)[e]) : a.kc[e]) : 0.f;
            const float vv = ok ? (a.kv_f16 ? __half2float(reinterpret_cast<const __half *>(a.vc)[e]) : a.vc[e]) : 0.f;
            __nv_bfloat16 h, l;
            split_bf16(kv, h, l);
            const int64_t ek = kbase + blk64(p, d, hd);
            a.kh[ek] = h;
            a.kl[ek] = l;
            asm_[pr * (hd + 1) + d] = vv;
        }
        __syncthreads();
        for (int i = tid; i < 64 * hd; i += 256) {
            const int d = i / 64, pr = i - d * 64;
            __nv_bfloat16 h, l;
            split_bf16(asm_[pr * (hd + 1) + d], h, l);
            const int64_t ev = vbase + blk64(d, p0 + pr, a.Lp);
            a.vh[ev] = h;
            a.vl[ev] = l;
        }
    } else {
        const int r0 = (blockIdx.x - nkb) * 64;
        const int rows = a.G * a.ntok;
        const int64_t qbase = (int64_t)g * a.rq * hd;
        for (int i = tid; i < 64 * hd; i += 256) {
            const int rr = i / hd, d = i - rr * hd, r = r0 + rr;
            if (r >= rows) continue;
            const int h = r / a.ntok, t = r - h * a.ntok;
            __nv_bfloat16 hi, lo;
            split_bf16(a.q[(int64_t)t * a.nh * hd + (int64_t)(g * a.G + h) * hd + d], hi, lo);
            const int64_t e = qbase + blk64(r, d, hd);
            a.qh[e] = hi;
            a.ql[e] = lo;
        }
    }
}

// Softmax of one score row per warp (model.go:297-313 on the scaled scores
// of positions <= the token's own): s = dot * scale, m = max s, e =
// fastExp(s - m), p = e / sum e; written as split bf16 into P (zero past the
// token's position).  grid (ceil(G*ntok / 8), nkv), 256 threads.
__global__ void __launch_bounds__(256) k_attn_softmax(const float *S, int ntok, int G, int Lp, int pos0, float scale,
                                                      int64_t rq, __nv_bfloat16 *ph, __nv_bfloat16 *pl) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int g = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows = G * ntok, r = blockIdx.x * 8 + warp;
    if (r >= rows) return;
    const int t = r % ntok, n = pos0 + t + 1;  // keys 0 .. pos0 + t
    const float *row = S + ((int64_t)g * rows + r) * Lp;
    float mx = -FLT_MAX;
    for (int p = lane; p < n; p += 32) mx = fmaxf(mx, __fmul_rn(__ldcg(row + p), scale));
    mx = warp_max(mx);
    float sum = 0.f;
    for (int p = lane; p < n; p += 32) sum += fast_exp(__fsub_rn(__fmul_rn(__ldcg(row + p), scale), mx));
    sum = warp_sum(sum);
    const int64_t base = (int64_t)g * rq * Lp;
    for (int p = lane; p < Lp; p += 32) {
        const float e = p < n ? fast_exp(__fsub_rn(__fmul_rn(__ldcg(row + p), scale), mx)) : 0.f;
        __nv_bfloat16 h, l;
        split_bf16(p < n ? __fdiv_rn(e, sum) : 0.f, h, l);
        const int64_t o = base + blk64(r, p, Lp);
        ph[o] = h;
        pl[o] = l;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool encode_fn() {
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}
}  // namespace

bool mma_available() {
    static int avail = -1;
    if (avail < 0) {
        int dev = 0, major = 0, minor = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        avail = (major == 10 && minor == 0 && encode_fn()) ? 1 : 0;
        const char *e = getenv("ACM_MMA");
        if (e && e[0] == '0') avail = 0;
    }
    return avail == 1;
}

// 2-D bf16 map over a 64x64-blocked [rows][k] matrix, seen as
// (ceil(rows/64) * k/64 * 64) rows of 64 elements; box {64, 64 rows}, 128-byte
// swizzle.  Boxes past the end read as zero.
static_assert(sizeof(TensorMap) == sizeof(CUtensorMap), "tensor map storage");
bool bf16_map(TensorMap *tmap, const void *base, int64_t rows, int64_t k) {
    CUtensorMap *map = reinterpret_cast<CUtensorMap *>(tmap);
    if (!encode_fn() || k % MBK || ((uintptr_t)base & 15)) return false;
    const int64_t rows2 = (rows + 63) / 64 * (k / 64) * 64;
    cuuint64_t dims[2] = {(cuuint64_t)MBK, (cuuint64_t)rows2};
    cuuint64_t strides[1] = {(cuuint64_t)MBK * 2};
    cuuint32_t box[2] = {MBK, 64};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

cudaError_t split_act_launch(const float *x, int ldx, int m, int k, void *hi, void *lo, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    if (k % 4 || ldx % 4) return cudaErrorInvalidValue;
    const int64_t total = (int64_t)m * k / 4;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    cudaError_t e = launch_pdl(k_split_act, dim3(grid), dim3(256), 0, st, x, ldx, m, k,
                               static_cast<__nv_bfloat16 *>(hi), static_cast<__nv_bfloat16 *>(lo));
    if (e != cudaSuccess) return e;
    return launched(1);
}

cudaError_t split_act_norm_launch(const float *x, int ldx, int m, int k, const float *norm_w, float eps, void *hi,
                                  void *lo, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    if (k % 4 || ldx % 4 || !norm_w || ((uintptr_t)x & 15) || ((uintptr_t)norm_w & 15)) return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(k_split_act_norm, dim3(m), dim3(256), 0, st, x, ldx, k, norm_w, eps,
                               static_cast<__nv_bfloat16 *>(hi), static_cast<__nv_bfloat16 *>(lo));
    if (e != cudaSuccess) return e;
    return launched(1);
}

cudaError_t split_act_reduce_norm_launch(const float *ws, int ks, int m, float *x, int k, const float *norm_w,
                                         float eps, void *hi, void *lo, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    if (ks < 1 || k % 4 || !norm_w || ((uintptr_t)x & 15) || ((uintptr_t)ws & 15) || ((uintptr_t)norm_w & 15))
        return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(k_split_act_reduce_norm, dim3(m), dim3(256), 0, st, ws, ks, m, x, k, norm_w, eps,
                               static_cast<__nv_bfloat16 *>(hi), static_cast<__nv_bfloat16 *>(lo));
    if (e != cudaSuccess) return e;
    return launched(1);
}

cudaError_t split_weight_launch(int type, const void *w, int64_t n, int k, void *hi, void *lo, cudaStream_t st) {
    if (k % 32) return cudaErrorInvalidValue;
    const int64_t total = n * (k / 32);
    const int grid = (int)std::min<int64_t>((total + 127) / 128, 148 * 16);
    auto *h = static_cast<__nv_bfloat16 *>(hi);
    auto *l = static_cast<__nv_bfloat16 *>(lo);
    const uint8_t *wb = static_cast<const uint8_t *>(w);
    switch (type) {
        case T_F32: k_split_weight<T_F32><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_F16: k_split_weight<T_F16><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_Q4_0: k_split_weight<T_Q4_0><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_Q5_0: k_split_weight<T_Q5_0><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_Q8_0: k_split_weight<T_Q8_0><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_Q4_K: k_split_weight<T_Q4_K><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_Q5_K: k_split_weight<T_Q5_K><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        case T_Q6_K: k_split_weight<T_Q6_K><<<grid, 128, 0, st>>>(wb, n, k, h, l); break;
        default: return cudaErrorInvalidValue;
    }
    return launched(1);
}

cudaError_t attn_split_launch(const AttnMmaOps &o, cudaStream_t st) {
    if (o.hd > 128 || o.hd % 64 || o.page_size % 64 || o.Lp % 64) return cudaErrorInvalidValue;
    AttnSplitArgs a{o.q,  o.kc, o.vc, o.kv_f16, o.page_row, o.layer_off, o.page_size, o.kvd, o.ntok, o.L,  o.Lp, o.G,
                    o.nh, o.hd, o.rq, static_cast<__nv_bfloat16 *>(o.qh), static_cast<__nv_bfloat16 *>(o.ql),
                    static_cast<__nv_bfloat16 *>(o.kh), static_cast<__nv_bfloat16 *>(o.kl),
                    static_cast<__nv_bfloat16 *>(o.vh), static_cast<__nv_bfloat16 *>(o.vl)};
    const size_t smem = (size_t)64 * (o.hd + 1) * sizeof(float);
    const int nqb = (int)((o.G * (int64_t)o.ntok + 63) / 64);
    cudaError_t e = launch_pdl(k_attn_split, dim3(o.Lp / 64 + nqb, o.nkv), dim3(256), smem, st, a);
    if (e != cudaSuccess) return e;
    return launched(1);
}

cudaError_t attn_softmax_launch(const AttnMmaOps &o, cudaStream_t st) {
    const int rows = o.G * o.ntok;
    cudaError_t e = launch_pdl(k_attn_softmax, dim3((rows + 7) / 8, o.nkv), dim3(256), 0, st, o.S, o.ntok, o.G, o.Lp,
                               o.pos0, o.scale, o.rq, static_cast<__nv_bfloat16 *>(o.ph),
                               static_cast<__nv_bfloat16 *>(o.pl));
    if (e != cudaSuccess) return e;
    return launched(1);
}

cudaError_t mma_gemm_launch(const MmaGemmSeg *segs, int nseg, const TensorMap *x_hi, const TensorMap *x_lo, int m,
                            int k, cudaStream_t st, float *ws, size_t ws_floats) {
    return mma_gemm_batched_launch(segs, nseg, x_hi, x_lo, m, k, MmaBatch{}, st, ws, ws_floats);
}

cudaError_t mma_gemm_batched_launch(const MmaGemmSeg *segs, int nseg, const TensorMap *x_hi, const TensorMap *x_lo,
                                    int m, int k, const MmaBatch &bt, cudaStream_t st, float *ws, size_t ws_floats) {
    if (nseg < 1 || nseg > MMA_MAX_SEG || m <= 0 || k % MBK || bt.n < 1 || (bt.n > 1 && nseg != 1))
        return cudaErrorInvalidValue;
    MmaArgs a;
    memset(&a, 0, sizeof(a));
    a.a_bstride = bt.a_stride;
    a.b_bstride = bt.b_stride;
    a.rmod = bt.rmod;
    a.rmul = bt.rmul;
    a.rdiv = bt.rdiv;
    a.rbatch = bt.rbatch;
    if (bt.causal && bt.cntok < 1) return cudaErrorInvalidValue;
    a.causal = bt.causal;
    a.cntok = bt.cntok;
    a.cpos0 = bt.cpos0;
    a.nseg = nseg;
    a.m = m;
    a.k = k;
    a.ttiles = (m + MBN - 1) / MBN;
    a.bhi = *reinterpret_cast<const CUtensorMap *>(x_hi);
    a.blo = *reinterpret_cast<const CUtensorMap *>(x_lo);
    int tiles = 0;
    for (int i = 0; i < nseg; i++) {
        const MmaGemmSeg &g = segs[i];
        MmaSeg &s = a.seg[i];
        s.ahi = *reinterpret_cast<const CUtensorMap *>(g.map_hi);
        s.alo = *reinterpret_cast<const CUtensorMap *>(g.map_lo);
        s.pair = g.map_hi2 != nullptr;
        if (s.pair) {
            s.ahi2 = *reinterpret_cast<const CUtensorMap *>(g.map_hi2);
            s.alo2 = *reinterpret_cast<const CUtensorMap *>(g.map_lo2);
        }
        s.n = (int)g.n;
        s.epi = g.epi;
        s.y = g.y;
        s.ldy = g.ldy;
        s.bias = g.bias;
        s.yrow = g.yrow;
        s.tile0 = tiles;
        const int rpt = s.pair ? MBM / 2 : MBM;
        tiles += (int)((g.n + rpt - 1) / rpt) * a.ttiles;
    }
    static std::atomic<bool> attr[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_mma_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, MMA_SMEM);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    // split-K when the tiles leave most SMs idle and K is long: one
    // segment, no SwiGLU pair, not batched, a workspace for the partials
    a.ksplit = 1;
    const int KTA = k / MBK;
    if (nseg == 1 && bt.n == 1 && !a.seg[0].pair && ws && tiles * 2 <= 148 && KTA >= 16) {
        int ks = std::min(KTA / 8, 148 / tiles);
        while (ks > 1 && (size_t)ks * m * segs[0].n > ws_floats) ks--;
        a.ksplit = std::max(1, ks);
        a.ws = ws;
    }
    cudaError_t e = launch_pdl(k_mma_gemm, dim3(tiles, bt.n, a.ksplit), dim3(MMA_THREADS), MMA_SMEM, st, a);
    if (e != cudaSuccess) return e;
    if (a.ksplit > 1) {
        e = split_reduce_launch(ws, a.ksplit, m, (int)segs[0].n, segs[0].y, segs[0].ldy, segs[0].epi, segs[0].bias,
                                segs[0].yrow, st);
        if (e != cudaSuccess) return e;
        return launched(2);
    }
    return launched(1);
}

cudaError_t split_reduce_launch(const float *ws, int ks, int m, int n, float *y, int ldy, int epi, const float *bias,
                                const int32_t *yrow, cudaStream_t st) {
    const int64_t total = (int64_t)m * n;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    return launch_pdl(k_split_reduce, dim3(grid), dim3(256), 0, st, ws, ks, m, n, y, ldy, epi, bias, yrow);
}

}  // namespace acm
