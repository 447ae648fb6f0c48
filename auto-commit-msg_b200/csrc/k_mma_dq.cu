// k_mma_dq.cu -- tensor-core GEMM for prefill with the weights dequantized
// in shared memory: y[m][n] (epi)= x[m][:] . W[n][:] (tensor.go:253-303 for
// M > 8 tokens) reading W as the GGUF blocks uploaded unchanged.
//
// The reference's matmul dequantizes a tile of rows into fp32 and dots it
// at once, never keeping fp32 weights (tensor.go:263-297).  Here likewise:
//   warp 0       producer: per 64 K-elements the TMA loads of the
//                activations' bf16 hi/lo tiles (as k_mma.cu);
//   warps 2..17  dequantizers.  Per 256 K-elements ("compact stage") they
//                copy each weight row's blocks that cover them (the
//                16-byte-aligned superset: Q6_K rows sit on 2-byte
//                boundaries) with 16-byte asynchronous copies, one or two
//                stages ahead; per 64 K-elements each thread decodes 16
//                elements of one row exactly (the reference's formulas, as
//                dequant_run32 computes them), splits them into bf16 hi + lo (as the
//                split cache of k_mma.cu does: the products are identical)
//                and writes both into the 128-byte-swizzled K-major A tiles
//                the MMA reads;
//   warp 1       allocates 128 TMEM columns; lane 0 issues the three
//                tcgen05.mma (hi.hi, hi.lo, lo.hi; M=128, N=128, K=16) per 16
//                K-elements and frees stages with tcgen05.commit;
//   warps 2..17  then the epilogue: each reads its TMEM lane quadrant
//                (warp % 4) for a quarter of the token columns; a SwiGLU
//                pair's gate and up rows meet in shared memory.
// A tile is 128 weight rows x 128 tokens, so each dequantized weight feeds
// 128 tokens' products: per 64 K-elements the CTA reads the rows' quantized
// bytes (4.6 KB for Q4_K) and 32 KB of activation splits, against 48 KB of
// split operands for half the tokens in k_mma.cu.  No cluster multicast.
#include <cuda.h>
#include <atomic>
#include <cuda_bf16.h>
#include <float.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "mma_dev.cuh"
#include "quant.cuh"

namespace acm {

namespace {

using namespace mma;

constexpr int DM = 128;  // weight rows per tile
constexpr int DBLK = 64;  // tokens per block of the activation splits (one TMA box)
constexpr int DBMAX = 3;  // blocks per token tile: N = 64, 128 or 192 tokens
constexpr int DN = DBLK * DBMAX;
constexpr int DK = 64;   // K elements per MMA stage (one 128-byte swizzle row of bf16)
constexpr int DKC = 256; // K elements per compact stage
constexpr int DCST_MAX = 3;  // compact stages (3 where shared memory allows, else 2)
constexpr int DAST = 2;  // A (dequantized) stages
constexpr int DBST = 2;  // B (activation) stages
constexpr int DA_BYTES = DM * DK * 2;  // 16 KB per half (hi or lo)
constexpr int DBOX = DBLK * DK * 2;    // 8 KB: one 64-token box of one half
constexpr int DQ_WARPS = 16;  // 512 dequantizing threads, 16 elements each per K step
constexpr int DQ_THREADS = (2 + DQ_WARPS) * 32;
constexpr uint32_t D_TMEM_COLS = 256;  // power of two >= DN

// Bytes one row needs for 256 elements, and its compact-stage slot (room
// for the 16-byte-aligned superset copy).
__host__ __device__ constexpr int rb256(int t) { return blk_bytes(t) * (256 / blk_elems(t)); }
__host__ __device__ constexpr int slot_bytes(int t) { return (rb256(t) + 15 + 15) & ~15; }

}  // namespace

struct DqSeg {
    const uint8_t *w, *w2;  // GGUF rows (w2: the up-projection of a SwiGLU pair)
    int type;
    int64_t rb;             // row bytes at K
    int n;
    int pair;
    int tile0;
    int epi;
    float *y;
    int ldy;
    const float *bias;
    const int32_t *yrow;
};
constexpr int DQ_MAX_SEG = 3;
struct DqArgs {
    DqSeg seg[DQ_MAX_SEG];
    int nseg;
    CUtensorMap bhi, blo;  // activations split, box {64, 64 rows}
    int m, k;
    int ttiles;            // token tiles: tile t spans blocks [t*nblk/ttiles, (t+1)*nblk/ttiles)
    int ksplit;            // K slices (blockIdx.z), partial sums to ws[slice][tok][n]
    float *ws;
    int slot;              // compact slot bytes of the launch's widest format
    int ncst;              // compact stages, 2 or 3 (copies run ncst - 1 stages ahead)
    int bmax;              // most blocks in one token tile of this launch (B stage: 2 * bmax boxes)
};

__device__ __forceinline__ void store_uint4(uint8_t *p, uint4 v) { *reinterpret_cast<uint4 *>(p) = v; }

// Run `run` (32 elements) of a row, exact (the reference's formulas, as
// dequant_run32), with the byte-to-float conversion on the 2^23 magic and
// the arithmetic on packed two-lane fp32: Q4_K d1*q - m1 as one fused
// multiply-add of an exact product (one rounding, the reference's); Q6_K
// (d*sc) * (q - 32) as the reference orders it.
template <int T>
__device__ __forceinline__ void dq_fast(const uint8_t *blk_row, int run, int sub, float (&v)[16]) {
    const float2 nmag = make_float2(-MAGIC, -MAGIC);
    if constexpr (T == T_Q4_K) {
        const uint8_t *blk = blk_row + (run >> 3) * 144;
        const int s = run & 7, g = s >> 1, hi = s & 1;
        uint32_t hw[4], q[4];
        ld_words_a2<4>(blk, hw);
        ld_words_a2<4>(blk + 16 + 32 * g + 16 * sub, q);
        float sc, mn;
        scale_min_k4(s, hw[1], hw[2], hw[3], sc, mn);
        const float d1 = f16u(hw[0]) * sc, m1 = f16u(hw[0] >> 16) * mn;
        const float2 dd = make_float2(d1, d1), mm = make_float2(-m1, -m1);
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t nb = hi ? ((q[w] >> 4) & 0x0F0F0F0Fu) : (q[w] & 0x0F0F0F0Fu);
            const float2 a = __fadd2_rn(make_float2(byte_m23(nb, 0), byte_m23(nb, 1)), nmag);
            const float2 b = __fadd2_rn(make_float2(byte_m23(nb, 2), byte_m23(nb, 3)), nmag);
            const float2 ra = __ffma2_rn(dd, a, mm), rb = __ffma2_rn(dd, b, mm);
            v[4 * w] = ra.x;
            v[4 * w + 1] = ra.y;
            v[4 * w + 2] = rb.x;
            v[4 * w + 3] = rb.y;
        }
    } else {  // Q6_K
        const uint8_t *blk = blk_row + (run >> 3) * 210;
        const int s = run & 7, h = s >> 2, t = s & 3;
        uint32_t ql[4], qh[4], sw[2];
        ld_words_a2<4>(blk + 64 * h + ((t & 1) ? 32 : 0) + 16 * sub, ql);
        ld_words_a2<4>(blk + 128 + 32 * h + 16 * sub, qh);
        ld_words_a2<2>(blk + 192 + 8 * h, sw);
        const float d = f16u(ld_u16_a2(blk + 208));
        const int si0 = 2 * t, si1 = 1 + 2 * t;  // sc index for l < 16 and l >= 16
        const float ds0 = d * (float)(int8_t)((sw[si0 >> 2] >> (8 * (si0 & 3))) & 0xFF);
        const float ds1 = d * (float)(int8_t)((sw[si1 >> 2] >> (8 * (si1 & 3))) & 0xFF);
        const float2 n32 = make_float2(-(MAGIC + 32.0f), -(MAGIC + 32.0f));
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t lo4 = (t < 2) ? (ql[w] & 0x0F0F0F0Fu) : ((ql[w] >> 4) & 0x0F0F0F0Fu);
            const uint32_t q6 = lo4 | (((qh[w] >> (2 * t)) & 0x03030303u) << 4);
            const float2 a = __fadd2_rn(make_float2(byte_m23(q6, 0), byte_m23(q6, 1)), n32);
            const float2 b = __fadd2_rn(make_float2(byte_m23(q6, 2), byte_m23(q6, 3)), n32);
            const float ds = sub ? ds1 : ds0;  // elements l < 16 or l >= 16 of the run
            const float2 dd = make_float2(ds, ds);
            const float2 ra = __fmul2_rn(dd, a), rb = __fmul2_rn(dd, b);
            v[4 * w] = ra.x;
            v[4 * w + 1] = ra.y;
            v[4 * w + 2] = rb.x;
            v[4 * w + 3] = rb.y;
        }
    }
}

// Elements 16 sub .. 16 sub + 15 of run `run` of a row into the A tiles
// (hi, lo), as chunks 4 half + 2 sub + {0, 1} of the row's 128-byte line.
template <int T>
__device__ __forceinline__ void dq_run(const uint8_t *slot_row, int run, int sub, uint8_t *ahi, uint8_t *alo, int row,
                                       int half, bool valid) {
    float v[16];
    if (valid) {
        if constexpr (T == T_Q4_K || T == T_Q6_K) {
            dq_fast<T>(slot_row, run, sub, v);
        } else {
            float w[32];
            dequant_run32<T>(slot_row, run, w);
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = sub ? w[16 + i] : w[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = 0.f;
    }
    // bf16 hi / lo of the 16 elements: 2 chunks of 8, chunk j = 4 half + 2 sub
    // + c of the row's 128-byte line, swizzled as TMA's 128-byte mode lays it out
#pragma unroll
    for (int c = 0; c < 2; c++) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            // hi = bf16(v), lo = bf16(v - hi), as split_bf16 does, two at a time
            const float2 ab = make_float2(v[8 * c + 2 * e], v[8 * c + 2 * e + 1]);
            const __nv_bfloat162 hb = __floats2bfloat162_rn(ab.x, ab.y);
            const float2 hf = __bfloat1622float2(hb);
            const float2 rest = __fadd2_rn(ab, make_float2(-hf.x, -hf.y));
            const __nv_bfloat162 lb = __floats2bfloat162_rn(rest.x, rest.y);
            h[e] = *reinterpret_cast<const uint32_t *>(&hb);
            l[e] = *reinterpret_cast<const uint32_t *>(&lb);
        }
        const int j = 4 * half + 2 * sub + c;
        const int off = row * 128 + ((j ^ (row & 7)) << 4);
        store_uint4(ahi + off, make_uint4(h[0], h[1], h[2], h[3]));
        store_uint4(alo + off, make_uint4(l[0], l[1], l[2], l[3]));
    }
}

template <int TA, int TB>
__global__ void __launch_bounds__(DQ_THREADS, 1) k_mma_dq(const __grid_constant__ DqArgs A) {
    extern __shared__ uint8_t dsm_raw[];
    uint8_t *dsm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
    // layout: A stages (hi, lo) | B stages (hi, lo) | compact stages | barriers
    uint8_t *astg = dsm;
    uint8_t *bstg = astg + DAST * 2 * DA_BYTES;
    const int bhalf = A.bmax * DBOX;  // bytes of one half (hi or lo) of a B stage
    uint8_t *cstg = bstg + DBST * 2 * bhalf;
    uint64_t *bars = reinterpret_cast<uint64_t *>(cstg + (size_t)A.ncst * DM * A.slot + 16);
    uint64_t *afull = bars, *aempty = afull + DAST;
    uint64_t *bfull = aempty + DAST, *bempty = bfull + DBST;
    uint64_t *accf = bempty + DBST;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int si = 0;
    while (si + 1 < A.nseg && (int)blockIdx.x >= A.seg[si + 1].tile0) si++;
    const DqSeg &S = A.seg[si];
    const int local = blockIdx.x - S.tile0;
    const int rt = local / A.ttiles, tt = local - rt * A.ttiles;
    const int rows_per_tile = S.pair ? DM / 2 : DM;
    const int nblk = (A.m + DBLK - 1) / DBLK;
    const int blk0 = tt * nblk / A.ttiles, nb = (tt + 1) * nblk / A.ttiles - blk0;  // 1..DBMAX blocks
    const int row0 = rt * rows_per_tile, tok0 = blk0 * DBLK, ntile = nb * DBLK;
    const uint32_t idesc = idesc_bf16(DM, ntile);
    const int KTA = A.k / DK;
    const int kb0 = (int)((int64_t)KTA * blockIdx.z / A.ksplit), kb1 = (int)((int64_t)KTA * (blockIdx.z + 1) / A.ksplit);
    const int KT = kb1 - kb0;          // MMA stages (64 K-elements); kb0 a multiple of 4
    const int NC = (KT + 3) / 4;       // compact stages (256 K-elements)

    if (tid == 0) {
        for (int i = 0; i < DAST; i++) {
            mbar_init(&afull[i], DQ_WARPS);
            mbar_init(&aempty[i], 1);
        }
        for (int i = 0; i < DBST; i++) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        mbar_init(accf, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(D_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    if (tid == 0) pdl_trigger();

    if (warp == 0) {
        // ---- producer: activation tiles ----
        int bissued = 0;
        bool stop = false;
        auto issue_b = [&](int kt) -> bool {
            const int bs = kt % DBST;
            if (lane == 0) {
                if (kt >= DBST && !mbar_wait(&bempty[bs], ((kt / DBST) & 1) ^ 1)) return false;
                uint8_t *st = bstg + (size_t)bs * 2 * bhalf;
                mbar_arrive_expect_tx(&bfull[bs], 2 * nb * DBOX);
                // one 64-row box per token block and half, contiguous: the
                // MMA reads the nb boxes as one K-major operand of 64 * nb rows
                for (int b = 0; b < nb; b++) {
                    const int yb = ((blk0 + b) * KTA + kb0 + kt) * 64;
                    tma_load_2d(st + b * DBOX, &A.bhi, 0, yb, &bfull[bs]);
                    tma_load_2d(st + bhalf + b * DBOX, &A.blo, 0, yb, &bfull[bs]);
                }
            }
            return true;
        };
        for (int kt = 0; kt < KT && !stop; kt++) {
            if (!__shfl_sync(0xffffffffu, issue_b(kt) ? 1 : 0, 0)) {
                stop = true;
                break;
            }
            bissued = kt + 1;
        }
        // no copy may still be landing when the CTA exits (fixed bound)
        if (lane == 0)
            for (int kt = max(0, bissued - DBST); kt < bissued; kt++)
                mbar_wait_limit(&bfull[kt % DBST], (kt / DBST) & 1, WAIT_LIMIT);
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            for (int kt = 0; kt < KT; kt++) {
                const int as = kt % DAST, bs = kt % DBST;
                if (!mbar_wait(&afull[as], (kt / DAST) & 1)) break;
                if (!mbar_wait(&bfull[bs], (kt / DBST) & 1)) break;
                tc_fence_after();
                const uint32_t ahi = smem_u32(astg + (size_t)as * 2 * DA_BYTES), alo = ahi + DA_BYTES;
                const uint32_t bhi = smem_u32(bstg + (size_t)bs * 2 * bhalf), blo = bhi + bhalf;
#pragma unroll
                for (int kk = 0; kk < DK / 16; kk++) {
                    const uint32_t off = kk * 32;
                    const uint64_t dah = sw128_desc(ahi + off), dal = sw128_desc(alo + off);
                    const uint64_t dbh = sw128_desc(bhi + off), dbl = sw128_desc(blo + off);
                    tc_mma(tmem, dah, dbh, idesc, (kt | kk) != 0);
                    tc_mma(tmem, dah, dbl, idesc, 1u);
                    tc_mma(tmem, dal, dbh, idesc, 1u);
                }
                tc_commit(&aempty[as]);
                tc_commit(&bempty[bs]);
            }
            tc_commit(accf);
        }
    } else {
        // ---- dequantizers (warps 2..17), then the epilogue ----
        const int q = (warp - 2) * 32 + lane;  // 0..511: row q / 4, run half, 16-element sub
        const int row = q >> 2, half = (q >> 1) & 1, sub = q & 1;
        const int lr = S.pair ? (row & 63) : row;
        const bool valid = row0 + lr < S.n;
        const uint8_t *wrow = (S.pair && row >= 64 ? S.w2 : S.w) + (int64_t)(row0 + lr) * S.rb;
        const int64_t cbytes = (int64_t)DKC / blk_elems(S.type) * blk_bytes(S.type);  // bytes of 256 elements
        // compact stage c: this row's blocks of K [kb0*64 + 256c, +256), the
        // 16-byte-aligned superset, copied by the row's four threads with
        // 16-byte asynchronous copies into the row's slot
        auto load_compact = [&](int c) {
            if (!valid) return;
            const uint8_t *src = wrow + (int64_t)(kb0 / 4 + c) * cbytes;
            const uintptr_t a0 = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
            const uintptr_t a1 = (reinterpret_cast<uintptr_t>(src) + cbytes + 15) & ~uintptr_t(15);
            uint8_t *dst = cstg + (size_t)(c % A.ncst) * DM * A.slot + (size_t)row * A.slot;
            for (uintptr_t o = (uintptr_t)(q & 3) * 16; a0 + o < a1; o += 64)
                cp_async16(dst + o, reinterpret_cast<const void *>(a0 + o));
        };
        load_compact(0);
        cp_async_commit();
        if (A.ncst == 3) {
            if (NC > 1) load_compact(1);
            cp_async_commit();
        }
        // A warp whose bounded wait gave up stops decoding but keeps taking
        // the loop's barriers, so that all dequantizers meet them alike.
        bool ok = true;
        for (int kt = 0; kt < KT; kt++) {
            const int c = kt >> 2, cs = c % A.ncst, as = kt % DAST;
            if ((kt & 3) == 0) {
                // stage c landed for every row (the newest group, stage c + 1
                // of a 3-stage ring, may still be in flight), and every
                // dequantizer is done with stage c - 1, whose slot the next
                // copies reuse
                const int ahead = A.ncst - 1;
                if (ahead == 2) cp_async_wait_group<1>();
                else cp_async_wait_all();
                named_sync(3, DQ_WARPS * 32);
                if (ok && c + ahead < NC) load_compact(c + ahead);
                cp_async_commit();
            }
            if (!ok) continue;
            if (kt >= DAST) ok = mbar_wait(&aempty[as], ((kt / DAST) - 1) & 1);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) continue;
            const uint8_t *src = wrow + (int64_t)(kb0 / 4 + c) * cbytes;
            const uint8_t *slot_row = cstg + (size_t)cs * DM * A.slot + (size_t)row * A.slot +
                                      (reinterpret_cast<uintptr_t>(src) & 15);
            uint8_t *ahi = astg + (size_t)as * 2 * DA_BYTES, *alo = ahi + DA_BYTES;
            const int run = (kt & 3) * 2 + half;  // 32-element run within the 256 of the slot
            if (S.type == TA) dq_run<TA>(slot_row, run, sub, ahi, alo, row, half, valid);
            else if constexpr (TB != TA) dq_run<TB>(slot_row, run, sub, ahi, alo, row, half, valid);
            // generic-proxy writes -> the tensor core's async-proxy reads
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[as]);
        }
        cp_async_wait_all();  // no copy lands after the CTA exits
        // ---- epilogue, on all dequantizer warps: a warp reads its TMEM lane
        // quadrant (warp % 4) and the column chunks cg*16 + 64 i ----
        const int qd = warp & 3, cg = (warp - 2) >> 2;
        const int et = tid - 64;  // 0 .. DQ_WARPS * 32 - 1
        const bool fin = named_and(1, DQ_WARPS * 32, mbar_wait(accf, 0));
        tc_fence_after();
        if (fin) {
            const int lrow = qd * 32 + lane;  // accumulator row (TMEM lane)
            const uint32_t tl = tmem + ((uint32_t)(qd * 32) << 16);
            if (S.pair) {
                // gate rows (lanes 0..63) and up rows (64..127) to the idle A/B
                // stages, [64][ntile + 1] floats each (2 * 64 * 193 * 4 bytes
                // <= the 64 KB of A stages + 2 * DBST * DBOX), then every
                // thread takes outputs with consecutive rows (coalesced stores)
                float *xg = reinterpret_cast<float *>(astg), *xu = xg + 64 * (ntile + 1);
                float *xr = (qd < 2 ? xg + lrow * (ntile + 1) : xu + (lrow - 64) * (ntile + 1));
                for (int c0 = cg * 16; c0 < ntile; c0 += 64) {
                    float v[16];
                    tc_ld16(tl + (uint32_t)c0, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) xr[c0 + j] = v[j];
                }
                named_sync(1, DQ_WARPS * 32);
                for (int i = et; i < 64 * ntile; i += DQ_WARPS * 32) {
                    const int r = i & 63, c = i >> 6;
                    const int n = row0 + r, tok = tok0 + c;
                    if (n < S.n && tok < A.m) {
                        const float g = xg[r * (ntile + 1) + c], u = xu[r * (ntile + 1) + c];
                        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_exp(-g)));
                        float *yp = S.y + (int64_t)(S.yrow ? S.yrow[tok] : tok) * S.ldy + n;
                        *yp = __fmul_rn(__fmul_rn(g, sg), u);
                    }
                }
            } else {
                const int n = row0 + lrow;
                for (int c0 = cg * 16; c0 < ntile; c0 += 64) {
                    float v[16];
                    tc_ld16(tl + (uint32_t)c0, v);  // warp-wide: before any lane-dependent branch
                    if (n >= S.n) {
                    } else if (A.ksplit > 1) {
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int tok = tok0 + c0 + j;
                            if (tok < A.m) A.ws[((int64_t)blockIdx.z * A.m + tok) * S.n + n] = v[j];
                        }
                    } else {
                        const float b = S.bias ? S.bias[n] : 0.f;
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            const int tok = tok0 + c0 + j;
                            if (tok < A.m) {
                                float *yp = S.y + (int64_t)(S.yrow ? S.yrow[tok] : tok) * S.ldy + n;
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
        // the accumulator must be idle before it is freed (fixed bound)
        mbar_wait_limit(accf, 0, WAIT_LIMIT);
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(D_TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
bool dq_type(int t) {
    return t == T_Q4_0 || t == T_Q5_0 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K;
}

static size_t dq_smem(int slot, int ncst, int bmax) {
    return 1024 + (size_t)DAST * 2 * DA_BYTES + (size_t)DBST * 2 * bmax * DBOX + (size_t)ncst * DM * slot + 16 + 256;
}

// SMs of the current device (queried once per device).
static int num_sms() {
    static int cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int &v = cache[dev & 63];
    if (!v && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) v = 148;
    return v;
}

template <int TA, int TB>
static cudaError_t dq_inst(const DqArgs &a, dim3 grid, size_t smem, cudaStream_t st) {
    static std::atomic<bool> attr[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_mma_dq<TA, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    return launch_pdl(k_mma_dq<TA, TB>, grid, dim3(DQ_THREADS), smem, st, a);
}

// Same interface as mma_gemm_launch, the weights given as GGUF rows
// (MmaGemmSeg::w / w2 / wtype); their types are one dq_type or {Q4_K, Q6_K}.
cudaError_t mma_dq_launch(const MmaGemmSeg *segs, int nseg, const TensorMap *x_hi, const TensorMap *x_lo, int m, int k,
                          cudaStream_t st, float *ws, size_t ws_floats, int *defer_ks) {
    if (defer_ks) *defer_ks = 0;
    if (nseg < 1 || nseg > DQ_MAX_SEG || m <= 0 || k % DKC) return cudaErrorInvalidValue;
    int ta = segs[0].wtype, tb = segs[0].wtype;
    for (int i = 0; i < nseg; i++) {
        const int t = segs[i].wtype;
        if (!dq_type(t) || !segs[i].w || (segs[i].map_hi2 && !segs[i].w2)) return cudaErrorInvalidValue;
        if (t != ta) tb = t;
    }
    for (int i = 0; i < nseg; i++)
        if (segs[i].wtype != ta && segs[i].wtype != tb) return cudaErrorInvalidValue;
    const bool q46 = (ta == T_Q4_K && tb == T_Q6_K) || (ta == T_Q6_K && tb == T_Q4_K);
    if (ta != tb && !q46) return cudaErrorInvalidValue;
    DqArgs a;
    memset(&a, 0, sizeof(a));
    a.nseg = nseg;
    a.m = m;
    a.k = k;
    a.bhi = *reinterpret_cast<const CUtensorMap *>(x_hi);
    a.blo = *reinterpret_cast<const CUtensorMap *>(x_lo);
    int rtiles = 0, slot = 0;
    for (int i = 0; i < nseg; i++) {
        const MmaGemmSeg &g = segs[i];
        DqSeg &s = a.seg[i];
        s.w = static_cast<const uint8_t *>(g.w);
        s.w2 = static_cast<const uint8_t *>(g.w2);
        s.type = g.wtype;
        s.rb = row_bytes(g.wtype, k);
        s.n = (int)g.n;
        s.pair = g.w2 != nullptr;
        if (s.pair && g.n % 64) return cudaErrorInvalidValue;
        s.epi = g.epi;
        s.y = g.y;
        s.ldy = g.ldy;
        s.bias = g.bias;
        s.yrow = g.yrow;
        const int rpt = s.pair ? DM / 2 : DM;
        rtiles += (int)((g.n + rpt - 1) / rpt);
        slot = std::max(slot, slot_bytes(g.wtype));
    }
    a.slot = slot;
    // Token tiles of whole 64-token blocks.  Every tile dequantizes its rows
    // once, so fewer, wider tiles cost less dequantization; the tile is the
    // narrowest that still fits the launch into one wave (a second, partial
    // wave would cost a whole tile's time).  Split-K launches keep 2 blocks.
    const int sms = num_sms();
    const int KTA = k / DK;
    const int nblk = (m + DBLK - 1) / DBLK;
    const bool splitk = nseg == 1 && !a.seg[0].pair && ws && KTA >= 16;
    int bm = 1;
    if (splitk) bm = 2;
    else
        while (bm < DBMAX && (int64_t)rtiles * ((nblk + bm - 1) / bm) > sms) bm++;
    bm = std::min(bm, nblk);
    while (bm > 1 && dq_smem(slot, 2, bm) > 227 * 1024) bm--;
    a.ttiles = (nblk + bm - 1) / bm;
    a.bmax = (nblk + a.ttiles - 1) / a.ttiles;  // blocks spread evenly: tiles differ by at most one
    int tiles = 0;
    for (int i = 0; i < nseg; i++) {
        DqSeg &s = a.seg[i];
        s.tile0 = tiles;
        const int rpt = s.pair ? DM / 2 : DM;
        tiles += (s.n + rpt - 1) / rpt * a.ttiles;
    }
    // split-K (one plain segment, long K): slices on 256-element boundaries
    a.ksplit = 1;
    if (splitk && tiles * 2 <= sms) {
        int ks = std::min(KTA / 8, sms / tiles);
        while (ks > 1 && ((size_t)ks * m * segs[0].n > ws_floats || (KTA / 4) % ks)) ks--;
        a.ksplit = std::max(1, ks);
        a.ws = ws;
    }
    a.ncst = dq_smem(slot, DCST_MAX, a.bmax) <= 227 * 1024 ? DCST_MAX : 2;
    const size_t smem = dq_smem(slot, a.ncst, a.bmax);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    const dim3 grid(tiles, 1, a.ksplit);
    cudaError_t e;
    if (q46) e = dq_inst<T_Q4_K, T_Q6_K>(a, grid, smem, st);
    else {
        switch (ta) {
            case T_Q4_K: e = dq_inst<T_Q4_K, T_Q4_K>(a, grid, smem, st); break;
            case T_Q6_K: e = dq_inst<T_Q6_K, T_Q6_K>(a, grid, smem, st); break;
            case T_Q8_0: e = dq_inst<T_Q8_0, T_Q8_0>(a, grid, smem, st); break;
            case T_Q5_K: e = dq_inst<T_Q5_K, T_Q5_K>(a, grid, smem, st); break;
            case T_Q4_0: e = dq_inst<T_Q4_0, T_Q4_0>(a, grid, smem, st); break;
            case T_Q5_0: e = dq_inst<T_Q5_0, T_Q5_0>(a, grid, smem, st); break;
            default: return cudaErrorInvalidValue;
        }
    }
    if (e != cudaSuccess) return e;
    if (a.ksplit > 1 && defer_ks) {
        *defer_ks = a.ksplit;  // the caller reduces
        return launched(1);
    }
    if (a.ksplit > 1) {
        e = split_reduce_launch(ws, a.ksplit, m, (int)segs[0].n, segs[0].y, segs[0].ldy, segs[0].epi, segs[0].bias,
                                segs[0].yrow, st);
        if (e != cudaSuccess) return e;
        return launched(2);
    }
    return launched(1);
}

}  // namespace acm
