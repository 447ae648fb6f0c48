// k_gemv.cu -- fused dequant-GEMV for decode (M = 1..8 tokens).
//
// The reference's matvec (internal/infer/tensor.go:253-303) dequantizes each
// weight row into an fp32 tile and dots it against the activations.  Decode
// is HBM-bound, so here the quantized GGUF bytes are streamed once, unchanged,
// and decoded in registers:
//   * one CTA per SM; each CTA owns a contiguous row range of one weight
//     matrix (several matrices -- q/k/v, gate/up -- share one launch);
//   * a producer warp moves whole rows into a ring of shared-memory stages
//     with the bulk-copy engine (cp.async.bulk + mbarrier), so every CTA has
//     tens of KB of HBM reads in flight from its first cycle;
//   * 8 consumer warps take one row at a time; lane l decodes units l, l+32,
//     ... (32 elements each) against the activation vector, which the CTA
//     stores in shared memory permuted into unit order (and optionally
//     RMS-normalised first: the norm before q/k/v, gate/up and lm_head);
//   * the row sum is a warp-shuffle reduction; the epilogue stores, adds to
//     the residual stream, or applies SwiGLU to a gate/up pair.
#include <stdio.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace acm {

__device__ int g_dev_error = 0;  // declared in common.cuh (relocatable device code)

template <int T, int MT>
__device__ __forceinline__ void prep_x(const GemvArgs &a, float *xs, float2 *xsum, float *red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.k;
    float sc[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) sc[m] = 1.0f;
    if (a.norm_w) {
        float ss[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) ss[m] = 0.f;
        for (int k = tid; k < K; k += 256)
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < a.m) {
                    float v = a.x[(int64_t)m * a.ldx + k];
                    ss[m] = fmaf(v, v, ss[m]);
                }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float w = warp_sum(ss[m]);
            if (lane == 0) red[warp * MT + m] = w;
        }
        named_sync(1, 256);
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float t = 0.f;
            for (int w = 0; w < 8; w++) t += red[w * MT + m];
            sc[m] = rms_scale(t, K, a.eps);
        }
    }
    for (int k = tid; k < K; k += 256) {
        int u, j;
        pos_unit<T>(k, K, u, j);
        const int off = u * 32 + (((j >> 2) ^ (u & 7)) << 2) + (j & 3);
        const float nw = a.norm_w ? a.norm_w[k] : 1.0f;
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float v = 0.f;
            if (m < a.m) {
                v = a.x[(int64_t)m * a.ldx + k];
                if (a.norm_w) v = __fmul_rn(__fmul_rn(v, sc[m]), nw);
            }
            xs[m * K + off] = v;
        }
    }
    named_sync(1, 256);
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        const int U = K / 32;
        for (int idx = tid; idx < MT * U; idx += 256) {
            const int m = idx / U, u = idx - m * U;
            const float *p = xs + m * K + u * 32;
            float lo = 0.f, hi = 0.f;
            // chunks 0..3 hold j < 16 (low sub-block), 4..7 j >= 16
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float4 a0 = *reinterpret_cast<const float4 *>(p + ((c ^ (u & 7)) << 2));
                const float4 a1 = *reinterpret_cast<const float4 *>(p + (((c + 4) ^ (u & 7)) << 2));
                lo += (a0.x + a0.y) + (a0.z + a0.w);
                hi += (a1.x + a1.y) + (a1.z + a1.w);
            }
            xsum[m * U + u] = make_float2(lo, hi);
        }
        named_sync(1, 256);
    }
}

template <int T, int MT>
__device__ __forceinline__ void gemv_consume(const GemvArgs &a, const GemvSeg &s, int r0, int r1, uint64_t *full,
                                             uint64_t *empty, const uint8_t *stg, const float *xs,
                                             const float2 *xsum) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.k, U = K / 32, R = s.rows_per_stage, NS = a.ns;
    const int nst = (r1 - r0 + R - 1) / R;
    const bool pair = s.w2 != nullptr;
    for (int i = 0; i < nst; i++) {
        const int slot = i % NS;
        if (!mbar_wait(&full[slot], (uint32_t)((i / NS) & 1))) return;
        const int ra = r0 + i * R, rbn = min(ra + R, r1);
        const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
        const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
        const int64_t c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
        const uint8_t *buf = stg + (size_t)slot * a.stage_bytes;
        for (int rr = warp; rr < rbn - ra; rr += 8) {
            const int n = ra + rr;
            const uint8_t *rp = buf + ((int64_t)n * s.rb - a0);
            float acc[MT], acc2[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) acc[m] = acc2[m] = 0.f;
            for (int u = lane; u < U; u += 32) {
                XView<MT> xv{xs + u * 32, K, u & 7};
                unit_dot<T, MT>(rp, u, K, xv, xsum + u, U, a.m, acc);
                if (pair) {
                    const uint8_t *rp2 = buf + (a1 - a0) + ((int64_t)n * s.rb2 - c0);
                    unit_dot<T, MT>(rp2, u, K, xv, xsum + u, U, a.m, acc2);
                }
            }
#pragma unroll
            for (int m = 0; m < MT; m++) {
                acc[m] = warp_sum(acc[m]);
                if (pair) acc2[m] = warp_sum(acc2[m]);
            }
            if (lane == 0) {
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    if (m < a.m) {
                        float v = acc[m];
                        if (s.bias) v += s.bias[n];
                        float *yp = s.y + (int64_t)(s.yrow ? s.yrow[m] : m) * s.ldy + n;
                        if (s.epi == EPI_ADD) {
                            *yp += v;
                        } else if (s.epi == EPI_SWIGLU) {
                            const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_exp(-v)));
                            *yp = __fmul_rn(__fmul_rn(v, sg), acc2[m]);
                        } else {
                            *yp = v;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
}

template <int MT>
__global__ void __launch_bounds__(GEMV_THREADS, 1) k_gemv(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    int sid = 0;
#pragma unroll 1
    for (int i = 1; i < a.nseg; i++)
        if ((int)blockIdx.x >= a.seg[i].cta0) sid = i;
    const GemvSeg &s = a.seg[sid];
    const int cta = (int)blockIdx.x - s.cta0;
    const int r0 = (int)((int64_t)s.n * cta / s.ncta), r1 = (int)((int64_t)s.n * (cta + 1) / s.ncta);
    const int K = a.k;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_NS_MAX;
    float *xs = reinterpret_cast<float *>(smem + 128);
    float2 *xsum = reinterpret_cast<float2 *>(xs + MT * K);
    float *red = reinterpret_cast<float *>(xsum + MT * (K / 32));
    uint8_t *stg = smem + a.stage_off;
    if (tid == 0) {
        for (int i = 0; i < a.ns; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 8);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (r1 <= r0) return;
    const int R = s.rows_per_stage, NS = a.ns;
    const int nst = (r1 - r0 + R - 1) / R;
    if (warp == 8) {
        if ((tid & 31) == 0) {
            for (int i = 0; i < nst; i++) {
                const int slot = i % NS;
                if (i >= NS && !mbar_wait(&empty[slot], (uint32_t)(((i / NS) - 1) & 1))) return;
                const int ra = r0 + i * R, rbn = min(ra + R, r1);
                const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
                const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
                uint32_t total = (uint32_t)(a1 - a0);
                int64_t c0 = 0, c1 = 0;
                if (s.w2) {
                    c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
                    c1 = ((int64_t)rbn * s.rb2 + 15) & ~int64_t(15);
                    total += (uint32_t)(c1 - c0);
                }
                uint8_t *dst = stg + (size_t)slot * a.stage_bytes;
                mbar_arrive_expect_tx(&full[slot], total);
                bulk_g2s(dst, s.w + a0, (uint32_t)(a1 - a0), &full[slot]);
                if (s.w2) bulk_g2s(dst + (a1 - a0), s.w2 + c0, (uint32_t)(c1 - c0), &full[slot]);
            }
        }
        return;
    }
    switch (s.type) {
#define ACM_GEMV_CASE(T)                                              \
    case T:                                                           \
        prep_x<T, MT>(a, xs, xsum, red);                              \
        gemv_consume<T, MT>(a, s, r0, r1, full, empty, stg, xs, xsum); \
        break;
        ACM_GEMV_CASE(T_Q4_K)
        ACM_GEMV_CASE(T_Q6_K)
        ACM_GEMV_CASE(T_Q8_0)
        ACM_GEMV_CASE(T_Q5_K)
        ACM_GEMV_CASE(T_Q4_0)
        ACM_GEMV_CASE(T_Q5_0)
        ACM_GEMV_CASE(T_F16)
        ACM_GEMV_CASE(T_F32)
#undef ACM_GEMV_CASE
        default:
            break;
    }
}

static const int SMEM_MAX = 227 * 1024;

static size_t x_bytes(int64_t k, int mt) {
    size_t b = 128 + (size_t)mt * k * 4 + (size_t)mt * (k / 32) * 8 + 8 * mt * 4;
    return (b + 127) & ~size_t(127);
}

bool gemv_supported(int type, int64_t k, int m) {
    if (!type_ok(type) || m < 1 || m > 8 || k % 32 || k % blk_elems(type)) return false;
    const int mt = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
    const size_t xb = x_bytes(k, mt);
    const int64_t rb = row_bytes(type, k);
    return xb + 2 * (size_t)(2 * rb + 64 + 128) + 16 <= (size_t)SMEM_MAX;
}

template <int MT>
static cudaError_t launch_mt(GemvArgs &a, int grid, size_t smem, cudaStream_t st) {
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
        if (e != cudaSuccess) return e;
        attr_done[dev & 63] = true;
    }
    k_gemv<MT><<<grid, GEMV_THREADS, smem, st>>>(a);
    return launched(1);
}

cudaError_t gemv_launch(const GemvSegDesc *segs, int nseg, const float *x, int ldx, int64_t k, int m,
                        const float *norm_w, float eps, int num_sms, cudaStream_t st) {
    if (nseg < 1 || nseg > GEMV_MAX_SEG || m < 1 || m > 8) return cudaErrorInvalidValue;
    const int mt = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
    GemvArgs a{};
    a.nseg = nseg;
    a.x = x;
    a.ldx = ldx;
    a.k = (int)k;
    a.m = m;
    a.norm_w = norm_w;
    a.eps = eps;
    const size_t xb = x_bytes(k, mt);
    // stage size: 32 KB target, at least two rows (pair: both matrices)
    int64_t maxrow = 0;
    double total_bytes = 0;
    for (int i = 0; i < nseg; i++) {
        const int64_t rb = row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1);
        maxrow = std::max(maxrow, rb);
        total_bytes += (double)rb * (double)segs[i].n;
    }
    // a stage holds R rows plus up to 60 bytes of 16-byte rounding (two
    // copies) and the 4-byte over-read of the unaligned word loader
    int64_t sb = std::max<int64_t>(32 * 1024, ((maxrow + 64 + 127) / 128) * 128);
    int ns = (int)std::min<int64_t>(6, ((int64_t)SMEM_MAX - (int64_t)xb - 16) / sb);
    if (ns < 2) {
        sb = ((maxrow + 64 + 127) / 128) * 128;
        ns = (int)std::min<int64_t>(GEMV_NS_MAX, ((int64_t)SMEM_MAX - (int64_t)xb - 16) / sb);
        if (ns < 2) return cudaErrorInvalidValue;
    }
    a.ns = ns;
    a.stage_bytes = (int)sb;
    a.stage_off = (int)xb;
    // CTAs per segment proportional to its bytes
    int grid = 0;
    for (int i = 0; i < nseg; i++) {
        GemvSeg &g = a.seg[i];
        const GemvSegDesc &d = segs[i];
        g.w = static_cast<const uint8_t *>(d.w);
        g.w2 = static_cast<const uint8_t *>(d.w2);
        g.type = d.type;
        g.rb = row_bytes(d.type, k);
        g.rb2 = d.w2 ? g.rb : 0;
        g.n = (int)d.n;
        g.epi = d.epi;
        g.y = d.y;
        g.ldy = d.ldy;
        g.bias = d.bias;
        g.yrow = d.yrow;
        const double share = (double)(g.rb + g.rb2) * (double)d.n / total_bytes;
        int nc = (int)(share * num_sms + 0.5);
        nc = std::max(1, std::min<int>(nc, (int)d.n));
        g.ncta = nc;
        g.cta0 = grid;
        grid += nc;
        g.rows_per_stage = (int)((sb - 64) / (g.rb + g.rb2));
        if (g.rows_per_stage < 1) return cudaErrorInvalidValue;
    }
    const size_t smem = xb + (size_t)ns * (size_t)sb + 16;
    switch (mt) {
        case 1: return launch_mt<1>(a, grid, smem, st);
        case 2: return launch_mt<2>(a, grid, smem, st);
        case 4: return launch_mt<4>(a, grid, smem, st);
        default: return launch_mt<8>(a, grid, smem, st);
    }
}

int read_and_clear_dev_error() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
    return v;
}

}  // namespace acm
