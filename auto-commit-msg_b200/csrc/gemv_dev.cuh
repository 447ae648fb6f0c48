// gemv_dev.cuh -- device side of the fused dequant-GEMV of k_gemv.cu (the
// lm_head and matvecs of 2..8 tokens).  A CTA consumes the stages of its row
// range from a ring of shared-memory stages; `cur` is the ring position of
// the range's first stage (0 for a single GEMV launch).
#pragma once
#include "common.cuh"
#include "kernels.h"
#include "quant.cuh"
#include "sbdot.cuh"

namespace acm {

template <int MT>
struct Cfg {
    static constexpr int NCW = MT <= 2 ? 16 : 8;  // consumer warps
    static constexpr int NT = NCW * 32 + 32;      // + producer warp
};

// Shared layout: [bars 128 B][x area][xsum area][red 16*MT floats][stages].
// Unit path x area: MT*K floats permuted into unit order, xsum MT*(K/32)
// float2 (low/high half sums per unit).  Wide path x area: MT*(K/256)*260
// floats (natural order, 4 floats of padding per 256), xsum MT*(K/32) floats.
__host__ __device__ inline size_t x_area_floats(int64_t k, int mt, int lpr) {
    return lpr ? (size_t)mt * (k / 256) * 260 : (size_t)mt * k;
}
__host__ __device__ inline size_t x_bytes(int64_t k, int mt, int lpr) {
    size_t b = 128 + x_area_floats(k, mt, lpr) * 4 + (size_t)mt * (k / 32) * 8 + 16 * mt * 4;
    return (b + 127) & ~size_t(127);
}

// Offset of activation element k in the x area (unit path: permuted into
// unit order with a bank swizzle; wide path: natural order, 4 floats of
// padding per 256).
template <int T>
__device__ __forceinline__ int x_off(int k, int K, bool wide) {
    if (wide) return (k >> 8) * 260 + (k & 255);
    int u, j;
    pos_unit<T>(k, K, u, j);
    return u * 32 + (((j >> 2) ^ (u & 7)) << 2) + (j & 3);
}

// Stage the activations (RMSNorm-ed when norm_w is set, model.go:213-222)
// into the x area.  The activations were written by other CTAs an instant
// ago, so each thread issues all of its loads (XB per token at a time, with
// the norm weights) before using any: one round trip instead of K / NC.
template <int T, int MT, int NCW = Cfg<MT>::NCW>
__device__ __forceinline__ void prep_x(const GemvArgs &a, float *xs, float *xsum, float *red) {
    constexpr int NC = NCW * 32;
    constexpr int XB = MT <= 2 ? 8 : 4;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.k;
    const bool wide = a.lpr != 0;
    const bool norm = a.norm_w != nullptr;
    const size_t xstr = wide ? (size_t)(K / 256) * 260 : (size_t)K;
    // norm weights first: in flight together with the activations
    float nw[XB];
    const bool one = K <= XB * NC;
    if (norm && one)
#pragma unroll
        for (int j = 0; j < XB; j++) nw[j] = j * NC + tid < K ? a.norm_w[j * NC + tid] : 0.f;
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) ss[m] = 0.f;
    // pass 1: raw values into the x area (and sum of squares)
    for (int k0 = 0; k0 < K; k0 += XB * NC) {
        float v[XB][MT];
#pragma unroll
        for (int j = 0; j < XB; j++) {
            const int k = k0 + j * NC + tid;
#pragma unroll
            for (int m = 0; m < MT; m++) v[j][m] = (k < K && m < a.m) ? __ldcg(a.x + (int64_t)m * a.ldx + k) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < XB; j++) {
            const int k = k0 + j * NC + tid;
            if (k < K) {
                const int off = x_off<T>(k, K, wide);
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    ss[m] = fmaf(v[j][m], v[j][m], ss[m]);
                    xs[m * xstr + off] = v[j][m];
                }
            }
        }
    }
    if (norm) {
        // pass 2 (same thread, same elements): scale by the row's RMS and the weight
#pragma unroll
        for (int m = 0; m < MT; m++) {
            const float w = warp_sum(ss[m]);
            if (lane == 0) red[warp * MT + m] = w;
        }
        named_sync(1, NC);
        float sc[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float t = 0.f;
            for (int w = 0; w < NCW; w++) t += red[w * MT + m];
            sc[m] = rms_scale(t, K, a.eps);
        }
        for (int k0 = 0; k0 < K; k0 += XB * NC) {
#pragma unroll
            for (int j = 0; j < XB; j++) {
                const int k = k0 + j * NC + tid;
                if (k < K) {
                    const float wk = one ? nw[j] : a.norm_w[k];
                    const int off = x_off<T>(k, K, wide);
#pragma unroll
                    for (int m = 0; m < MT; m++)
                        if (m < a.m) xs[m * xstr + off] = __fmul_rn(__fmul_rn(xs[m * xstr + off], sc[m]), wk);
                }
            }
        }
    }
    named_sync(1, NC);
    const int U = K / 32;
    if (wide) {
        // per-32 sums for the min terms of K-quants
        const int xstr = (K / 256) * 260;
        for (int idx = tid; idx < MT * U; idx += NC) {
            const int m = idx / U, u = idx - m * U;
            const float *p = xs + m * xstr + (u >> 3) * 260 + (u & 7) * 32;
            float s = 0.f;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float4 v = *reinterpret_cast<const float4 *>(p + 4 * c);
                s += (v.x + v.y) + (v.z + v.w);
            }
            xsum[m * U + u] = s;
        }
        named_sync(1, NC);
    } else if constexpr (T == T_Q4_K || T == T_Q5_K) {
        float2 *xs2 = reinterpret_cast<float2 *>(xsum);
        for (int idx = tid; idx < MT * U; idx += NC) {
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
            xs2[m * U + u] = make_float2(lo, hi);
        }
        named_sync(1, NC);
    }
}

// Residual values of row n for the EPI_ADD epilogue, loaded before the row's
// dot products so the read overlaps them.
template <int MT>
__device__ __forceinline__ void prefetch_res(const GemvSeg &s, int n, int m_used, bool active, float (&res)[MT]) {
#pragma unroll
    for (int m = 0; m < MT; m++)
        res[m] = (active && s.epi == EPI_ADD && m < m_used)
                     ? __ldcg(s.y + (int64_t)(s.yrow ? s.yrow[m] : m) * s.ldy + n)
                     : 0.f;
}

// Epilogue of one finished row n (values for tokens 0..m_used-1); res holds
// the residual values (prefetch_res) for EPI_ADD.
template <int MT>
__device__ __forceinline__ void row_out(const GemvSeg &s, int n, int m_used, const float (&acc)[MT],
                                        const float (&acc2)[MT], const float (&res)[MT],
                                        unsigned long long (&best)[MT]) {
#pragma unroll
    for (int m = 0; m < MT; m++) {
        if (m < m_used) {
            float v = acc[m];
            if (s.bias) v += s.bias[n];
            float *yp = s.y + (int64_t)(s.yrow ? s.yrow[m] : m) * s.ldy + n;
            if (s.epi == EPI_ADD) {
                *yp = res[m] + v;
            } else if (s.epi == EPI_SWIGLU) {
                const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_exp(-v)));
                *yp = __fmul_rn(__fmul_rn(v, sg), acc2[m]);
            } else {
                *yp = v;
            }
            if (s.amax) {
                const unsigned long long k = logit_key(v, n);
                best[m] = k > best[m] ? k : best[m];
            }
        }
    }
}

template <int MT>
__device__ __forceinline__ void flush_argmax(const GemvSeg &s, int m_used, unsigned long long (&best)[MT]) {
    if (!s.amax) return;
#pragma unroll
    for (int m = 0; m < MT; m++) {
        unsigned long long b = best[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(0xffffffffu, b, o);
            b = x > b ? x : b;
        }
        if ((threadIdx.x & 31) == 0 && m < m_used && b) atomicMax(&s.amax[m], b);
    }
}

template <int T, int MT, int NCW = Cfg<MT>::NCW>
__device__ __forceinline__ void consume_unit(const GemvArgs &a, const GemvSeg &s, int r0, int r1, uint64_t *full,
                                             uint64_t *empty, const uint8_t *stg, const float *xs,
                                             const float2 *xsum, uint32_t cur = 0) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.k, U = K / 32, R = s.rows_per_stage, NS = a.ns;
    const int nst = (r1 - r0 + R - 1) / R;
    const bool pair = s.w2 != nullptr;
    unsigned long long best[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) best[m] = 0ull;
    for (int i = 0; i < nst; i++) {
        const uint32_t ring = cur + (uint32_t)i;
        const int slot = (int)(ring % (uint32_t)NS);
        if (!mbar_wait(&full[slot], (ring / (uint32_t)NS) & 1u)) return;
        const int ra = r0 + i * R, rbn = min(ra + R, r1);
        const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
        const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
        const int64_t c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
        const uint8_t *buf = stg + (size_t)slot * a.stage_bytes;
        for (int rr = warp; rr < rbn - ra; rr += NCW) {
            const int n = ra + rr;
            float res[MT];
            prefetch_res<MT>(s, n, a.m, lane == 0, res);
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
            if (lane == 0) row_out<MT>(s, n, a.m, acc, acc2, res, best);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    flush_argmax<MT>(s, a.m, best);
}

template <int T, int MT, int NCW = Cfg<MT>::NCW>
__device__ __forceinline__ void consume_wide(const GemvArgs &a, const GemvSeg &s, int r0, int r1, uint64_t *full,
                                             uint64_t *empty, const uint8_t *stg, const float *xw,
                                             const float *xs32, uint32_t cur = 0) {
    if constexpr (sb_supported<T>()) {
        constexpr int SB = SpanBytes<T>::v;
        const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
        const int K = a.k, NSB = K / 256, R = s.rows_per_stage, NS = a.ns;
        const int lpr = a.lpr, rpw = 32 / lpr, spl = NSB / lpr;
        const int xstr = NSB * 260, sstr = K / 32;
        const int nst = (r1 - r0 + R - 1) / R;
        const bool pair = s.w2 != nullptr;
        const int sub = lane % lpr;
        unsigned long long best[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) best[m] = 0ull;
        for (int i = 0; i < nst; i++) {
            const uint32_t ring = cur + (uint32_t)i;
            const int slot = (int)(ring % (uint32_t)NS);
            if (!mbar_wait(&full[slot], (ring / (uint32_t)NS) & 1u)) return;
            const int ra = r0 + i * R, rbn = min(ra + R, r1);
            const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
            const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
            const int64_t c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
            const uint8_t *buf = stg + (size_t)slot * a.stage_bytes;
            for (int gb = warp * rpw; gb < rbn - ra; gb += NCW * rpw) {
                const int rr = gb + lane / lpr;
                const bool valid = rr < rbn - ra;
                const int n = ra + rr;
                float res[MT];
                prefetch_res<MT>(s, n, a.m, valid && sub == 0, res);
                float acc[MT], acc2[MT];
#pragma unroll
                for (int m = 0; m < MT; m++) acc[m] = acc2[m] = 0.f;
                if (valid) {
                    const uint8_t *rp = buf + ((int64_t)n * s.rb - a0);
                    const uint8_t *rp2 = pair ? buf + (a1 - a0) + ((int64_t)n * s.rb2 - c0) : nullptr;
                    for (int j = 0; j < spl; j++) {
                        const int sb = sub + j * lpr;
                        sb_dot<T, MT>(rp + (int64_t)sb * SB, xw + sb * 260, xstr, xs32 + sb * 8, sstr, a.m, acc);
                        if (pair)
                            sb_dot<T, MT>(rp2 + (int64_t)sb * SB, xw + sb * 260, xstr, xs32 + sb * 8, sstr, a.m, acc2);
                    }
                }
#pragma unroll
                for (int m = 0; m < MT; m++)
                    for (int o = lpr >> 1; o > 0; o >>= 1) {
                        acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
                        if (pair) acc2[m] += __shfl_xor_sync(0xffffffffu, acc2[m], o);
                    }
                if (valid && sub == 0) row_out<MT>(s, n, a.m, acc, acc2, res, best);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        flush_argmax<MT>(s, a.m, best);
    }
}

}  // namespace acm
