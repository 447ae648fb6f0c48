// sbdot.cuh -- dot products of one 256-element span of a weight row with the
// activations, decoding the block headers once per span (the wide GEMV path,
// where each lane owns whole super-blocks of a row).  x256 holds the span's
// activations of token 0 in natural order (token m at x256 + m*xstr); xs32
// the span's eight 32-element activation sums (token m at xs32 + m*sstr).
// The arithmetic is the factored form of unit_dot: per 32/16-element
// sub-block, d*sc * sum(q*x) - dmin*m * sum(x).
#pragma once
#include "quant.cuh"

namespace acm {

template <int T>
struct SpanBytes;
template <> struct SpanBytes<T_Q4_K> { static constexpr int v = 144; };
template <> struct SpanBytes<T_Q5_K> { static constexpr int v = 176; };
template <> struct SpanBytes<T_Q6_K> { static constexpr int v = 210; };
template <> struct SpanBytes<T_Q8_0> { static constexpr int v = 272; };
template <> struct SpanBytes<T_F16> { static constexpr int v = 512; };

template <int T>
__host__ __device__ constexpr bool sb_supported() {
    return T == T_Q4_K || T == T_Q5_K || T == T_Q6_K || T == T_Q8_0 || T == T_F16;
}

template <int T, int MT>
__device__ __forceinline__ void sb_dot(const uint8_t *blk, const float *x256, int xstr, const float *xs32, int sstr,
                                       int m_used, float (&acc)[MT]) {
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        const uint4 hv = *reinterpret_cast<const uint4 *>(blk);
        const float d = f16u(hv.x), dmin = f16u(hv.x >> 16);
        uint4 qh0, qh1;
        if constexpr (T == T_Q5_K) {
            qh0 = *reinterpret_cast<const uint4 *>(blk + 16);
            qh1 = *reinterpret_cast<const uint4 *>(blk + 32);
        }
#pragma unroll
        for (int g = 0; g < 4; g++) {
            float sc0, mn0, sc1, mn1;
            scale_min_k4(2 * g, hv.y, hv.z, hv.w, sc0, mn0);
            scale_min_k4(2 * g + 1, hv.y, hv.z, hv.w, sc1, mn1);
            const uint8_t *qs = blk + (T == T_Q4_K ? 16 : 48) + 32 * g;
            const uint4 qa = *reinterpret_cast<const uint4 *>(qs), qb = *reinterpret_cast<const uint4 *>(qs + 16);
            const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            // packed two-lane fp32 (sm_100 FADD2 / FFMA2): element pairs share one
            // instruction; each accumulator pair holds the even / odd elements
            float2 slo2[MT], shi2[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) slo2[m] = shi2[m] = make_float2(0.f, 0.f);
            const float2 nmag = make_float2(-MAGIC, -MAGIC);
#pragma unroll
            for (int w = 0; w < 8; w++) {
                uint32_t lo, hi;
                if constexpr (T == T_Q4_K) {
                    lo = qw[w] & 0x0F0F0F0Fu;
                    hi = qw[w] & 0xF0F0F0F0u;  // 16*q
                } else {
                    const uint32_t hw[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
                    lo = (qw[w] & 0x0F0F0F0Fu) | (((hw[w] >> (2 * g)) & 0x01010101u) << 4);
                    hi = ((qw[w] >> 4) & 0x0F0F0F0Fu) | (((hw[w] >> (2 * g + 1)) & 0x01010101u) << 4);
                }
                // bytes into the low mantissa of 2^23, then minus 2^23: the exact integers
                const float2 fl01 = __fadd2_rn(make_float2(byte_m23(lo, 0), byte_m23(lo, 1)), nmag);
                const float2 fl23 = __fadd2_rn(make_float2(byte_m23(lo, 2), byte_m23(lo, 3)), nmag);
                const float2 fh01 = __fadd2_rn(make_float2(byte_m23(hi, 0), byte_m23(hi, 1)), nmag);
                const float2 fh23 = __fadd2_rn(make_float2(byte_m23(hi, 2), byte_m23(hi, 3)), nmag);
#pragma unroll
                for (int m = 0; m < MT; m++)
                    if (m < m_used) {
                        const float4 xl = *reinterpret_cast<const float4 *>(x256 + m * xstr + 64 * g + 4 * w);
                        const float4 xh = *reinterpret_cast<const float4 *>(x256 + m * xstr + 64 * g + 32 + 4 * w);
                        slo2[m] = __ffma2_rn(fl01, make_float2(xl.x, xl.y), slo2[m]);
                        slo2[m] = __ffma2_rn(fl23, make_float2(xl.z, xl.w), slo2[m]);
                        shi2[m] = __ffma2_rn(fh01, make_float2(xh.x, xh.y), shi2[m]);
                        shi2[m] = __ffma2_rn(fh23, make_float2(xh.z, xh.w), shi2[m]);
                    }
            }
            float slo[MT], shi[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) {
                slo[m] = slo2[m].x + slo2[m].y;
                shi[m] = shi2[m].x + shi2[m].y;
            }
            const float d1 = d * sc0, m1 = dmin * mn0, m2 = dmin * mn1;
            const float d2 = (T == T_Q4_K) ? d * sc1 * 0.0625f : d * sc1;
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used)
                    acc[m] += d1 * slo[m] - m1 * xs32[m * sstr + 2 * g] + d2 * shi[m] - m2 * xs32[m * sstr + 2 * g + 1];
        }
    } else if constexpr (T == T_Q6_K) {
        const float d = f16u(ld_u16_a2(blk + 208));
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t A[8], B[8], H[8], sw[2];
            ld_words_a2<8>(blk + 64 * h, A);
            ld_words_a2<8>(blk + 64 * h + 32, B);
            ld_words_a2<8>(blk + 128 + 32 * h, H);
            ld_words_a2<2>(blk + 192 + 8 * h, sw);
#pragma unroll
            for (int half = 0; half < 2; half++) {  // l < 16, l >= 16 (a scale boundary)
                float st[4][MT];
#pragma unroll
                for (int t = 0; t < 4; t++)
#pragma unroll
                    for (int m = 0; m < MT; m++) st[t][m] = 0.f;
#pragma unroll
                for (int ww = 0; ww < 4; ww++) {
                    const int w = 4 * half + ww;
                    const uint32_t q6[4] = {(A[w] & 0x0F0F0F0Fu) | ((H[w] << 4) & 0x30303030u),
                                            (B[w] & 0x0F0F0F0Fu) | ((H[w] << 2) & 0x30303030u),
                                            ((A[w] >> 4) & 0x0F0F0F0Fu) | (H[w] & 0x30303030u),
                                            ((B[w] >> 4) & 0x0F0F0F0Fu) | ((H[w] >> 2) & 0x30303030u)};
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        float f[4];
#pragma unroll
                        for (int b = 0; b < 4; b++) f[b] = byte_f(q6[t], b, MAGIC + 32.0f);
#pragma unroll
                        for (int m = 0; m < MT; m++)
                            if (m < m_used) {
                                const float4 x = *reinterpret_cast<const float4 *>(x256 + m * xstr + 128 * h + 32 * t + 4 * w);
                                st[t][m] = fmaf(f[0], x.x, st[t][m]);
                                st[t][m] = fmaf(f[1], x.y, st[t][m]);
                                st[t][m] = fmaf(f[2], x.z, st[t][m]);
                                st[t][m] = fmaf(f[3], x.w, st[t][m]);
                            }
                    }
                }
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int si = 2 * t + half;
                    const float ds = d * (float)(int8_t)((sw[si >> 2] >> (8 * (si & 3))) & 0xFF);
#pragma unroll
                    for (int m = 0; m < MT; m++)
                        if (m < m_used) acc[m] = fmaf(ds, st[t][m], acc[m]);
                }
            }
        }
    } else if constexpr (T == T_Q8_0) {
#pragma unroll 2
        for (int b = 0; b < 8; b++) {
            const uint8_t *p = blk + 34 * b;
            const float d = f16u(ld_u16_a2(p));
            uint32_t q[8];
            ld_words_a2<8>(p + 2, q);
            float s[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) s[m] = 0.f;
#pragma unroll
            for (int w = 0; w < 8; w++) {
                const uint32_t vb = q[w] ^ 0x80808080u;
                float f[4];
#pragma unroll
                for (int c = 0; c < 4; c++) f[c] = byte_f(vb, c, MAGIC + 128.0f);
#pragma unroll
                for (int m = 0; m < MT; m++)
                    if (m < m_used) {
                        const float4 x = *reinterpret_cast<const float4 *>(x256 + m * xstr + 32 * b + 4 * w);
                        s[m] = fmaf(f[0], x.x, s[m]);
                        s[m] = fmaf(f[1], x.y, s[m]);
                        s[m] = fmaf(f[2], x.z, s[m]);
                        s[m] = fmaf(f[3], x.w, s[m]);
                    }
            }
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) acc[m] = fmaf(d, s[m], acc[m]);
        }
    } else if constexpr (T == T_F16) {
#pragma unroll 4
        for (int c = 0; c < 32; c++) {
            const uint4 hv = *reinterpret_cast<const uint4 *>(blk + 16 * c);
            const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
            float f[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&hw[i]));
                f[2 * i] = t.x;
                f[2 * i + 1] = t.y;
            }
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) {
                    const float4 x0 = *reinterpret_cast<const float4 *>(x256 + m * xstr + 8 * c);
                    const float4 x1 = *reinterpret_cast<const float4 *>(x256 + m * xstr + 8 * c + 4);
                    float s = acc[m];
                    s = fmaf(f[0], x0.x, s);
                    s = fmaf(f[1], x0.y, s);
                    s = fmaf(f[2], x0.z, s);
                    s = fmaf(f[3], x0.w, s);
                    s = fmaf(f[4], x1.x, s);
                    s = fmaf(f[5], x1.y, s);
                    s = fmaf(f[6], x1.z, s);
                    s = fmaf(f[7], x1.w, s);
                    acc[m] = s;
                }
        }
    }
}

}  // namespace acm
