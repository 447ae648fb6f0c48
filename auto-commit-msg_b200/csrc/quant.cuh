// quant.cuh -- device decoders for the ggml block formats the reference reads
// (internal/infer/tensor.go:83-226).  Blocks are read straight from the GGUF
// bytes as uploaded; nothing is repacked.
//
// Every format is walked in "units" of 32 elements.  A unit is what one lane
// of a warp decodes per step:
//   Q4_K/Q5_K  8 units per 256-element super-block; unit ub = 2g + half covers
//              elements 64g + 16half + [0,16) (low nibbles, sub-block 2g) and
//              64g + 32 + 16half + [0,16) (high nibbles, sub-block 2g + 1)
//   Q6_K       8 units per super-block; unit ub = 4h + q covers elements
//              128h + 32t + 8q + [0,8) for t = 0..3
//   Q4_0/Q5_0/Q8_0  one 32-element block
//   F16        elements 8u + (K/4)c + [0,8), c = 0..3
//   F32        elements 4u + (K/8)c + [0,4), c = 0..7
// Within a unit, element j (0..31) is ordered as the decoders produce it; the
// GEMV kernel stores the activation vector permuted into the same order.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace acm {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

// BlockSize, gguf.go:70-90
__host__ __device__ constexpr int blk_elems(int t) {
    return t == T_F32 || t == T_F16 ? 1 : (t == T_Q4_K || t == T_Q5_K || t == T_Q6_K) ? 256 : 32;
}
__host__ __device__ constexpr int blk_bytes(int t) {
    return t == T_F32 ? 4 : t == T_F16 ? 2 : t == T_Q4_0 ? 18 : t == T_Q5_0 ? 22 : t == T_Q8_0 ? 34
         : t == T_Q4_K ? 144 : t == T_Q5_K ? 176 : t == T_Q6_K ? 210 : 0;
}
__host__ __device__ constexpr bool type_ok(int t) { return blk_bytes(t) != 0; }
__host__ __device__ inline int64_t row_bytes(int t, int64_t k) { return k / blk_elems(t) * blk_bytes(t); }

// f16, tensor.go:17-40.  The hardware conversion is exact for every half
// (normals, subnormals, infinities, NaN).
__device__ __forceinline__ float f16u(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFF))); }

// Load NW little-endian 32-bit words starting at a 2-byte aligned address
// with aligned loads and funnel shifts (reads one word past the run; every
// buffer is padded for that).
template <int NW>
__device__ __forceinline__ void ld_words_a2(const uint8_t *p, uint32_t (&w)[NW]) {
    const uint32_t *base = reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(p) & 3) * 8u;
    uint32_t a[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; i++) a[i] = base[i];
#pragma unroll
    for (int i = 0; i < NW; i++) w[i] = __funnelshift_r(a[i], a[i + 1], sh);
}
__device__ __forceinline__ uint32_t ld_u16_a2(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }

// Unsigned byte b of v as an exact float via the 2^23 magic (one PRMT + one
// FADD, no int->float conversion unit): returns (v.byte[b]) - off.
__device__ __forceinline__ float byte_f(uint32_t v, int b, float off_plus_magic) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | (uint32_t)b)) - off_plus_magic;
}
constexpr float MAGIC = 8388608.0f;  // 2^23
// Byte b of v in the low mantissa bits of 2^23: the float 2^23 + byte.
__device__ __forceinline__ float byte_m23(uint32_t v, int b) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | (uint32_t)b));
}

// scaleMinK4, tensor.go:123-130, for a runtime index j and the 12 scale
// bytes held in three words.
__device__ __forceinline__ void scale_min_k4(int j, uint32_t s0, uint32_t s1, uint32_t s2, float &sc, float &mn) {
    const int jj = j & 3;
    const uint32_t sh = 8u * (uint32_t)jj;
    uint32_t a = (s0 >> sh) & 0xFF, b = (s1 >> sh) & 0xFF, c = (s2 >> sh) & 0xFF;
    uint32_t sc_lo = a & 63, mn_lo = b & 63;
    uint32_t sc_hi = (c & 0x0F) | ((a >> 6) << 4);
    uint32_t mn_hi = (c >> 4) | ((b >> 6) << 4);
    sc = (float)(j < 4 ? sc_lo : sc_hi);
    mn = (float)(j < 4 ? mn_lo : mn_hi);
}

// ---------------------------------------------------------------------------
// Element position of (unit u, index j) inside a row of K elements, and the
// inverse.  Used to scatter exact dequant output and to permute activations.
// ---------------------------------------------------------------------------
template <int T>
__host__ __device__ __forceinline__ int unit_pos(int u, int j, int K) {
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        int sb = u >> 3, ub = u & 7, g = ub >> 1, half = ub & 1;
        return sb * 256 + g * 64 + (j >> 4) * 32 + half * 16 + (j & 15);
    } else if constexpr (T == T_Q6_K) {
        int sb = u >> 3, ub = u & 7, h = ub >> 2, q = ub & 3;
        return sb * 256 + h * 128 + (j >> 3) * 32 + q * 8 + (j & 7);
    } else if constexpr (T == T_F16) {
        return 8 * u + (K / 4) * (j >> 3) + (j & 7);
    } else if constexpr (T == T_F32) {
        return 4 * u + (K / 8) * (j >> 2) + (j & 3);
    } else {
        return u * 32 + j;
    }
}

template <int T>
__host__ __device__ __forceinline__ void pos_unit(int pos, int K, int &u, int &j) {
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        int sb = pos >> 8, r = pos & 255, g = r >> 6, rr = r & 63, hi = rr >> 5, l = rr & 31;
        u = sb * 8 + g * 2 + (l >> 4);
        j = hi * 16 + (l & 15);
    } else if constexpr (T == T_Q6_K) {
        int sb = pos >> 8, r = pos & 255, h = r >> 7, rr = r & 127, t = rr >> 5, l = rr & 31;
        u = sb * 8 + h * 4 + (l >> 3);
        j = t * 8 + (l & 7);
    } else if constexpr (T == T_F16) {
        int q = K / 4, c = pos / q, rem = pos - c * q;
        u = rem >> 3;
        j = c * 8 + (rem & 7);
    } else if constexpr (T == T_F32) {
        int q = K / 8, c = pos / q, rem = pos - c * q;
        u = rem >> 2;
        j = c * 4 + (rem & 3);
    } else {
        u = pos >> 5;
        j = pos & 31;
    }
}

// ---------------------------------------------------------------------------
// Exact dequant of run r = elements [32r, 32r + 32) of a row into v[32].
// Each value is computed with the reference's formula and is bit-identical
// to dequantRowSlow: the scale products are exact in fp32, so the only
// rounding is the one the reference makes (tensor.go:148-153, :182-190,
// :219-222).
// ---------------------------------------------------------------------------
template <int T>
__device__ __forceinline__ void dequant_run32(const uint8_t *row, int r, float (&v)[32]) {
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        constexpr int BB = (T == T_Q4_K) ? 144 : 176;
        const uint8_t *blk = row + (r >> 3) * BB;
        const int s = r & 7, g = s >> 1, hi = s & 1;
        uint32_t hw[4];
        ld_words_a2<4>(blk, hw);  // d, dmin, scales[0..11]
        const float d = f16u(hw[0]), dmin = f16u(hw[0] >> 16);
        float sc, mn;
        scale_min_k4(s, hw[1], hw[2], hw[3], sc, mn);
        const float d1 = d * sc, m1 = dmin * mn;
        uint32_t q[8], qh[8];
        ld_words_a2<8>(blk + (T == T_Q4_K ? 16 : 48) + 32 * g, q);
        if constexpr (T == T_Q5_K) ld_words_a2<8>(blk + 16, qh);
#pragma unroll
        for (int w = 0; w < 8; w++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const uint32_t byte = (q[w] >> (8 * b)) & 0xFF;
                const uint32_t nib = hi ? (byte >> 4) : (byte & 15);
                if constexpr (T == T_Q4_K) {
                    v[4 * w + b] = d1 * (float)nib - m1;
                } else {
                    const uint32_t hb = (qh[w] >> (8 * b)) & 0xFF;
                    const float add = (hb & (1u << s)) ? 16.0f : 0.0f;
                    v[4 * w + b] = d1 * ((float)nib + add) - m1;
                }
            }
    } else if constexpr (T == T_Q6_K) {
        const uint8_t *blk = row + (r >> 3) * 210;
        const int s = r & 7, h = s >> 2, t = s & 3;
        uint32_t ql[8], qh[8], sw[2];
        ld_words_a2<8>(blk + 64 * h + ((t & 1) ? 32 : 0), ql);
        ld_words_a2<8>(blk + 128 + 32 * h, qh);
        ld_words_a2<2>(blk + 192 + 8 * h, sw);
        const float d = f16u(ld_u16_a2(blk + 208));
        const int si0 = 2 * t, si1 = 1 + 2 * t;  // sc index for l < 16 and l >= 16
        const float ds0 = d * (float)(int8_t)((sw[si0 >> 2] >> (8 * (si0 & 3))) & 0xFF);
        const float ds1 = d * (float)(int8_t)((sw[si1 >> 2] >> (8 * (si1 & 3))) & 0xFF);
#pragma unroll
        for (int w = 0; w < 8; w++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const uint32_t L = (ql[w] >> (8 * b)) & 0xFF, H = (qh[w] >> (8 * b)) & 0xFF;
                const uint32_t lo4 = (t < 2) ? (L & 15) : (L >> 4);
                const uint32_t q6 = lo4 | (((H >> (2 * t)) & 3) << 4);
                v[4 * w + b] = ((w < 4) ? ds0 : ds1) * (float)((int)q6 - 32);
            }
    } else if constexpr (T == T_Q8_0) {
        const uint8_t *blk = row + r * 34;
        const float d = f16u(ld_u16_a2(blk));
        uint32_t q[8];
        ld_words_a2<8>(blk + 2, q);
#pragma unroll
        for (int w = 0; w < 8; w++)
#pragma unroll
            for (int b = 0; b < 4; b++) v[4 * w + b] = d * (float)(int8_t)((q[w] >> (8 * b)) & 0xFF);
    } else if constexpr (T == T_Q4_0) {
        const uint8_t *blk = row + r * 18;
        const float d = f16u(ld_u16_a2(blk));
        uint32_t q[4];
        ld_words_a2<4>(blk + 2, q);
#pragma unroll
        for (int w = 0; w < 4; w++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const uint32_t byte = (q[w] >> (8 * b)) & 0xFF;
                v[4 * w + b] = d * (float)((int)(byte & 15) - 8);
                v[16 + 4 * w + b] = d * (float)((int)(byte >> 4) - 8);
            }
    } else if constexpr (T == T_Q5_0) {
        const uint8_t *blk = row + r * 22;
        const float d = f16u(ld_u16_a2(blk));
        uint32_t qh[1], q[4];
        ld_words_a2<1>(blk + 2, qh);
        ld_words_a2<4>(blk + 6, q);
#pragma unroll
        for (int w = 0; w < 4; w++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int jj = 4 * w + b;
                const uint32_t byte = (q[w] >> (8 * b)) & 0xFF;
                const int x0 = (int)(byte & 15) | (int)((qh[0] >> jj) & 1) << 4;
                const int x1 = (int)(byte >> 4) | (int)((qh[0] >> (jj + 16)) & 1) << 4;
                v[jj] = d * (float)(x0 - 16);
                v[16 + jj] = d * (float)(x1 - 16);
            }
    } else if constexpr (T == T_F16) {
        uint32_t w[16];
        ld_words_a2<16>(row + 64 * r, w);
#pragma unroll
        for (int i = 0; i < 16; i++) {
            v[2 * i] = f16u(w[i]);
            v[2 * i + 1] = f16u(w[i] >> 16);
        }
    } else {  // F32
        const float *p = reinterpret_cast<const float *>(row) + 32 * r;
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = p[i];
    }
}

// ---------------------------------------------------------------------------
// Factored unit dot products for the decode GEMV.  For every token m the lane
// adds  sum_j w_j * x_m[j]  to acc[m], where w_j is the dequantized weight.
// The block scale is applied once per sub-block (d1 * sum q x - m1 * sum x)
// instead of once per element, which is the same sum in exact arithmetic.
// xs: permuted activations of this unit for token 0 (16-byte aligned, chunk c
// at xs[((c ^ (u & 7)) << 2)]), token stride XS floats; xsum: per-unit
// (low, high) sums of the activations, token stride XSUM float2s.
// ---------------------------------------------------------------------------
template <int MT>
struct XView {
    const float *xs;   // token 0, this unit
    int stride;        // floats between tokens
    int swz;           // u & 7
    __device__ __forceinline__ float4 chunk(int m, int c) const {
        return *reinterpret_cast<const float4 *>(xs + m * stride + ((c ^ swz) << 2));
    }
};

__device__ __forceinline__ float f4get(const float4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

template <int T, int MT>
__device__ __forceinline__ void unit_dot(const uint8_t *row, int u, int K, const XView<MT> &xv, const float2 *xsum,
                                         int xsum_stride, int m_used, float (&acc)[MT]) {
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        constexpr int BB = (T == T_Q4_K) ? 144 : 176;
        const uint8_t *blk = row + (u >> 3) * BB;
        const int ub = u & 7, g = ub >> 1, half = ub & 1;
        const uint4 hv = *reinterpret_cast<const uint4 *>(blk);  // d, dmin, scales[12]
        float d = f16u(hv.x), dmin = f16u(hv.x >> 16);
        float sc0, mn0, sc1, mn1;
        scale_min_k4(2 * g, hv.y, hv.z, hv.w, sc0, mn0);
        scale_min_k4(2 * g + 1, hv.y, hv.z, hv.w, sc1, mn1);
        uint4 qv, qhv;
        if constexpr (T == T_Q4_K) {
            qv = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * g + 16 * half);
        } else {
            qv = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * g + 16 * half);
            qhv = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * half);
        }
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
        // packed two-lane fp32 (sm_100 FADD2 / FFMA2): half the instructions and
        // half the length of each accumulation chain (even / odd elements)
        float2 slo2[MT], shi2[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) slo2[m] = shi2[m] = make_float2(0.f, 0.f);
        const float2 nmag = make_float2(-MAGIC, -MAGIC);
#pragma unroll
        for (int w = 0; w < 4; w++) {
            uint32_t lo, hi;
            if constexpr (T == T_Q4_K) {
                lo = qw[w] & 0x0F0F0F0Fu;
                hi = qw[w] & 0xF0F0F0F0u;  // 16*q, rescaled below
            } else {
                const uint32_t qhw[4] = {qhv.x, qhv.y, qhv.z, qhv.w};
                lo = (qw[w] & 0x0F0F0F0Fu) | (((qhw[w] >> (2 * g)) & 0x01010101u) << 4);
                hi = ((qw[w] >> 4) & 0x0F0F0F0Fu) | (((qhw[w] >> (2 * g + 1)) & 0x01010101u) << 4);
            }
            const float2 fl01 = __fadd2_rn(make_float2(byte_m23(lo, 0), byte_m23(lo, 1)), nmag);
            const float2 fl23 = __fadd2_rn(make_float2(byte_m23(lo, 2), byte_m23(lo, 3)), nmag);
            const float2 fh01 = __fadd2_rn(make_float2(byte_m23(hi, 0), byte_m23(hi, 1)), nmag);
            const float2 fh23 = __fadd2_rn(make_float2(byte_m23(hi, 2), byte_m23(hi, 3)), nmag);
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if (m < m_used) {
                    float4 xl = xv.chunk(m, w), xh = xv.chunk(m, 4 + w);
                    slo2[m] = __ffma2_rn(fl01, make_float2(xl.x, xl.y), slo2[m]);
                    slo2[m] = __ffma2_rn(fl23, make_float2(xl.z, xl.w), slo2[m]);
                    shi2[m] = __ffma2_rn(fh01, make_float2(xh.x, xh.y), shi2[m]);
                    shi2[m] = __ffma2_rn(fh23, make_float2(xh.z, xh.w), shi2[m]);
                }
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
        for (int m = 0; m < MT; m++) {
            if (m < m_used) {
                const float2 xsm = xsum[m * xsum_stride];
                acc[m] += d1 * slo[m] - m1 * xsm.x + d2 * shi[m] - m2 * xsm.y;
            }
        }
    } else if constexpr (T == T_Q6_K) {
        const uint8_t *blk = row + (u >> 3) * 210;
        const int ub = u & 7, h = ub >> 2, qq = ub & 3, l0 = 8 * qq;
        uint32_t a[2], b2[2], hh[2], sw[2];
        ld_words_a2<2>(blk + 64 * h + l0, a);
        ld_words_a2<2>(blk + 64 * h + 32 + l0, b2);
        ld_words_a2<2>(blk + 128 + 32 * h + l0, hh);
        ld_words_a2<2>(blk + 192 + 8 * h, sw);
        const float d = f16u(ld_u16_a2(blk + 208));
        const int is = l0 >> 4;
        float st[4][MT];
#pragma unroll
        for (int t = 0; t < 4; t++)
#pragma unroll
            for (int m = 0; m < MT; m++) st[t][m] = 0.f;
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t A = a[w], B = b2[w], H = hh[w];
            const uint32_t q6[4] = {(A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u),
                                    (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u),
                                    ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u),
                                    ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u)};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                float f[4];
#pragma unroll
                for (int b = 0; b < 4; b++) f[b] = byte_f(q6[t], b, MAGIC + 32.0f);
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    if (m < m_used) {
                        float4 x = xv.chunk(m, 2 * t + w);
                        st[t][m] = fmaf(f[0], x.x, st[t][m]);
                        st[t][m] = fmaf(f[1], x.y, st[t][m]);
                        st[t][m] = fmaf(f[2], x.z, st[t][m]);
                        st[t][m] = fmaf(f[3], x.w, st[t][m]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int si = is + 2 * t;
            const float ds = d * (float)(int8_t)((sw[si >> 2] >> (8 * (si & 3))) & 0xFF);
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) acc[m] = fmaf(ds, st[t][m], acc[m]);
        }
    } else if constexpr (T == T_Q8_0 || T == T_Q4_0 || T == T_Q5_0) {
        constexpr int BB = blk_bytes(T);
        const uint8_t *blk = row + u * BB;
        const float d = f16u(ld_u16_a2(blk));
        float s[MT], s2[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) s[m] = s2[m] = 0.f;
        if constexpr (T == T_Q8_0) {
            uint32_t q[8];
            ld_words_a2<8>(blk + 2, q);
#pragma unroll
            for (int w = 0; w < 8; w++) {
                const uint32_t vb = q[w] ^ 0x80808080u;  // int8 -> biased byte
                float f[4];
#pragma unroll
                for (int b = 0; b < 4; b++) f[b] = byte_f(vb, b, MAGIC + 128.0f);
#pragma unroll
                for (int m = 0; m < MT; m++)
                    if (m < m_used) {
                        float4 x = xv.chunk(m, w);
                        s[m] = fmaf(f[0], x.x, s[m]);
                        s[m] = fmaf(f[1], x.y, s[m]);
                        s[m] = fmaf(f[2], x.z, s[m]);
                        s[m] = fmaf(f[3], x.w, s[m]);
                    }
            }
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) acc[m] = fmaf(d, s[m], acc[m]);
        } else {
            uint32_t q[4], qh0 = 0;
            if constexpr (T == T_Q4_0) {
                ld_words_a2<4>(blk + 2, q);
            } else {
                uint32_t t1[1];
                ld_words_a2<1>(blk + 2, t1);
                qh0 = t1[0];
                ld_words_a2<4>(blk + 6, q);
            }
#pragma unroll
            for (int w = 0; w < 4; w++) {
                uint32_t lo, hi;
                float offl, offh;
                if constexpr (T == T_Q4_0) {
                    lo = q[w] & 0x0F0F0F0Fu;
                    hi = q[w] & 0xF0F0F0F0u;  // 16*q
                    offl = MAGIC + 8.0f;
                    offh = MAGIC + 128.0f;
                } else {
                    const uint32_t n0 = (qh0 >> (4 * w)) & 0xF, n1 = (qh0 >> (16 + 4 * w)) & 0xF;
                    lo = (q[w] & 0x0F0F0F0Fu) | (((n0 * 0x00204081u) & 0x01010101u) << 4);
                    hi = ((q[w] >> 4) & 0x0F0F0F0Fu) | (((n1 * 0x00204081u) & 0x01010101u) << 4);
                    offl = offh = MAGIC + 16.0f;
                }
                float fl[4], fh[4];
#pragma unroll
                for (int b = 0; b < 4; b++) {
                    fl[b] = byte_f(lo, b, offl);
                    fh[b] = byte_f(hi, b, offh);
                }
#pragma unroll
                for (int m = 0; m < MT; m++)
                    if (m < m_used) {
                        float4 xl = xv.chunk(m, w), xh = xv.chunk(m, 4 + w);
                        s[m] = fmaf(fl[0], xl.x, s[m]);
                        s[m] = fmaf(fl[1], xl.y, s[m]);
                        s[m] = fmaf(fl[2], xl.z, s[m]);
                        s[m] = fmaf(fl[3], xl.w, s[m]);
                        s2[m] = fmaf(fh[0], xh.x, s2[m]);
                        s2[m] = fmaf(fh[1], xh.y, s2[m]);
                        s2[m] = fmaf(fh[2], xh.z, s2[m]);
                        s2[m] = fmaf(fh[3], xh.w, s2[m]);
                    }
            }
            const float dh = (T == T_Q4_0) ? d * 0.0625f : d;
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) acc[m] += d * s[m] + dh * s2[m];
        }
    } else if constexpr (T == T_F16) {
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 hv = *reinterpret_cast<const uint4 *>(row + 2 * (8 * u + (K / 4) * c));
            const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
            float f[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&hw[i]));
                f[2 * i] = t.x;
                f[2 * i + 1] = t.y;
            }
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) {
                    float4 x0 = xv.chunk(m, 2 * c), x1 = xv.chunk(m, 2 * c + 1);
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
    } else {  // F32
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const float4 wv = *reinterpret_cast<const float4 *>(row + 4 * (4 * u + (K / 8) * c));
#pragma unroll
            for (int m = 0; m < MT; m++)
                if (m < m_used) {
                    float4 x = xv.chunk(m, c);
                    float s = acc[m];
                    s = fmaf(wv.x, x.x, s);
                    s = fmaf(wv.y, x.y, s);
                    s = fmaf(wv.z, x.z, s);
                    s = fmaf(wv.w, x.w, s);
                    acc[m] = s;
                }
        }
    }
}

// fastExp, internal/infer/model.go:282-295: 2^i * p5(f) with the
// reference's degree-5 polynomial, evaluated without contraction as the
// reference evaluates it.
__device__ __forceinline__ float fast_exp(float x) {
    if (x < -87.0f) return 0.0f;
    const float t = __fmul_rn(x, 1.4426950408889634f);
    const float fi = floorf(t);
    const float f = __fsub_rn(t, fi);
    float p = __fadd_rn(0.00961813f, __fmul_rn(f, 0.00133336f));
    p = __fadd_rn(0.05550411f, __fmul_rn(f, p));
    p = __fadd_rn(0.24022650f, __fmul_rn(f, p));
    p = __fadd_rn(0.69314718f, __fmul_rn(f, p));
    p = __fadd_rn(1.0000001f, __fmul_rn(f, p));
    const int i = (int)fi;
    if (i > 127) return __int_as_float(0x7f800000);  // overflow -> +Inf
    return p * __int_as_float((i + 127) << 23);       // i >= -126 here: 2^i is a normal float
}

}  // namespace acm
