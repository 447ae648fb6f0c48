// gemv1.cuh -- the batch-1 decode GEMV (one token), device side.
//
// The reference's matvec (internal/infer/tensor.go:253-303, matvec :301)
// dequantizes a tile of weight rows and dots it with the activations.  A
// batch-1 decode token is a chain of ~140 such matvecs of 1-4 MB each, so a
// matvec costs its latency, not its bytes.  Shaped for that:
//   * the activations are staged once per CTA (coalesced loads, RMSNorm in
//     place) and each lane keeps the ones of its "lane unit" in registers for
//     every row, so the inner loop reads shared memory only for weights;
//   * a lane unit is 64 elements for Q4_K / Q5_K / Q6_K (one sub-block pair
//     of a super-block, whose scales are decoded once per 64 weights) and 32
//     for the other formats (quant.cuh's units); a row of K elements is
//     K / unit lanes: half a warp (two rows per warp step) when that is at
//     most 16, else a warp, else a team of warps whose partial sums meet in
//     shared memory;
//   * the factored sub-block dot (d*sc * sum q*x - dmin*m * sum x) on packed
//     two-lane fp32 (FADD2 / FFMA2), a shuffle reduction per row, and the
//     epilogues (store + bias, residual add, SwiGLU of a gate/up pair, greedy
//     argmax key).
// User: k_gemv1.cu (one launch per matvec; each team moves its rows into its
// own stages with the bulk-copy engine before the dependency wait).
#pragma once
#include "common.cuh"
#include "gemv_dev.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace acm {

// ---------------------------------------------------------------------------
// Lane units
// ---------------------------------------------------------------------------
template <int T>
__host__ __device__ constexpr int lane_elems() {
    return (T == T_Q4_K || T == T_Q5_K || T == T_Q6_K) ? 64 : 32;
}
__host__ __device__ inline int lane_elems_rt(int t) { return (t == T_Q4_K || t == T_Q5_K || t == T_Q6_K) ? 64 : 32; }

// Row geometry of a format at K: lane units per row, lanes a row takes (16
// or 32: two rows per warp step when 16), warps per row team.
struct RowGeo {
    int U, lpr, ts;
};
__host__ __device__ inline RowGeo row_geo(int type, int K) {
    const int U = K / lane_elems_rt(type);
    RowGeo g;
    g.U = U;
    g.lpr = (lane_elems_rt(type) == 64 && U <= 16) ? 16 : 32;
    g.ts = g.lpr == 16 ? 1 : (U + 31) / 32;
    return g;
}

// Element order of a 64-element unit (group G): Q4_K / Q5_K: the natural
// elements 64G .. 64G + 63 (low nibbles of 32 bytes, then high nibbles);
// Q6_K: group (super-block sb, half h, l0 = 16 * (G & 1)) element 16t + i is
// position 256 sb + 128 h + 32 t + l0 + i (t = 0..3, i = 0..15).
template <int T>
__host__ __device__ __forceinline__ int group_pos(int G, int e) {
    if constexpr (T == T_Q6_K) {
        const int sb = G >> 2, h = (G >> 1) & 1, l0 = 16 * (G & 1);
        return sb * 256 + h * 128 + 32 * (e >> 4) + l0 + (e & 15);
    } else {
        return 64 * G + e;
    }
}
template <int T>
__host__ __device__ __forceinline__ void pos_group(int p, int &G, int &e) {
    if constexpr (T == T_Q6_K) {
        const int sb = p >> 8, r = p & 255, h = r >> 7, rr = r & 127, t = rr >> 5, l = rr & 31;
        G = sb * 4 + h * 2 + (l >> 4);
        e = 16 * t + (l & 15);
    } else {
        G = p >> 6;
        e = p & 63;
    }
}

// Staged activations: the unit's chunk c (elements 4c .. 4c + 3 of the unit)
// at u * E + ((c ^ (u & 7)) << 2), so a quarter warp reading chunk c of eight
// consecutive units hits distinct banks.  Offset of natural position p (a
// multiple of 4: four consecutive positions are four consecutive unit
// elements).
template <int T>
__device__ __forceinline__ int xs_off(int p, int K) {
    if constexpr (lane_elems<T>() == 64) {
        int G, e;
        pos_group<T>(p, G, e);
        return G * 64 + (((e >> 2) ^ (G & 7)) << 2);
    } else {
        return x_off<T>(p, K, false);
    }
}

template <int NC>
struct XRegN {
    float4 c[NC];  // unit elements 4i .. 4i + 3
};

template <int NC>
__device__ __forceinline__ void load_lane_x(const float *xs, int u, XRegN<NC> &r) {
#pragma unroll
    for (int c = 0; c < NC; c++) r.c[c] = *reinterpret_cast<const float4 *>(xs + u * (4 * NC) + ((c ^ (u & 7)) << 2));
}

// ---------------------------------------------------------------------------
// Activation staging, once per CTA: coalesced loads, RMSNorm (model.go:213-222,
// dst = x * scale * w) when norm_w is set, stored in lane-unit order (xs_off).
// XPER float4s per thread are held in registers (larger K is read twice).
// ---------------------------------------------------------------------------
constexpr int XPER = 2;
struct XStage {
    float4 v[XPER], w[XPER];
};

// Before the dependency wait: the norm weights (they never change).
__device__ __forceinline__ void stage_x_pre(const float *norm_w, int K, XStage &r, int nthr) {
    const int n4 = K >> 2;
#pragma unroll
    for (int i = 0; i < XPER; i++) {
        const int q = threadIdx.x + i * nthr;
        r.w[i] = (norm_w && q < n4) ? __ldg(reinterpret_cast<const float4 *>(norm_w) + q)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// nthr threads (0 .. nthr - 1) take part; bar: 0 for the whole CTA, else the
// named barrier they share.
__device__ __forceinline__ void stage_sync(int bar, int nthr) {
    if (bar) named_sync(bar, nthr);
    else __syncthreads();
}

// After the wait: the activations (written by earlier kernels or phases), the
// norm, the store.  red: 32 floats of scratch.
template <int T>
__device__ __forceinline__ void stage_x(const float *x, const float *norm_w, int K, float eps, float *xs, float *red,
                                        XStage &r, int nthr, int bar) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n4 = K >> 2;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < XPER; i++) {
        const int q = tid + i * nthr;
        r.v[i] = q < n4 ? __ldcg(reinterpret_cast<const float4 *>(x) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (norm_w) {
        for (int q = tid + XPER * nthr; q < n4; q += nthr) {
            const float4 t = __ldcg(reinterpret_cast<const float4 *>(x) + q);
            ss = fmaf(t.x, t.x, fmaf(t.y, t.y, fmaf(t.z, t.z, fmaf(t.w, t.w, ss))));
        }
    }
    float sc = 1.f;
    if (norm_w) {
#pragma unroll
        for (int i = 0; i < XPER; i++) {
            ss = fmaf(r.v[i].x, r.v[i].x, ss);
            ss = fmaf(r.v[i].y, r.v[i].y, ss);
            ss = fmaf(r.v[i].z, r.v[i].z, ss);
            ss = fmaf(r.v[i].w, r.v[i].w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        stage_sync(bar, nthr);
        float t = 0.f;
        for (int i = 0; i < (nthr >> 5); i++) t += red[i];
        sc = rms_scale(t, K, eps);
    }
    auto put = [&](int q, float4 a, float4 b) {
        if (norm_w)
            a = make_float4(__fmul_rn(__fmul_rn(a.x, sc), b.x), __fmul_rn(__fmul_rn(a.y, sc), b.y),
                            __fmul_rn(__fmul_rn(a.z, sc), b.z), __fmul_rn(__fmul_rn(a.w, sc), b.w));
        *reinterpret_cast<float4 *>(xs + xs_off<T>(4 * q, K)) = a;
    };
#pragma unroll
    for (int i = 0; i < XPER; i++) {
        const int q = tid + i * nthr;
        if (q < n4) put(q, r.v[i], r.w[i]);
    }
    for (int q = tid + XPER * nthr; q < n4; q += nthr)
        put(q, __ldcg(reinterpret_cast<const float4 *>(x) + q),
            norm_w ? __ldg(reinterpret_cast<const float4 *>(norm_w) + q) : make_float4(0.f, 0.f, 0.f, 0.f));
    stage_sync(bar, nthr);
}

// ---------------------------------------------------------------------------
// Dot products of one lane unit of a row
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// acc += sum_j w_j x_j over unit u of a row (MT = 1, activations in
// registers).  xs: the unit's (low half, high half) activation sums, used by
// the K-quant min terms.
template <int T>
__device__ __forceinline__ float unit_dot1(const uint8_t *row, int u, int K, const XRegN<8> &x, float2 xs) {
    const float2 nmag = f2(-MAGIC, -MAGIC);
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        constexpr int BB = (T == T_Q4_K) ? 144 : 176;
        const uint8_t *blk = row + (u >> 3) * BB;
        const int ub = u & 7, g = ub >> 1, half = ub & 1;
        const uint4 hv = *reinterpret_cast<const uint4 *>(blk);  // d, dmin, scales[12]
        uint4 qv, qhv;
        if constexpr (T == T_Q4_K) {
            qv = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * g + 16 * half);
        } else {
            qv = *reinterpret_cast<const uint4 *>(blk + 48 + 32 * g + 16 * half);
            qhv = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * half);
        }
        const float d = f16u(hv.x), dmin = f16u(hv.x >> 16);
        float sc0, mn0, sc1, mn1;
        scale_min_k4(2 * g, hv.y, hv.z, hv.w, sc0, mn0);
        scale_min_k4(2 * g + 1, hv.y, hv.z, hv.w, sc1, mn1);
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
        float2 slo = f2(0.f, 0.f), shi = f2(0.f, 0.f);
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
            const float2 l01 = __fadd2_rn(f2(byte_m23(lo, 0), byte_m23(lo, 1)), nmag);
            const float2 l23 = __fadd2_rn(f2(byte_m23(lo, 2), byte_m23(lo, 3)), nmag);
            const float2 h01 = __fadd2_rn(f2(byte_m23(hi, 0), byte_m23(hi, 1)), nmag);
            const float2 h23 = __fadd2_rn(f2(byte_m23(hi, 2), byte_m23(hi, 3)), nmag);
            const float4 xl = x.c[w], xh = x.c[4 + w];
            slo = __ffma2_rn(l01, f2(xl.x, xl.y), slo);
            slo = __ffma2_rn(l23, f2(xl.z, xl.w), slo);
            shi = __ffma2_rn(h01, f2(xh.x, xh.y), shi);
            shi = __ffma2_rn(h23, f2(xh.z, xh.w), shi);
        }
        const float d1 = d * sc0, m1 = dmin * mn0, m2 = dmin * mn1;
        const float d2 = (T == T_Q4_K) ? d * sc1 * 0.0625f : d * sc1;
        return d1 * (slo.x + slo.y) - m1 * xs.x + d2 * (shi.x + shi.y) - m2 * xs.y;
    } else if constexpr (T == T_Q6_K) {
        // unit (h, qq): ql bytes [64h + 8qq, +8) and [64h + 32 + 8qq, +8), qh
        // bytes [128 + 32h + 8qq, +8); element 32t + j of the unit is
        // position 128h + 32t + 8qq + j
        const uint8_t *blk = row + (u >> 3) * 210;
        const int ub = u & 7, h = ub >> 2, qq = ub & 3, l0 = 8 * qq;
        uint32_t a[2], b2[2], hh[2], sw[2];
        ld_words_a2<2>(blk + 64 * h + l0, a);
        ld_words_a2<2>(blk + 64 * h + 32 + l0, b2);
        ld_words_a2<2>(blk + 128 + 32 * h + l0, hh);
        ld_words_a2<2>(blk + 192 + 8 * h, sw);
        const float d = f16u(ld_u16_a2(blk + 208));
        const float2 nm32 = f2(-(MAGIC + 32.0f), -(MAGIC + 32.0f));
        float2 st[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t A = a[w], B = b2[w], H = hh[w];
            const uint32_t q6[4] = {(A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u),
                                    (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u),
                                    ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u),
                                    ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u)};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const float2 f01 = __fadd2_rn(f2(byte_m23(q6[t], 0), byte_m23(q6[t], 1)), nm32);
                const float2 f23 = __fadd2_rn(f2(byte_m23(q6[t], 2), byte_m23(q6[t], 3)), nm32);
                const float4 xv = x.c[2 * t + w];
                st[t] = __ffma2_rn(f01, f2(xv.x, xv.y), st[t]);
                st[t] = __ffma2_rn(f23, f2(xv.z, xv.w), st[t]);
            }
        }
        const int is = l0 >> 4;
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int si = is + 2 * t;
            const float ds = d * (float)(int8_t)((sw[si >> 2] >> (8 * (si & 3))) & 0xFF);
            acc = fmaf(ds, st[t].x + st[t].y, acc);
        }
        return acc;
    } else if constexpr (T == T_Q8_0) {
        const uint8_t *blk = row + u * 34;
        const float d = f16u(ld_u16_a2(blk));
        uint32_t q[8];
        ld_words_a2<8>(blk + 2, q);
        const float2 nm = f2(-(MAGIC + 128.0f), -(MAGIC + 128.0f));
        float2 s0 = f2(0.f, 0.f), s1 = f2(0.f, 0.f);
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const uint32_t vb = q[w] ^ 0x80808080u;  // int8 -> biased byte
            const float2 f01 = __fadd2_rn(f2(byte_m23(vb, 0), byte_m23(vb, 1)), nm);
            const float2 f23 = __fadd2_rn(f2(byte_m23(vb, 2), byte_m23(vb, 3)), nm);
            const float4 xv = x.c[w];
            s0 = __ffma2_rn(f01, f2(xv.x, xv.y), s0);
            s1 = __ffma2_rn(f23, f2(xv.z, xv.w), s1);
        }
        return d * ((s0.x + s0.y) + (s1.x + s1.y));
    } else if constexpr (T == T_Q4_0 || T == T_Q5_0) {
        constexpr int BB = blk_bytes(T);
        const uint8_t *blk = row + u * BB;
        const float d = f16u(ld_u16_a2(blk));
        uint32_t q[4], qh0 = 0;
        if constexpr (T == T_Q4_0) {
            ld_words_a2<4>(blk + 2, q);
        } else {
            uint32_t t1[1];
            ld_words_a2<1>(blk + 2, t1);
            qh0 = t1[0];
            ld_words_a2<4>(blk + 6, q);
        }
        float2 sl = f2(0.f, 0.f), sh = f2(0.f, 0.f);
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
            const float2 nl = f2(-offl, -offl), nh = f2(-offh, -offh);
            const float2 l01 = __fadd2_rn(f2(byte_m23(lo, 0), byte_m23(lo, 1)), nl);
            const float2 l23 = __fadd2_rn(f2(byte_m23(lo, 2), byte_m23(lo, 3)), nl);
            const float2 h01 = __fadd2_rn(f2(byte_m23(hi, 0), byte_m23(hi, 1)), nh);
            const float2 h23 = __fadd2_rn(f2(byte_m23(hi, 2), byte_m23(hi, 3)), nh);
            const float4 xl = x.c[w], xh = x.c[4 + w];
            sl = __ffma2_rn(l01, f2(xl.x, xl.y), sl);
            sl = __ffma2_rn(l23, f2(xl.z, xl.w), sl);
            sh = __ffma2_rn(h01, f2(xh.x, xh.y), sh);
            sh = __ffma2_rn(h23, f2(xh.z, xh.w), sh);
        }
        const float dh = (T == T_Q4_0) ? d * 0.0625f : d;
        return d * (sl.x + sl.y) + dh * (sh.x + sh.y);
    } else if constexpr (T == T_F16) {
        float2 s0 = f2(0.f, 0.f), s1 = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 hv = *reinterpret_cast<const uint4 *>(row + 2 * (8 * u + (K / 4) * c));
            const float2 w0 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.x));
            const float2 w1 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.y));
            const float2 w2 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.z));
            const float2 w3 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.w));
            const float4 x0 = x.c[2 * c], x1 = x.c[2 * c + 1];
            s0 = __ffma2_rn(w0, f2(x0.x, x0.y), s0);
            s1 = __ffma2_rn(w1, f2(x0.z, x0.w), s1);
            s0 = __ffma2_rn(w2, f2(x1.x, x1.y), s0);
            s1 = __ffma2_rn(w3, f2(x1.z, x1.w), s1);
        }
        return (s0.x + s0.y) + (s1.x + s1.y);
    } else {  // F32
        float2 s0 = f2(0.f, 0.f), s1 = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const float4 wv = *reinterpret_cast<const float4 *>(row + 4 * (4 * u + (K / 8) * c));
            const float4 xv = x.c[c];
            s0 = __ffma2_rn(f2(wv.x, wv.y), f2(xv.x, xv.y), s0);
            s1 = __ffma2_rn(f2(wv.z, wv.w), f2(xv.z, xv.w), s1);
        }
        return (s0.x + s0.y) + (s1.x + s1.y);
    }
}


// The four 6-bit (scale, min) pairs of sub-blocks 2g, 2g + 1 of a Q4_K / Q5_K
// super-block (scaleMinK4, tensor.go:123-130) from its 12 scale bytes s0..s2,
// as bytes [sc0, sc1, m0, m1]; g is a lane constant, so the byte selectors
// are too and no lane branches.
__device__ __forceinline__ uint32_t scales_k4_pair(uint32_t s0, uint32_t s1, uint32_t s2, int g) {
    const uint32_t jj = (uint32_t)(2 * g) & 3u;
    const uint32_t a = __byte_perm(s0, s1, jj | ((jj + 1) << 4) | ((4 + jj) << 8) | ((5 + jj) << 12));
    if (g < 2) return a & 0x3F3F3F3Fu;
    const uint32_t b = __byte_perm(s2, 0u, jj | ((jj + 1) << 4) | (jj << 8) | ((jj + 1) << 12));
    return ((b & 0x00000F0Fu) | ((b >> 4) & 0x0F0F0000u)) | ((a >> 2) & 0x30303030u);
}

// sum_j w_j x_j over group G of a row (64 elements, group_pos order).
// xs: (sum of the group's low 32 activations, of the high 32) for the min
// terms of Q4_K / Q5_K.
template <int T>
__device__ __forceinline__ float group_dot(const uint8_t *row, int G, const XRegN<16> &x, float2 xs) {
    const float2 nmag = f2(-MAGIC, -MAGIC);
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        constexpr int BB = (T == T_Q4_K) ? 144 : 176, QO = (T == T_Q4_K) ? 16 : 48;
        const uint8_t *blk = row + (G >> 2) * BB;
        const int g = G & 3;
        const uint4 hv = *reinterpret_cast<const uint4 *>(blk);  // d, dmin, scales[12]
        const uint4 qa = *reinterpret_cast<const uint4 *>(blk + QO + 32 * g);
        const uint4 qb = *reinterpret_cast<const uint4 *>(blk + QO + 32 * g + 16);
        uint4 ha, hb;
        if constexpr (T == T_Q5_K) {
            ha = *reinterpret_cast<const uint4 *>(blk + 16);
            hb = *reinterpret_cast<const uint4 *>(blk + 32);
        }
        const uint32_t sm = scales_k4_pair(hv.y, hv.z, hv.w, g);
        const float2 d2 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.x));  // d, dmin
        const float2 scf = __fadd2_rn(f2(byte_m23(sm, 0), byte_m23(sm, 1)), nmag);
        const float2 mnf = __fadd2_rn(f2(byte_m23(sm, 2), byte_m23(sm, 3)), nmag);
        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        float2 slo = f2(0.f, 0.f), shi = f2(0.f, 0.f);
#pragma unroll
        for (int w = 0; w < 8; w++) {
            uint32_t lo, hi;
            if constexpr (T == T_Q4_K) {
                lo = qw[w] & 0x0F0F0F0Fu;
                hi = qw[w] & 0xF0F0F0F0u;  // 16*q, rescaled below
            } else {
                const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
                lo = (qw[w] & 0x0F0F0F0Fu) | (((hw[w] >> (2 * g)) & 0x01010101u) << 4);
                hi = ((qw[w] >> 4) & 0x0F0F0F0Fu) | (((hw[w] >> (2 * g + 1)) & 0x01010101u) << 4);
            }
            const float2 l01 = __fadd2_rn(f2(byte_m23(lo, 0), byte_m23(lo, 1)), nmag);
            const float2 l23 = __fadd2_rn(f2(byte_m23(lo, 2), byte_m23(lo, 3)), nmag);
            const float2 h01 = __fadd2_rn(f2(byte_m23(hi, 0), byte_m23(hi, 1)), nmag);
            const float2 h23 = __fadd2_rn(f2(byte_m23(hi, 2), byte_m23(hi, 3)), nmag);
            const float4 xl = x.c[w], xh = x.c[8 + w];
            slo = __ffma2_rn(l01, f2(xl.x, xl.y), slo);
            slo = __ffma2_rn(l23, f2(xl.z, xl.w), slo);
            shi = __ffma2_rn(h01, f2(xh.x, xh.y), shi);
            shi = __ffma2_rn(h23, f2(xh.z, xh.w), shi);
        }
        // d1 = d*sc (exact), m1 = dmin*m (exact), as the reference forms them
        const float d1 = d2.x * scf.x, m1 = d2.y * mnf.x, m2 = d2.y * mnf.y;
        const float dh = (T == T_Q4_K) ? d2.x * scf.y * 0.0625f : d2.x * scf.y;
        return d1 * (slo.x + slo.y) - m1 * xs.x + dh * (shi.x + shi.y) - m2 * xs.y;
    } else {  // Q6_K: group (sb, h, l0)
        const uint8_t *blk = row + (G >> 2) * 210;
        const int h = (G >> 1) & 1, l0 = 16 * (G & 1), is = G & 1;
        uint32_t A[4], B[4], H[4], sw[2];
        ld_words_a2<4>(blk + 64 * h + l0, A);
        ld_words_a2<4>(blk + 64 * h + 32 + l0, B);
        ld_words_a2<4>(blk + 128 + 32 * h + l0, H);
        ld_words_a2<2>(blk + 192 + 8 * h, sw);
        const float d = f16u(ld_u16_a2(blk + 208));
        const float2 nm32 = f2(-(MAGIC + 32.0f), -(MAGIC + 32.0f));
        float2 st[4] = {f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t q6[4] = {(A[w] & 0x0F0F0F0Fu) | ((H[w] << 4) & 0x30303030u),
                                    (B[w] & 0x0F0F0F0Fu) | ((H[w] << 2) & 0x30303030u),
                                    ((A[w] >> 4) & 0x0F0F0F0Fu) | (H[w] & 0x30303030u),
                                    ((B[w] >> 4) & 0x0F0F0F0Fu) | ((H[w] >> 2) & 0x30303030u)};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const float2 f01 = __fadd2_rn(f2(byte_m23(q6[t], 0), byte_m23(q6[t], 1)), nm32);
                const float2 f23 = __fadd2_rn(f2(byte_m23(q6[t], 2), byte_m23(q6[t], 3)), nm32);
                const float4 xv = x.c[4 * t + w];
                st[t] = __ffma2_rn(f01, f2(xv.x, xv.y), st[t]);
                st[t] = __ffma2_rn(f23, f2(xv.z, xv.w), st[t]);
            }
        }
        // scales sc[8h + is + 2t]: bytes is, is+2, is+4, is+6 of the two words
        const uint32_t sel = is ? 0x7531u : 0x6420u;
        const uint32_t s4 = __byte_perm(sw[0], sw[1], sel);
        float acc = 0.f;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const float ds = d * (float)(int8_t)((s4 >> (8 * t)) & 0xFF);
            acc = fmaf(ds, st[t].x + st[t].y, acc);
        }
        return acc;
    }
}

// One lane unit u of a row: group_dot or unit_dot1 by the format's unit.
template <int T, int NC>
__device__ __forceinline__ float lane_dot(const uint8_t *row, int u, int K, const XRegN<NC> &x, float2 xs) {
    if constexpr (NC == 16) return group_dot<T>(row, u, x, xs);
    else return unit_dot1<T>(row, u, K, x, xs);
}

// The (low half, high half) activation sums of a lane unit (K-quant mins).
template <int T, int NC>
__device__ __forceinline__ float2 lane_xsum(const XRegN<NC> &x) {
    float2 s = make_float2(0.f, 0.f);
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
#pragma unroll
        for (int c = 0; c < NC / 2; c++) {
            const float4 v = x.c[c], w = x.c[NC / 2 + c];
            s.x += (v.x + v.y) + (v.z + v.w);
            s.y += (w.x + w.y) + (w.z + w.w);
        }
    }
    return s;
}

// ---------------------------------------------------------------------------
// Launch arguments of the per-matvec kernel (k_gemv1.cu)
// ---------------------------------------------------------------------------
struct Gemv1Args {
    GemvSeg seg[GEMV_MAX_SEG];
    int nseg;
    const float *x;       // activations of the token (16-byte aligned)
    int k;
    const float *norm_w;  // optional RMSNorm weight applied to x
    float eps;
    int nstage;           // stages per team (1: the team's rows in one copy; 2: double-buffered)
    int stage_bytes;      // bytes per stage (multiple of 128)
    int stage_off;        // byte offset of the first team's stages
    int part_off;         // byte offset of the teams' partial-sum area (teams of more than one warp)
    int part_rows;        // rows per stage the partial area holds
    unsigned long long *trace;  // optional per-CTA timeline of this launch [GEMV1_TRACE_CTAS][8]
    L2Range pf[GEMV_MAX_PF];    // weights of the next matvecs, pulled into L2 (split over the CTAs)
    int npf;
};
// Timeline stamps (thread 0 of each CTA, %globaltimer ns): 0 entry, 1 copies
// issued, 2 dependency wait over, 3 activations staged, 4 first stage
// landed, 5 its rows done; 6 the SM id.
constexpr int GEMV1_TRACE_CTAS = 160;
__device__ __forceinline__ void trace_stamp(unsigned long long *tr, int i) {
    if (tr && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        tr[(size_t)blockIdx.x * 8 + i] = t;
    }
}
constexpr int GEMV1_BAR_BYTES = 256;  // mbarriers: 2 per team, up to 16 teams
constexpr int GEMV1_MAX_TS = 16;       // row teams of up to 16 warps

// Bulk-copy chunk i of a team's rows [wr0, wr1) (rows_per_stage rows; the
// 16-byte rounded byte range of the matrix, then of the pair's second
// matrix) into stage i % nstage, completing on that stage's mbarrier.
__device__ __forceinline__ void gemv1_issue(const Gemv1Args &a, const GemvSeg &s, int wr0, int wr1, int i,
                                            uint64_t *bar, uint8_t *wbuf) {
    const int st = i % a.nstage, R = s.rows_per_stage;
    const int ra = wr0 + i * R, rbn = min(ra + R, wr1);
    const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
    const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
    uint32_t total = (uint32_t)(a1 - a0);
    int64_t c0 = 0, c1 = 0;
    if (s.w2) {
        c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
        c1 = ((int64_t)rbn * s.rb2 + 15) & ~int64_t(15);
        total += (uint32_t)(c1 - c0);
    }
    uint8_t *dst = wbuf + (size_t)st * a.stage_bytes;
    mbar_arrive_expect_tx(&bar[st], total);
    bulk_g2s(dst, s.w + a0, (uint32_t)(a1 - a0), &bar[st]);
    if (s.w2) bulk_g2s(dst + (a1 - a0), s.w2 + c0, (uint32_t)(c1 - c0), &bar[st]);
}

// Wait for the copies of chunks [first, last) of a team's stages (a bounded
// drain after a timed-out wait, so no bulk copy lands after the CTA exits).
__device__ __forceinline__ void gemv1_drain(uint64_t *bar, int nstg, int first, int last) {
    for (int i = first; i < last; i++) {
        const int st = i % nstg;
        mbar_wait_limit(&bar[st], (uint32_t)((i / nstg) & 1), WAIT_LIMIT);
    }
}

// ---------------------------------------------------------------------------
// One team's rows of one stage.  The team's rows are r(j) = base + j * step
// for j in [0, cnt); this warp is number tw of the team (ts warps).  Rows go
// out two at a time per row slot (a half warp when lpr == 16, else the
// warp / team), so each lane has two independent dot products in flight.
// ts == 1: the row sums end in the slot's lanes and one of them runs the
// epilogue; ts > 1: the warps' partial sums meet in part[j][2][ts] and the
// team's first warp finishes the rows, lane j % 32 for row j.  (For
// 64-element units a slot has one row in flight, the lanes' 64 activations
// taking the registers a second would use.)
// ---------------------------------------------------------------------------
struct RowCtx {
    const GemvSeg *s;
    float *yb;       // output row of the token
    float resv;      // this lane's prefetched residual (EPI_ADD)
    int res_j0;      // team-wide index of the row whose residual lane 0 holds
    int res_step;    // ... and its stride over the lanes
    unsigned long long best;
};

__device__ __forceinline__ void row_epilogue(RowCtx &c, int n, int jglob, float v, float v2) {
    const GemvSeg &s = *c.s;
    const int lane = threadIdx.x & 31;
    float o[1] = {v}, o2[1] = {v2}, res[1] = {0.f};
    if (s.epi == EPI_ADD) res[0] = (jglob == c.res_j0 + lane * c.res_step) ? c.resv : __ldcg(c.yb + n);
    unsigned long long b1[1] = {c.best};
    row_out<1>(s, n, 1, o, o2, res, b1);
    c.best = b1[0];
}

template <int T, int NC>
__device__ __forceinline__ void stage_rows(RowCtx &c, const RowGeo &geo, int K, const uint8_t *buf, int64_t a0,
                                           const uint8_t *buf2, int64_t c0, int base, int step, int cnt,
                                           int jglob0, int tw, int team_bar, float *part, const XRegN<NC> &xr,
                                           float2 xsm) {
    const GemvSeg &s = *c.s;
    const int lane = threadIdx.x & 31;
    const bool pair = s.w2 != nullptr;
    const int rpi = 32 / geo.lpr;               // rows per slot step (1 or 2 slots per warp)
    const int half = rpi == 2 ? lane >> 4 : 0;  // this lane's row slot
    const int lu = rpi == 2 ? lane & 15 : lane;
    const int u = 32 * tw + lu;
    const bool has_u = u < geo.U;
    // rows in flight per slot: two for 32-element units, one for 64-element
    // ones (their 64 activations per lane leave no registers for a second)
    constexpr int RU = NC == 16 ? 1 : 2;
    for (int j0 = 0; j0 < cnt; j0 += RU * rpi) {
        const int ja = j0 + half, jb = RU == 2 ? j0 + rpi + half : cnt;
        const int na = base + ja * step, nb = base + jb * step;
        float pa = 0.f, qa = 0.f, pb = 0.f, qb = 0.f;
        if (has_u) {
            if (ja < cnt) {
                pa = lane_dot<T, NC>(buf + ((int64_t)na * s.rb - a0), u, K, xr, xsm);
                if (pair) qa = lane_dot<T, NC>(buf2 + ((int64_t)na * s.rb2 - c0), u, K, xr, xsm);
            }
            if (jb < cnt) {
                pb = lane_dot<T, NC>(buf + ((int64_t)nb * s.rb - a0), u, K, xr, xsm);
                if (pair) qb = lane_dot<T, NC>(buf2 + ((int64_t)nb * s.rb2 - c0), u, K, xr, xsm);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            if (o >= geo.lpr) continue;
            pa += __shfl_xor_sync(0xffffffffu, pa, o);
            pb += __shfl_xor_sync(0xffffffffu, pb, o);
            if (pair) {
                qa += __shfl_xor_sync(0xffffffffu, qa, o);
                qb += __shfl_xor_sync(0xffffffffu, qb, o);
            }
        }
        if (geo.ts == 1) {
            // rows ja, jb of this slot: epilogue on the slot's lanes 0 and 1
            // (one lane per row when a warp is one slot: lanes ja % 32, jb % 32)
            const int ea = rpi == 2 ? 16 * half : (ja & 31), eb = rpi == 2 ? 16 * half + 1 : (jb & 31);
            if (ja < cnt && lane == ea) row_epilogue(c, na, jglob0 + ja, pa, qa);
            if (jb < cnt && lane == eb) row_epilogue(c, nb, jglob0 + jb, pb, qb);
        } else if (lane == 0) {
            const int TS = geo.ts;
            part[(ja * 2) * TS + tw] = pa;
            part[(ja * 2 + 1) * TS + tw] = qa;
            if (jb < cnt) {
                part[(jb * 2) * TS + tw] = pb;
                part[(jb * 2 + 1) * TS + tw] = qb;
            }
        }
    }
    if (geo.ts > 1) {
        const int TS = geo.ts;
        named_sync(team_bar, TS * 32);
        if (tw == 0) {
            for (int j = lane; j < cnt; j += 32) {
                float o = 0.f, o2 = 0.f;
                for (int t = 0; t < TS; t++) {
                    o += part[(j * 2) * TS + t];
                    o2 += part[(j * 2 + 1) * TS + t];
                }
                row_epilogue(c, base + j * step, jglob0 + j, o, o2);
            }
        }
        named_sync(team_bar, TS * 32);  // the parts and the stage are free again
    }
}

// The lane's activations and unit sums, and the residual prefetch of the
// team's first rows (team-wide indices res_j0 + lane * res_step).
template <int T, int NC>
__device__ __forceinline__ void lane_setup(RowCtx &c, const GemvSeg &s, const float *xs, const RowGeo &geo, int tw,
                                           int first_row, int row_step, int nrows, XRegN<NC> &xr, float2 &xsm) {
    const int lane = threadIdx.x & 31;
    const int rpi = 32 / geo.lpr;
    const int u = 32 * tw + (rpi == 2 ? (lane & 15) : lane);
    if (u < geo.U) {
        load_lane_x<NC>(xs, u, xr);
    } else {
#pragma unroll
        for (int i = 0; i < NC; i++) xr.c[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    xsm = lane_xsum<T, NC>(xr);
    c.s = &s;
    c.yb = s.y + (int64_t)(s.yrow ? s.yrow[0] : 0) * s.ldy;
    c.best = 0ull;
    c.resv = 0.f;
    c.res_j0 = 0;
    c.res_step = 1;
    if (s.epi == EPI_ADD && tw == 0 && lane < nrows) c.resv = __ldcg(c.yb + first_row + lane * row_step);
}

__device__ __forceinline__ void flush_best(RowCtx &c) {
    if (!c.s->amax) return;
    const int lane = threadIdx.x & 31;
    unsigned long long best = c.best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long x = __shfl_xor_sync(0xffffffffu, best, o);
        best = x > best ? x : best;
    }
    if (lane == 0 && best) atomicMax(&c.s->amax[0], best);
}

// ---------------------------------------------------------------------------
// Per-matvec kernel: a team's contiguous rows [wr0, wr1) through its own
// stages (filled by gemv1_issue).  red: ts ints (flags); part: the team's
// partial sums [part_rows][2][ts].
// ---------------------------------------------------------------------------
template <int T>
__device__ __forceinline__ void gemv1_rows(const Gemv1Args &a, const GemvSeg &s, const RowGeo &geo, int wr0,
                                           int wr1, uint64_t *bar, uint8_t *wbuf, int nst, int tw, int team_bar,
                                           float *part, float *red, const float *xs) {
    constexpr int NC = lane_elems<T>() / 4;
    const int lane = threadIdx.x & 31;
    const int K = a.k, TS = geo.ts, NSTG = a.nstage, R = s.rows_per_stage;
    RowCtx c;
    XRegN<NC> xr;
    float2 xsm;
    lane_setup<T, NC>(c, s, xs, geo, tw, wr0, 1, wr1 - wr0, xr, xsm);
    for (int i = 0; i < nst; i++) {
        const int st = i % NSTG;
        // every warp of the team sees the stage land, or the whole team leaves
        bool ok = __all_sync(0xffffffffu, mbar_wait(&bar[st], (uint32_t)((i / NSTG) & 1)));
        if (i == 0) trace_stamp(a.trace, 4);
        if (TS > 1) {
            int *flag = reinterpret_cast<int *>(red);
            if (lane == 0) flag[tw] = ok ? 1 : 0;
            named_sync(team_bar, TS * 32);
            for (int t = 0; t < TS; t++) ok = ok && flag[t] != 0;
        }
        if (!ok) {
            if (lane == 0 && tw == 0) gemv1_drain(bar, NSTG, i, min(i + NSTG, nst));
            return;
        }
        const int ra = wr0 + i * R, rbn = min(ra + R, wr1);
        const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
        const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
        const int64_t c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
        const uint8_t *buf = wbuf + (size_t)st * a.stage_bytes;
        stage_rows<T, NC>(c, geo, K, buf, a0, buf + (a1 - a0), c0, ra, 1, rbn - ra, ra - wr0, tw, team_bar, part, xr,
                          xsm);
        if (TS == 1) __syncwarp();
        if (lane == 0 && tw == 0 && i + NSTG < nst) {
            // the team is done reading this stage: refill it with chunk i + NSTG
            fence_proxy_async_smem();
            gemv1_issue(a, s, wr0, wr1, i + NSTG, bar, wbuf);
        }
    }
    trace_stamp(a.trace, 5);
    flush_best(c);
}

}  // namespace acm
