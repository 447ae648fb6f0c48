// gemv1.cuh -- the batch-1 decode GEMV (one token), device side.
//
// The reference's matvec (internal/infer/tensor.go:253-303, matvec :301)
// dequantizes a tile of weight rows and dots it with the activations.  A
// batch-1 decode token is a chain of ~140 such matvecs of 1-4 MB each, so the
// cost of one launch is its latency, not its bytes.  This kernel is shaped
// for that:
//   * lean CTAs (4-16 warps, no producer warp, a few KB of shared memory per
//     warp), so the CTAs of the next kernels of the token fit on the SMs
//     beside the running one (programmatic dependent launch lets them start
//     as soon as every CTA of this kernel has started);
//   * each warp owns a contiguous row range and moves it into its own
//     shared-memory stages with the bulk-copy engine, issued before the
//     kernel waits for its predecessor -- weights never depend on earlier
//     kernels, so they land while the previous matvec is still running;
//   * each lane keeps the activations of its 32-element units in registers
//     (loaded once, RMSNorm applied in registers, reused for every row), so
//     the inner loop reads shared memory only for weight bytes;
//   * the factored sub-block dot of unit_dot (d*sc * sum q*x - dmin*m * sum x)
//     on packed two-lane fp32 (FADD2 / FFMA2), a shuffle reduction per row,
//     and the epilogues of the other GEMVs (store + bias, residual add,
//     SwiGLU of a gate/up pair, greedy argmax key).
// Units and their element order are those of quant.cuh (unit_pos).
#pragma once
#include "common.cuh"
#include "gemv_dev.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace acm {

// Activations of one 32-element unit in unit order: c[i] holds the unit's
// elements 4i .. 4i + 3 (positions unit_pos<T>(u, 4i + j, K)).
struct XReg {
    float4 c[8];
};

// Activation staging, once per CTA: coalesced loads, RMSNorm (model.go:213-222,
// dst = x * scale * w) when norm_w is set, stored in the unit order of format
// T with the chunk swizzle of x_off, so that each lane then reads its unit's
// 32 values with conflict-free 16-byte loads.  XPER float4s per thread are
// held in registers (K <= XPER * 4 * blockDim.x; larger K is read twice).
constexpr int XPER = 2;
struct XStage {
    float4 v[XPER], w[XPER];
};

// Before the dependency wait: the norm weights (they never change).
__device__ __forceinline__ void stage_x_pre(const float *norm_w, int K, XStage &r) {
    const int n4 = K >> 2;
#pragma unroll
    for (int i = 0; i < XPER; i++) {
        const int q = threadIdx.x + i * blockDim.x;
        r.w[i] = (norm_w && q < n4) ? __ldg(reinterpret_cast<const float4 *>(norm_w) + q)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// After the wait: the activations (written by the previous kernel), the
// norm, the store.  red: 32 floats of scratch.  Every thread takes part.
template <int T>
__device__ __forceinline__ void stage_x(const float *x, const float *norm_w, int K, float eps, float *xs, float *red,
                                        XStage &r) {
    const int tid = threadIdx.x, nthr = blockDim.x, warp = tid >> 5, lane = tid & 31;
    const int n4 = K >> 2;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < XPER; i++) {
        const int q = tid + i * nthr;
        r.v[i] = q < n4 ? __ldcg(reinterpret_cast<const float4 *>(x) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int q = tid + XPER * nthr; q < n4; q += nthr) {
        const float4 t = __ldcg(reinterpret_cast<const float4 *>(x) + q);
        ss = fmaf(t.x, t.x, fmaf(t.y, t.y, fmaf(t.z, t.z, fmaf(t.w, t.w, ss))));
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
        __syncthreads();
        float t = 0.f;
        for (int i = 0; i < (nthr >> 5); i++) t += red[i];
        sc = rms_scale(t, K, eps);
    }
    auto put = [&](int q, float4 a, float4 b) {
        if (norm_w)
            a = make_float4(__fmul_rn(__fmul_rn(a.x, sc), b.x), __fmul_rn(__fmul_rn(a.y, sc), b.y),
                            __fmul_rn(__fmul_rn(a.z, sc), b.z), __fmul_rn(__fmul_rn(a.w, sc), b.w));
        // 4 consecutive positions are 4 consecutive elements of one unit
        *reinterpret_cast<float4 *>(xs + x_off<T>(4 * q, K, false)) = a;
    };
#pragma unroll
    for (int i = 0; i < XPER; i++) {
        const int q = tid + i * nthr;
        if (q < n4) put(q, r.v[i], r.w[i]);
    }
    for (int q = tid + XPER * nthr; q < n4; q += nthr)
        put(q, __ldcg(reinterpret_cast<const float4 *>(x) + q),
            norm_w ? __ldg(reinterpret_cast<const float4 *>(norm_w) + q) : make_float4(0.f, 0.f, 0.f, 0.f));
    __syncthreads();
}

__device__ __forceinline__ void load_xreg_smem(const float *xs, int u, XReg &r) {
#pragma unroll
    for (int c = 0; c < 8; c++) r.c[c] = *reinterpret_cast<const float4 *>(xs + u * 32 + ((c ^ (u & 7)) << 2));
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// acc += sum_j w_j x_j over unit u of a row (MT = 1, activations in
// registers).  xs: the unit's (low half, high half) activation sums, used by
// the K-quant min terms.
template <int T>
__device__ __forceinline__ float unit_dot1(const uint8_t *row, int u, int K, const XReg &x, float2 xs) {
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

struct Gemv1Args {
    GemvSeg seg[GEMV_MAX_SEG];
    int nseg;
    const float *x;       // activations of the token (16-byte aligned)
    int k;
    const float *norm_w;  // optional RMSNorm weight applied to x
    float eps;
    int ts;               // warps per row team: ceil(K / 1024), each warp 32 units of a row
    int nstage;           // stages per team (1: the team's rows in one copy; 2: double-buffered)
    int stage_bytes;      // bytes per stage (multiple of 128)
    int stage_off;        // byte offset of the first team's stages
    int part_off;         // byte offset of the teams' partial-sum area (teams of more than one warp)
    int part_rows;        // rows per stage the partial area holds
    unsigned long long *trace;  // optional per-CTA timeline of this launch [GEMV1_TRACE_CTAS][8]
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
constexpr int GEMV1_MAX_TS = 16;       // K <= 16384

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

// Rows [wr0, wr1) of matrix s for one team of a.ts warps; this warp is
// number tw of its team and owns units 32 tw + lane of every row.  team_bar:
// named barrier of the team (teams of more than one warp); part: the team's
// partial sums [part_rows][2][ts]; red: ts ints (flags); xs: the staged
// activations (stage_x).  Two rows are in flight per warp; the epilogue of
// the team's row wr0 + j runs on lane j % 32 (which prefetched its residual).
template <int T>
__device__ __forceinline__ void gemv1_rows(const Gemv1Args &a, const GemvSeg &s, int wr0, int wr1, uint64_t *bar,
                                           uint8_t *wbuf, int nst, int tw, int team_bar, float *part, float *red,
                                           const float *xs) {
    const int lane = threadIdx.x & 31;
    const int K = a.k, U = K >> 5, TS = a.ts;
    const int NSTG = a.nstage, R = s.rows_per_stage;
    const bool pair = s.w2 != nullptr;
    const int u = 32 * tw + lane;
    const bool has_u = u < U;
    float *yb = s.y + (int64_t)(s.yrow ? s.yrow[0] : 0) * s.ldy;
    // residual stream values (EPI_ADD) of the team's first 32 rows, one per lane
    float resv = 0.f;
    if (s.epi == EPI_ADD && tw == 0 && wr0 + lane < wr1) resv = __ldcg(yb + wr0 + lane);
    auto epilogue = [&](int n, float v, float v2, unsigned long long &best) {
        float o[1] = {v}, o2[1] = {v2}, res[1] = {0.f};
        if (s.epi == EPI_ADD) res[0] = (n - wr0 == lane) ? resv : __ldcg(yb + n);
        unsigned long long b1[1] = {best};
        row_out<1>(s, n, 1, o, o2, res, b1);
        best = b1[0];
    };
    // this lane's activations (unit u), staged and RMSNorm-ed by stage_x
    XReg xr;
    if (has_u) {
        load_xreg_smem(xs, u, xr);
    } else {
#pragma unroll
        for (int c = 0; c < 8; c++) xr.c[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float2 xsm = make_float2(0.f, 0.f);
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const float4 v = xr.c[c], w = xr.c[4 + c];
            xsm.x += (v.x + v.y) + (v.z + v.w);
            xsm.y += (w.x + w.y) + (w.z + w.w);
        }
    }
    unsigned long long best = 0ull;
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
        const uint8_t *buf2 = buf + (a1 - a0);
        for (int n = ra; n < rbn; n += 2) {
            const bool two = n + 1 < rbn;
            float p0 = 0.f, q0 = 0.f, p1 = 0.f, q1 = 0.f;
            if (has_u) {
                p0 = unit_dot1<T>(buf + ((int64_t)n * s.rb - a0), u, K, xr, xsm);
                if (pair) q0 = unit_dot1<T>(buf2 + ((int64_t)n * s.rb2 - c0), u, K, xr, xsm);
                if (two) {
                    p1 = unit_dot1<T>(buf + ((int64_t)(n + 1) * s.rb - a0), u, K, xr, xsm);
                    if (pair) q1 = unit_dot1<T>(buf2 + ((int64_t)(n + 1) * s.rb2 - c0), u, K, xr, xsm);
                }
            }
            p0 = warp_sum(p0);
            p1 = warp_sum(p1);
            if (pair) {
                q0 = warp_sum(q0);
                q1 = warp_sum(q1);
            }
            if (TS == 1) {
                if (lane == ((n - wr0) & 31)) epilogue(n, p0, q0, best);
                if (two && lane == ((n + 1 - wr0) & 31)) epilogue(n + 1, p1, q1, best);
            } else if (lane == 0) {
                part[((n - ra) * 2) * TS + tw] = p0;
                part[((n - ra) * 2 + 1) * TS + tw] = q0;
                if (two) {
                    part[((n + 1 - ra) * 2) * TS + tw] = p1;
                    part[((n + 1 - ra) * 2 + 1) * TS + tw] = q1;
                }
            }
        }
        if (TS == 1) {
            __syncwarp();
        } else {
            // the team's partial sums of this stage are in: warp 0 finishes
            // the rows, one lane per row, summing the parts in unit order
            named_sync(team_bar, TS * 32);
            if (tw == 0) {
                for (int j = lane; j < rbn - ra; j += 32) {
                    float o = 0.f, o2 = 0.f;
                    for (int t = 0; t < TS; t++) {
                        o += part[(j * 2) * TS + t];
                        o2 += part[(j * 2 + 1) * TS + t];
                    }
                    epilogue(ra + j, o, o2, best);
                }
            }
            named_sync(team_bar, TS * 32);  // parts and the stage are free again
        }
        if (lane == 0 && tw == 0 && i + NSTG < nst) {
            // the team is done reading this stage: refill it with chunk i + NSTG
            fence_proxy_async_smem();
            gemv1_issue(a, s, wr0, wr1, i + NSTG, bar, wbuf);
        }
    }
    trace_stamp(a.trace, 5);
    if (s.amax) {
        // lanes hold row maxima: reduce, one atomic per warp
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(0xffffffffu, best, o);
            best = x > best ? x : best;
        }
        if (lane == 0 && best) atomicMax(&s.amax[0], best);
    }
}

}  // namespace acm
