// attn_dev.cuh -- device helpers of the attention kernels: paged cache
// addressing, the per-head RMSNorm + RoPE of model.go:362-382 and the
// batch-1 decode attention item.
#pragma once
#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace acm {

// One cache element at element offset `off` of a pool (fp32, or IEEE half
// for the reduced-precision cache: round to nearest even on store).
__device__ __forceinline__ void kv_store(float *pool, int64_t off, float v, bool f16) {
    if (f16) reinterpret_cast<__half *>(pool)[off] = __float2half_rn(v);
    else pool[off] = v;
}
__device__ __forceinline__ float kv_load(const float *pool, int64_t off, bool f16) {
    return f16 ? __half2float(reinterpret_cast<const __half *>(pool)[off]) : pool[off];
}

__device__ __forceinline__ const float *kv_row(const float *pool, const KVDesc &kv, int layer, int seq, int pos) {
    const int page = kv.page_table[(int64_t)seq * kv.max_pages + (pos / kv.page_size)];
    return pool + (int64_t)layer * kv.layer_stride + ((int64_t)page * kv.page_size + (pos % kv.page_size)) * kv.kvd;
}

template <int HD>
__device__ __forceinline__ void head_norm_rope(float *v, const float *nw, const RopeDesc &r, int pos, int lane) {
    // v: HD floats in shared memory (one warp); rmsnorm (model.go:213-222)
    // then rope (model.go:237-251) in place
    if (nw) {
        float ss = 0.f;
        for (int d = lane; d < HD; d += 32) ss = fmaf(v[d], v[d], ss);
        ss = warp_sum(ss);
        const float sc = rms_scale(ss, HD, r.eps);
        __syncwarp();
        for (int d = lane; d < HD; d += 32) v[d] = __fmul_rn(__fmul_rn(v[d], sc), nw[d]);
    }
    __syncwarp();
    const int half = r.rope_dim / 2;
    const float2 *tab = r.tab + (int64_t)pos * half;
    for (int i = lane; i < half; i += 32) {
        const int ia = r.interleaved ? 2 * i : i, ib = r.interleaved ? 2 * i + 1 : i + half;
        const float a = v[ia], b = v[ib];
        const float2 cs = tab[i];
        v[ia] = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        v[ib] = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
    }
    __syncwarp();
}

// The same per-head RMSNorm + RoPE on a head already held in registers (lane
// owns elements lane + 32e) with its norm weights (nw, when has_nw) and its
// rope table entries (cs[j] for pair lane + 32j) preloaded; the result is
// written to v (shared memory).  Same arithmetic as head_norm_rope.
template <int HD, int NR>
__device__ __forceinline__ void norm_rope_regs(float *v, const float (&x)[HD / 32], bool has_nw,
                                               const float (&nw)[HD / 32], const float2 (&cs)[NR], int half,
                                               int interleaved, float eps, int lane) {
    constexpr int PER = HD / 32;
    if (has_nw) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < PER; e++) ss = fmaf(x[e], x[e], ss);
        ss = warp_sum(ss);
        const float sc = rms_scale(ss, HD, eps);
#pragma unroll
        for (int e = 0; e < PER; e++) v[lane + 32 * e] = __fmul_rn(__fmul_rn(x[e], sc), nw[e]);
    } else {
#pragma unroll
        for (int e = 0; e < PER; e++) v[lane + 32 * e] = x[e];
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < NR; j++) {
        const int i = lane + 32 * j;
        if (i < half) {
            const int ia = interleaved ? 2 * i : i, ib = interleaved ? 2 * i + 1 : i + half;
            const float a = v[ia], b = v[ib];
            v[ia] = __fsub_rn(__fmul_rn(a, cs[j].x), __fmul_rn(b, cs[j].y));
            v[ib] = __fadd_rn(__fmul_rn(a, cs[j].y), __fmul_rn(b, cs[j].x));
        }
    }
    __syncwarp();
}

// Stride (floats) of one partial row of the decode attention: HD values of
// sum e*v, then max and sum e, padded to 16 bytes for bulk copies.
__host__ __device__ constexpr int dec_part_stride(int HD) { return HD + 4; }

// Shared-memory floats one decode attention item needs (a multiple of 4).
__host__ __device__ constexpr int dec_item_floats(int HD, int CH, int G) {
    return (G * (HD + 4) + CH * (HD + 4) + CH * HD + G * CH + 2 * G + (HD < 128 ? HD : 0) + 4 + 3) & ~3;
}

// Partial rows the merge buffer of an item holds (its K and V staging area).
__host__ __device__ constexpr int dec_merge_rows(int HD, int CH) {
    return (CH * (HD + 4) + CH * HD) / dec_part_stride(HD);
}

// Query heads per decode attention item: a divisor h of the group size G
// whose partial rows (h x nch slices) fit the merge buffer in one round of
// copies.  Among those, the largest that still gives at least min_items
// items (nkv x nch x G/h), else the smallest; min_items 0 takes the largest.
// Splitting a group over items re-reads its K/V rows (from L2) but lets
// several CTAs merge at once, each over fewer rows.
__host__ __device__ inline int dec_heads_per_item(int G, int nch, int nkv, int HD, int CH, int min_items) {
    const int cap = dec_merge_rows(HD, CH);
    int small = 0;
    for (int h = G; h >= 1; h--) {
        if (G % h || h * nch > cap) continue;
        if (min_items <= 0 || nkv * nch * (G / h) >= min_items) return h;
        small = h;
    }
    return small ? small : 1;
}

// Cache offsets of a decode attention item, without the layer term: `base`
// of the slice's first position (the slice lies in one page, CH dividing the
// page size) and `newo` of the new position `pos`; both include kv head g.
__device__ __forceinline__ void dec_item_offsets(const KVDesc &kv, int seq, int pos, int g, int lo, int hd,
                                                 int64_t &base, int64_t &newo) {
    const int32_t *pt = kv.page_table + (int64_t)seq * kv.max_pages;
    base = ((int64_t)pt[lo / kv.page_size] * kv.page_size + (lo % kv.page_size)) * kv.kvd + g * hd;
    newo = ((int64_t)pt[pos / kv.page_size] * kv.page_size + (pos % kv.page_size)) * kv.kvd + g * hd;
}

// One decode attention item: token t (new position pos), query heads
// g*G + h0 .. g*G + h0 + hn - 1 of kv head g, positions [c*CH, c*CH + CH) --
// model.go:362-408 for that slice, flash-decoding style -- run by 128 threads
// (gtid 0..127) that synchronise on named barrier `bid`.  The items whose
// slice holds `pos` also normalise and rope the new key (model.go:362-382);
// the one with h0 == 0 appends key and value to the cache.  With more than
// one slice, each writes an unnormalised partial (sum e*v, max, sum e) per
// head and the last slice of (t, g, h0) to finish merges them.  sm:
// dec_item_floats(HD, CH, G) floats, 16-byte aligned.  base / newo:
// dec_item_offsets.
//
// Latency is what matters at this size (a few KB per item): the cached rows
// are requested first, every other global load is issued before any is
// consumed, and the merge pulls whole partial rows into shared memory with
// asynchronous copies (one round trip for every head's rows while hn x
// slices fits dec_merge_rows, else per head in tiles); per-head maxima and
// weights are warp reductions, the outputs one (head, dim) per thread.
// Register use stays small (a fast CTA launch, several items per SM).  KH:
// the cache holds IEEE half (the
// reduced-precision cache); its rows are loaded into registers first,
// widened into the same fp32 staging rows once the query heads are ready,
// and the appended key/value are rounded to half before they are used.
template <int HD, int CH, bool KH = false>
__device__ void decode_attn_item(const RopeDesc &r, const float *q_nw, const float *k_nw, const AttnDesc &a,
                                 const KVDesc &kv, int layer, int t, int pos, int g, int c, int64_t base,
                                 int64_t newo, float *sm, int gtid, int bid, int h0, int hn) {
    constexpr int PER = HD / 32, QS = HD + 4, KS = HD + 4, NR = (HD / 2 + 31) / 32;
    constexpr int GROUPS = 128 / HD, PS = dec_part_stride(HD);
    static_assert(CH == 16 || CH == 32, "chunk must be 16 or 32 positions");
    const int warp = gtid >> 5, lane = gtid & 31;
    const int G = a.n_head / a.n_head_kv, nh = a.n_head, qd = nh * HD, kvd = a.n_head_kv * HD;
    const int L = pos + 1, lo = c * CH, hi = min(L, lo + CH), n = hi - lo;
    const int nchunk = (L + CH - 1) / CH;
    float *qs = sm;                 // [hn][QS]; merge: weights
    float *ks = qs + G * QS;        // [CH][KS]   } merge: partial rows
    float *vs = ks + CH * KS;       // [CH][HD]   }
    float *sc = vs + CH * HD;       // [G][CH]
    float *stat = sc + G * CH;      // [G][2]
    float *gred = stat + 2 * G;     // [HD] second position group (HD < 128)
    int *flag = reinterpret_cast<int *>(gred + (HD < 128 ? HD : 0));
    const bool has_new = pos >= lo && pos < hi;
    const int ncopy = has_new ? n - 1 : n;
    const bool kwarp = has_new && warp == (hn & 3);
    const int half = r.rope_dim / 2;
    const int64_t lofs = (int64_t)layer * kv.layer_stride;

    // ---- cached rows of the slice: asynchronous copies, all in flight ----
    constexpr int CPH = HD / 8;                    // 16-byte pieces per fp16 row
    constexpr int NPH = KH ? (CH * CPH + 127) / 128 : 1;
    uint4 kreg[NPH], vreg[NPH];
    if constexpr (!KH) {
        constexpr int CPR = HD / 4;  // 16-byte pieces per row
        const float *kb = kv.k + lofs + base, *vb = kv.v + lofs + base;
        for (int i = gtid; i < ncopy * CPR; i += 128) {  // K and V piece together, constant divisors
            const int p = i / CPR, piece = i - p * CPR;
            cp_async16(ks + p * KS + piece * 4, kb + (int64_t)p * kv.kvd + piece * 4);
            cp_async16(vs + p * HD + piece * 4, vb + (int64_t)p * kv.kvd + piece * 4);
        }
    } else {
        const __half *kb = reinterpret_cast<const __half *>(kv.k) + lofs + base;
        const __half *vb = reinterpret_cast<const __half *>(kv.v) + lofs + base;
#pragma unroll
        for (int j = 0; j < NPH; j++) {
            const int i = gtid + 128 * j, p = i / CPH, piece = i - p * CPH;
            if (i < ncopy * CPH) {
                kreg[j] = __ldg(reinterpret_cast<const uint4 *>(kb + (int64_t)p * kv.kvd + piece * 8));
                vreg[j] = __ldg(reinterpret_cast<const uint4 *>(vb + (int64_t)p * kv.kvd + piece * 8));
            }
        }
    }
    // ---- query heads (and the new key): loads, then norm + rope ----
    {
        float nq[PER];
        float2 cs[NR];
#pragma unroll
        for (int e = 0; e < PER; e++) nq[e] = q_nw ? q_nw[lane + 32 * e] : 0.f;
#pragma unroll
        for (int j = 0; j < NR; j++) {
            const int i = lane + 32 * j;
            cs[j] = i < half ? r.tab[(int64_t)pos * half + i] : make_float2(0.f, 0.f);
        }
        for (int h = warp; h < hn; h += 4) {
            const float *src = a.q + (int64_t)t * qd + (int64_t)(g * G + h0 + h) * HD;
            float qv[PER];
#pragma unroll
            for (int e = 0; e < PER; e++) qv[e] = __ldcg(src + lane + 32 * e);
            norm_rope_regs<HD, NR>(qs + h * QS, qv, q_nw != nullptr, nq, cs, half, r.interleaved, r.eps, lane);
        }
        if (kwarp) {
            const float *ksrc = r.k + (int64_t)t * kvd + g * HD, *vsrc = r.v + (int64_t)t * kvd + g * HD;
            float kx[PER], nk[PER];
            float *kn = ks + (n - 1) * KS, *vn = vs + (n - 1) * HD;
#pragma unroll
            for (int e = 0; e < PER; e++) {
                kx[e] = __ldcg(ksrc + lane + 32 * e);
                vn[lane + 32 * e] = __ldcg(vsrc + lane + 32 * e);
                nk[e] = k_nw ? k_nw[lane + 32 * e] : 0.f;
            }
            norm_rope_regs<HD, NR>(kn, kx, k_nw != nullptr, nk, cs, half, r.interleaved, r.eps, lane);
            if constexpr (KH) {  // the values later steps will read back
#pragma unroll
                for (int e = 0; e < PER; e++) {
                    kn[lane + 32 * e] = __half2float(__float2half_rn(kn[lane + 32 * e]));
                    vn[lane + 32 * e] = __half2float(__float2half_rn(vn[lane + 32 * e]));
                }
            }
            if (h0 == 0) {  // one item of the group appends the new position
#pragma unroll
                for (int e = 0; e < PER; e++) {
                    kv_store(kv.k, lofs + newo + lane + 32 * e, kn[lane + 32 * e], KH);
                    kv_store(kv.v, lofs + newo + lane + 32 * e, vn[lane + 32 * e], KH);
                }
            }
        }
    }
    if constexpr (KH) {  // widen the fp16 rows into the staging rows
#pragma unroll
        for (int j = 0; j < NPH; j++) {
            const int i = gtid + 128 * j, p = i / CPH, piece = i - p * CPH;
            if (i < ncopy * CPH) {
                const uint32_t kw[4] = {kreg[j].x, kreg[j].y, kreg[j].z, kreg[j].w};
                const uint32_t vw[4] = {vreg[j].x, vreg[j].y, vreg[j].z, vreg[j].w};
                float4 *kd = reinterpret_cast<float4 *>(ks + p * KS + piece * 8);
                float4 *vd = reinterpret_cast<float4 *>(vs + p * HD + piece * 8);
#pragma unroll
                for (int w = 0; w < 2; w++) {
                    const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&kw[2 * w]));
                    const float2 k1 = __half22float2(*reinterpret_cast<const __half2 *>(&kw[2 * w + 1]));
                    const float2 v0 = __half22float2(*reinterpret_cast<const __half2 *>(&vw[2 * w]));
                    const float2 v1 = __half22float2(*reinterpret_cast<const __half2 *>(&vw[2 * w + 1]));
                    kd[w] = make_float4(k0.x, k0.y, k1.x, k1.y);
                    vd[w] = make_float4(v0.x, v0.y, v1.x, v1.y);
                }
            }
        }
    }
    cp_async_wait_all();
    named_sync(bid, 128);

    // ---- scores (one lane per (head, position)) and the slice softmax ----
    for (int b0 = warp * 32; b0 < hn * CH; b0 += 128) {
        const int i = b0 + lane, h = i / CH, p = i - h * CH;
        const bool ok = i < hn * CH && p < n;
        float s = -FLT_MAX;
        if (ok) {
            const float4 *qh = reinterpret_cast<const float4 *>(qs + h * QS);
            const float4 *kp = reinterpret_cast<const float4 *>(ks + p * KS);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
            for (int d4 = 0; d4 < HD / 4; d4++) {
                const float4 x = qh[d4], y = kp[d4];
                acc.x = fmaf(x.x, y.x, acc.x);
                acc.y = fmaf(x.y, y.y, acc.y);
                acc.z = fmaf(x.z, y.z, acc.z);
                acc.w = fmaf(x.w, y.w, acc.w);
            }
            s = __fmul_rn((acc.x + acc.y) + (acc.z + acc.w), a.scale);
        }
        float mx = s;
#pragma unroll
        for (int o = CH / 2; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e = ok ? fast_exp(__fsub_rn(s, mx)) : 0.f;
        float sum = e;
#pragma unroll
        for (int o = CH / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (i < hn * CH) {
            sc[h * CH + p] = nchunk == 1 ? __fdiv_rn(e, sum) : e;
            if (p == 0) {
                stat[2 * h] = mx;
                stat[2 * h + 1] = sum;
            }
        }
    }
    named_sync(bid, 128);

    // ---- P.V, head by head; single chunk: the output, else the partial ----
    const int d = gtid % HD, gp = gtid / HD;
    for (int h = 0; h < hn; h++) {
        const float *sh = sc + h * CH;
        float acc = 0.f;
#pragma unroll 4
        for (int p = gp; p < n; p += GROUPS) acc = fmaf(sh[p], vs[p * HD + d], acc);
        if (GROUPS > 1) {
            if (gp > 0) gred[d] = acc;
            named_sync(bid, 128);
            if (gp == 0) acc += gred[d];
            named_sync(bid, 128);
        }
        if (gp == 0) {
            if (nchunk == 1) {
                a.out[(int64_t)t * qd + (int64_t)(g * G + h0 + h) * HD + d] = acc;
            } else {
                float *pp = a.part + (((int64_t)t * nh + g * G + h0 + h) * a.nsplit + c) * PS;
                pp[d] = acc;
                if (d == 0) {
                    pp[HD] = stat[2 * h];
                    pp[HD + 1] = stat[2 * h + 1];
                }
            }
        }
    }
    if (nchunk == 1) {
        named_sync(bid, 128);
        return;
    }

    // ---- arrival count; the last slice of (t, g, h0) merges ----
    __threadfence();
    named_sync(bid, 128);
    if (gtid == 0) {
        int *cnt = a.counter + (int64_t)t * nh + g * G + h0;
        const int old = atomicAdd(cnt, 1);
        const int last = old == nchunk - 1;
        if (last) *cnt = 0;  // ready for the next step
        *flag = last;
    }
    named_sync(bid, 128);
    if (*flag) {
        __threadfence();
        // merge buffer: the ks..vs region, CAP partial rows at a time
        float *buf = ks;
        constexpr int CAP = dec_merge_rows(HD, CH);
        if (hn * nchunk <= CAP) {
            // every head's partial rows in one round of copies (row hh * nchunk + cc)
            for (int i = gtid; i < hn * nchunk * (PS / 4); i += 128) {
                const int row = i / (PS / 4), piece = i - row * (PS / 4);
                const int hh = row / nchunk, cc = row - hh * nchunk;
                cp_async16(buf + row * PS + piece * 4,
                           a.part + (((int64_t)t * nh + g * G + h0 + hh) * a.nsplit + cc) * PS + piece * 4);
            }
            cp_async_wait_all();
            named_sync(bid, 128);
            // per head (one warp each): maximum over the slices, their weights
            // exp(m_c - M) and the softmax denominator sum_c w_c * (sum e)_c
            float *wb = qs;  // [hn][nchunk]: hn * nchunk <= CAP <= QS
            for (int hh = warp; hh < hn; hh += 4) {
                const float *bh = buf + hh * nchunk * PS;
                float M = -FLT_MAX;
                for (int cc = lane; cc < nchunk; cc += 32) M = fmaxf(M, bh[cc * PS + HD]);
                M = warp_max(M);
                float den = 0.f;
                for (int cc = lane; cc < nchunk; cc += 32) {
                    const float w = fast_exp(bh[cc * PS + HD] - M);
                    wb[hh * nchunk + cc] = w;
                    den = fmaf(w, bh[cc * PS + HD + 1], den);
                }
                den = warp_sum(den);
                if (lane == 0) stat[2 * hh + 1] = den;
            }
            named_sync(bid, 128);
            for (int o = gtid; o < hn * HD; o += 128) {
                const int hh = o / HD, dd = o - hh * HD;
                const float *bh = buf + hh * nchunk * PS + dd, *wh = wb + hh * nchunk;
                float num = 0.f;
                for (int cc = 0; cc < nchunk; cc++) num = fmaf(wh[cc], bh[cc * PS], num);
                a.out[(int64_t)t * qd + (int64_t)(g * G + h0 + hh) * HD + dd] = num / stat[2 * hh + 1];
            }
        } else
        for (int h = 0; h < hn; h++) {
            const float *ph = a.part + ((int64_t)t * nh + g * G + h0 + h) * a.nsplit * PS;
            float M = -FLT_MAX, num = 0.f, den = 0.f;
            for (int c0 = 0; c0 < nchunk; c0 += CAP) {
                const int nt = min(CAP, nchunk - c0);
                for (int i = gtid; i < nt * (PS / 4); i += 128) {
                    const int cc = i / (PS / 4), piece = i - cc * (PS / 4);
                    cp_async16(buf + cc * PS + piece * 4, ph + (int64_t)(c0 + cc) * PS + piece * 4);
                }
                cp_async_wait_all();
                named_sync(bid, 128);
                float mt = -FLT_MAX;
                for (int cc = 0; cc < nt; cc++) mt = fmaxf(mt, buf[cc * PS + HD]);
                const float Mn = fmaxf(M, mt);
                if (c0 > 0) {  // contexts longer than one buffer: rescale what came before
                    const float r0 = fast_exp(M - Mn);
                    num *= r0;
                    den *= r0;
                }
                M = Mn;
                for (int cc = gp; cc < nt; cc += GROUPS) {
                    const float w = fast_exp(buf[cc * PS + HD] - M);
                    num = fmaf(w, buf[cc * PS + d], num);
                    den = fmaf(w, buf[cc * PS + HD + 1], den);
                }
                named_sync(bid, 128);
            }
            if (GROUPS > 1) {
                if (gp > 0) {
                    gred[d] = num;
                    if (d == 0) stat[0] = den;
                }
                named_sync(bid, 128);
                if (gp == 0) {
                    num += gred[d];
                    den += stat[0];
                }
                named_sync(bid, 128);
            }
            if (gp == 0) a.out[(int64_t)t * qd + (int64_t)(g * G + h0 + h) * HD + d] = num / den;
        }
    }
    named_sync(bid, 128);
}

}  // namespace acm
