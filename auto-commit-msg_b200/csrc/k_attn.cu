// k_attn.cu -- GQA attention over the paged KV cache (model.go:384-408).
//
// One CTA handles one (token, kv-head) pair and a contiguous range of cache
// positions; the G = n_head / n_head_kv query heads that share the kv head
// are processed together so each K/V row is read once for all of them.
//   phase 1: warp w scores positions w, w+4, ... (lane-split dot product,
//            shuffle reduction), times 1/sqrt(head_dim) as the reference;
//   phase 2: per head, max, fastExp(s - max), sum (softmax, model.go:297-313);
//   phase 3: out[d] = sum_p p_p * v_p[d], positions in increasing order
//            (axpy loop, model.go:404-406).
// Decode batches are small, so the position range of a token is split over
// `nsplit` CTAs (flash-decoding); a second kernel merges the partial
// (sum e*v, max, sum e) triples.
#include <float.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>

#include "attn_dev.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "quant.cuh"

namespace acm {

template <int HD>
__global__ void __launch_bounds__(128) k_attn(const AttnDesc a, const KVDesc kv, int layer, TokMeta tm,
                                              int chunk_max) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    extern __shared__ float sm[];
    constexpr int PER = HD / 32;  // q/k elements per lane
    const int t = blockIdx.x, g = blockIdx.y, split = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.n_head / a.n_head_kv;
    const int nh = a.n_head, qd = nh * HD;
    const int seq = tm.seq[t], pos = tm.pos[t];
    const int L = pos + 1;
    int lo = 0, hi = L;
    if (a.nsplit > 1) {
        const int chunk = (L + a.nsplit - 1) / a.nsplit;
        lo = min(L, split * chunk);
        hi = min(L, lo + chunk);
    }
    const int n = hi - lo;
    float *qs = sm;                    // [G][HD]
    float *sc = sm + G * HD;           // [G][chunk_max]
    float *stat = sc + G * chunk_max;  // [G][2] (max, sum)
    float *red = stat + 2 * G;         // [(128/HD - 1)][G][HD] position-group partials
    if (n <= 0) {
        // empty split: neutral partial
        if (threadIdx.x < G) {
            float *pp = a.part + (((int64_t)t * nh + g * G + threadIdx.x) * a.nsplit + split) * (HD + 2);
            pp[HD] = -FLT_MAX;
            pp[HD + 1] = 0.f;
        }
        for (int i = threadIdx.x; i < G * HD; i += 128) {
            const int hh = i / HD, d = i - hh * HD;
            a.part[(((int64_t)t * nh + g * G + hh) * a.nsplit + split) * (HD + 2) + d] = 0.f;
        }
        return;
    }
    for (int i = threadIdx.x; i < G * HD; i += 128) qs[i] = a.q[(int64_t)t * qd + (int64_t)g * G * HD + i];
    __syncthreads();
    // phase 1: scores
    for (int p = lo + warp; p < hi; p += 4) {
        const float *kr = kv_row(kv.k, kv, layer, seq, p) + g * HD;
        float kk[PER];
#pragma unroll
        for (int e = 0; e < PER; e++) kk[e] = kr[lane + 32 * e];
        for (int h = 0; h < G; h++) {
            float s = 0.f;
#pragma unroll
            for (int e = 0; e < PER; e++) s = fmaf(qs[h * HD + lane + 32 * e], kk[e], s);
            s = warp_sum(s);
            if (lane == 0) sc[h * chunk_max + (p - lo)] = __fmul_rn(s, a.scale);
        }
    }
    __syncthreads();
    // phase 2: softmax per head (warp h handles heads h, h+4, ...)
    for (int h = warp; h < G; h += 4) {
        float *s = sc + h * chunk_max;
        float mx = -FLT_MAX;
        for (int i = lane; i < n; i += 32) mx = fmaxf(mx, s[i]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int i = lane; i < n; i += 32) {
            const float e = fast_exp(__fsub_rn(s[i], mx));
            s[i] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (a.nsplit == 1) {
            for (int i = lane; i < n; i += 32) s[i] = __fdiv_rn(s[i], sum);
        }
        if (lane == 0) {
            stat[2 * h] = mx;
            stat[2 * h + 1] = sum;
        }
    }
    __syncthreads();
    // phase 3: P.V ; 128 threads cover HD dims x (128/HD) position groups
    constexpr int GROUPS = 128 / HD;
    const int d = threadIdx.x % HD, grp = threadIdx.x / HD;
    float acc[8];
#pragma unroll
    for (int h = 0; h < 8; h++) acc[h] = 0.f;
    for (int p = lo + grp; p < hi; p += GROUPS) {
        const float v = kv_row(kv.v, kv, layer, seq, p)[g * HD + d];
#pragma unroll
        for (int h = 0; h < 8; h++)
            if (h < G) acc[h] = fmaf(sc[h * chunk_max + (p - lo)], v, acc[h]);
    }
    if (GROUPS > 1) {
        if (grp > 0)
            for (int h = 0; h < G; h++) red[((grp - 1) * G + h) * HD + d] = acc[h];
        __syncthreads();
        if (grp == 0)
            for (int gg = 1; gg < GROUPS; gg++)
                for (int h = 0; h < G; h++) acc[h] += red[((gg - 1) * G + h) * HD + d];
    }
    if (grp != 0) return;
    if (a.nsplit == 1) {
        for (int h = 0; h < G; h++) a.out[(int64_t)t * qd + (int64_t)(g * G + h) * HD + d] = acc[h];
    } else {
        for (int h = 0; h < G; h++) {
            float *pp = a.part + (((int64_t)t * nh + g * G + h) * a.nsplit + split) * (HD + 2);
            pp[d] = acc[h];
            if (d == 0) {
                pp[HD] = stat[2 * h];
                pp[HD + 1] = stat[2 * h + 1];
            }
        }
    }
}

// Merge split partials: out = sum_s w_s * o_s / sum_s w_s * l_s with
// w_s = fastExp(m_s - max_s m_s).
template <int HD>
__global__ void k_attn_combine(const AttnDesc a) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int t = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const float *pp = a.part + ((int64_t)t * a.n_head + h) * a.nsplit * (HD + 2);
    float mx = -FLT_MAX;
    for (int s = 0; s < a.nsplit; s++)
        if (pp[s * (HD + 2) + HD + 1] > 0.f) mx = fmaxf(mx, pp[s * (HD + 2) + HD]);
    float num = 0.f, den = 0.f;
    for (int s = 0; s < a.nsplit; s++) {
        const float l = pp[s * (HD + 2) + HD + 1];
        if (l > 0.f) {
            const float w = fast_exp(pp[s * (HD + 2) + HD] - mx);
            num = fmaf(w, pp[s * (HD + 2) + d], num);
            den = fmaf(w, l, den);
        }
    }
    a.out[(int64_t)t * a.n_head * HD + (int64_t)h * HD + d] = num / den;
}

// ---------------------------------------------------------------------------
// Decode attention with the new token's QK-norm / RoPE / cache append fused
// in.  Tokens belong to distinct sequences.  CTA (t, g, c) covers positions
// [32c, 32c + 32) of token t's sequence for kv head g; CTAs past the
// sequence's length exit at once.  Each CTA stages its K/V rows in shared
// memory with asynchronous copies issued together, rotates its G query heads
// itself, and -- when its range holds the new position -- normalises and
// rotates the new key, writes key and value to the cache and uses them
// directly.  With one chunk the CTA writes the normalised output; otherwise
// it writes (sum e*v, max, sum e) and the last CTA to arrive merges.
// ---------------------------------------------------------------------------
constexpr int ATT_CHUNK = 32;

template <int HD>
__global__ void __launch_bounds__(128) k_attn_decode(const RopeDesc r, const AttnDesc a, const KVDesc kv, int layer,
                                                     TokMeta tm) {
    extern __shared__ __align__(16) float sm[];
    const int G = a.n_head / a.n_head_kv, nsub = (int)gridDim.y / a.n_head_kv;  // nsub: 1 or G
    const int t = blockIdx.x, g = blockIdx.y / nsub, j = blockIdx.y - g * nsub, c = blockIdx.z;
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    const int seq = tm.seq[t], pos = tm.pos[t];
    if (c * ATT_CHUNK > pos) return;  // beyond this token's context
    // head subset j of hn heads (chosen from this token's slice count; the
    // launch's tokens share the item target); one subset when the launch has
    // no room for more
    const int mi = (a.min_items + (int)gridDim.x - 1) / (int)gridDim.x;
    const int hn = nsub == 1 ? G : dec_heads_per_item(G, (pos + ATT_CHUNK) / ATT_CHUNK, a.n_head_kv, HD, ATT_CHUNK, mi);
    if ((j + 1) * hn > G) return;
    int64_t base, newo;
    dec_item_offsets(kv, seq, pos, g, c * ATT_CHUNK, HD, base, newo);
    if (kv.f16)
        decode_attn_item<HD, ATT_CHUNK, true>(r, r.q_nw, r.k_nw, a, kv, layer, t, pos, g, c, base, newo, sm,
                                              threadIdx.x, 1, j * hn, hn);
    else
        decode_attn_item<HD, ATT_CHUNK, false>(r, r.q_nw, r.k_nw, a, kv, layer, t, pos, g, c, base, newo, sm,
                                               threadIdx.x, 1, j * hn, hn);
}

// ---------------------------------------------------------------------------
// Batched decode attention (many tokens per launch, so that (token, kv head)
// pairs alone fill the GPU): CTA (t, g, s) streams its range of token t's
// context for the G query heads of kv head g in 32-position tiles,
// double-buffered in shared memory in the cache's own format, with the
// softmax maximum found as it goes (running maximum, sums and accumulators
// rescaled by fastExp(m_old - m_new)) -- model.go:384-408.  The CTA whose
// range holds the new position normalises and ropes the new key and appends
// key and value to the cache before streaming.  With several splits, each
// writes (sum e*v, max, sum e) and the last to arrive merges them.
// ---------------------------------------------------------------------------
constexpr int TT = 32;  // positions per tile

__host__ __device__ constexpr int tiled_smem_floats(int HD, int G, int kt_bytes) {
    // qs [G][HD+4] | K 2 x [TT][HD + 16/kt] | V 2 x [TT][HD] | sc [G][TT] | stat 3G+1 | gred [G][HD] | knew [HD] | flag
    return (G * (HD + 4) + (2 * TT * (HD + 16 / kt_bytes) + 2 * TT * HD) * kt_bytes / 4 + G * TT + 4 * G +
            (HD < 128 ? G * HD : 0) + HD + 4 + 3) & ~3;
}

__device__ __forceinline__ float kt_f(float v) { return v; }
__device__ __forceinline__ float kt_f(__half v) { return __half2float(v); }

template <int HD, typename KT>
__global__ void __launch_bounds__(128) k_attn_decode_tiled(const RopeDesc r, const AttnDesc a, const KVDesc kv,
                                                           int layer, TokMeta tm, int nsplit) {
    extern __shared__ __align__(16) float sm[];
    constexpr int PER = HD / 32, NR = (HD / 2 + 31) / 32, QS = HD + 4;
    constexpr int EPR = 16 / (int)sizeof(KT);  // elements per 16-byte piece
    constexpr int CPR = HD / EPR;              // pieces per row
    constexpr int KSE = HD + EPR;              // K row stride (elements)
    constexpr int GROUPS = 128 / HD, PS = dec_part_stride(HD);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int G = a.n_head / a.n_head_kv, nh = a.n_head, qd = nh * HD, kvd = a.n_head_kv * HD;
    if (tid == 0) pdl_trigger();
    pdl_wait();
    const int seq = tm.seq[t], pos = tm.pos[t], L = pos + 1;
    const int tiles_all = (L + TT - 1) / TT, tps = (tiles_all + nsplit - 1) / nsplit;
    const int nsp = (tiles_all + tps - 1) / tps;  // splits this token uses
    if (s >= nsp) return;
    const int lo = s * tps * TT, hi = min(L, lo + tps * TT), ntile = (hi - lo + TT - 1) / TT;
    float *qs = sm;
    KT *kbuf = reinterpret_cast<KT *>(qs + G * QS);
    KT *vbuf = kbuf + 2 * TT * KSE;
    float *sc = reinterpret_cast<float *>(vbuf + 2 * TT * HD);
    float *st_m = sc + G * TT, *st_l = st_m + G, *st_r = st_l + G;
    float *gred = st_r + 2 * G;
    float *knew = gred + (HD < 128 ? G * HD : 0);
    int *flag = reinterpret_cast<int *>(knew + HD);
    const int64_t lofs = (int64_t)layer * kv.layer_stride;
    const int32_t *pt = kv.page_table + (int64_t)seq * kv.max_pages;
    const KT *kpool = reinterpret_cast<const KT *>(kv.k), *vpool = reinterpret_cast<const KT *>(kv.v);
    auto load_tile = [&](int ti, int buf) {  // a tile lies in one page (page size a multiple of TT)
        const int p0 = lo + ti * TT, n = min(TT, hi - p0);
        const int64_t base =
            lofs + ((int64_t)pt[p0 / kv.page_size] * kv.page_size + (p0 % kv.page_size)) * kv.kvd + g * HD;
        KT *kd = kbuf + buf * TT * KSE, *vd = vbuf + buf * TT * HD;
        for (int i = tid; i < n * CPR; i += 128) {
            const int p = i / CPR, c = i - p * CPR;
            cp_async16(kd + p * KSE + c * EPR, kpool + base + (int64_t)p * kv.kvd + c * EPR);
            cp_async16(vd + p * HD + c * EPR, vpool + base + (int64_t)p * kv.kvd + c * EPR);
        }
        cp_async_commit();
    };
    // ---- query heads, and the new key / value appended before streaming ----
    const int half = r.rope_dim / 2;
    const bool has_new = pos >= lo && pos < hi;
    {
        float nq[PER];
        float2 cs[NR];
#pragma unroll
        for (int e = 0; e < PER; e++) nq[e] = r.q_nw ? r.q_nw[lane + 32 * e] : 0.f;
#pragma unroll
        for (int j = 0; j < NR; j++) {
            const int i = lane + 32 * j;
            cs[j] = i < half ? r.tab[(int64_t)pos * half + i] : make_float2(0.f, 0.f);
        }
        for (int h = warp; h < G; h += 4) {
            float qv[PER];
#pragma unroll
            for (int e = 0; e < PER; e++) qv[e] = __ldcg(a.q + (int64_t)t * qd + (int64_t)(g * G + h) * HD + lane + 32 * e);
            norm_rope_regs<HD, NR>(qs + h * QS, qv, r.q_nw != nullptr, nq, cs, half, r.interleaved, r.eps, lane);
        }
        if (has_new && warp == (G & 3)) {
            float kx[PER], nk[PER], vx[PER];
#pragma unroll
            for (int e = 0; e < PER; e++) {
                kx[e] = __ldcg(r.k + (int64_t)t * kvd + g * HD + lane + 32 * e);
                vx[e] = __ldcg(r.v + (int64_t)t * kvd + g * HD + lane + 32 * e);
                nk[e] = r.k_nw ? r.k_nw[lane + 32 * e] : 0.f;
            }
            norm_rope_regs<HD, NR>(knew, kx, r.k_nw != nullptr, nk, cs, half, r.interleaved, r.eps, lane);
            const int64_t no = lofs + ((int64_t)pt[pos / kv.page_size] * kv.page_size + (pos % kv.page_size)) * kv.kvd +
                               g * HD;
#pragma unroll
            for (int e = 0; e < PER; e++) {
                kv_store(kv.k, no + lane + 32 * e, knew[lane + 32 * e], kv.f16);
                kv_store(kv.v, no + lane + 32 * e, vx[e], kv.f16);
            }
            __threadfence();  // the row is read back through L2 by this CTA's tile copies
        }
        if (tid < G) {
            st_m[tid] = -FLT_MAX;
            st_l[tid] = 0.f;
        }
    }
    __syncthreads();  // queries ready; the appended row visible to this CTA's copies
    // ---- stream the tiles ----
    const int d = tid % HD, gp = tid / HD;
    float acc[8];
#pragma unroll
    for (int h = 0; h < 8; h++) acc[h] = 0.f;
    load_tile(0, 0);
    for (int ti = 0; ti < ntile; ti++) {
        const int buf = ti & 1;
        if (ti + 1 < ntile) {
            load_tile(ti + 1, buf ^ 1);
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();
        const int n = min(TT, hi - (lo + ti * TT));
        const KT *kt = kbuf + buf * TT * KSE, *vt = vbuf + buf * TT * HD;
        // scores, one lane per (head, position); a head's 32 positions are one warp
        for (int b0 = warp * 32; b0 < G * TT; b0 += 128) {
            const int i = b0 + lane, h = i / TT, p = i - h * TT;
            const bool in = i < G * TT, ok = in && p < n;
            float sv = -FLT_MAX;
            if (ok) {
                const float *qh = qs + h * QS;
                const KT *kp = kt + p * KSE;
                float4 ac = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
                for (int d4 = 0; d4 < HD / 4; d4++) {
                    const float4 x = *reinterpret_cast<const float4 *>(qh + 4 * d4);
                    float y0, y1, y2, y3;
                    if constexpr (sizeof(KT) == 4) {
                        const float4 y = *reinterpret_cast<const float4 *>(kp + 4 * d4);
                        y0 = y.x, y1 = y.y, y2 = y.z, y3 = y.w;
                    } else {
                        const uint2 hv = *reinterpret_cast<const uint2 *>(kp + 4 * d4);
                        const float2 a0 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.x));
                        const float2 a1 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.y));
                        y0 = a0.x, y1 = a0.y, y2 = a1.x, y3 = a1.y;
                    }
                    ac.x = fmaf(x.x, y0, ac.x);
                    ac.y = fmaf(x.y, y1, ac.y);
                    ac.z = fmaf(x.z, y2, ac.z);
                    ac.w = fmaf(x.w, y3, ac.w);
                }
                sv = __fmul_rn((ac.x + ac.y) + (ac.z + ac.w), a.scale);
            }
            if (in) {  // whole warps: every lane of a head's warp takes part
                const float mold = st_m[h];
                const float mnew = fmaxf(mold, warp_max(sv));
                const float e = ok ? fast_exp(__fsub_rn(sv, mnew)) : 0.f;
                const float sum = warp_sum(e);
                sc[h * TT + p] = e;
                if (p == 0) {
                    const float rs = mold == -FLT_MAX ? 0.f : fast_exp(__fsub_rn(mold, mnew));
                    st_r[h] = rs;
                    st_m[h] = mnew;
                    st_l[h] = fmaf(st_l[h], rs, sum);
                }
            }
        }
        __syncthreads();
        // P.V with the running rescale
#pragma unroll
        for (int h = 0; h < 8; h++) {
            if (h < G) {
                const float *sh = sc + h * TT;
                float a2 = acc[h] * st_r[h];
#pragma unroll 4
                for (int p = gp; p < n; p += GROUPS) a2 = fmaf(sh[p], kt_f(vt[p * HD + d]), a2);
                acc[h] = a2;
            }
        }
        __syncthreads();  // the tile's buffers are free for the load two tiles on
    }
    // ---- combine the position groups (HD < 128) ----
    if (GROUPS > 1) {
#pragma unroll
        for (int h = 0; h < 8; h++)
            if (h < G && gp > 0) gred[h * HD + d] = acc[h];
        __syncthreads();
        if (gp == 0) {
#pragma unroll
            for (int h = 0; h < 8; h++)
                if (h < G) acc[h] += gred[h * HD + d];
        }
    }
    if (nsp == 1) {
        if (gp == 0) {
#pragma unroll
            for (int h = 0; h < 8; h++)
                if (h < G) a.out[(int64_t)t * qd + (int64_t)(g * G + h) * HD + d] = acc[h] / st_l[h];
        }
        return;
    }
    if (gp == 0) {
#pragma unroll
        for (int h = 0; h < 8; h++) {
            if (h < G) {
                float *pp = a.part + (((int64_t)t * nh + g * G + h) * a.nsplit + s) * PS;
                pp[d] = acc[h];
                if (d == 0) {
                    pp[HD] = st_m[h];
                    pp[HD + 1] = st_l[h];
                }
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int *cnt = a.counter + (int64_t)t * nh + g * G;
        const int old = atomicAdd(cnt, 1);
        const int last = old == nsp - 1;
        if (last) *cnt = 0;  // ready for the next step
        *flag = last;
    }
    __syncthreads();
    if (*flag) {  // the last split merges every split's rows (few: direct loads)
        __threadfence();
        for (int o = tid; o < G * HD; o += 128) {
            const int h = o / HD, dd = o - h * HD;
            const float *ph = a.part + ((int64_t)t * nh + g * G + h) * a.nsplit * PS;
            float M = -FLT_MAX;
            for (int c = 0; c < nsp; c++) M = fmaxf(M, __ldcg(ph + c * PS + HD));
            float num = 0.f, den = 0.f;
            for (int c = 0; c < nsp; c++) {
                const float w = fast_exp(__fsub_rn(__ldcg(ph + c * PS + HD), M));
                num = fmaf(w, __ldcg(ph + c * PS + dd), num);
                den = fmaf(w, __ldcg(ph + c * PS + HD + 1), den);
            }
            a.out[(int64_t)t * qd + (int64_t)(g * G + h) * HD + dd] = num / den;
        }
    }
}

template <int HD, typename KT>
static cudaError_t launch_tiled(const RopeDesc &r, const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm,
                               int ntok, int nsplit, cudaStream_t st) {
    const int G = a.n_head / a.n_head_kv;
    const size_t smem = (size_t)tiled_smem_floats(HD, G, (int)sizeof(KT)) * sizeof(float);
    static std::atomic<bool> attr[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_decode_tiled<HD, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    return launch_pdl(k_attn_decode_tiled<HD, KT>, dim3(ntok, a.n_head_kv, nsplit), dim3(128), smem, st, r, a, kv,
                      layer, tm, nsplit);
}

cudaError_t attention_decode_launch(const RopeDesc &r, const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm,
                                    int ntok, int max_pos, cudaStream_t st) {
    if (ntok <= 0) return cudaSuccess;
    const int G = a.n_head / a.n_head_kv;
    if (G > 8 || a.n_head % a.n_head_kv || (a.head_dim != 64 && a.head_dim != 128)) return cudaErrorInvalidValue;
    const int nchunk = (max_pos + 1 + ATT_CHUNK - 1) / ATT_CHUNK;
    if (nchunk > a.nsplit) return cudaErrorInvalidValue;  // partial buffer capacity
    if (kv.page_size % ATT_CHUNK) return cudaErrorInvalidValue;
    const int HD = a.head_dim;
    const size_t smem = (size_t)dec_item_floats(HD, ATT_CHUNK, G) * sizeof(float);
    // Many (token, kv head) pairs: the streaming kernel, a few splits per pair.
    const bool batched = (int64_t)ntok * a.n_head_kv * 4 >= (a.min_items > 1 ? a.min_items : 1);
    if (batched && a.min_items > 0) {
        const int target = 6 * a.min_items;  // ~3 resident CTAs per SM, two waves
        int ns = (int)std::min<int64_t>(16, (target + (int64_t)ntok * a.n_head_kv - 1) / ((int64_t)ntok * a.n_head_kv));
        ns = std::max(1, std::min(ns, a.nsplit));
        cudaError_t e = kv.f16 ? (HD == 128 ? launch_tiled<128, __half>(r, a, kv, layer, tm, ntok, ns, st)
                                            : launch_tiled<64, __half>(r, a, kv, layer, tm, ntok, ns, st))
                               : (HD == 128 ? launch_tiled<128, float>(r, a, kv, layer, tm, ntok, ns, st)
                                            : launch_tiled<64, float>(r, a, kv, layer, tm, ntok, ns, st));
        if (e != cudaSuccess) return e;
        return launched(1);
    }
    // y: kv head x head subset (unused subsets exit).  Query heads are split
    // over items only while the launch has few (token, kv head) pairs: with
    // many tokens the extra CTAs would mostly exit at once.
    const int nsub = batched ? 1 : G;
    dim3 grid(ntok, a.n_head_kv * nsub, nchunk);
    cudaError_t e = HD == 128 ? launch_pdl(k_attn_decode<128>, grid, dim3(128), smem, st, r, a, kv, layer, tm)
                              : launch_pdl(k_attn_decode<64>, grid, dim3(128), smem, st, r, a, kv, layer, tm);
    if (e != cudaSuccess) return e;
    return launched(1);
}

// ---------------------------------------------------------------------------
// Prefill attention: the tokens of the batch are consecutive positions of one
// sequence (keys/values already appended).  CTA (tile, g): QT query tokens x
// the G query heads of kv head g = R = QT*G rows.  Two passes over 32-position
// key tiles staged in shared memory: pass 1 finds each row's maximum score,
// pass 2 forms e = fastExp(s - max) exactly as the reference's softmax
// (model.go:297-313) and accumulates e*v and sum e; out = sum(e*v) / sum(e).
// Scores and P.V are register-tiled FFMA (4 rows x 4 keys, 8 rows x 8 dims).
// ---------------------------------------------------------------------------
constexpr int PQT = 16;  // query tokens per CTA
constexpr int PKT = 32;  // keys per tile

template <int HD>
__global__ void __launch_bounds__(256) k_attn_prefill(const AttnDesc a, const KVDesc kv, int layer, TokMeta tm,
                                                      int ntok) {
    extern __shared__ __align__(16) float psm[];
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int G = a.n_head / a.n_head_kv, nh = a.n_head, qd = nh * HD;
    const int tile = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
    const int t0 = tile * PQT, nt = min(PQT, ntok - t0);
    const int R = PQT * G;  // rows (token-major: r = tq*G + h)
    const int seq = tm.seq[t0], pos0 = tm.pos[t0];
    const int max_pos = pos0 + nt - 1;
    constexpr int QS = HD + 4;  // padded row strides
    float *qs = psm;                     // [R][QS]
    float *ks = qs + R * QS;             // [PKT][QS]
    float *vs = ks + PKT * QS;           // [PKT][HD]
    float *ss = vs + PKT * HD;           // [R][PKT + 1]
    float *rmax = ss + R * (PKT + 1);    // [R]
    float *rsum = rmax + R;              // [R]
    for (int i = tid; i < R * HD; i += 256) {
        const int r = i / HD, d = i - r * HD, tq = r / G, h = r - tq * G;
        qs[r * QS + d] = tq < nt ? a.q[(int64_t)(t0 + tq) * qd + (int64_t)(g * G + h) * HD + d] : 0.f;
    }
    for (int r = tid; r < R; r += 256) {
        rmax[r] = -FLT_MAX;
        rsum[r] = 0.f;
    }
    const int nkt = (max_pos + PKT) / PKT;  // key tiles covering [0, max_pos]
    // thread tiles: scores 4 rows x 4 keys (R <= 128 rows, 32 keys -> <= 256 threads)
    const int sr = (tid / 8) * 4, sk = (tid % 8) * 4;
    // P.V: 8 rows x 8 dims per thread over R x HD
    const int prow = (tid / (HD / 8)) * 8, pdim = (tid % (HD / 8)) * 8;
    float o[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) o[i][j] = 0.f;
    for (int pass = 0; pass < 2; pass++) {
        for (int kt = 0; kt < nkt; kt++) {
            const int k0 = kt * PKT, kn = min(PKT, max_pos + 1 - k0);
            __syncthreads();
            // stage keys (and values in pass 2); a tile lies in one page
            const int64_t base = (int64_t)layer * kv.layer_stride +
                                 ((int64_t)kv.page_table[(int64_t)seq * kv.max_pages + k0 / kv.page_size] * kv.page_size +
                                  (k0 % kv.page_size)) * kv.kvd + g * HD;
            const int pieces = kn * (HD / 4);
            if (kv.f16) {  // fp16 cache: 4 halves per piece, widened on the way in
                for (int i = tid; i < pieces * (pass + 1); i += 256) {
                    const int which = i / pieces, rem = i - which * pieces;
                    const int p = rem / (HD / 4), c = rem - p * (HD / 4);
                    const __half *src = reinterpret_cast<const __half *>(which ? kv.v : kv.k) + base +
                                        (int64_t)p * kv.kvd + c * 4;
                    const uint2 hv = *reinterpret_cast<const uint2 *>(src);
                    const float2 a0 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.x));
                    const float2 a1 = __half22float2(*reinterpret_cast<const __half2 *>(&hv.y));
                    *reinterpret_cast<float4 *>(which ? vs + p * HD + c * 4 : ks + p * QS + c * 4) =
                        make_float4(a0.x, a0.y, a1.x, a1.y);
                }
            } else {
                for (int i = tid; i < pieces * (pass + 1); i += 256) {
                    const int which = i / pieces, rem = i - which * pieces;
                    const int p = rem / (HD / 4), c = rem - p * (HD / 4);
                    const float *src = (which ? kv.v : kv.k) + base + (int64_t)p * kv.kvd + c * 4;
                    cp_async16(which ? vs + p * HD + c * 4 : ks + p * QS + c * 4, src);
                }
            }
            cp_async_wait_all();
            __syncthreads();
            // scores for rows sr..sr+3, keys sk..sk+3
            if (sr < R) {
                float acc[4][4];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
                for (int d = 0; d < HD; d += 4) {
                    float4 qv[4], kv4[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const float4 *>(qs + (sr + i) * QS + d);
#pragma unroll
                    for (int j = 0; j < 4; j++) kv4[j] = *reinterpret_cast<const float4 *>(ks + (sk + j) * QS + d);
#pragma unroll
                    for (int i = 0; i < 4; i++)
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            acc[i][j] = fmaf(qv[i].x, kv4[j].x, acc[i][j]);
                            acc[i][j] = fmaf(qv[i].y, kv4[j].y, acc[i][j]);
                            acc[i][j] = fmaf(qv[i].z, kv4[j].z, acc[i][j]);
                            acc[i][j] = fmaf(qv[i].w, kv4[j].w, acc[i][j]);
                        }
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = sr + i, tq = r / G;
                    const int qpos = pos0 + tq;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int kp = k0 + sk + j;
                        const bool ok = sk + j < kn && kp <= qpos && tq < nt;
                        ss[r * (PKT + 1) + sk + j] = ok ? __fmul_rn(acc[i][j], a.scale) : -FLT_MAX;
                    }
                }
            }
            __syncthreads();
            if (pass == 0) {
                // running row maxima
                for (int r = tid; r < R; r += 256) {
                    float m = rmax[r];
                    for (int j = 0; j < kn; j++) m = fmaxf(m, ss[r * (PKT + 1) + j]);
                    rmax[r] = m;
                }
            } else {
                // e = fastExp(s - max) in place, row sums
                for (int r = tid; r < R; r += 256) {
                    const float m = rmax[r];
                    float s = rsum[r];
                    for (int j = 0; j < kn; j++) {
                        float *e = ss + r * (PKT + 1) + j;
                        const float v = *e == -FLT_MAX ? 0.f : fast_exp(__fsub_rn(*e, m));
                        *e = v;
                        s += v;
                    }
                    rsum[r] = s;
                }
                __syncthreads();
                if (prow < R) {
                    for (int j = 0; j < kn; j++) {
                        const float4 v0 = *reinterpret_cast<const float4 *>(vs + j * HD + pdim);
                        const float4 v1 = *reinterpret_cast<const float4 *>(vs + j * HD + pdim + 4);
                        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const float p = ss[(prow + i) * (PKT + 1) + j];
#pragma unroll
                            for (int dd = 0; dd < 8; dd++) o[i][dd] = fmaf(p, vv[dd], o[i][dd]);
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
    if (prow < R) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int r = prow + i, tq = r / G, h = r - tq * G;
            if (tq >= nt) continue;
            const float inv = rsum[r];
            float *dst = a.out + (int64_t)(t0 + tq) * qd + (int64_t)(g * G + h) * HD + pdim;
#pragma unroll
            for (int dd = 0; dd < 8; dd++) dst[dd] = __fdiv_rn(o[i][dd], inv);
        }
    }
}

cudaError_t attention_prefill_launch(const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm, int ntok,
                                     cudaStream_t st) {
    if (ntok <= 0) return cudaSuccess;
    const int G = a.n_head / a.n_head_kv, HD = a.head_dim;
    if (G > 8 || a.n_head % a.n_head_kv || (HD != 64 && HD != 128) || kv.page_size % PKT) return cudaErrorInvalidValue;
    const int R = PQT * G;
    if ((R / 4) * 8 > 256 && R > 128) return cudaErrorInvalidValue;
    const int QS = HD + 4;
    const size_t smem = ((size_t)R * QS + PKT * QS + PKT * HD + (size_t)R * (PKT + 1) + 2 * R) * sizeof(float);
    static std::atomic<bool> attr[64][2] = {};  // per device and variant: attributes set
    int dev = 0;
    cudaGetDevice(&dev);
    const int hi = HD == 128 ? 0 : 1;
    if (!attr[dev & 63][hi]) {
        cudaFuncSetAttribute(HD == 128 ? k_attn_prefill<128> : k_attn_prefill<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr[dev & 63][hi] = true;
    }
    dim3 grid((ntok + PQT - 1) / PQT, a.n_head_kv);
    cudaError_t e = HD == 128 ? launch_pdl(k_attn_prefill<128>, grid, dim3(256), smem, st, a, kv, layer, tm, ntok)
                              : launch_pdl(k_attn_prefill<64>, grid, dim3(256), smem, st, a, kv, layer, tm, ntok);
    if (e != cudaSuccess) return e;
    return launched(1);
}

cudaError_t attention_launch(const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm, int ntok, int max_pos,
                             cudaStream_t st) {
    if (ntok <= 0) return cudaSuccess;
    const int G = a.n_head / a.n_head_kv;
    if (G > 8 || a.n_head % a.n_head_kv || kv.f16) return cudaErrorInvalidValue;  // fp32 cache only
    const int L = max_pos + 1;
    const int chunk_max = (L + a.nsplit - 1) / a.nsplit;
    const int HD = a.head_dim;
    const size_t red = (size_t)(128 / HD > 1 ? (128 / HD - 1) : 0) * G * HD;
    const size_t smem = ((size_t)G * HD + (size_t)G * chunk_max + 2 * G + red) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    dim3 grid(ntok, a.n_head_kv, a.nsplit);
    static std::atomic<bool> attr[64][2] = {};  // per device and variant: attributes set
    int dev = 0;
    cudaGetDevice(&dev);
    if (HD == 128) {
        if (!attr[dev & 63][0]) {
            cudaFuncSetAttribute(k_attn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            attr[dev & 63][0] = true;
        }
        launch_pdl(k_attn<128>, grid, dim3(128), smem, st, a, kv, layer, tm, chunk_max);
        if (a.nsplit > 1) launch_pdl(k_attn_combine<128>, dim3(ntok, a.n_head), dim3(128), 0, st, a);
    } else if (HD == 64) {
        if (!attr[dev & 63][1]) {
            cudaFuncSetAttribute(k_attn<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            attr[dev & 63][1] = true;
        }
        launch_pdl(k_attn<64>, grid, dim3(128), smem, st, a, kv, layer, tm, chunk_max);
        if (a.nsplit > 1) launch_pdl(k_attn_combine<64>, dim3(ntok, a.n_head), dim3(64), 0, st, a);
    } else {
        return cudaErrorInvalidValue;
    }
    return launched(a.nsplit > 1 ? 2 : 1);
}

}  // namespace acm
