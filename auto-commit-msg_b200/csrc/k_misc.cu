// k_misc.cu -- the small per-token kernels of the token loop:
//   exact dequant / embedding gather   (tensor.go:55-81, model.go:338-340)
//   RMSNorm                           (model.go:213-222)
//   QK-norm + RoPE + KV-cache append  (model.go:362-382, :237-251)
//   top-k / greedy sampler            (sampler.go:19-98)
#include <float.h>

#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "attn_dev.cuh"
#include "quant.cuh"

namespace acm {

// ---------------------------------------------------------------------------
// Dequantize rows; one thread per 32-element run (consecutive threads take
// consecutive runs of a row, so the output stores coalesce).
// ---------------------------------------------------------------------------
template <int T>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t *w, int64_t rb, int64_t K, int64_t nrows,
                                                 const int32_t *ids, int64_t src_rows, float *out, int64_t ldo) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int64_t runs = K / 32, total = nrows * runs;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / runs;
        const int run = (int)(idx - r * runs);
        int64_t src = r;
        if (ids) {
            src = ids[r];
            if (src < 0 || src >= src_rows) {
                atomicExch(&g_dev_error, DEV_ERR_BOUNDS);
                continue;
            }
        }
        float v[32];
        dequant_run32<T>(w + src * rb, run, v);
        float4 *o = reinterpret_cast<float4 *>(out + r * ldo + 32 * run);
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
}

cudaError_t dequant_launch(int type, const void *w, int64_t k, int64_t nrows, const int32_t *row_ids,
                           int64_t src_rows, float *out, int64_t ldo, cudaStream_t st) {
    if (!type_ok(type) || k % 32 || (k % blk_elems(type)) || nrows < 0 || (ldo % 4)) return cudaErrorInvalidValue;
    if (nrows == 0) return cudaSuccess;
    const int64_t total = nrows * (k / 32);
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    const uint8_t *wb = static_cast<const uint8_t *>(w);
    const int64_t rb = row_bytes(type, k);
    switch (type) {
#define ACM_DQ(T) \
    case T: launch_pdl(k_dequant<T>, dim3(grid), dim3(256), 0, st, wb, rb, k, nrows, row_ids, src_rows, out, ldo); break;
        ACM_DQ(T_F32) ACM_DQ(T_F16) ACM_DQ(T_Q4_0) ACM_DQ(T_Q5_0) ACM_DQ(T_Q8_0) ACM_DQ(T_Q4_K) ACM_DQ(T_Q5_K)
        ACM_DQ(T_Q6_K)
#undef ACM_DQ
    }
    return launched(1);
}

// ---------------------------------------------------------------------------
// RMSNorm, one CTA per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const float *x, int ldx, const float *w, float *y, int ldy, int n,
                                                 float eps) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    __shared__ float red[8];
    const float *xr = x + (int64_t)blockIdx.x * ldx;
    float *yr = y + (int64_t)blockIdx.x * ldy;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += red[i];
    const float sc = rms_scale(t, n, eps);
    for (int i = threadIdx.x; i < n; i += 256) yr[i] = __fmul_rn(__fmul_rn(xr[i], sc), w[i]);
}

cudaError_t rmsnorm_launch(const float *x, int ldx, const float *w, float *y, int ldy, int m, int n, float eps,
                           cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    launch_pdl(k_rmsnorm, dim3(m), dim3(256), 0, st, x, ldx, w, y, ldy, n, eps);
    return launched(1);
}

// ---------------------------------------------------------------------------
// QK-norm + RoPE + KV append.  One warp per head of one token: warps
// [0, n_head) take the query heads (rotated in place), warps
// [n_head, n_head + n_head_kv) take the key heads and also copy the value
// head; both key and value land in the token's page of the paged cache.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t kv_off(const KVDesc &kv, int layer, int seq, int pos) {
    const int page = kv.page_table[(int64_t)seq * kv.max_pages + (pos / kv.page_size)];
    return (int64_t)layer * kv.layer_stride + ((int64_t)page * kv.page_size + (pos % kv.page_size)) * kv.kvd;
}

__global__ void __launch_bounds__(256) k_rope_append(const RopeDesc r, const KVDesc kv, int layer, TokMeta tm) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    extern __shared__ float sh[];  // 8 warps x head_dim
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hh = blockIdx.y * 8 + warp;
    const int hd = r.head_dim, nh = r.n_head, nkv = r.n_head_kv;
    if (hh >= nh + nkv) return;
    const int pos = tm.pos[t], seq = tm.seq[t];
    const bool isq = hh < nh;
    const int qd = nh * hd, kvd = nkv * hd;
    float *vec = sh + warp * hd;
    const float *src = isq ? r.q + (int64_t)t * qd + hh * hd : r.k + (int64_t)t * kvd + (hh - nh) * hd;
    const float *nw = isq ? r.q_nw : r.k_nw;
    float ss = 0.f;
    for (int d = lane; d < hd; d += 32) {
        const float x = src[d];
        vec[d] = x;
        ss = fmaf(x, x, ss);
    }
    if (nw) {
        ss = warp_sum(ss);
        const float sc = rms_scale(ss, hd, r.eps);
        for (int d = lane; d < hd; d += 32) vec[d] = __fmul_rn(__fmul_rn(vec[d], sc), nw[d]);
    }
    __syncwarp();
    const int half = r.rope_dim / 2;
    const float2 *tab = r.tab + (int64_t)pos * half;
    for (int i = lane; i < half; i += 32) {
        const int ia = r.interleaved ? 2 * i : i, ib = r.interleaved ? 2 * i + 1 : i + half;
        const float a = vec[ia], b = vec[ib];
        const float2 cs = tab[i];
        const float na = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        const float nb = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        vec[ia] = na;
        vec[ib] = nb;
    }
    __syncwarp();
    if (isq) {
        float *dst = r.q + (int64_t)t * qd + hh * hd;
        for (int d = lane; d < hd; d += 32) dst[d] = vec[d];
    } else {
        const int g = hh - nh;
        const int64_t off = kv_off(kv, layer, seq, pos) + (int64_t)g * hd;
        const float *vs = r.v + (int64_t)t * kvd + g * hd;
        for (int d = lane; d < hd; d += 32) {
            kv_store(kv.k, off + d, vec[d], kv.f16);
            kv_store(kv.v, off + d, vs[d], kv.f16);
        }
    }
}

cudaError_t rope_append_launch(const RopeDesc &r, const KVDesc &kv, int layer, TokMeta tm, int ntok,
                               cudaStream_t st) {
    if (ntok <= 0) return cudaSuccess;
    dim3 grid(ntok, (r.n_head + r.n_head_kv + 7) / 8);
    launch_pdl(k_rope_append, grid, dim3(256), 8 * r.head_dim * sizeof(float), st, r, kv, layer, tm);
    return launched(1);
}

// ---------------------------------------------------------------------------
// Sampler.  A candidate is a 64-bit key: the order-preserving image of the
// logit in the high word and (~index) in the low word, so sorting keys in
// descending order ranks by logit and, among equal logits, by lower index --
// the order of greedy() and topK() (sampler.go:19-27, :80-98).  NaN logits
// rank last (the reference's comparisons never select them).
// ---------------------------------------------------------------------------
constexpr int SAMPLE_CHUNK = 2048;
constexpr int TOPK_MAX = 64;

// Bitonic sort of n (power of two) keys in shared memory, descending.
__device__ void bitonic_desc(uint64_t *s, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t a = s[i], b = s[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        s[i] = b;
                        s[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// The TOPK_MAX largest keys of s[0..n) (0 = empty; n a power of two and a
// multiple of 32), in descending order, into s[0..TOPK_MAX) (fewer non-empty
// keys: the rest 0).  A radix select over the keys' high words (the logit's
// order bits; 4 digits of 8 bits, most significant first) finds the high word
// T of the TOPK_MAX-th largest key; the keys whose high word is >= T --
// TOPK_MAX of them unless several logits equal that one -- are gathered into
// `work` (n keys) and sorted, the full key (value, then lower index) deciding.
// hist: 256 words; ctl: 4 ints.  Every thread of the block calls it.
__device__ void block_top64(uint64_t *s, int n, uint64_t *work, uint32_t *hist, int *ctl) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) ctl[0] = 0;
    __syncthreads();
    int local = 0;
    for (int i = tid; i < n; i += nt) local += s[i] != 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if (lane == 0 && local) atomicAdd(&ctl[0], local);
    __syncthreads();
    const int total = ctl[0];
    uint32_t T = 0;
    if (total > TOPK_MAX) {
        uint32_t prefix = 0, pmask = 0;
        int want = TOPK_MAX;  // rank sought among the keys that match the prefix
        for (int dg = 3; dg >= 0; dg--) {
            for (int i = tid; i < 256; i += nt) hist[i] = 0u;
            __syncthreads();
            for (int i = tid; i < n; i += nt) {  // n is a multiple of 32: whole warps iterate together
                const uint64_t k = s[i];
                const uint32_t h = (uint32_t)(k >> 32);
                const uint32_t bin = (k && (h & pmask) == prefix) ? (h >> (8 * dg)) & 255u : 256u;
                const unsigned same = __match_any_sync(0xffffffffu, bin);
                if (bin < 256u && lane == __ffs(same) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(same));
            }
            __syncthreads();
            if (warp == 0) {  // lane l: bins 255 - 8l down to 248 - 8l; ranks counted from the top
                uint32_t c[8], tot = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    c[j] = hist[255 - 8 * lane - j];
                    tot += c[j];
                }
                uint32_t incl = tot;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += x;
                }
                const uint32_t excl = incl - tot, w = (uint32_t)want;
                if (excl < w && w <= incl) {
                    uint32_t acc = excl;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (acc + c[j] >= w) {
                            ctl[1] = 255 - 8 * lane - j;
                            ctl[2] = (int)(w - acc);
                            break;
                        }
                        acc += c[j];
                    }
                }
            }
            __syncthreads();
            prefix |= (uint32_t)ctl[1] << (8 * dg);
            pmask |= 0xFFu << (8 * dg);
            want = ctl[2];
            __syncthreads();
        }
        T = prefix;
    }
    if (tid == 0) ctl[3] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += nt) {
        const uint64_t k = s[i];
        if (k && (uint32_t)(k >> 32) >= T) work[atomicAdd(&ctl[3], 1)] = k;
    }
    __syncthreads();
    const int m = ctl[3];
    int mp = TOPK_MAX;
    while (mp < m) mp <<= 1;
    for (int i = m + tid; i < mp; i += nt) work[i] = 0ull;
    __syncthreads();
    bitonic_desc(work, mp);
    for (int i = tid; i < TOPK_MAX; i += nt) s[i] = work[i];
    __syncthreads();
}

// Per chunk of SAMPLE_CHUNK logits: the top `kk` keys (kk = 1 or 64).
__global__ void __launch_bounds__(256) k_topk_partial(const float *logits, const int32_t *rows, int64_t ld,
                                                      int vocab, int kk, uint64_t *cand, int nchunks) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    __shared__ uint64_t s[SAMPLE_CHUNK];
    const int t = blockIdx.y, c = blockIdx.x;
    const float *lg = logits + (int64_t)(rows ? rows[t] : t) * ld;
    const int base = c * SAMPLE_CHUNK;
    uint64_t *out = cand + ((int64_t)t * nchunks + c) * TOPK_MAX;
    if (kk == 1) {
        uint64_t best = 0;
        for (int i = base + threadIdx.x; i < min(base + SAMPLE_CHUNK, vocab); i += 256) {
            const uint64_t k = logit_key(lg[i], i);
            best = k > best ? k : best;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t x = __shfl_xor_sync(0xffffffffu, best, o);
            best = x > best ? x : best;
        }
        if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint64_t b = 0;
            for (int i = 0; i < 8; i++) b = s[i] > b ? s[i] : b;
            out[0] = b;
        }
        return;
    }
    __shared__ uint64_t work[SAMPLE_CHUNK];
    __shared__ uint32_t hist[256];
    __shared__ int ctl[4];
    for (int i = threadIdx.x; i < SAMPLE_CHUNK; i += 256) {
        const int v = base + i;
        s[i] = v < vocab ? logit_key(lg[v], v) : 0ull;
    }
    __syncthreads();
    block_top64(s, SAMPLE_CHUNK, work, hist, ctl);
    for (int i = threadIdx.x; i < TOPK_MAX; i += 256) out[i] = s[i];
}

// Philox4x32-10 (Salmon et al., SC'11) -> uniform in [0,1) with 53 bits.
__device__ __forceinline__ double philox_uniform(uint64_t seed, uint64_t step) {
    uint32_t c0 = (uint32_t)step, c1 = (uint32_t)(step >> 32), c2 = 0x5A4D4341u, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; r++) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0;
        c1 = n1;
        c2 = n2;
        c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    const uint64_t u = ((uint64_t)c1 << 32) | c0;
    return (double)(u >> 11) * 0x1p-53;
}

// Merge the per-chunk candidates of one token and draw (Sample,
// sampler.go:30-76; the fp64 part runs on one thread in the reference's order).
__global__ void __launch_bounds__(1024) k_sample_final(SampleDesc d, int kk) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    extern __shared__ uint64_t s[];
    const int t = blockIdx.x;
    const int n = d.nchunks * kk;
    int np = 32;  // as the launch sized the shared memory
    while (np < n) np <<= 1;
    const uint64_t *cand = d.cand + (int64_t)t * d.nchunks * TOPK_MAX;
    for (int i = threadIdx.x; i < np; i += blockDim.x)
        s[i] = i < n ? cand[(i / kk) * TOPK_MAX + (i % kk)] : 0ull;
    __syncthreads();
    if (kk > 1) {
        uint64_t *work = s + np;
        uint32_t *hist = reinterpret_cast<uint32_t *>(work + np);
        block_top64(s, np, work, hist, reinterpret_cast<int *>(hist + 256));
    }
    if (threadIdx.x != 0) return;
    const double temp = d.temp ? d.temp[t] : 0.0;
    if (kk == 1 || temp <= 0.0) {
        uint64_t b = s[0];
        if (kk == 1)
            for (int i = 1; i < n; i++) b = s[i] > b ? s[i] : b;
        d.out[t] = key_index(b);
        return;
    }
    int k = TOPK_MAX;
    const int tk = d.top_k ? d.top_k[t] : 0;
    if (tk > 0 && tk < k) k = tk;
    const int cnt = min(k, d.vocab);
    double p[TOPK_MAX];
    const double mx = (double)key_logit(s[0]);
    double sum = 0.0;
    for (int i = 0; i < cnt; i++) {
        p[i] = exp(((double)key_logit(s[i]) - mx) / temp);
        sum += p[i];
    }
    int cut = cnt;
    const double tp = d.top_p ? d.top_p[t] : 0.0;
    if (tp > 0.0 && tp < 1.0) {
        double acc = 0.0;
        for (int i = 0; i < cnt; i++) {
            acc += p[i] / sum;
            if (acc >= tp) {
                cut = i + 1;
                break;
            }
        }
        sum = 0.0;
        for (int i = 0; i < cut; i++) sum += p[i];
    }
    double r = philox_uniform(d.seed ? d.seed[t] : 0, d.step ? d.step[t] : 0) * sum;
    for (int i = 0; i < cut; i++) {
        r -= p[i];
        if (r <= 0.0) {
            d.out[t] = key_index(s[i]);
            return;
        }
    }
    d.out[t] = key_index(s[cut - 1]);
}

cudaError_t sample_launch(const SampleDesc &d, int ntok, bool all_greedy, cudaStream_t st) {
    if (ntok <= 0) return cudaSuccess;
    const int kk = all_greedy ? 1 : TOPK_MAX;
    dim3 g1(d.nchunks, ntok);
    launch_pdl(k_topk_partial, g1, dim3(256), 0, st, d.logits, d.rows, d.ld, d.vocab, kk, d.cand, d.nchunks);
    int np = 32;
    while (np < d.nchunks * kk) np <<= 1;
    // keys, the top-64 gather buffer, histogram and control words
    const size_t smem = kk > 1 ? 2 * (size_t)np * sizeof(uint64_t) + 256 * 4 + 16 : (size_t)np * sizeof(uint64_t);
    static std::atomic<bool> attr[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaFuncSetAttribute(k_sample_final, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr[dev & 63] = true;
    }
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    launch_pdl(k_sample_final, dim3(ntok), dim3(1024), smem, st, d, kk);
    return launched(2);
}

// ---------------------------------------------------------------------------
__global__ void k_swiglu(const float *g, const float *u, float *y, int64_t n) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = g[i];
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, fast_exp(-v)));
        y[i] = __fmul_rn(__fmul_rn(v, sg), u[i]);
    }
}

cudaError_t swiglu_launch(const float *g, const float *u, float *y, int64_t n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    launch_pdl(k_swiglu, dim3((unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8)), dim3(256), 0, st, g, u, y, n);
    return launched(1);
}

__global__ void k_advance(int32_t *tok, int32_t *pos, uint64_t *step, int32_t *out, unsigned long long *amax,
                          int32_t *hist, int hist_ld, int32_t *hist_col, int ntok) {
    pdl_wait();
    if (threadIdx.x == 0) pdl_trigger();
    const int t = threadIdx.x;
    if (t < ntok) {
        const int col = *hist_col;
        int32_t id;
        if (amax) {  // greedy: the lm_head epilogue folded every row into amax[t]
            id = key_index(amax[t]);
            amax[t] = 0ull;
            out[t] = id;
        } else {
            id = out[t];
        }
        tok[t] = id;
        pos[t] += 1;
        step[t] += 1;
        if (hist && col >= 0 && col < hist_ld) hist[(int64_t)t * hist_ld + col] = id;
    }
    __syncthreads();
    if (t == 0) *hist_col += 1;
}

cudaError_t advance_launch(int32_t *tok, int32_t *pos, uint64_t *step, int32_t *out, unsigned long long *amax,
                           int32_t *hist, int hist_ld, int32_t *hist_col, int ntok, cudaStream_t st) {
    if (ntok <= 0 || ntok > 1024) return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(k_advance, dim3(1), dim3(((ntok + 31) / 32) * 32), 0, st, tok, pos, step, out, amax,
                               hist, hist_ld, hist_col, ntok);
    if (e != cudaSuccess) return e;
    return launched(1);
}

}  // namespace acm
