// engine.cu -- host runtime of libacmcuda.so and the C ABI (include/acm.h).
//
// A model holds the GGUF tensors exactly as uploaded, fp32 norm/bias vectors,
// the RoPE cos/sin table, a paged fp32 KV cache shared by `max_seqs`
// sequence slots, and activation buffers for up to TMAX tokens per pass.
// Every pass runs a batch of tokens; each token carries (slot, position), so a
// prefill chunk (one slot, consecutive positions) and a batched decode step
// (many slots, one token each) go through the same kernels.  Decode steps of
// a fixed batch size are captured once into a CUDA graph and replayed; the
// graph reads its token ids and positions from device memory and ends with a
// kernel that advances them, so the token loop can run on the device without
// a host round trip per token.
#include <fcntl.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <memory>
#include <string>
#include <initializer_list>
#include <unordered_map>
#include <vector>

#include "acm.h"
#include "gguf_host.h"
#include "kernels.h"
#include "quant.cuh"

using namespace acm;

std::atomic<unsigned long long> acm::g_kernel_launches{0};

namespace {

constexpr int TMAX = 1024;        // tokens per pass (the reference's prefill chunk, sampler.go:116)
constexpr int PAGE = 64;          // KV positions per page
constexpr int NSPLIT_MAX = 32;
constexpr int PART_TOKSPLIT = 4096;
constexpr int HIST_MAX = 64;      // decode steps per device-side chunk

std::string fmt(const char *f, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}

}  // namespace

struct acm_engine {
    int device = 0;
    int models = 0;       // live models created on this engine
    bool closed = false;  // acm_close called; freed when the last model goes
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    std::string err;
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    void *scratch2 = nullptr;  // operand splits of acm_matmul_dev's tensor-core path
    size_t scratch2_bytes = 0;
    int kv_f16 = 0;            // KV cache type of models created from now on (1: IEEE half)
};

namespace {

struct DevTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;
    int64_t numel = 0;
    size_t nbytes = 0;
    uint8_t *d = nullptr;
    // bf16 hi/lo split of the dequantized weights for the tensor-core GEMM
    // (built on first use; split_state 1 ready, -1 unavailable)
    void *whi = nullptr, *wlo = nullptr;
    TensorMap mhi, mlo;
    int split_state = 0;
    int64_t k() const { return dims.empty() ? numel : (int64_t)dims[0]; }
    int64_t rows() const { return dims.size() < 2 ? 1 : numel / (int64_t)dims[0]; }
};

struct Layer {
    DevTensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *gate = nullptr, *up = nullptr,
              *down = nullptr;
    float *attn_nw = nullptr, *ffn_nw = nullptr, *q_nw = nullptr, *k_nw = nullptr;
    float *q_b = nullptr, *k_b = nullptr, *v_b = nullptr;
};

struct Seq {
    bool open = false;
    int pos = 0;
    std::vector<int> pages;
};

template <typename T>
struct Pinned {
    T *p = nullptr;
    size_t n = 0;
    cudaError_t alloc(size_t cnt) {
        n = cnt;
        return cudaMallocHost(reinterpret_cast<void **>(&p), sizeof(T) * std::max<size_t>(cnt, 1));
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
    }
};

}  // namespace

struct acm_model {
    acm_engine *e = nullptr;
    acm_config c{};
    int max_seqs = 1;
    std::string err;
    std::unordered_map<std::string, DevTensor> tensors;
    std::vector<void *> allocs;
    bool finalized = false;

    DevTensor *embd = nullptr, *out = nullptr;
    float *out_nw = nullptr;
    std::vector<Layer> layers;
    float2 *rope_tab = nullptr;

    // paged KV cache
    int max_pages = 0, n_pages = 0;
    float *kpool = nullptr, *vpool = nullptr;  // fp32, or IEEE half elements when kv_f16
    int64_t layer_stride = 0;                  // elements
    int kv_f16 = 0;
    std::vector<int> free_pages;
    int32_t *d_page_table = nullptr;
    Pinned<int32_t> h_page_table;
    std::vector<Seq> seqs;

    // activations
    int tdec = 8;  // largest decode batch (max(8, max_seqs))
    float *x = nullptr, *h = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *hb = nullptr,
          *hb2 = nullptr, *part = nullptr, *logits = nullptr;

    // tensor-core GEMM: activations split into bf16 hi/lo [T][kmax] and their
    // tensor maps for K = n_embd, q_dim, n_ff
    void *xs_hi = nullptr, *xs_lo = nullptr;
    float *mma_ws = nullptr;  // split-K partial sums [4][T][max(n_embd, q_dim)]
    size_t mma_ws_floats = 0;
    TensorMap xmap_hi[3], xmap_lo[3];
    int xmap_k[3] = {0, 0, 0};
    int mma_state = 0;  // 0 untried, 1 usable, -1 unavailable
    // prefill attention on the tensor cores: split operands, scores, weights
    void *aq_hi = nullptr, *aq_lo = nullptr, *ak_hi = nullptr, *ak_lo = nullptr, *av_hi = nullptr, *av_lo = nullptr,
         *ap_hi = nullptr, *ap_lo = nullptr;
    float *as = nullptr;
    int attn_mma_state = 0;

    // per-token metadata and sampler state (device + pinned staging)
    int32_t *d_tok = nullptr, *d_seq = nullptr, *d_pos = nullptr, *d_out = nullptr, *d_topk = nullptr;
    double *d_temp = nullptr, *d_topp = nullptr;
    uint64_t *d_seed = nullptr, *d_step = nullptr, *d_cand = nullptr;
    int32_t *d_hist = nullptr, *d_hist_col = nullptr;
    unsigned long long *d_amax = nullptr;  // per-token argmax keys (greedy decode)
    int *d_attn_cnt = nullptr;              // decode attention split counters
    int dec_nsplit = 1;                     // chunk capacity of the decode attention
    unsigned long long *d_gtrace = nullptr; // per-CTA timelines of batch-1 GEMV launches (tracing on)
    float *d_dbg = nullptr;                 // per-layer residual of the pass's last token (DebugLayer on)
    bool dbg_layers = false;
    int gtrace_slots = 0, gtrace_on = 0;
    int nchunks = 0;
    Pinned<int32_t> h_tok, h_seq, h_pos, h_out, h_topk, h_hist;
    Pinned<double> h_temp, h_topp;
    Pinned<uint64_t> h_seed, h_step;

    struct Graph {
        cudaGraphExec_t exec = nullptr;
        unsigned long long kernels = 0;  // kernel launches captured in the graph
    };
    std::map<std::pair<int, int>, Graph> graphs;
    Graph gemv_bench;
    cudaEvent_t ev[4] = {};
    double last_prefill_s = 0, last_decode_s = 0;
};

namespace {

int set_err(acm_model *m, int code, const std::string &msg) {
    if (m) m->err = msg;
    return code;
}
int set_eerr(acm_engine *e, int code, const std::string &msg) {
    if (e) e->err = msg;
    return code;
}

#define CK_M(call)                                                                                  \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return set_err(m, e_ == cudaErrorMemoryAllocation ? ACM_ERR_OOM : ACM_ERR_CUDA,         \
                           fmt("%s: %s", #call, cudaGetErrorString(e_)));                           \
    } while (0)
#define CK_E(call)                                                                                  \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            return set_eerr(e, e_ == cudaErrorMemoryAllocation ? ACM_ERR_OOM : ACM_ERR_CUDA,        \
                            fmt("%s: %s", #call, cudaGetErrorString(e_)));                          \
    } while (0)

template <typename T>
cudaError_t dalloc(acm_model *m, T **p, size_t count) {
    void *v = nullptr;
    cudaError_t e = cudaMalloc(&v, sizeof(T) * std::max<size_t>(count, 1));
    if (e == cudaSuccess) {
        m->allocs.push_back(v);
        *p = static_cast<T *>(v);
    }
    return e;
}

// Synchronise the model stream and turn device-side error flags into status.
int sync_check(acm_model *m) {
    cudaError_t e = cudaStreamSynchronize(m->e->stream);
    if (e != cudaSuccess) return set_err(m, ACM_ERR_CUDA, fmt("device error: %s", cudaGetErrorString(e)));
    const int de = read_and_clear_dev_error();
    if (de == DEV_ERR_TIMEOUT) return set_err(m, ACM_ERR_TIMEOUT, "a device-side wait timed out");
    if (de == DEV_ERR_BOUNDS) return set_err(m, ACM_ERR_INVALID, "token id out of range (device check)");
    return ACM_OK;
}

int ensure_pages(acm_model *m, int seq, int upto) {
    Seq &s = m->seqs[seq];
    const int need = (upto + PAGE - 1) / PAGE;
    if (need > m->max_pages) return set_err(m, ACM_ERR_CTX_EXCEEDED, "context length exceeded");
    bool dirty = false;
    while ((int)s.pages.size() < need) {
        if (m->free_pages.empty()) return set_err(m, ACM_ERR_OOM, "KV cache pages exhausted");
        const int pg = m->free_pages.back();
        m->free_pages.pop_back();
        m->h_page_table.p[(size_t)seq * m->max_pages + s.pages.size()] = pg;
        s.pages.push_back(pg);
        dirty = true;
    }
    if (dirty) {
        CK_M(cudaMemcpyAsync(m->d_page_table + (size_t)seq * m->max_pages,
                             m->h_page_table.p + (size_t)seq * m->max_pages, sizeof(int32_t) * m->max_pages,
                             cudaMemcpyHostToDevice, m->e->stream));
    }
    return ACM_OK;
}

int attn_nsplit(acm_model *m, int ntok, int max_pos) {
    const int nkv = m->c.n_head_kv;
    if ((int64_t)ntok * nkv >= 2 * m->e->num_sms) return 1;
    int ns = (2 * m->e->num_sms + ntok * nkv - 1) / (ntok * nkv);
    ns = std::min(ns, NSPLIT_MAX);
    ns = std::min(ns, std::max(1, (max_pos + 1 + 15) / 16));
    ns = std::min(ns, std::max(1, PART_TOKSPLIT / ntok));
    return std::max(ns, 1);
}

// One pass over `ntok` tokens whose ids/slots/positions are already in
// d_tok/d_seq/d_pos.  Logits are produced for tokens [lm_first, lm_first +
// lm_count) into their slots' rows of m->logits.  Enqueues only (capturable).
// ---- tensor-core GEMM plumbing ----
// The split cache of a weight tensor (exact dequant -> bf16 hi/lo), built on
// first use.  False when the tensor cannot take the tensor-core path.
bool ensure_split(acm_model *m, DevTensor *t) {
    if (t->split_state) return t->split_state > 0;
    t->split_state = -1;
    const int64_t n = t->rows(), k = t->k();
    if (k % 64 || n <= 0) return false;
    if (dalloc(m, reinterpret_cast<uint16_t **>(&t->whi), (size_t)rows64(n) * k) != cudaSuccess ||
        dalloc(m, reinterpret_cast<uint16_t **>(&t->wlo), (size_t)rows64(n) * k) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (split_weight_launch((int)t->type, t->d, n, (int)k, t->whi, t->wlo, m->e->stream) != cudaSuccess) return false;
    if (!bf16_map(&t->mhi, t->whi, n, k) || !bf16_map(&t->mlo, t->wlo, n, k)) return false;
    t->split_state = 1;
    return true;
}

// Activation split buffers and their maps (once per model).
bool mma_ready(acm_model *m) {
    if (m->mma_state) return m->mma_state > 0;
    m->mma_state = -1;
    if (!mma_available()) return false;
    const acm_config &c = m->c;
    const int qd = c.n_head * c.head_dim;
    const int ks[3] = {c.n_embd, qd, c.n_ff};
    const int kmax = std::max(ks[0], std::max(ks[1], ks[2]));
    const size_t T = (size_t)rows64(std::max(TMAX, m->tdec));
    if (dalloc(m, reinterpret_cast<uint16_t **>(&m->xs_hi), T * kmax) != cudaSuccess ||
        dalloc(m, reinterpret_cast<uint16_t **>(&m->xs_lo), T * kmax) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    m->mma_ws_floats = 4 * T * (size_t)std::max(c.n_embd, qd);
    if (dalloc(m, &m->mma_ws, m->mma_ws_floats) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    for (int i = 0; i < 3; i++) {
        if (ks[i] % 64) return false;
        m->xmap_k[i] = ks[i];
        if (!bf16_map(&m->xmap_hi[i], m->xs_hi, (int64_t)T, ks[i]) ||
            !bf16_map(&m->xmap_lo[i], m->xs_lo, (int64_t)T, ks[i]))
            return false;
    }
    m->mma_state = 1;
    return true;
}

// Split fp32 activations x [ntok][k] into the model's bf16 buffers and
// return the maps for this K (nullptr when the tensor-core path is off).
// norm_w: RMSNorm the rows first (one fused launch).
int mma_split_x(acm_model *m, const float *x, int ldx, int ntok, int k, const TensorMap **hi, const TensorMap **lo,
                const float *norm_w = nullptr, float eps = 0.f) {
    int i = 0;
    while (i < 3 && m->xmap_k[i] != k) i++;
    if (i == 3) return set_err(m, ACM_ERR_INVALID, "no activation map for this K");
    if (norm_w) CK_M(split_act_norm_launch(x, ldx, ntok, k, norm_w, eps, m->xs_hi, m->xs_lo, m->e->stream));
    else CK_M(split_act_launch(x, ldx, ntok, k, m->xs_hi, m->xs_lo, m->e->stream));
    *hi = &m->xmap_hi[i];
    *lo = &m->xmap_lo[i];
    return ACM_OK;
}

// Buffers of the tensor-core prefill attention, for chunks of up to TMAX
// tokens and contexts of up to max_ctx positions (limited to 8192: the score
// matrix is [kv heads][G * TMAX][max_ctx] fp32).
bool attn_mma_ready(acm_model *m) {
    if (m->attn_mma_state) return m->attn_mma_state > 0;
    m->attn_mma_state = -1;
    const acm_config &c = m->c;
    const char *env = getenv("ACM_ATTN_MMA");
    if ((env && env[0] == '0') || !mma_ready(m)) return false;
    const int hd = c.head_dim, nkv = c.n_head_kv, G = c.n_head / c.n_head_kv;
    if (hd % 64 || hd > 128 || c.max_ctx > 8192 || PAGE % 64) return false;
    const size_t rq = (size_t)rows64((int64_t)G * TMAX), lp = (size_t)rows64(c.max_ctx);
    const size_t nq = nkv * rq * hd, nk = nkv * lp * hd, np = nkv * rq * lp;
    auto al16 = [&](void **p, size_t n) {
        return dalloc(m, reinterpret_cast<uint16_t **>(p), n) == cudaSuccess;
    };
    if (!al16(&m->aq_hi, nq) || !al16(&m->aq_lo, nq) || !al16(&m->ak_hi, nk) || !al16(&m->ak_lo, nk) ||
        !al16(&m->av_hi, nk) || !al16(&m->av_lo, nk) || !al16(&m->ap_hi, np) || !al16(&m->ap_lo, np) ||
        dalloc(m, &m->as, (size_t)nkv * G * TMAX * lp) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    m->attn_mma_state = 1;
    return true;
}

// Prefill attention of one layer on the tensor cores: the chunk's tokens are
// consecutive positions pos0 .. pos0 + ntok - 1 of sequence `seq` (keys and
// values already appended).  S = Q.K^T and O = P.V as batched split-bf16
// GEMMs over the kv heads, the reference's softmax between them.
int attention_prefill_mma(acm_model *m, int layer, int seq, int pos0, int ntok) {
    const acm_config &c = m->c;
    cudaStream_t st = m->e->stream;
    const int hd = c.head_dim, nkv = c.n_head_kv, G = c.n_head / c.n_head_kv, nh = c.n_head;
    const int L = pos0 + ntok, Lp = (int)rows64(L), rows = G * ntok;
    const int64_t rq = rows64(rows);
    AttnMmaOps o{};
    o.q = m->q;
    o.kc = m->kpool;
    o.vc = m->vpool;
    o.kv_f16 = m->kv_f16;
    o.page_row = m->d_page_table + (int64_t)seq * m->max_pages;
    o.layer_off = (int64_t)layer * m->layer_stride;
    o.page_size = PAGE;
    o.kvd = nkv * hd;
    o.ntok = ntok;
    o.L = L;
    o.Lp = Lp;
    o.G = G;
    o.nh = nh;
    o.hd = hd;
    o.nkv = nkv;
    o.pos0 = pos0;
    o.rq = rq;
    o.scale = 1.0f / (float)sqrt((double)hd);
    o.qh = m->aq_hi; o.ql = m->aq_lo; o.kh = m->ak_hi; o.kl = m->ak_lo;
    o.vh = m->av_hi; o.vl = m->av_lo; o.ph = m->ap_hi; o.pl = m->ap_lo;
    o.S = m->as;
    CK_M(attn_split_launch(o, st));
    TensorMap kh, kl, qh, ql, vh, vl, ph, pl;
    if (!bf16_map(&kh, m->ak_hi, (int64_t)nkv * Lp, hd) || !bf16_map(&kl, m->ak_lo, (int64_t)nkv * Lp, hd) ||
        !bf16_map(&qh, m->aq_hi, nkv * rq, hd) || !bf16_map(&ql, m->aq_lo, nkv * rq, hd) ||
        !bf16_map(&vh, m->av_hi, (int64_t)nkv * hd, Lp) || !bf16_map(&vl, m->av_lo, (int64_t)nkv * hd, Lp) ||
        !bf16_map(&ph, m->ap_hi, nkv * rq, Lp) || !bf16_map(&pl, m->ap_lo, nkv * rq, Lp))
        return set_err(m, ACM_ERR_CUDA, "tensor map encoding failed");
    // S[g][r][p] = Qs[g][r] . Ks[g][p]
    MmaGemmSeg sq{&kh, &kl, nullptr, nullptr, L, EPI_STORE, m->as, Lp, nullptr, nullptr};
    MmaBatch bq;
    bq.n = nkv;
    bq.a_stride = (Lp / 64) * (hd / 64) * 64;
    bq.b_stride = (int)(rq / 64) * (hd / 64) * 64;
    bq.rbatch = rows;
    bq.causal = 1;  // key tiles above the diagonal: never read by the softmax
    bq.cntok = ntok;
    bq.cpos0 = pos0;
    CK_M(mma_gemm_batched_launch(&sq, 1, &qh, &ql, rows, hd, bq, st));
    CK_M(attn_softmax_launch(o, st));
    // att[t][(g*G + h)*hd + d] = P[g][h*ntok + t] . Vt[g][d]
    MmaGemmSeg sv{&vh, &vl, nullptr, nullptr, hd, EPI_STORE, m->att, hd, nullptr, nullptr};
    MmaBatch bv;
    bv.n = nkv;
    bv.a_stride = (hd / 64) * (Lp / 64) * 64;
    bv.b_stride = (int)(rq / 64) * (Lp / 64) * 64;
    bv.rmod = ntok;
    bv.rmul = nh;
    bv.rdiv = 1;
    bv.rbatch = G;
    bv.causal = 2;  // P is zero past each token's position
    bv.cntok = ntok;
    bv.cpos0 = pos0;
    CK_M(mma_gemm_batched_launch(&sv, 1, &ph, &pl, rows, Lp, bv, st));
    return ACM_OK;
}

// Whether the in-kernel dequant tensor-core GEMM (k_mma_dq.cu) serves these
// weights: every one a quantized GGUF type (one type, or Q4_K with Q6_K) and
// K a multiple of 256.  No split cache is built for them.
bool use_mma_dq(acm_model *m, std::initializer_list<DevTensor *> ts, int64_t k) {
    if (k % 256 || !mma_ready(m)) return false;
    int ta = -1, tb = -1;
    for (DevTensor *t : ts) {
        if (!t) continue;
        const int ty = (int)t->type;
        if (!dq_type(ty)) return false;
        if (ta < 0) ta = ty;
        else if (ty != ta) tb = ty;
    }
    if (tb >= 0 && !((ta == T_Q4_K && tb == T_Q6_K) || (ta == T_Q6_K && tb == T_Q4_K))) return false;
    for (DevTensor *t : ts)
        if (t && (int)t->type != ta && (int)t->type != tb) return false;
    return true;
}

// Launch a tensor-core GEMM: weights dequantized in the kernel when the
// segments carry GGUF rows (wtype >= 0), else from their split caches.
cudaError_t mma_run(const MmaGemmSeg *segs, int nseg, const TensorMap *xh, const TensorMap *xl, int m, int k,
                    cudaStream_t st, float *ws = nullptr, size_t wsf = 0, int *defer_ks = nullptr) {
    if (defer_ks) *defer_ks = 0;
    if (segs[0].wtype >= 0) return mma_dq_launch(segs, nseg, xh, xl, m, k, st, ws, wsf, defer_ks);
    return mma_gemm_launch(segs, nseg, xh, xl, m, k, st, ws, wsf);
}

// Whether the tensor-core GEMM serves a GEMM of these weights (batches of
// more than 8 tokens; exact split caches built here).
bool use_mma(acm_model *m, std::initializer_list<DevTensor *> ts) {
    if (!mma_ready(m)) return false;
    for (DevTensor *t : ts)
        if (t && !ensure_split(m, t)) return false;
    return true;
}

// `decode`: every token belongs to a different sequence (one new token each),
// which enables the fused decode attention; `amax`: fold the lm_head rows
// into per-token argmax keys (greedy sampling) instead of only storing logits.
int forward_pass(acm_model *m, int ntok, int max_pos, int lm_first, int lm_count, bool decode = false,
                 unsigned long long *amax = nullptr) {
    const acm_config &c = m->c;
    cudaStream_t st = m->e->stream;
    const int E = c.n_embd, hd = c.head_dim, qd = c.n_head * hd, kvd = c.n_head_kv * hd, F = c.n_ff;
    const int S = m->e->num_sms;
    const float eps = c.rms_eps;
    CK_M(dequant_launch(m->embd->type, m->embd->d, E, ntok, m->d_tok, m->embd->rows(), m->x, E, st));
    KVDesc kv{m->kpool, m->vpool, m->d_page_table, m->max_pages, PAGE, m->layer_stride, kvd, m->kv_f16};
    TokMeta tm{m->d_seq, m->d_pos};
    const float scale = 1.0f / (float)sqrt((double)hd);
    const int nsplit = attn_nsplit(m, ntok, max_pos);
    for (int l = 0; l < c.n_layers; l++) {
        const Layer &L = m->layers[l];
        // q, k, v (+ bias) from RMSNorm(x)
        const bool gv = gemv_supported(L.q->type, E, ntok) && gemv_supported(L.k->type, E, ntok) &&
                        gemv_supported(L.v->type, E, ntok);
        if (gv) {
            GemvSegDesc sg[3] = {{L.q->d, nullptr, (int)L.q->type, qd, EPI_STORE, m->q, qd, L.q_b, nullptr},
                                 {L.k->d, nullptr, (int)L.k->type, kvd, EPI_STORE, m->k, kvd, L.k_b, nullptr},
                                 {L.v->d, nullptr, (int)L.v->type, kvd, EPI_STORE, m->v, kvd, L.v_b, nullptr}};
            // each matvec pulls the next one's weights into L2 (decode: weights
            // > L2 per token, so without this the next kernel's first stages
            // pay a DRAM round trip on the critical path)
            const L2Range pf_o[1] = {{L.o->d, (int64_t)L.o->nbytes}};
            CK_M(gemv_launch(sg, 3, m->x, E, E, ntok, L.attn_nw, eps, S, st, pf_o, 1));
        } else if (use_mma_dq(m, {L.q, L.k, L.v}, E) || use_mma(m, {L.q, L.k, L.v})) {
            const bool dq = use_mma_dq(m, {L.q, L.k, L.v}, E);
            const TensorMap *xh, *xl;
            if (int rc = mma_split_x(m, m->x, E, ntok, E, &xh, &xl, L.attn_nw, eps)) return rc;
            MmaGemmSeg sg[3] = {{&L.q->mhi, &L.q->mlo, nullptr, nullptr, qd, EPI_STORE, m->q, qd, L.q_b, nullptr,
                                 L.q->d, nullptr, dq ? (int)L.q->type : -1},
                                {&L.k->mhi, &L.k->mlo, nullptr, nullptr, kvd, EPI_STORE, m->k, kvd, L.k_b, nullptr,
                                 L.k->d, nullptr, dq ? (int)L.k->type : -1},
                                {&L.v->mhi, &L.v->mlo, nullptr, nullptr, kvd, EPI_STORE, m->v, kvd, L.v_b, nullptr,
                                 L.v->d, nullptr, dq ? (int)L.v->type : -1}};
            CK_M(mma_run(sg, 3, xh, xl, ntok, E, st));
        } else {
            CK_M(rmsnorm_launch(m->x, E, L.attn_nw, m->h, E, ntok, E, eps, st));
            CK_M(gemm_launch({L.q->d, nullptr, (int)L.q->type, qd, E, ntok, m->h, E, m->q, qd, EPI_STORE, L.q_b, nullptr}, st));
            CK_M(gemm_launch({L.k->d, nullptr, (int)L.k->type, kvd, E, ntok, m->h, E, m->k, kvd, EPI_STORE, L.k_b, nullptr}, st));
            CK_M(gemm_launch({L.v->d, nullptr, (int)L.v->type, kvd, E, ntok, m->h, E, m->v, kvd, EPI_STORE, L.v_b, nullptr}, st));
        }
        RopeDesc rd{m->q, m->k, m->v, L.q_nw, L.k_nw, m->rope_tab, c.n_head, c.n_head_kv, hd, c.rope_dim,
                    c.rope_interleaved, eps};
        if (decode) {
            AttnDesc ad{m->q, m->att, c.n_head, c.n_head_kv, hd, scale, m->part, m->dec_nsplit, m->d_attn_cnt,
                        m->e->num_sms};
            CK_M(attention_decode_launch(rd, ad, kv, l, tm, ntok, max_pos, st));
        } else {
            CK_M(rope_append_launch(rd, kv, l, tm, ntok, st));
            // a prefill chunk: consecutive positions of one sequence
            if (ntok > 8 && attn_mma_ready(m)) {
                if (int rc = attention_prefill_mma(m, l, m->h_seq.p[0], m->h_pos.p[0], ntok)) return rc;
            } else {
                AttnDesc ad{m->q, m->att, c.n_head, c.n_head_kv, hd, scale, m->part, nsplit, nullptr};
                CK_M(attention_prefill_launch(ad, kv, l, tm, ntok, st));
            }
        }
        // the gate/up GEMM on the tensor cores (its RMSNorm fused into the
        // activations' split, and then the o GEMM's split-K reduce too)
        const bool pair = L.gate->type == L.up->type;
        const bool gu_mma = !(gemv_supported(L.gate->type, E, ntok) && gemv_supported(L.up->type, E, ntok)) &&
                            F % 64 == 0 && ((pair && use_mma_dq(m, {L.gate, L.up}, E)) || use_mma(m, {L.gate, L.up}));
        int o_ks = 0;  // split-K slices of the o GEMM left for the gate/up staging to reduce
        // x += Wo att
        if (gemv_supported(L.o->type, qd, ntok)) {
            GemvSegDesc so{L.o->d, nullptr, (int)L.o->type, E, EPI_ADD, m->x, E, nullptr, nullptr};
            const L2Range pf_f[2] = {{L.gate->d, (int64_t)L.gate->nbytes}, {L.up->d, (int64_t)L.up->nbytes}};
            CK_M(gemv_launch(&so, 1, m->att, qd, qd, ntok, nullptr, eps, S, st, pf_f, 2));
        } else if (use_mma_dq(m, {L.o}, qd) || use_mma(m, {L.o})) {
            const bool dq = use_mma_dq(m, {L.o}, qd);
            const TensorMap *xh, *xl;
            if (int rc = mma_split_x(m, m->att, qd, ntok, qd, &xh, &xl)) return rc;
            MmaGemmSeg so{&L.o->mhi, &L.o->mlo, nullptr, nullptr, E, EPI_ADD, m->x, E, nullptr, nullptr,
                          L.o->d, nullptr, dq ? (int)L.o->type : -1};
            CK_M(mma_run(&so, 1, xh, xl, ntok, qd, st, m->mma_ws, m->mma_ws_floats, gu_mma ? &o_ks : nullptr));
        } else {
            CK_M(gemm_launch({L.o->d, nullptr, (int)L.o->type, E, qd, ntok, m->att, qd, m->x, E, EPI_ADD, nullptr, nullptr}, st));
        }
        // hb = silu(Wg h) * (Wu h), h = RMSNorm(x)
        if (!gu_mma && gemv_supported(L.gate->type, E, ntok) && gemv_supported(L.up->type, E, ntok)) {
            if (pair) {
                GemvSegDesc sf{L.gate->d, L.up->d, (int)L.gate->type, F, EPI_SWIGLU, m->hb, F, nullptr, nullptr};
                const L2Range pf_d[1] = {{L.down->d, (int64_t)L.down->nbytes}};
                CK_M(gemv_launch(&sf, 1, m->x, E, E, ntok, L.ffn_nw, eps, S, st, pf_d, 1));
            } else {
                GemvSegDesc sf[2] = {{L.gate->d, nullptr, (int)L.gate->type, F, EPI_STORE, m->hb, F, nullptr, nullptr},
                                     {L.up->d, nullptr, (int)L.up->type, F, EPI_STORE, m->hb2, F, nullptr, nullptr}};
                CK_M(gemv_launch(sf, 2, m->x, E, E, ntok, L.ffn_nw, eps, S, st));
                CK_M(swiglu_launch(m->hb, m->hb2, m->hb, (int64_t)ntok * F, st));
            }
        } else if (gu_mma) {
            // one paired launch: both projections dequantized in the kernel
            // (same type), else both split to bf16 whatever their types
            const bool dq = pair && use_mma_dq(m, {L.gate, L.up}, E);
            const TensorMap *xh, *xl;
            if (o_ks > 0) {
                // x += the o GEMM's partial sums, RMSNorm, split: one launch
                int i = 0;
                while (i < 3 && m->xmap_k[i] != E) i++;
                if (i == 3) return set_err(m, ACM_ERR_INVALID, "no activation map for this K");
                CK_M(split_act_reduce_norm_launch(m->mma_ws, o_ks, ntok, m->x, E, L.ffn_nw, eps, m->xs_hi, m->xs_lo,
                                                  st));
                xh = &m->xmap_hi[i];
                xl = &m->xmap_lo[i];
            } else if (int rc = mma_split_x(m, m->x, E, ntok, E, &xh, &xl, L.ffn_nw, eps)) {
                return rc;
            }
            MmaGemmSeg sf{&L.gate->mhi, &L.gate->mlo, &L.up->mhi, &L.up->mlo, F, EPI_SWIGLU, m->hb, F, nullptr, nullptr,
                          L.gate->d, L.up->d, dq ? (int)L.gate->type : -1};
            CK_M(mma_run(&sf, 1, xh, xl, ntok, E, st));
        } else {
            CK_M(rmsnorm_launch(m->x, E, L.ffn_nw, m->h, E, ntok, E, eps, st));
            if (pair) {
                CK_M(gemm_launch({L.gate->d, L.up->d, (int)L.gate->type, F, E, ntok, m->h, E, m->hb, F, EPI_SWIGLU, nullptr, nullptr}, st));
            } else {
                CK_M(gemm_launch({L.gate->d, nullptr, (int)L.gate->type, F, E, ntok, m->h, E, m->hb, F, EPI_STORE, nullptr, nullptr}, st));
                CK_M(gemm_launch({L.up->d, nullptr, (int)L.up->type, F, E, ntok, m->h, E, m->hb2, F, EPI_STORE, nullptr, nullptr}, st));
                CK_M(swiglu_launch(m->hb, m->hb2, m->hb, (int64_t)ntok * F, st));
            }
        }
        // x += Wd hb
        if (gemv_supported(L.down->type, F, ntok)) {
            GemvSegDesc sd{L.down->d, nullptr, (int)L.down->type, E, EPI_ADD, m->x, E, nullptr, nullptr};
            L2Range pf_n[3] = {};
            int npf = 0;
            if (l + 1 < c.n_layers) {
                const Layer &N = m->layers[l + 1];
                pf_n[0] = {N.q->d, (int64_t)N.q->nbytes};
                pf_n[1] = {N.k->d, (int64_t)N.k->nbytes};
                pf_n[2] = {N.v->d, (int64_t)N.v->nbytes};
                npf = 3;
            }
            CK_M(gemv_launch(&sd, 1, m->hb, F, F, ntok, nullptr, eps, S, st, pf_n, npf));
        } else if (use_mma_dq(m, {L.down}, F) || use_mma(m, {L.down})) {
            const bool dq = use_mma_dq(m, {L.down}, F);
            const TensorMap *xh, *xl;
            if (int rc = mma_split_x(m, m->hb, F, ntok, F, &xh, &xl)) return rc;
            MmaGemmSeg sd{&L.down->mhi, &L.down->mlo, nullptr, nullptr, E, EPI_ADD, m->x, E, nullptr, nullptr,
                          L.down->d, nullptr, dq ? (int)L.down->type : -1};
            CK_M(mma_run(&sd, 1, xh, xl, ntok, F, st, m->mma_ws, m->mma_ws_floats));
        } else {
            CK_M(gemm_launch({L.down->d, nullptr, (int)L.down->type, E, F, ntok, m->hb, F, m->x, E, EPI_ADD, nullptr, nullptr}, st));
        }
        if (m->dbg_layers)  // DebugLayer (model.go:427-429): the residual after layer l, last token
            CK_M(cudaMemcpyAsync(m->d_dbg + (size_t)l * E, m->x + (size_t)(ntok - 1) * E, sizeof(float) * E,
                                 cudaMemcpyDeviceToDevice, st));
    }
    if (lm_count > 0) {
        // final RMSNorm + lm_head for the requested tokens, into their slots' logits rows
        const float *xin = m->x + (size_t)lm_first * E;
        const int V = (int)m->out->rows();
        if (gemv_supported(m->out->type, E, lm_count)) {
            GemvSegDesc so{m->out->d, nullptr, (int)m->out->type, V, EPI_STORE, m->logits, c.vocab, nullptr,
                           m->d_seq + lm_first, amax};
            CK_M(gemv_launch(&so, 1, xin, E, E, lm_count, m->out_nw, eps, S, st));
        } else if (use_mma_dq(m, {m->out}, E) || use_mma(m, {m->out})) {
            const bool dq = use_mma_dq(m, {m->out}, E);
            CK_M(rmsnorm_launch(xin, E, m->out_nw, m->h, E, lm_count, E, eps, st));
            const TensorMap *xh, *xl;
            if (int rc = mma_split_x(m, m->h, E, lm_count, E, &xh, &xl)) return rc;
            MmaGemmSeg sl{&m->out->mhi, &m->out->mlo, nullptr, nullptr, V, EPI_STORE, m->logits, c.vocab, nullptr,
                          m->d_seq + lm_first, m->out->d, nullptr, dq ? (int)m->out->type : -1};
            CK_M(mma_run(&sl, 1, xh, xl, lm_count, E, st));
        } else {
            CK_M(rmsnorm_launch(xin, E, m->out_nw, m->h, E, lm_count, E, eps, st));
            CK_M(gemm_launch({m->out->d, nullptr, (int)m->out->type, V, E, lm_count, m->h, E, m->logits, c.vocab,
                              EPI_STORE, nullptr, m->d_seq + lm_first}, st));
        }
    }
    return ACM_OK;
}

int sample_pass(acm_model *m, int ntok, bool greedy) {
    SampleDesc sd{m->logits, m->d_seq, m->c.vocab, m->c.vocab, m->d_temp, m->d_topk, m->d_topp, m->d_seed,
                  m->d_step, m->d_out, m->d_cand, m->nchunks};
    CK_M(sample_launch(sd, ntok, greedy, m->e->stream));
    return ACM_OK;
}

// Upload ids/slots/positions of a token batch from the pinned staging.
int upload_meta(acm_model *m, int ntok) {
    cudaStream_t st = m->e->stream;
    CK_M(cudaMemcpyAsync(m->d_tok, m->h_tok.p, sizeof(int32_t) * ntok, cudaMemcpyHostToDevice, st));
    CK_M(cudaMemcpyAsync(m->d_seq, m->h_seq.p, sizeof(int32_t) * ntok, cudaMemcpyHostToDevice, st));
    CK_M(cudaMemcpyAsync(m->d_pos, m->h_pos.p, sizeof(int32_t) * ntok, cudaMemcpyHostToDevice, st));
    return ACM_OK;
}

int upload_sampler(acm_model *m, int ntok) {
    cudaStream_t st = m->e->stream;
    CK_M(cudaMemcpyAsync(m->d_temp, m->h_temp.p, sizeof(double) * ntok, cudaMemcpyHostToDevice, st));
    CK_M(cudaMemcpyAsync(m->d_topp, m->h_topp.p, sizeof(double) * ntok, cudaMemcpyHostToDevice, st));
    CK_M(cudaMemcpyAsync(m->d_topk, m->h_topk.p, sizeof(int32_t) * ntok, cudaMemcpyHostToDevice, st));
    CK_M(cudaMemcpyAsync(m->d_seed, m->h_seed.p, sizeof(uint64_t) * ntok, cudaMemcpyHostToDevice, st));
    CK_M(cudaMemcpyAsync(m->d_step, m->h_step.p, sizeof(uint64_t) * ntok, cudaMemcpyHostToDevice, st));
    return ACM_OK;
}

// A decode step for `ntok` tokens: forward + sample + advance, replayed from
// a CUDA graph captured on first use for this (batch size, greedy) pair.
int decode_graph_launch(acm_model *m, int ntok, bool greedy) {
    const auto key = std::make_pair(ntok, greedy ? 1 : 0);
    auto it = m->graphs.find(key);
    cudaStream_t st = m->e->stream;
    // greedy batches whose lm_head runs as a matvec fold the argmax into its
    // epilogue; larger batches (GEMM lm_head) take the greedy sampler pass
    const bool fold = greedy && gemv_supported((int)m->out->type, m->c.n_embd, ntok);
    unsigned long long *amax = fold ? m->d_amax : nullptr;
    if (it == m->graphs.end()) {
        // warm-up run outside capture (first launches set kernel attributes)
        int rc = forward_pass(m, ntok, m->c.max_ctx - 1, 0, ntok, true, amax);
        if (rc) return rc;
        if (!fold && (rc = sample_pass(m, ntok, greedy))) return rc;
        CK_M(cudaMemsetAsync(m->d_amax, 0, sizeof(unsigned long long) * ntok, st));
        if ((rc = sync_check(m))) return rc;
        cudaGraph_t g = nullptr;
        const unsigned long long before = g_kernel_launches.load();
        CK_M(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        // greedy: the lm_head epilogue keeps the argmax and advance reads it;
        // otherwise the top-k sampler runs between them
        rc = forward_pass(m, ntok, m->c.max_ctx - 1, 0, ntok, true, amax);
        if (!rc && !fold) rc = sample_pass(m, ntok, greedy);
        cudaError_t ae = advance_launch(m->d_tok, m->d_pos, m->d_step, m->d_out, amax,
                                        m->d_hist, HIST_MAX, m->d_hist_col, ntok, st);
        cudaError_t ce = cudaStreamEndCapture(st, &g);
        const unsigned long long captured = g_kernel_launches.load() - before;
        g_kernel_launches -= captured;  // capturing is not executing
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ae != cudaSuccess || ce != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return set_err(m, ACM_ERR_CUDA, fmt("graph capture failed: %s", cudaGetErrorString(ae ? ae : ce)));
        }
        cudaGraphExec_t ex = nullptr;
        cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return set_err(m, ACM_ERR_CUDA, fmt("graph instantiate: %s", cudaGetErrorString(ie)));
        acm_model::Graph gr;
        gr.exec = ex;
        gr.kernels = captured;
        it = m->graphs.emplace(key, gr).first;
        // the warm-up pass above advanced nothing on the device; restore inputs
        int rc2 = upload_meta(m, ntok);
        if (rc2) return rc2;
        if ((rc2 = upload_sampler(m, ntok))) return rc2;
    }
    CK_M(cudaGraphLaunch(it->second.exec, st));
    g_kernel_launches += it->second.kernels;
    return ACM_OK;
}

int check_seq(acm_model *m, int seq) {
    if (!m || !m->finalized) return set_err(m, ACM_ERR_INVALID, "model not finalized");
    if (seq < 0 || seq >= m->max_seqs || !m->seqs[seq].open) return set_err(m, ACM_ERR_NO_SEQ, fmt("sequence %d is not open", seq));
    return ACM_OK;
}

void fill_sampler(acm_model *m, int t, const acm_sampler *s, uint64_t step) {
    m->h_temp.p[t] = s ? s->temp : 0.0;
    m->h_topk.p[t] = s ? s->top_k : 0;
    m->h_topp.p[t] = s ? s->top_p : 0.0;
    m->h_seed.p[t] = s ? s->seed : 0;
    m->h_step.p[t] = step;
}

double ev_seconds(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    return ms * 1e-3;
}

// Forward over n tokens of one sequence (chunks of TMAX), logits of the last
// token into the slot's row.  Caller has validated the context length.
int forward_seq(acm_model *m, int seq, const int32_t *toks, int n) {
    Seq &s = m->seqs[seq];
    int rc;
    if ((rc = ensure_pages(m, seq, s.pos + n))) return rc;
    for (int i = 0; i < n; i += TMAX) {
        const int cnt = std::min(TMAX, n - i);
        if (i > 0 && (rc = sync_check(m))) return rc;  // staging reuse
        for (int j = 0; j < cnt; j++) {
            m->h_tok.p[j] = toks[i + j];
            m->h_seq.p[j] = seq;
            m->h_pos.p[j] = s.pos + i + j;
        }
        if ((rc = upload_meta(m, cnt))) return rc;
        const bool last = i + cnt == n;
        if ((rc = forward_pass(m, cnt, s.pos + i + cnt - 1, cnt - 1, last ? 1 : 0, cnt == 1))) return rc;
    }
    s.pos += n;
    return ACM_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

ACM_API const char *acm_version(void) { return "acm-b200 0.1 (sm_100a)"; }

ACM_API int acm_open(int device, acm_engine **out) {
    if (!out) return ACM_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return ACM_ERR_CUDA;
    auto *e = new acm_engine();
    e->device = device;
    cudaError_t ce = cudaSetDevice(device);
    if (ce == cudaSuccess) ce = cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (ce != cudaSuccess) {
        delete e;
        return ACM_ERR_CUDA;
    }
    *out = e;
    return ACM_OK;
}

static void engine_free(acm_engine *e) {
    cudaSetDevice(e->device);
    if (e->scratch) cudaFree(e->scratch);
    if (e->scratch2) cudaFree(e->scratch2);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

ACM_API int acm_close(acm_engine *e) {
    if (!e) return ACM_ERR_INVALID;
    if (e->models > 0) {  // models still alive: free with the last of them
        e->closed = true;
        return ACM_OK;
    }
    engine_free(e);
    return ACM_OK;
}

ACM_API const char *acm_engine_error(acm_engine *e) { return e ? e->err.c_str() : "null engine"; }
ACM_API void *acm_engine_stream(acm_engine *e) { return e ? (void *)e->stream : nullptr; }
ACM_API int acm_engine_sync(acm_engine *e) {
    if (!e) return ACM_ERR_INVALID;
    cudaSetDevice(e->device);
    CK_E(cudaStreamSynchronize(e->stream));
    return ACM_OK;
}

ACM_API int acm_engine_set_kv_f16(acm_engine *e, int32_t enable) {
    if (!e) return ACM_ERR_INVALID;
    e->kv_f16 = enable ? 1 : 0;
    return ACM_OK;
}

ACM_API int acm_engine_set_wait_limit(acm_engine *e, int64_t polls) {
    if (!e) return ACM_ERR_INVALID;
    cudaSetDevice(e->device);
    CK_E(cudaStreamSynchronize(e->stream));
    const uint32_t v = polls < 0 ? WAIT_LIMIT_DEFAULT : (uint32_t)std::min<int64_t>(polls, 0xFFFFFFFFll);
    CK_E(set_wait_limit(v));
    return ACM_OK;
}

ACM_API int acm_model_create(acm_engine *e, const acm_config *cfg, int32_t max_seqs, acm_model **out) {
    if (!e || !cfg || !out || max_seqs < 1 || max_seqs > 1024) return ACM_ERR_INVALID;
    *out = nullptr;
    const acm_config &c = *cfg;
    if (c.n_layers <= 0 || c.n_embd <= 0 || c.n_head <= 0 || c.n_head_kv <= 0 || c.head_dim <= 0 || c.n_ff <= 0 ||
        c.vocab <= 0 || c.max_ctx <= 0)
        return set_eerr(e, ACM_ERR_INVALID, "invalid model configuration");
    if (c.arch < 0 || c.arch > 2) return set_eerr(e, ACM_ERR_UNSUPPORTED_ARCH, "unsupported architecture");
    auto *m = new acm_model();
    m->e = e;
    e->models++;
    m->c = c;
    m->max_seqs = max_seqs;
    m->kv_f16 = e->kv_f16;
    *out = m;
    return ACM_OK;
}

}  // extern "C"

namespace {
// Shape checks of one GGUF tensor (the part of acm_model_add_tensor before
// any device work); fills t.
int tensor_meta(acm_model *m, const char *name, uint32_t ggml_type, const uint64_t *dims, int32_t ndims,
                size_t nbytes, DevTensor &t) {
    if (m->finalized) return set_err(m, ACM_ERR_INVALID, "model already finalized");
    if (!type_ok((int)ggml_type))
        return set_err(m, ACM_ERR_UNSUPPORTED_TYPE, fmt("tensor %s: unsupported type %u", name, ggml_type));
    t.name = name;
    t.type = ggml_type;
    t.numel = 1;
    for (int i = 0; i < ndims; i++) {
        t.dims.push_back(dims[i]);
        t.numel *= (int64_t)dims[i];
    }
    const int be = blk_elems((int)ggml_type);
    if (ndims == 0 || t.numel <= 0 || t.dims[0] % be)
        return set_err(m, ACM_ERR_INVALID, fmt("tensor %s: bad shape", name));
    t.nbytes = (size_t)(t.numel / be) * blk_bytes((int)ggml_type);
    if (nbytes != t.nbytes)
        return set_err(m, ACM_ERR_INVALID, fmt("tensor %s: %zu bytes given, %zu expected", name, nbytes, t.nbytes));
    return ACM_OK;
}

// Upload of a whole GGUF (the fast path of acm_model_load_gguf) to n models,
// one per engine (the same device may repeat): per model one device arena for
// every used tensor (256-byte aligned slots, 64 zero bytes after each), filled
// through two portable pinned staging buffers.  The host copies each chunk
// out of the mapping ONCE and every device's copy engine takes it from the
// same staging buffer, while the host fills the other buffer: the reference
// maps the file once per process (app/model_unix.go:15-34), and a host that
// drives several GPUs from one process reads it once for all of them.
int upload_gguf(acm_model *const *ms, int n, const gguf::File &f, const std::vector<const std::string *> &names) {
    std::vector<std::vector<DevTensor>> ts(n, std::vector<DevTensor>(names.size()));
    std::vector<size_t> offs(names.size());
    std::vector<uint8_t *> arena(n, nullptr);
    size_t total = 0;
    for (size_t i = 0; i < names.size(); i++) {
        const gguf::Tensor &t = f.tensors.at(*names[i]);
        for (int d = 0; d < n; d++)
            if (int rc = tensor_meta(ms[d], names[i]->c_str(), t.type, t.dims.data(), (int)t.dims.size(), t.nbytes,
                                     ts[d][i]))
                return rc;
        offs[i] = total;
        total += (t.nbytes + 64 + 255) & ~size_t(255);
    }
    for (int d = 0; d < n; d++) {
        acm_model *m = ms[d];
        cudaSetDevice(m->e->device);
        CK_M(dalloc(m, &arena[d], total));
    }
    constexpr size_t CH = 64u << 20;
    uint8_t *stage[2] = {nullptr, nullptr};
    std::vector<cudaEvent_t> done(2 * (size_t)n, nullptr);  // [buffer][model]
    int rc = ACM_OK;
    for (int b = 0; b < 2 && !rc; b++)
        if (cudaHostAlloc(reinterpret_cast<void **>(&stage[b]), CH, cudaHostAllocPortable) != cudaSuccess)
            rc = set_err(ms[0], ACM_ERR_OOM, "pinned staging buffer");
    for (int d = 0; d < n && !rc; d++) {
        cudaSetDevice(ms[d]->e->device);
        for (int b = 0; b < 2 && !rc; b++)
            if (cudaEventCreateWithFlags(&done[(size_t)b * n + d], cudaEventDisableTiming) != cudaSuccess)
                rc = set_err(ms[d], ACM_ERR_CUDA, "upload event");
    }
    // the arena's bytes in order, CH at a time: tensor bytes from the mapping,
    // zeros for the padding after each tensor
    bool pending[2] = {false, false};
    size_t ti = 0;
    int b = 0;
    for (size_t pos = 0; pos < total && !rc; pos += CH) {
        if (pending[b]) {
            // staging buffer b is free again once every device has copied it
            for (int d = 0; d < n && !rc; d++) {
                cudaError_t e = cudaEventSynchronize(done[(size_t)b * n + d]);
                if (e != cudaSuccess) rc = set_err(ms[d], ACM_ERR_CUDA, fmt("upload: %s", cudaGetErrorString(e)));
            }
            if (rc) break;
        }
        const size_t len = std::min(CH, total - pos);
        for (size_t q = 0; q < len;) {
            const size_t at = pos + q;
            while (ti + 1 < names.size() && offs[ti + 1] <= at) ti++;
            const gguf::Tensor &t = f.tensors.at(*names[ti]);
            const size_t end_t = offs[ti] + t.nbytes, end_slot = ti + 1 < names.size() ? offs[ti + 1] : total;
            if (at < end_t) {
                const size_t c = std::min(end_t - at, len - q);
                memcpy(stage[b] + q, static_cast<const uint8_t *>(t.data) + (at - offs[ti]), c);
                q += c;
            } else {
                const size_t c = std::min(end_slot - at, len - q);
                memset(stage[b] + q, 0, c);
                q += c;
            }
        }
        for (int d = 0; d < n && !rc; d++) {
            acm_model *m = ms[d];
            cudaSetDevice(m->e->device);
            if (cudaMemcpyAsync(arena[d] + pos, stage[b], len, cudaMemcpyHostToDevice, m->e->stream) != cudaSuccess ||
                cudaEventRecord(done[(size_t)b * n + d], m->e->stream) != cudaSuccess)
                rc = set_err(m, ACM_ERR_CUDA, "upload copy failed");
        }
        pending[b] = true;
        b ^= 1;
    }
    // no copy may still read a staging buffer when it is freed
    for (int d = 0; d < n; d++) {
        acm_model *m = ms[d];
        cudaSetDevice(m->e->device);
        cudaError_t e = cudaStreamSynchronize(m->e->stream);
        if (!rc && e != cudaSuccess) rc = set_err(m, ACM_ERR_CUDA, fmt("upload: %s", cudaGetErrorString(e)));
    }
    for (cudaEvent_t ev : done)
        if (ev) cudaEventDestroy(ev);
    for (int k = 0; k < 2; k++)
        if (stage[k]) cudaFreeHost(stage[k]);
    if (rc) return rc;
    for (int d = 0; d < n; d++)
        for (size_t i = 0; i < names.size(); i++) {
            ts[d][i].d = arena[d] + offs[i];
            ms[d]->tensors[*names[i]] = std::move(ts[d][i]);
        }
    return ACM_OK;
}

// Read-only private mapping of a file, as the reference's readModel
// (app/model_unix.go:15-34).
struct FileMap {
    void *p = MAP_FAILED;
    size_t len = 0;
    std::string err;
    explicit FileMap(const char *path) {
        const int fd = open(path, O_RDONLY);
        if (fd < 0) {
            err = fmt("open %s: %s", path, strerror(errno));
            return;
        }
        struct stat sb;
        if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
            close(fd);
            err = fmt("stat %s failed", path);
            return;
        }
        len = (size_t)sb.st_size;
        p = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (p == MAP_FAILED) {
            err = fmt("mmap %s failed", path);
            return;
        }
        madvise(p, len, MADV_WILLNEED);
    }
    ~FileMap() {
        if (p != MAP_FAILED) munmap(p, len);
    }
    bool ok() const { return p != MAP_FAILED; }
    const uint8_t *data() const { return static_cast<const uint8_t *>(p); }
};

// gguf.Parse + infer.Load's metadata and tensor rules + the upload, from the
// file's bytes, to one model per engine (outs[i] on es[i]).  On failure no
// model is left and es[0] (or the engine whose model failed) holds the error.
int load_gguf_bytes(acm_engine *const *es, int n, const uint8_t *data, size_t len, int32_t max_ctx, int32_t max_seqs,
                    acm_model **outs) {
    for (int i = 0; i < n; i++) outs[i] = nullptr;
    gguf::File f;
    std::string err;
    int rc = gguf::parse(data, len, f, err);
    acm_config c;
    if (!rc) rc = gguf::load_config(f, max_ctx, c, err);
    if (rc) return set_eerr(es[0], rc, err);
    std::vector<acm_model *> ms(n, nullptr);
    for (int i = 0; i < n && !rc; i++) {
        rc = acm_model_create(es[i], &c, max_seqs, &ms[i]);
        if (rc && i) es[0]->err = es[i]->err;
    }
    std::vector<const std::string *> names;
    for (const std::string &name : f.order)
        if (name == "token_embd.weight" || name == "output.weight" || name == "output_norm.weight" ||
            name.rfind("blk.", 0) == 0)
            names.push_back(&name);
    if (!rc) rc = upload_gguf(ms.data(), n, f, names);
    for (int i = 0; i < n && !rc; i++) {
        cudaSetDevice(es[i]->device);
        rc = acm_model_finalize(ms[i]);
    }
    if (rc) {
        for (int i = 0; i < n; i++)
            if (ms[i]) {
                if (!ms[i]->err.empty()) es[0]->err = ms[i]->err;
                acm_model_destroy(ms[i]);
            }
        return rc;
    }
    for (int i = 0; i < n; i++) outs[i] = ms[i];
    return ACM_OK;
}

int config_bytes(const uint8_t *data, size_t len, int32_t max_ctx, acm_config *out, char *err, int32_t errlen) {
    gguf::File f;
    std::string e;
    int rc = gguf::parse(data, len, f, e);
    if (!rc) rc = gguf::load_config(f, max_ctx, *out, e);
    if (rc && err && errlen > 0) snprintf(err, (size_t)errlen, "%s", e.c_str());
    return rc;
}
}  // namespace

extern "C" {

ACM_API int acm_model_add_tensor(acm_model *m, const char *name, uint32_t ggml_type, const uint64_t *dims,
                                 int32_t ndims, const void *host_bytes, size_t nbytes) {
    if (!m || !name || (ndims > 0 && !dims) || ndims < 0 || ndims > 8 || (!host_bytes && nbytes))
        return set_err(m, ACM_ERR_INVALID, "invalid tensor arguments");
    DevTensor t;
    if (int rc = tensor_meta(m, name, ggml_type, dims, ndims, nbytes, t)) return rc;
    cudaSetDevice(m->e->device);
    // 16 bytes of padding: the bulk copies round spans up to 16 bytes and the
    // unaligned word loader reads one word past a run
    CK_M(dalloc(m, &t.d, t.nbytes + 64));
    CK_M(cudaMemcpy(t.d, host_bytes, t.nbytes, cudaMemcpyHostToDevice));
    CK_M(cudaMemset(t.d + t.nbytes, 0, 64));
    m->tensors[name] = std::move(t);
    return ACM_OK;
}

static int norm_vec(acm_model *m, const DevTensor *t, int64_t n, float **out, const char *what) {
    *out = nullptr;
    if (!t) return ACM_OK;
    if (t->numel != n) return set_err(m, ACM_ERR_INVALID, fmt("%s: %lld elements, %lld expected", what,
                                                              (long long)t->numel, (long long)n));
    CK_M(dalloc(m, out, (size_t)n + 4));
    if (n % 32 == 0) {
        CK_M(dequant_launch((int)t->type, t->d, n, 1, nullptr, 1, *out, n, m->e->stream));
    } else {
        // short vectors not a multiple of 32 elements: F32 only
        if (t->type != T_F32) return set_err(m, ACM_ERR_UNSUPPORTED_TYPE, fmt("%s: unsupported type", what));
        CK_M(cudaMemcpyAsync(*out, t->d, sizeof(float) * n, cudaMemcpyDeviceToDevice, m->e->stream));
    }
    return ACM_OK;
}

ACM_API int acm_model_finalize(acm_model *m) {
    if (!m) return ACM_ERR_INVALID;
    if (m->finalized) return set_err(m, ACM_ERR_INVALID, "model already finalized");
    cudaSetDevice(m->e->device);
    acm_config &c = m->c;
    auto get = [&](const std::string &n) -> DevTensor * {
        auto it = m->tensors.find(n);
        return it == m->tensors.end() ? nullptr : &it->second;
    };
    const int E = c.n_embd, hd = c.head_dim, qd = c.n_head * hd, kvd = c.n_head_kv * hd, F = c.n_ff;
    if (c.n_head % c.n_head_kv || c.n_head / c.n_head_kv > 8)
        return set_err(m, ACM_ERR_INVALID, "unsupported head grouping");
    if (hd != 64 && hd != 128) return set_err(m, ACM_ERR_INVALID, fmt("unsupported head_dim %d", hd));
    if (c.rope_dim <= 0 || c.rope_dim > hd || c.rope_dim % 2)
        return set_err(m, ACM_ERR_INVALID, fmt("unsupported rope dimension %d", c.rope_dim));
    // model.go:161-169
    m->embd = get("token_embd.weight");
    m->out = get("output.weight");
    DevTensor *on = get("output_norm.weight");
    if (!m->embd || !on) return set_err(m, ACM_ERR_MISSING_TENSOR, "missing embedding or output norm tensors");
    if (!m->out) m->out = m->embd;
    int rc;
    if ((rc = norm_vec(m, on, E, &m->out_nw, "output_norm.weight"))) return rc;
    auto shape_ok = [&](const DevTensor *t, int64_t k, int64_t n) { return t->k() == k && t->rows() == n; };
    if (m->embd->k() != E) return set_err(m, ACM_ERR_INVALID, "token_embd.weight: bad shape");
    if (m->out->k() != E || m->out->rows() != c.vocab)
        return set_err(m, ACM_ERR_INVALID, "output tensor rows do not match the token list");
    m->layers.assign(c.n_layers, Layer());
    for (int i = 0; i < c.n_layers; i++) {
        const std::string b = "blk." + std::to_string(i) + ".";
        Layer &L = m->layers[i];
        L.q = get(b + "attn_q.weight");
        L.k = get(b + "attn_k.weight");
        L.v = get(b + "attn_v.weight");
        L.o = get(b + "attn_output.weight");
        L.gate = get(b + "ffn_gate.weight");
        L.up = get(b + "ffn_up.weight");
        L.down = get(b + "ffn_down.weight");
        DevTensor *an = get(b + "attn_norm.weight"), *fn = get(b + "ffn_norm.weight");
        if (!an || !L.q || !L.k || !L.v || !L.o || !fn || !L.gate || !L.up || !L.down)
            return set_err(m, ACM_ERR_MISSING_TENSOR, fmt("layer %d: missing tensors", i));  // model.go:196-199
        if (!shape_ok(L.q, E, qd) || !shape_ok(L.k, E, kvd) || !shape_ok(L.v, E, kvd) || !shape_ok(L.o, qd, E) ||
            !shape_ok(L.gate, E, F) || !shape_ok(L.up, E, F) || !shape_ok(L.down, F, E))
            return set_err(m, ACM_ERR_INVALID, fmt("layer %d: tensor shapes do not match the configuration", i));
        if ((rc = norm_vec(m, an, E, &L.attn_nw, "attn_norm"))) return rc;
        if ((rc = norm_vec(m, fn, E, &L.ffn_nw, "ffn_norm"))) return rc;
        if ((rc = norm_vec(m, get(b + "attn_q_norm.weight"), hd, &L.q_nw, "attn_q_norm"))) return rc;
        if ((rc = norm_vec(m, get(b + "attn_k_norm.weight"), hd, &L.k_nw, "attn_k_norm"))) return rc;
        if ((rc = norm_vec(m, get(b + "attn_q.bias"), qd, &L.q_b, "attn_q.bias"))) return rc;
        if ((rc = norm_vec(m, get(b + "attn_k.bias"), kvd, &L.k_b, "attn_k.bias"))) return rc;
        if ((rc = norm_vec(m, get(b + "attn_v.bias"), kvd, &L.v_b, "attn_v.bias"))) return rc;
    }
    // RoPE table: ropeFreqs (model.go:253-280) then cos/sin per position as
    // rope() computes them (model.go:240): float32(cos(float64(float32(pos)*f)))
    {
        const int half = c.rope_dim / 2;
        std::vector<float> f(half);
        for (int i = 0; i < half; i++) f[i] = 1.0f / (float)pow((double)c.rope_base, (double)(2 * i) / (double)c.rope_dim);
        if (c.rope_scaling == ACM_ROPE_LINEAR) {
            for (int i = 0; i < half; i++) f[i] /= c.rope_factor;
        } else if (c.rope_scaling == ACM_ROPE_LLAMA3) {
            const float lo_wl = c.rope_orig_ctx / c.rope_lo_f, hi_wl = c.rope_orig_ctx / c.rope_hi_f;
            for (int i = 0; i < half; i++) {
                const double wl = 2 * M_PI / (double)f[i];
                if (wl < (double)hi_wl) {
                } else if (wl > (double)lo_wl) {
                    f[i] /= c.rope_factor;
                } else {
                    const float smooth = (c.rope_orig_ctx / (float)wl - c.rope_lo_f) / (c.rope_hi_f - c.rope_lo_f);
                    f[i] = (1 - smooth) * f[i] / c.rope_factor + smooth * f[i];
                }
            }
        }
        std::vector<float2> tab((size_t)c.max_ctx * half);
        for (int p = 0; p < c.max_ctx; p++)
            for (int i = 0; i < half; i++) {
                volatile float a = (float)p * f[i];
                tab[(size_t)p * half + i] = make_float2((float)cos((double)a), (float)sin((double)a));
            }
        CK_M(dalloc(m, &m->rope_tab, tab.size()));
        CK_M(cudaMemcpy(m->rope_tab, tab.data(), sizeof(float2) * tab.size(), cudaMemcpyHostToDevice));
    }
    // paged KV cache: enough pages for every slot at full context
    m->max_pages = (c.max_ctx + PAGE - 1) / PAGE;
    m->n_pages = m->max_pages * m->max_seqs;
    m->layer_stride = (int64_t)m->n_pages * PAGE * kvd;
    const size_t pool_floats = m->kv_f16 ? ((size_t)m->layer_stride * c.n_layers + 1) / 2
                                         : (size_t)m->layer_stride * c.n_layers;
    CK_M(dalloc(m, &m->kpool, pool_floats));
    CK_M(dalloc(m, &m->vpool, pool_floats));
    m->free_pages.clear();
    for (int p = m->n_pages - 1; p >= 0; p--) m->free_pages.push_back(p);
    CK_M(dalloc(m, &m->d_page_table, (size_t)m->max_seqs * m->max_pages));
    CK_M(m->h_page_table.alloc((size_t)m->max_seqs * m->max_pages));
    for (size_t i = 0; i < (size_t)m->max_seqs * m->max_pages; i++) m->h_page_table.p[i] = 0;
    CK_M(cudaMemcpy(m->d_page_table, m->h_page_table.p, sizeof(int32_t) * m->max_seqs * m->max_pages,
                    cudaMemcpyHostToDevice));
    m->seqs.assign(m->max_seqs, Seq());
    // activations
    m->tdec = std::max(8, m->max_seqs);
    const size_t T = (size_t)std::max(TMAX, m->tdec);
    CK_M(dalloc(m, &m->x, T * E));
    CK_M(dalloc(m, &m->h, T * E));
    CK_M(dalloc(m, &m->q, T * qd));
    CK_M(dalloc(m, &m->k, T * kvd));
    CK_M(dalloc(m, &m->v, T * kvd));
    CK_M(dalloc(m, &m->att, T * qd));
    CK_M(dalloc(m, &m->hb, T * F));
    CK_M(dalloc(m, &m->hb2, T * F));
    m->dec_nsplit = (c.max_ctx + 31) / 32;  // 32-position chunks of the decode attention
    const size_t part_rows = std::max<size_t>((size_t)PART_TOKSPLIT, (size_t)m->tdec * m->dec_nsplit);
    // rows of hd + 4 floats: the decode attention's partial stride (dec_part_stride)
    CK_M(dalloc(m, &m->part, part_rows * c.n_head * (hd + 4)));
    CK_M(dalloc(m, &m->d_attn_cnt, (size_t)m->tdec * c.n_head));
    CK_M(cudaMemset(m->d_attn_cnt, 0, sizeof(int) * (size_t)m->tdec * c.n_head));
    CK_M(dalloc(m, &m->logits, (size_t)m->max_seqs * c.vocab));
    CK_M(cudaMemset(m->logits, 0, sizeof(float) * (size_t)m->max_seqs * c.vocab));
    CK_M(dalloc(m, &m->d_tok, T));
    CK_M(dalloc(m, &m->d_seq, T));
    CK_M(dalloc(m, &m->d_pos, T));
    CK_M(dalloc(m, &m->d_out, T));
    CK_M(dalloc(m, &m->d_topk, T));
    CK_M(dalloc(m, &m->d_temp, T));
    CK_M(dalloc(m, &m->d_topp, T));
    CK_M(dalloc(m, &m->d_seed, T));
    CK_M(dalloc(m, &m->d_step, T));
    m->nchunks = (c.vocab + 2047) / 2048;
    CK_M(dalloc(m, &m->d_cand, (size_t)m->tdec * m->nchunks * 64));
    CK_M(dalloc(m, &m->d_hist, (size_t)m->tdec * HIST_MAX));
    CK_M(dalloc(m, &m->d_hist_col, 1));
    CK_M(dalloc(m, &m->d_amax, T));
    CK_M(cudaMemset(m->d_amax, 0, sizeof(unsigned long long) * T));
    CK_M(m->h_tok.alloc(T));
    CK_M(m->h_seq.alloc(T));
    CK_M(m->h_pos.alloc(T));
    CK_M(m->h_out.alloc(T));
    CK_M(m->h_topk.alloc(T));
    CK_M(m->h_temp.alloc(T));
    CK_M(m->h_topp.alloc(T));
    CK_M(m->h_seed.alloc(T));
    CK_M(m->h_step.alloc(T));
    CK_M(m->h_hist.alloc((size_t)m->tdec * HIST_MAX));
    for (int i = 0; i < 4; i++) CK_M(cudaEventCreate(&m->ev[i]));
    rc = sync_check(m);
    if (rc) return rc;
    m->finalized = true;
    return ACM_OK;
}

ACM_API int acm_model_destroy(acm_model *m) {
    if (m && m->gtrace_on) gemv1_trace(nullptr, 0);
    if (!m) return ACM_ERR_INVALID;
    cudaSetDevice(m->e->device);
    cudaStreamSynchronize(m->e->stream);
    for (auto &g : m->graphs) cudaGraphExecDestroy(g.second.exec);
    if (m->gemv_bench.exec) cudaGraphExecDestroy(m->gemv_bench.exec);
    for (void *p : m->allocs) cudaFree(p);
    m->h_page_table.release();
    m->h_tok.release();
    m->h_seq.release();
    m->h_pos.release();
    m->h_out.release();
    m->h_topk.release();
    m->h_temp.release();
    m->h_topp.release();
    m->h_seed.release();
    m->h_step.release();
    m->h_hist.release();
    for (int i = 0; i < 4; i++)
        if (m->ev[i]) cudaEventDestroy(m->ev[i]);
    acm_engine *e = m->e;
    delete m;
    if (--e->models == 0 && e->closed) engine_free(e);
    return ACM_OK;
}

ACM_API const char *acm_last_error(acm_model *m) { return m ? m->err.c_str() : "null model"; }

ACM_API int acm_model_config(acm_model *m, acm_config *out) {
    if (!m || !out) return ACM_ERR_INVALID;
    *out = m->c;
    return ACM_OK;
}

ACM_API int acm_model_load_gguf(acm_engine *e, const char *path, int32_t max_ctx, int32_t max_seqs,
                                acm_model **out) {
    if (!e || !path || !out) return ACM_ERR_INVALID;
    *out = nullptr;
    FileMap map(path);
    if (!map.ok()) return set_eerr(e, ACM_ERR_IO, map.err);
    return load_gguf_bytes(&e, 1, map.data(), map.len, max_ctx, max_seqs, out);
}

ACM_API int acm_model_load_gguf_mem(acm_engine *e, const void *data, size_t nbytes, int32_t max_ctx, int32_t max_seqs,
                                    acm_model **out) {
    if (!e || !data || !out) return ACM_ERR_INVALID;
    *out = nullptr;
    return load_gguf_bytes(&e, 1, static_cast<const uint8_t *>(data), nbytes, max_ctx, max_seqs, out);
}

ACM_API int acm_model_load_gguf_multi(acm_engine *const *es, int32_t n, const char *path, int32_t max_ctx,
                                      int32_t max_seqs, acm_model **outs) {
    if (!es || n < 1 || n > 64 || !path || !outs) return ACM_ERR_INVALID;
    for (int i = 0; i < n; i++)
        if (!es[i]) return ACM_ERR_INVALID;
    for (int i = 0; i < n; i++) outs[i] = nullptr;
    FileMap map(path);
    if (!map.ok()) return set_eerr(es[0], ACM_ERR_IO, map.err);
    return load_gguf_bytes(es, n, map.data(), map.len, max_ctx, max_seqs, outs);
}

ACM_API int acm_load_config(const char *path, int32_t max_ctx, acm_config *out, char *err, int32_t errlen) {
    if (!path || !out) {
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "null argument");
        return ACM_ERR_INVALID;
    }
    FileMap map(path);
    if (!map.ok()) {
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", map.err.c_str());
        return ACM_ERR_IO;
    }
    return config_bytes(map.data(), map.len, max_ctx, out, err, errlen);
}

ACM_API int acm_load_config_mem(const void *data, size_t nbytes, int32_t max_ctx, acm_config *out, char *err,
                                int32_t errlen) {
    if (!data || !out) {
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "null argument");
        return ACM_ERR_INVALID;
    }
    return config_bytes(static_cast<const uint8_t *>(data), nbytes, max_ctx, out, err, errlen);
}

ACM_API int acm_seq_open(acm_model *m, int32_t *seq_out) {
    if (!m || !seq_out || !m->finalized) return set_err(m, ACM_ERR_INVALID, "model not finalized");
    for (int i = 0; i < m->max_seqs; i++)
        if (!m->seqs[i].open) {
            m->seqs[i].open = true;
            m->seqs[i].pos = 0;
            *seq_out = i;
            return ACM_OK;
        }
    return set_err(m, ACM_ERR_NO_SEQ, "no free sequence slot");
}

ACM_API int acm_seq_close(acm_model *m, int32_t seq) {
    int rc = check_seq(m, seq);
    if (rc) return rc;
    Seq &s = m->seqs[seq];
    for (int pg : s.pages) m->free_pages.push_back(pg);
    s.pages.clear();
    s.open = false;
    s.pos = 0;
    return ACM_OK;
}

ACM_API int acm_seq_reset(acm_model *m, int32_t seq) {
    int rc = check_seq(m, seq);
    if (rc) return rc;
    m->seqs[seq].pos = 0;  // Reset keeps the cache pages, model.go:458-460
    return ACM_OK;
}

ACM_API int acm_seq_pos(acm_model *m, int32_t seq, int32_t *pos_out) {
    int rc = check_seq(m, seq);
    if (rc) return rc;
    if (!pos_out) return ACM_ERR_INVALID;
    *pos_out = m->seqs[seq].pos;
    return ACM_OK;
}

ACM_API int acm_forward(acm_model *m, int32_t seq, const int32_t *toks, int32_t n, float *logits_out) {
    int rc = check_seq(m, seq);
    if (rc) return rc;
    if (n <= 0 || !toks) return set_err(m, ACM_ERR_INVALID, "empty token batch");
    cudaSetDevice(m->e->device);
    Seq &s = m->seqs[seq];
    if (s.pos + n > m->c.max_ctx)  // model.go:320-321
        return set_err(m, ACM_ERR_CTX_EXCEEDED, fmt("context length exceeded (%d > %d)", s.pos + n, m->c.max_ctx));
    const int64_t erows = m->embd->rows();
    for (int i = 0; i < n; i++)
        if (toks[i] < 0 || toks[i] >= erows) return set_err(m, ACM_ERR_INVALID, fmt("token id %d out of range", toks[i]));
    CK_M(cudaEventRecord(m->ev[0], m->e->stream));
    const int pos0 = s.pos;
    rc = forward_seq(m, seq, toks, n);
    if (rc) {
        s.pos = pos0;
        return rc;
    }
    CK_M(cudaEventRecord(m->ev[1], m->e->stream));
    if (logits_out)
        CK_M(cudaMemcpyAsync(logits_out, m->logits + (size_t)seq * m->c.vocab, sizeof(float) * m->c.vocab,
                             cudaMemcpyDeviceToHost, m->e->stream));
    if ((rc = sync_check(m))) return rc;
    m->last_prefill_s = ev_seconds(m->ev[0], m->ev[1]);
    return ACM_OK;
}

ACM_API int acm_sample(acm_model *m, int32_t seq, const acm_sampler *s, uint64_t step, int32_t *tok_out) {
    int rc = check_seq(m, seq);
    if (rc) return rc;
    if (!tok_out) return ACM_ERR_INVALID;
    cudaSetDevice(m->e->device);
    m->h_seq.p[0] = seq;
    fill_sampler(m, 0, s, step);
    CK_M(cudaMemcpyAsync(m->d_seq, m->h_seq.p, sizeof(int32_t), cudaMemcpyHostToDevice, m->e->stream));
    if ((rc = upload_sampler(m, 1))) return rc;
    if ((rc = sample_pass(m, 1, !s || s->temp <= 0))) return rc;
    CK_M(cudaMemcpyAsync(m->h_out.p, m->d_out, sizeof(int32_t), cudaMemcpyDeviceToHost, m->e->stream));
    if ((rc = sync_check(m))) return rc;
    *tok_out = m->h_out.p[0];
    return ACM_OK;
}

ACM_API int acm_decode_step(acm_model *m, int32_t nseq, const int32_t *seqs, const int32_t *in_tok,
                            const acm_sampler *samplers, const uint64_t *steps, int32_t *out_tok,
                            float *logits_out) {
    if (!m || !m->finalized) return set_err(m, ACM_ERR_INVALID, "model not finalized");
    if (nseq <= 0 || nseq > m->tdec || !seqs || !in_tok || !out_tok)
        return set_err(m, ACM_ERR_INVALID, "bad decode batch");
    cudaSetDevice(m->e->device);
    std::vector<char> seen(m->max_seqs, 0);
    bool greedy = true;
    const int64_t erows = m->embd->rows();
    for (int i = 0; i < nseq; i++) {
        int rc = check_seq(m, seqs[i]);
        if (rc) return rc;
        if (seen[seqs[i]]) return set_err(m, ACM_ERR_INVALID, "sequence repeated in a decode batch");
        seen[seqs[i]] = 1;
        const Seq &s = m->seqs[seqs[i]];
        if (s.pos + 1 > m->c.max_ctx)
            return set_err(m, ACM_ERR_CTX_EXCEEDED, fmt("context length exceeded (%d > %d)", s.pos + 1, m->c.max_ctx));
        if (in_tok[i] < 0 || in_tok[i] >= erows) return set_err(m, ACM_ERR_INVALID, fmt("token id %d out of range", in_tok[i]));
        if ((rc = ensure_pages(m, seqs[i], s.pos + 1))) return rc;
        m->h_tok.p[i] = in_tok[i];
        m->h_seq.p[i] = seqs[i];
        m->h_pos.p[i] = s.pos;
        fill_sampler(m, i, samplers ? &samplers[i] : nullptr, steps ? steps[i] : 0);
        if (samplers && samplers[i].temp > 0) greedy = false;
    }
    int rc;
    if ((rc = upload_meta(m, nseq))) return rc;
    if ((rc = upload_sampler(m, nseq))) return rc;
    CK_M(cudaMemsetAsync(m->d_hist_col, 0, sizeof(int32_t), m->e->stream));
    CK_M(cudaEventRecord(m->ev[2], m->e->stream));
    if ((rc = decode_graph_launch(m, nseq, greedy))) return rc;
    CK_M(cudaEventRecord(m->ev[3], m->e->stream));
    CK_M(cudaMemcpyAsync(m->h_out.p, m->d_out, sizeof(int32_t) * nseq, cudaMemcpyDeviceToHost, m->e->stream));
    if ((rc = sync_check(m))) return rc;
    m->last_decode_s = ev_seconds(m->ev[2], m->ev[3]);
    for (int i = 0; i < nseq; i++) {
        out_tok[i] = m->h_out.p[i];
        m->seqs[seqs[i]].pos += 1;
    }
    if (logits_out)
        for (int i = 0; i < nseq; i++)
            CK_M(cudaMemcpy(logits_out + (size_t)i * m->c.vocab, m->logits + (size_t)seqs[i] * m->c.vocab,
                            sizeof(float) * m->c.vocab, cudaMemcpyDeviceToHost));
    return ACM_OK;
}

ACM_API int acm_generate(acm_model *m, int32_t seq, const int32_t *prompt, int32_t n_prompt, const acm_sampler *s,
                         int32_t max_tok, int32_t stop_on_eos, int32_t *out_ids, int32_t *n_out, acm_stats *stats) {
    int rc = check_seq(m, seq);
    if (rc) return rc;
    if (!n_out || (max_tok > 0 && !out_ids) || n_prompt < 0 || (n_prompt > 0 && !prompt))
        return set_err(m, ACM_ERR_INVALID, "bad generate arguments");
    cudaSetDevice(m->e->device);
    *n_out = 0;
    acm_stats st{0, 0, 0, 0};
    Seq &sq = m->seqs[seq];
    cudaStream_t stream = m->e->stream;
    // sampler.go:116-121: chunk = min(1024, MaxCtx - pos)
    const int chunk = std::min(TMAX, m->c.max_ctx - sq.pos);
    if (chunk <= 0) return set_err(m, ACM_ERR_CTX_EXCEEDED, "context length exceeded");
    const int64_t erows = m->embd->rows();
    for (int i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || prompt[i] >= erows) return set_err(m, ACM_ERR_INVALID, fmt("token id %d out of range", prompt[i]));
    for (int i = 0; i < n_prompt; i += chunk) {
        const int end = std::min(i + chunk, n_prompt);
        if (sq.pos + (end - i) > m->c.max_ctx)
            return set_err(m, ACM_ERR_CTX_EXCEEDED,
                           fmt("context length exceeded (%d > %d)", sq.pos + end - i, m->c.max_ctx));
        CK_M(cudaEventRecord(m->ev[0], stream));
        if ((rc = forward_seq(m, seq, prompt + i, end - i))) return rc;
        CK_M(cudaEventRecord(m->ev[1], stream));
        if ((rc = sync_check(m))) return rc;
        st.prefill_s += ev_seconds(m->ev[0], m->ev[1]);
        st.prefill_toks += end - i;
    }
    m->last_prefill_s = st.prefill_s;
    if (n_prompt == 0 || max_tok <= 0) {
        if (stats) *stats = st;
        return ACM_OK;
    }
    const bool greedy = !s || s->temp <= 0;
    // id_0 from the prefill logits (step 0)
    m->h_seq.p[0] = seq;
    fill_sampler(m, 0, s, 0);
    CK_M(cudaMemcpyAsync(m->d_seq, m->h_seq.p, sizeof(int32_t), cudaMemcpyHostToDevice, stream));
    if ((rc = upload_sampler(m, 1))) return rc;
    if ((rc = sample_pass(m, 1, greedy))) return rc;
    CK_M(cudaMemcpyAsync(m->h_out.p, m->d_out, sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
    if ((rc = sync_check(m))) return rc;
    // sampler.go:136-157: sample -> stop check -> append -> Forward.  The
    // Forward+Sample pairs run on the device in chunks of up to HIST_MAX graph
    // replays; step i of a chunk forwards the pending id and samples hist[i]
    // with the draw of sample call n + 1 + i.
    int n = 0;
    int32_t id = m->h_out.p[0];
    double dec = 0;
    while (n < max_tok) {
        if (stop_on_eos && (id == m->c.eos || id == m->c.eos2)) break;
        const int room = m->c.max_ctx - sq.pos;
        if (room <= 0) {
            out_ids[n++] = id;
            *n_out = n;
            st.decode_s = dec;
            if (stats) *stats = st;
            return set_err(m, ACM_ERR_CTX_EXCEEDED, fmt("context length exceeded (%d > %d)", sq.pos + 1, m->c.max_ctx));
        }
        const int steps = std::min(std::min(HIST_MAX, max_tok - n), room);
        if ((rc = ensure_pages(m, seq, sq.pos + steps))) return rc;
        m->h_tok.p[0] = id;
        m->h_seq.p[0] = seq;
        m->h_pos.p[0] = sq.pos;
        fill_sampler(m, 0, s, (uint64_t)n + 1);
        if ((rc = upload_meta(m, 1))) return rc;
        if ((rc = upload_sampler(m, 1))) return rc;
        CK_M(cudaMemsetAsync(m->d_hist_col, 0, sizeof(int32_t), stream));
        CK_M(cudaEventRecord(m->ev[2], stream));
        for (int i = 0; i < steps; i++)
            if ((rc = decode_graph_launch(m, 1, greedy))) return rc;
        CK_M(cudaEventRecord(m->ev[3], stream));
        CK_M(cudaMemcpyAsync(m->h_hist.p, m->d_hist, sizeof(int32_t) * steps, cudaMemcpyDeviceToHost, stream));
        if ((rc = sync_check(m))) return rc;
        dec += ev_seconds(m->ev[2], m->ev[3]);
        for (int i = 0; i < steps; i++) {
            out_ids[n++] = id;  // step i forwarded `id`
            sq.pos += 1;
            st.decode_toks++;
            id = m->h_hist.p[i];
            if (n >= max_tok) break;
            if (stop_on_eos && (id == m->c.eos || id == m->c.eos2)) break;  // later steps are discarded
        }
    }
    m->last_decode_s = dec;
    st.decode_s = dec;
    *n_out = n;
    if (stats) *stats = st;
    return ACM_OK;
}

// Continuous batching over independent requests (no reference counterpart:
// the reference serves one prompt per process).  Each request follows
// Generate's loop (sampler.go:108-157) exactly as acm_generate does -- id_0
// from the prefill logits with draw 0, then Forward + Sample with draw n + 1
// -- while up to max_batch of them share each decode step.
ACM_API int acm_serve(acm_model *m, acm_request *reqs, int32_t n, int32_t max_batch, int32_t stop_on_eos,
                      acm_stats *stats) {
    if (!m || !m->finalized) return set_err(m, ACM_ERR_INVALID, "model not finalized");
    if (n < 0 || (n > 0 && !reqs)) return set_err(m, ACM_ERR_INVALID, "bad request list");
    for (int i = 0; i < n; i++)
        if (reqs[i].n_prompt < 0 || (reqs[i].n_prompt > 0 && !reqs[i].prompt) ||
            (reqs[i].max_tok > 0 && !reqs[i].out_ids))
            return set_err(m, ACM_ERR_INVALID, fmt("bad request %d", i));
    cudaSetDevice(m->e->device);
    const int B = std::max(1, std::min(max_batch > 0 ? max_batch : m->tdec, m->tdec));
    cudaStream_t stream = m->e->stream;
    const int64_t erows = m->embd->rows();
    struct Act {
        int r, seq;
        int32_t id;
    };
    std::vector<Act> act;
    acm_stats st{0, 0, 0, 0};
    for (int i = 0; i < n; i++) {
        reqs[i].n_out = 0;
        reqs[i].status = ACM_OK;
    }
    auto is_stop = [&](int32_t id) { return stop_on_eos && (id == m->c.eos || id == m->c.eos2); };
    int next = 0, rc = ACM_OK;
    std::vector<int32_t> seqs, toks, outs;
    std::vector<acm_sampler> sams;
    std::vector<uint64_t> steps;
    while (next < n || !act.empty()) {
        // ---- admission: prefill new requests into free slots ----
        std::vector<Act> fresh;
        while ((int)(act.size() + fresh.size()) < B && next < n) {
            acm_request &q = reqs[next];
            int32_t seq = -1;
            if (acm_seq_open(m, &seq) != ACM_OK) {
                if (act.empty() && fresh.empty()) return set_err(m, ACM_ERR_INVALID, "no free sequence slot");
                break;  // retry once a slot frees up
            }
            const int r = next++;
            Seq &sq = m->seqs[seq];
            int qrc = ACM_OK;
            for (int i = 0; i < q.n_prompt && !qrc; i++)
                if (q.prompt[i] < 0 || q.prompt[i] >= erows) qrc = set_err(m, ACM_ERR_INVALID, fmt("token id %d out of range", q.prompt[i]));
            const int chunk = std::max(1, std::min(TMAX, m->c.max_ctx));
            for (int i = 0; i < q.n_prompt && !qrc; i += chunk) {
                const int end = std::min(i + chunk, q.n_prompt);
                if (sq.pos + (end - i) > m->c.max_ctx) {
                    qrc = set_err(m, ACM_ERR_CTX_EXCEEDED,
                                  fmt("context length exceeded (%d > %d)", sq.pos + end - i, m->c.max_ctx));
                    break;
                }
                CK_M(cudaEventRecord(m->ev[0], stream));
                if ((rc = forward_seq(m, seq, q.prompt + i, end - i))) return rc;
                CK_M(cudaEventRecord(m->ev[1], stream));
                if ((rc = sync_check(m))) return rc;
                st.prefill_s += ev_seconds(m->ev[0], m->ev[1]);
                st.prefill_toks += end - i;
            }
            if (qrc || q.n_prompt == 0 || q.max_tok <= 0) {
                q.status = qrc;
                acm_seq_close(m, seq);
                continue;
            }
            fresh.push_back(Act{r, seq, 0});
        }
        if (!fresh.empty()) {
            // id_0 of every new request from its prefill logits (draw 0)
            const int k = (int)fresh.size();
            bool greedy = true;
            for (int i = 0; i < k; i++) {
                m->h_seq.p[i] = fresh[i].seq;
                fill_sampler(m, i, &reqs[fresh[i].r].sampler, 0);
                if (reqs[fresh[i].r].sampler.temp > 0) greedy = false;
            }
            CK_M(cudaMemcpyAsync(m->d_seq, m->h_seq.p, sizeof(int32_t) * k, cudaMemcpyHostToDevice, stream));
            if ((rc = upload_sampler(m, k))) return rc;
            if ((rc = sample_pass(m, k, greedy))) return rc;
            CK_M(cudaMemcpyAsync(m->h_out.p, m->d_out, sizeof(int32_t) * k, cudaMemcpyDeviceToHost, stream));
            if ((rc = sync_check(m))) return rc;
            for (int i = 0; i < k; i++) {
                fresh[i].id = m->h_out.p[i];
                act.push_back(fresh[i]);
            }
        }
        // ---- retire: stop id sampled, or no room for another position ----
        for (size_t i = 0; i < act.size();) {
            acm_request &q = reqs[act[i].r];
            bool done = is_stop(act[i].id);
            if (!done && m->seqs[act[i].seq].pos + 1 > m->c.max_ctx) {
                q.out_ids[q.n_out++] = act[i].id;  // appended, then Forward fails (as acm_generate)
                q.status = ACM_ERR_CTX_EXCEEDED;
                done = true;
            }
            if (done) {
                acm_seq_close(m, act[i].seq);
                act[i] = act.back();
                act.pop_back();
            } else {
                i++;
            }
        }
        if (act.empty()) continue;
        // ---- one batched decode step: Forward(id) + Sample with draw n + 1 ----
        const int na = (int)act.size();
        seqs.resize(na);
        toks.resize(na);
        outs.resize(na);
        sams.resize(na);
        steps.resize(na);
        for (int i = 0; i < na; i++) {
            const acm_request &q = reqs[act[i].r];
            seqs[i] = act[i].seq;
            toks[i] = act[i].id;
            sams[i] = q.sampler;
            steps[i] = (uint64_t)q.n_out + 1;
        }
        if ((rc = acm_decode_step(m, na, seqs.data(), toks.data(), sams.data(), steps.data(), outs.data(), nullptr)))
            return rc;
        st.decode_s += m->last_decode_s;
        st.decode_toks += na;
        for (size_t i = 0; i < act.size();) {
            acm_request &q = reqs[act[i].r];
            q.out_ids[q.n_out++] = act[i].id;
            act[i].id = outs[i];
            if (q.n_out >= q.max_tok) {
                acm_seq_close(m, act[i].seq);
                act[i] = act.back();
                outs[i] = outs[act.size() - 1];
                act.pop_back();
            } else {
                i++;
            }
        }
    }
    m->last_prefill_s = st.prefill_s;
    m->last_decode_s = st.decode_s;
    if (stats) *stats = st;
    return ACM_OK;
}

ACM_API int32_t acm_max_logit(const float *logits, int32_t n) {
    int32_t best = 0;
    for (int32_t i = 1; i < n; i++)
        if (logits[i] > logits[best]) best = i;
    return best;
}

ACM_API int acm_model_last_timing(acm_model *m, double *prefill_s, double *decode_s) {
    if (!m) return ACM_ERR_INVALID;
    if (prefill_s) *prefill_s = m->last_prefill_s;
    if (decode_s) *decode_s = m->last_decode_s;
    return ACM_OK;
}

ACM_API uint64_t acm_kernel_launches(void) { return g_kernel_launches.load(); }


ACM_API int acm_model_debug_layers(acm_model *m, int32_t enable) {
    if (!m || !m->finalized) return set_err(m, ACM_ERR_INVALID, "model not finalized");
    cudaSetDevice(m->e->device);
    if (enable && !m->d_dbg) {
        CK_M(dalloc(m, &m->d_dbg, (size_t)m->c.n_layers * m->c.n_embd));
        CK_M(cudaMemset(m->d_dbg, 0, sizeof(float) * m->c.n_layers * m->c.n_embd));
    }
    if ((bool)enable != m->dbg_layers) {
        m->dbg_layers = enable != 0;
        // captured decode graphs hold (or lack) the copies: rebuild them
        for (auto &g : m->graphs) cudaGraphExecDestroy(g.second.exec);
        m->graphs.clear();
    }
    return ACM_OK;
}

ACM_API int acm_model_debug_layers_read(acm_model *m, float *out, int64_t cap) {
    if (!m || !m->dbg_layers || !m->d_dbg || !out) return set_err(m, ACM_ERR_INVALID, "layer dumps not enabled");
    const int64_t n = (int64_t)m->c.n_layers * m->c.n_embd;
    if (cap < n) return set_err(m, ACM_ERR_INVALID, "buffer too small");
    cudaSetDevice(m->e->device);
    CK_M(cudaStreamSynchronize(m->e->stream));
    CK_M(cudaMemcpy(out, m->d_dbg, sizeof(float) * n, cudaMemcpyDeviceToHost));
    return ACM_OK;
}

ACM_API int acm_model_trace_gemv(acm_model *m, int32_t slots) {
    if (!m || !m->finalized || slots < 0) return set_err(m, ACM_ERR_INVALID, "bad arguments");
    cudaSetDevice(m->e->device);
    if (slots > m->gtrace_slots) {
        CK_M(dalloc(m, &m->d_gtrace, (size_t)slots * 160 * 8));
        m->gtrace_slots = slots;
    }
    if (slots) CK_M(cudaMemset(m->d_gtrace, 0, sizeof(unsigned long long) * (size_t)slots * 160 * 8));
    m->gtrace_on = slots;
    // captured graphs bake each launch's slot in: rebuild them
    for (auto &g : m->graphs) cudaGraphExecDestroy(g.second.exec);
    m->graphs.clear();
    gemv1_trace(slots ? m->d_gtrace : nullptr, slots);
    return ACM_OK;
}

ACM_API int acm_model_trace_gemv_read(acm_model *m, uint64_t *out, int64_t cap, int32_t *used) {
    if (!m || !m->gtrace_on || !out) return set_err(m, ACM_ERR_INVALID, "GEMV tracing not enabled");
    cudaSetDevice(m->e->device);
    const int n = std::min(gemv1_trace_used(), m->gtrace_on);
    if (cap < (int64_t)n * 160 * 8) return set_err(m, ACM_ERR_INVALID, "trace buffer too small");
    CK_M(cudaMemcpy(out, m->d_gtrace, sizeof(uint64_t) * (size_t)n * 160 * 8, cudaMemcpyDeviceToHost));
    if (used) *used = n;
    return ACM_OK;
}

ACM_API int acm_model_bench_gemm(acm_model *m, int32_t ntok, int32_t reps, double *sec_per_pass,
                                 double *flops_per_pass, int32_t *launches_per_pass) {
    if (!m || !m->finalized || reps <= 0 || ntok < 9 || ntok > TMAX) return set_err(m, ACM_ERR_INVALID, "bad arguments");
    cudaSetDevice(m->e->device);
    const acm_config &c = m->c;
    cudaStream_t st = m->e->stream;
    const int E = c.n_embd, hd = c.head_dim, qd = c.n_head * hd, kvd = c.n_head_kv * hd, F = c.n_ff;
    // the GEMM kind forward_pass takes for each group of weights
    struct Kinds {
        bool qkv, o, gu, down;
    };
    std::vector<Kinds> kinds;
    for (const Layer &L : m->layers) {
        Kinds k{use_mma_dq(m, {L.q, L.k, L.v}, E), use_mma_dq(m, {L.o}, qd),
                L.gate->type == L.up->type && use_mma_dq(m, {L.gate, L.up}, E), use_mma_dq(m, {L.down}, F)};
        if ((!k.qkv && !use_mma(m, {L.q, L.k, L.v})) || (!k.o && !use_mma(m, {L.o})) ||
            (!k.gu && !use_mma(m, {L.gate, L.up})) || (!k.down && !use_mma(m, {L.down})) || F % 64)
            return set_err(m, ACM_ERR_INVALID, "tensor-core GEMM unavailable for this model");
        kinds.push_back(k);
    }
    // activation maps: the split buffers as they are (contents do not matter for timing)
    const TensorMap *xe_h = &m->xmap_hi[0], *xe_l = &m->xmap_lo[0];
    const TensorMap *xq_h = &m->xmap_hi[1], *xq_l = &m->xmap_lo[1];
    const TensorMap *xf_h = &m->xmap_hi[2], *xf_l = &m->xmap_lo[2];
    double flops = 0;
    int nl = 0;
    auto pass = [&]() -> int {
        flops = 0;
        nl = 0;
        for (size_t li = 0; li < m->layers.size(); li++) {
            const Layer &L = m->layers[li];
            const Kinds &kd = kinds[li];
            MmaGemmSeg sg[3] = {{&L.q->mhi, &L.q->mlo, nullptr, nullptr, qd, EPI_STORE, m->q, qd, L.q_b, nullptr,
                                 L.q->d, nullptr, kd.qkv ? (int)L.q->type : -1},
                                {&L.k->mhi, &L.k->mlo, nullptr, nullptr, kvd, EPI_STORE, m->k, kvd, L.k_b, nullptr,
                                 L.k->d, nullptr, kd.qkv ? (int)L.k->type : -1},
                                {&L.v->mhi, &L.v->mlo, nullptr, nullptr, kvd, EPI_STORE, m->v, kvd, L.v_b, nullptr,
                                 L.v->d, nullptr, kd.qkv ? (int)L.v->type : -1}};
            CK_M(mma_run(sg, 3, xe_h, xe_l, ntok, E, st));
            MmaGemmSeg so{&L.o->mhi, &L.o->mlo, nullptr, nullptr, E, EPI_STORE, m->h, E, nullptr, nullptr,
                          L.o->d, nullptr, kd.o ? (int)L.o->type : -1};
            CK_M(mma_run(&so, 1, xq_h, xq_l, ntok, qd, st, m->mma_ws, m->mma_ws_floats));
            MmaGemmSeg sf{&L.gate->mhi, &L.gate->mlo, &L.up->mhi, &L.up->mlo, F, EPI_SWIGLU, m->hb2, F, nullptr, nullptr,
                          L.gate->d, L.up->d, kd.gu ? (int)L.gate->type : -1};
            CK_M(mma_run(&sf, 1, xe_h, xe_l, ntok, E, st));
            MmaGemmSeg sd{&L.down->mhi, &L.down->mlo, nullptr, nullptr, E, EPI_STORE, m->h, E, nullptr, nullptr,
                          L.down->d, nullptr, kd.down ? (int)L.down->type : -1};
            CK_M(mma_run(&sd, 1, xf_h, xf_l, ntok, F, st, m->mma_ws, m->mma_ws_floats));
            flops += 2.0 * ntok * ((double)(qd + 2 * kvd) * E + (double)E * qd + 2.0 * F * E + (double)E * F);
            nl += 4;
        }
        return ACM_OK;
    };
    int rc;
    if ((rc = pass())) return rc;  // warm-up
    if ((rc = sync_check(m))) return rc;
    CK_M(cudaEventRecord(m->ev[0], st));
    for (int i = 0; i < reps; i++)
        if ((rc = pass())) return rc;
    CK_M(cudaEventRecord(m->ev[1], st));
    if ((rc = sync_check(m))) return rc;
    if (sec_per_pass) *sec_per_pass = ev_seconds(m->ev[0], m->ev[1]) / reps;
    if (flops_per_pass) *flops_per_pass = flops;
    if (launches_per_pass) *launches_per_pass = nl;
    return ACM_OK;
}

ACM_API int acm_model_bench_gemv(acm_model *m, int32_t reps, double *sec_per_pass, double *bytes_per_pass,
                                 int32_t *launches_per_pass) {
    if (!m || !m->finalized || reps <= 0) return set_err(m, ACM_ERR_INVALID, "bad arguments");
    cudaSetDevice(m->e->device);
    const acm_config &c = m->c;
    cudaStream_t st = m->e->stream;
    const int E = c.n_embd, hd = c.head_dim, qd = c.n_head * hd, kvd = c.n_head_kv * hd, F = c.n_ff, S = m->e->num_sms;
    const float eps = c.rms_eps;
    double B = 0;
    int nl = 0;
    auto ops = [&]() -> int {
        B = 0;
        nl = 0;
        for (int l = 0; l < c.n_layers; l++) {
            const Layer &L = m->layers[l];
            GemvSegDesc sg[3] = {{L.q->d, nullptr, (int)L.q->type, qd, EPI_STORE, m->q, qd, L.q_b, nullptr},
                                 {L.k->d, nullptr, (int)L.k->type, kvd, EPI_STORE, m->k, kvd, L.k_b, nullptr},
                                 {L.v->d, nullptr, (int)L.v->type, kvd, EPI_STORE, m->v, kvd, L.v_b, nullptr}};
            const L2Range pf_o[1] = {{L.o->d, (int64_t)L.o->nbytes}};
            CK_M(gemv_launch(sg, 3, m->x, E, E, 1, L.attn_nw, eps, S, st, pf_o, 1));
            B += (double)(L.q->nbytes + L.k->nbytes + L.v->nbytes) + 4.0 * (2 * E + qd + 2 * kvd);
            GemvSegDesc so{L.o->d, nullptr, (int)L.o->type, E, EPI_ADD, m->x, E, nullptr, nullptr};
            const L2Range pf_f[2] = {{L.gate->d, (int64_t)L.gate->nbytes}, {L.up->d, (int64_t)L.up->nbytes}};
            CK_M(gemv_launch(&so, 1, m->att, qd, qd, 1, nullptr, eps, S, st, pf_f, 2));
            B += (double)L.o->nbytes + 4.0 * (qd + 2 * E);
            if (L.gate->type == L.up->type) {
                GemvSegDesc sf{L.gate->d, L.up->d, (int)L.gate->type, F, EPI_SWIGLU, m->hb, F, nullptr, nullptr};
                const L2Range pf_d[1] = {{L.down->d, (int64_t)L.down->nbytes}};
                CK_M(gemv_launch(&sf, 1, m->x, E, E, 1, L.ffn_nw, eps, S, st, pf_d, 1));
            } else {
                GemvSegDesc sf[2] = {{L.gate->d, nullptr, (int)L.gate->type, F, EPI_STORE, m->hb, F, nullptr, nullptr},
                                     {L.up->d, nullptr, (int)L.up->type, F, EPI_STORE, m->hb2, F, nullptr, nullptr}};
                CK_M(gemv_launch(sf, 2, m->x, E, E, 1, L.ffn_nw, eps, S, st));
            }
            B += (double)(L.gate->nbytes + L.up->nbytes) + 4.0 * (2 * E + F);
            GemvSegDesc sd{L.down->d, nullptr, (int)L.down->type, E, EPI_ADD, m->x, E, nullptr, nullptr};
            L2Range pf_n[3] = {};
            int npf = 0;
            if (l + 1 < c.n_layers) {
                const Layer &N = m->layers[l + 1];
                pf_n[0] = {N.q->d, (int64_t)N.q->nbytes};
                pf_n[1] = {N.k->d, (int64_t)N.k->nbytes};
                pf_n[2] = {N.v->d, (int64_t)N.v->nbytes};
                npf = 3;
            }
            CK_M(gemv_launch(&sd, 1, m->hb, F, F, 1, nullptr, eps, S, st, pf_n, npf));
            B += (double)L.down->nbytes + 4.0 * (F + 2 * E);
            nl += 4;
        }
        GemvSegDesc so{m->out->d, nullptr, (int)m->out->type, m->out->rows(), EPI_STORE, m->logits, c.vocab, nullptr,
                       m->d_seq};
        CK_M(gemv_launch(&so, 1, m->x, E, E, 1, m->out_nw, eps, S, st));
        B += (double)m->out->nbytes + 4.0 * (2 * E + (double)m->out->rows());
        nl += 1;
        return ACM_OK;
    };
    m->h_seq.p[0] = 0;
    CK_M(cudaMemcpyAsync(m->d_seq, m->h_seq.p, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    int rc;
    if (!m->gemv_bench.exec) {
        if ((rc = ops())) return rc;  // warm-up (kernel attributes) outside capture
        if ((rc = sync_check(m))) return rc;
        const unsigned long long before = g_kernel_launches.load();
        cudaGraph_t g = nullptr;
        CK_M(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = ops();
        cudaError_t ce = cudaStreamEndCapture(st, &g);
        const unsigned long long captured = g_kernel_launches.load() - before;
        g_kernel_launches -= captured;
        if (rc || ce != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return rc ? rc : set_err(m, ACM_ERR_CUDA, "capture failed");
        }
        cudaError_t ie = cudaGraphInstantiate(&m->gemv_bench.exec, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return set_err(m, ACM_ERR_CUDA, "instantiate failed");
        m->gemv_bench.kernels = captured;
    } else {
        // recompute byte/launch counts without launching: run ops under a
        // throwaway capture
        cudaGraph_t g = nullptr;
        const unsigned long long before = g_kernel_launches.load();
        CK_M(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = ops();
        cudaStreamEndCapture(st, &g);
        g_kernel_launches -= g_kernel_launches.load() - before;
        if (g) cudaGraphDestroy(g);
        if (rc) return rc;
    }
    CK_M(cudaGraphLaunch(m->gemv_bench.exec, st));  // warm
    CK_M(cudaEventRecord(m->ev[0], st));
    for (int i = 0; i < reps; i++) CK_M(cudaGraphLaunch(m->gemv_bench.exec, st));
    CK_M(cudaEventRecord(m->ev[1], st));
    if ((rc = sync_check(m))) return rc;
    g_kernel_launches += (unsigned long long)(reps + 1) * m->gemv_bench.kernels;
    if (sec_per_pass) *sec_per_pass = ev_seconds(m->ev[0], m->ev[1]) / reps;
    if (bytes_per_pass) *bytes_per_pass = B;
    if (launches_per_pass) *launches_per_pass = nl;
    return ACM_OK;
}

// ---- kernel-level entry points ----

static int scratch(acm_engine *e, size_t bytes, uint8_t **p) {
    if (e->scratch_bytes < bytes) {
        if (e->scratch) cudaFree(e->scratch);
        e->scratch = nullptr;
        e->scratch_bytes = 0;
        CK_E(cudaMalloc(&e->scratch, bytes));
        e->scratch_bytes = bytes;
    }
    *p = static_cast<uint8_t *>(e->scratch);
    return ACM_OK;
}

static size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

static int scratch2(acm_engine *e, size_t bytes, uint8_t **p) {
    if (e->scratch2_bytes < bytes) {
        if (e->scratch2) cudaFree(e->scratch2);
        e->scratch2 = nullptr;
        e->scratch2_bytes = 0;
        CK_E(cudaMalloc(&e->scratch2, bytes));
        e->scratch2_bytes = bytes;
    }
    *p = static_cast<uint8_t *>(e->scratch2);
    return ACM_OK;
}

ACM_API int acm_dequant(acm_engine *e, uint32_t ggml_type, const void *host_bytes, int64_t nrows, int64_t k,
                        float *host_out) {
    if (!e || !host_bytes || !host_out || nrows <= 0 || k <= 0) return ACM_ERR_INVALID;
    if (!type_ok((int)ggml_type)) return set_eerr(e, ACM_ERR_UNSUPPORTED_TYPE, "unsupported type");
    if (k % 32 || k % blk_elems((int)ggml_type)) return set_eerr(e, ACM_ERR_INVALID, "row length not a multiple of 32");
    cudaSetDevice(e->device);
    const size_t wb = (size_t)nrows * row_bytes((int)ggml_type, k), ob = sizeof(float) * nrows * k;
    uint8_t *s = nullptr;
    int rc = scratch(e, al256(wb + 64) + ob, &s);
    if (rc) return rc;
    float *o = reinterpret_cast<float *>(s + al256(wb + 64));
    CK_E(cudaMemcpyAsync(s, host_bytes, wb, cudaMemcpyHostToDevice, e->stream));
    CK_E(cudaMemsetAsync(s + wb, 0, 64, e->stream));
    CK_E(dequant_launch((int)ggml_type, s, k, nrows, nullptr, nrows, o, k, e->stream));
    CK_E(cudaMemcpyAsync(host_out, o, ob, cudaMemcpyDeviceToHost, e->stream));
    CK_E(cudaStreamSynchronize(e->stream));
    if (read_and_clear_dev_error()) return set_eerr(e, ACM_ERR_TIMEOUT, "device-side error flag set");
    return ACM_OK;
}

ACM_API int acm_matmul_dev(acm_engine *e, uint32_t ggml_type, const void *d_w, int64_t n, int64_t k,
                           const float *d_x, int32_t m, float *d_y) {
    if (!e || !d_w || !d_x || !d_y || n <= 0 || k <= 0 || m <= 0) return ACM_ERR_INVALID;
    if (!type_ok((int)ggml_type)) return set_eerr(e, ACM_ERR_UNSUPPORTED_TYPE, "unsupported type");
    if (k % 32 || k % blk_elems((int)ggml_type)) return set_eerr(e, ACM_ERR_INVALID, "row length not a multiple of 32");
    if (n > INT32_MAX) return set_eerr(e, ACM_ERR_INVALID, "too many rows");
    if (gemv_supported((int)ggml_type, k, m)) {
        GemvSegDesc sg{d_w, nullptr, (int)ggml_type, n, EPI_STORE, d_y, (int)n, nullptr, nullptr};
        CK_E(gemv_launch(&sg, 1, d_x, (int)k, k, m, nullptr, 0.f, e->num_sms, e->stream));
    } else if (k % 256 == 0 && dq_type((int)ggml_type) && mma_available()) {
        // tensor-core path, W dequantized in the kernel: split x only
        const size_t xbs = al256((size_t)rows64(m) * k * 2);
        const size_t wsf = std::min<size_t>(4 * (size_t)m * n, (size_t)148 * 128 * 64);
        uint8_t *s2 = nullptr;
        if (int rc = scratch2(e, 2 * xbs + wsf * 4, &s2)) return rc;
        uint8_t *xhi = s2, *xlo = s2 + xbs;
        float *ws = reinterpret_cast<float *>(xlo + xbs);
        CK_E(split_act_launch(d_x, (int)k, m, (int)k, xhi, xlo, e->stream));
        TensorMap mxh, mxl;
        if (!bf16_map(&mxh, xhi, m, k) || !bf16_map(&mxl, xlo, m, k))
            return set_eerr(e, ACM_ERR_CUDA, "tensor map encoding failed");
        MmaGemmSeg sg{nullptr, nullptr, nullptr, nullptr, n, EPI_STORE, d_y, (int)n, nullptr, nullptr,
                      d_w, nullptr, (int)ggml_type};
        CK_E(mma_dq_launch(&sg, 1, &mxh, &mxl, m, (int)k, e->stream, ws, wsf));
    } else if (k % 64 == 0 && mma_available()) {
        // tensor-core path: split W and x to bf16 hi/lo in the second scratch
        const size_t wbs = al256((size_t)rows64(n) * k * 2), xbs = al256((size_t)rows64(m) * k * 2);
        // split-K partial sums: split-K runs only when the tiles fill at most
        // half the SMs, so ks * m * n stays within 148 tiles of 128 x 64
        const size_t wsf = std::min<size_t>(4 * (size_t)m * n, (size_t)148 * 128 * 64);
        uint8_t *s2 = nullptr;
        if (int rc = scratch2(e, 2 * wbs + 2 * xbs + wsf * 4, &s2)) return rc;
        uint8_t *whi = s2, *wlo = s2 + wbs, *xhi = s2 + 2 * wbs, *xlo = xhi + xbs;
        float *ws = reinterpret_cast<float *>(xlo + xbs);
        CK_E(split_weight_launch((int)ggml_type, d_w, n, (int)k, whi, wlo, e->stream));
        CK_E(split_act_launch(d_x, (int)k, m, (int)k, xhi, xlo, e->stream));
        TensorMap mwh, mwl, mxh, mxl;
        if (!bf16_map(&mwh, whi, n, k) || !bf16_map(&mwl, wlo, n, k) || !bf16_map(&mxh, xhi, m, k) ||
            !bf16_map(&mxl, xlo, m, k))
            return set_eerr(e, ACM_ERR_CUDA, "tensor map encoding failed");
        MmaGemmSeg sg{&mwh, &mwl, nullptr, nullptr, n, EPI_STORE, d_y, (int)n, nullptr, nullptr};
        CK_E(mma_gemm_launch(&sg, 1, &mxh, &mxl, m, (int)k, e->stream, ws, wsf));
    } else {
        CK_E(gemm_launch({d_w, nullptr, (int)ggml_type, n, k, m, d_x, (int)k, d_y, (int)n, EPI_STORE, nullptr, nullptr},
                         e->stream));
    }
    return ACM_OK;
}

ACM_API int acm_bench_matmul(acm_engine *e, uint32_t ggml_type, const void *d_w, int64_t w_stride, int32_t copies,
                             int64_t n, int64_t k, const float *d_x, int32_t m, float *d_y, int32_t reps,
                             double *sec_per_call) {
    if (!e || !d_w || !sec_per_call || copies <= 0 || reps <= 0 || w_stride < 0 || w_stride % 256)
        return ACM_ERR_INVALID;
    if (copies > 1 && w_stride < (int64_t)n * row_bytes((int)ggml_type, k) + 16)
        return set_eerr(e, ACM_ERR_INVALID, "weight copies overlap");
    cudaSetDevice(e->device);
    const uint8_t *w0 = static_cast<const uint8_t *>(d_w);
    for (int i = 0; i < copies; i++)  // untimed pass over every copy
        if (int rc = acm_matmul_dev(e, ggml_type, w0 + (int64_t)i * w_stride, n, k, d_x, m, d_y)) return rc;
    cudaEvent_t ev[2];
    CK_E(cudaEventCreate(&ev[0]));
    if (cudaEventCreate(&ev[1]) != cudaSuccess) {
        cudaEventDestroy(ev[0]);
        return set_eerr(e, ACM_ERR_CUDA, "cudaEventCreate failed");
    }
    int rc = ACM_OK;
    float ms = 0.f;
    if (cudaEventRecord(ev[0], e->stream) != cudaSuccess) rc = set_eerr(e, ACM_ERR_CUDA, "cudaEventRecord failed");
    for (int i = 0; i < reps && rc == ACM_OK; i++)
        rc = acm_matmul_dev(e, ggml_type, w0 + (int64_t)(i % copies) * w_stride, n, k, d_x, m, d_y);
    if (rc == ACM_OK && (cudaEventRecord(ev[1], e->stream) != cudaSuccess || cudaEventSynchronize(ev[1]) != cudaSuccess ||
                         cudaEventElapsedTime(&ms, ev[0], ev[1]) != cudaSuccess))
        rc = set_eerr(e, ACM_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    cudaEventDestroy(ev[0]);
    cudaEventDestroy(ev[1]);
    if (rc == ACM_OK) *sec_per_call = 1e-3 * ms / reps;
    return rc;
}

ACM_API int acm_matmul(acm_engine *e, uint32_t ggml_type, const void *host_w, int64_t n, int64_t k,
                       const float *host_x, int32_t m, float *host_y) {
    if (!e || !host_w || !host_x || !host_y || n <= 0 || k <= 0 || m <= 0) return ACM_ERR_INVALID;
    if (!type_ok((int)ggml_type)) return set_eerr(e, ACM_ERR_UNSUPPORTED_TYPE, "unsupported type");
    if (k % 32 || k % blk_elems((int)ggml_type)) return set_eerr(e, ACM_ERR_INVALID, "row length not a multiple of 32");
    cudaSetDevice(e->device);
    const size_t wb = (size_t)n * row_bytes((int)ggml_type, k), xb = sizeof(float) * m * k, yb = sizeof(float) * m * n;
    uint8_t *s = nullptr;
    int rc = scratch(e, al256(wb + 64) + al256(xb) + yb, &s);
    if (rc) return rc;
    float *dx = reinterpret_cast<float *>(s + al256(wb + 64));
    float *dy = reinterpret_cast<float *>(s + al256(wb + 64) + al256(xb));
    CK_E(cudaMemcpyAsync(s, host_w, wb, cudaMemcpyHostToDevice, e->stream));
    CK_E(cudaMemsetAsync(s + wb, 0, 64, e->stream));
    CK_E(cudaMemcpyAsync(dx, host_x, xb, cudaMemcpyHostToDevice, e->stream));
    if ((rc = acm_matmul_dev(e, ggml_type, s, n, k, dx, m, dy))) return rc;
    CK_E(cudaMemcpyAsync(host_y, dy, yb, cudaMemcpyDeviceToHost, e->stream));
    CK_E(cudaStreamSynchronize(e->stream));
    if (read_and_clear_dev_error()) return set_eerr(e, ACM_ERR_TIMEOUT, "a device-side wait timed out");
    return ACM_OK;
}

ACM_API int acm_sample_logits(acm_engine *e, const float *host_logits, int32_t n, const acm_sampler *s,
                              uint64_t step, int32_t *tok_out) {
    if (!e || !host_logits || n <= 0 || !tok_out) return ACM_ERR_INVALID;
    cudaSetDevice(e->device);
    const int nchunks = (n + 2047) / 2048;
    const size_t lb = al256(sizeof(float) * n), cb = al256(sizeof(uint64_t) * nchunks * 64);
    uint8_t *p = nullptr;
    int rc = scratch(e, lb + cb + 256 * 8, &p);
    if (rc) return rc;
    float *dl = reinterpret_cast<float *>(p);
    uint64_t *cand = reinterpret_cast<uint64_t *>(p + lb);
    uint8_t *par = p + lb + cb;
    double *temp = reinterpret_cast<double *>(par);
    double *topp = temp + 1;
    uint64_t *seed = reinterpret_cast<uint64_t *>(par + 16), *stp = seed + 1;
    int32_t *topk = reinterpret_cast<int32_t *>(par + 32), *out = topk + 1;
    uint8_t hostpar[64] = {};
    const double tv = s ? s->temp : 0.0, pv = s ? s->top_p : 0.0;
    const uint64_t sv = s ? s->seed : 0;
    const int32_t kv = s ? s->top_k : 0;
    memcpy(hostpar, &tv, 8);
    memcpy(hostpar + 8, &pv, 8);
    memcpy(hostpar + 16, &sv, 8);
    memcpy(hostpar + 24, &step, 8);
    memcpy(hostpar + 32, &kv, 4);
    CK_E(cudaMemcpyAsync(dl, host_logits, sizeof(float) * n, cudaMemcpyHostToDevice, e->stream));
    CK_E(cudaMemcpyAsync(par, hostpar, 40, cudaMemcpyHostToDevice, e->stream));
    SampleDesc sd{dl, nullptr, n, n, temp, topk, topp, seed, stp, out, cand, nchunks};
    CK_E(sample_launch(sd, 1, !s || s->temp <= 0, e->stream));
    int32_t res = -1;
    CK_E(cudaMemcpyAsync(&res, out, sizeof(int32_t), cudaMemcpyDeviceToHost, e->stream));
    CK_E(cudaStreamSynchronize(e->stream));
    *tok_out = res;
    return ACM_OK;
}

}  // extern "C"

namespace acm {
int sample_noalloc(int dev, cudaStream_t st, const float *d_logits, int64_t ld, int nrows, int vocab,
                   const acm_sampler *samplers, const uint64_t *steps, int32_t *d_out, std::string *err);
}

extern "C" {

// The sampler on device logits with its scratch in a fixed buffer of the
// library image (k_noalloc.cu): nothing is allocated, nothing is copied back,
// nothing waits; the ids land in d_out when the engine stream reaches them.
ACM_API int acm_sample_dev_noalloc(acm_engine *e, const float *d_logits, int64_t ld, int32_t nrows, int32_t vocab,
                                   const acm_sampler *samplers, const uint64_t *steps, int32_t *d_out) {
    if (!e) return ACM_ERR_INVALID;
    CK_E(cudaSetDevice(e->device));
    std::string msg;
    const int rc = acm::sample_noalloc(e->device, e->stream, d_logits, ld, nrows, vocab, samplers, steps, d_out, &msg);
    if (rc == 0) return ACM_OK;
    return set_eerr(e, rc == 1 ? ACM_ERR_INVALID : ACM_ERR_CUDA, msg);
}

}  // extern "C"
