// kernels.h -- launch interfaces of the engine's CUDA kernels (host side).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <vector>

namespace acm {

// Device error flag values (set by kernels, read by the host after a sync).
enum : int { DEV_ERR_NONE = 0, DEV_ERR_TIMEOUT = 1, DEV_ERR_BOUNDS = 2 };

// Programmatic dependent launch on the decode path (env ACM_PDL=0 disables).
extern bool g_pdl;

// Epilogues shared by the GEMV and GEMM kernels.
enum : int {
    EPI_STORE = 0,   // y = W x (+ bias)
    EPI_ADD = 1,     // y += W x          (residual update, model.go:411-413, :424-426)
    EPI_SWIGLU = 2,  // y = silu(Wg x) * (Wu x)   (model.go:420-422)
};

// One weight matrix (or gate/up pair) of a multi-segment GEMV launch.
struct GemvSeg {
    const uint8_t *w, *w2;  // tensor bytes (w2: up-projection of a SwiGLU pair)
    int64_t rb, rb2;        // row bytes
    int type;               // ggml type (w2 has the same type)
    int n;                  // rows
    int cta0, ncta;         // this segment's CTA range
    int rows_per_stage;
    int epi;
    float *y;               // output [m][ldy]
    int ldy;
    const float *bias;      // optional, n floats
    const int32_t *yrow;    // optional: output row of token m (default m)
    unsigned long long *amax;  // optional: per-token running argmax key (greedy sampling)
};

constexpr int GEMV_MAX_SEG = 4;
constexpr int GEMV_NS_MAX = 8;

// An HBM range pulled into L2 ahead of its use: the weights of the next
// matvec, prefetched by this one's producer warps (split across its CTAs), so
// the next kernel's first stages come from L2 instead of DRAM.
struct L2Range {
    const void *p;
    int64_t bytes;
};
constexpr int GEMV_MAX_PF = 3;

struct GemvArgs {
    GemvSeg seg[GEMV_MAX_SEG];
    int nseg;
    const float *x;      // activations [m][ldx] (fp32)
    int ldx;
    int k;
    int m;
    const float *norm_w; // optional RMSNorm weight applied to x in the prologue
    float eps;
    int ns;              // pipeline stages
    int stage_bytes;
    int stage_off;       // byte offset of the stage ring in shared memory
    int lpr;             // 0: one row per warp (unit path); else lanes per row (wide path)
    L2Range pf[GEMV_MAX_PF];
    int npf;
};

struct GemvSegDesc {
    const void *w, *w2;
    int type;
    int64_t n;
    int epi;
    float *y;
    int ldy;
    const float *bias;
    const int32_t *yrow;
    unsigned long long *amax;
};
// Plans CTA ranges / stages and launches (possibly several launches when the
// segments' types have no common kernel instance).  Returns a cudaError_t.
cudaError_t gemv_launch(const GemvSegDesc *segs, int nseg, const float *x, int ldx, int64_t k, int m,
                        const float *norm_w, float eps, int num_sms, cudaStream_t st, const L2Range *pf = nullptr,
                        int npf = 0);
bool gemv_supported(int type, int64_t k, int m);

// Prefill / batched GEMM: y[m][n] (epi) x[m][k] . W[n][k]^T.
struct GemmDesc {
    const void *w, *w2;
    int type;
    int64_t n, k;
    int m;
    const float *x;
    int ldx;
    float *y;
    int ldy;
    int epi;
    const float *bias;
    const int32_t *yrow;    // optional: output row of token m (default m)
};
cudaError_t gemm_launch(const GemmDesc &d, cudaStream_t st);

// ---------------------------------------------------------------------------
// Tensor-core GEMM (k_mma.cu): bf16 hi/lo split operands, three tcgen05 MMAs
// per K step, fp32 accumulation in TMEM.
struct alignas(64) TensorMap {
    uint64_t w[16];  // CUtensorMap
};
bool mma_available();
// Split operands are stored 64x64-blocked; buffers hold ceil(rows/64)*64 rows.
// Tensor map over such a [rows][k] buffer for the GEMM's 64x64 boxes.
bool bf16_map(TensorMap *map, const void *base, int64_t rows, int64_t k);
inline int64_t rows64(int64_t rows) { return (rows + 63) / 64 * 64; }
// fp32 [m][ldx] -> bf16 hi, lo (blocked)
cudaError_t split_act_launch(const float *x, int ldx, int m, int k, void *hi, void *lo, cudaStream_t st);
// x[m][k] += the ks partial sums of ws (a deferred split-K reduce, EPI_ADD),
// then RMSNorm and split of the rows, in one launch
cudaError_t split_act_reduce_norm_launch(const float *ws, int ks, int m, float *x, int k, const float *norm_w,
                                         float eps, void *hi, void *lo, cudaStream_t st);
// RMSNorm of each row (weight norm_w) and its split in one launch
cudaError_t split_act_norm_launch(const float *x, int ldx, int m, int k, const float *norm_w, float eps, void *hi,
                                  void *lo, cudaStream_t st);
// exact dequant of W [n][k] -> bf16 hi, lo (blocked)
cudaError_t split_weight_launch(int type, const void *w, int64_t n, int k, void *hi, void *lo, cudaStream_t st);
struct MmaGemmSeg {
    const TensorMap *map_hi, *map_lo;    // W split cache
    const TensorMap *map_hi2, *map_lo2;  // SwiGLU pair: up-projection (else null)
    int64_t n;                           // rows (a multiple of 64 for pairs)
    int epi;
    float *y;
    int ldy;
    const float *bias;
    const int32_t *yrow;
    // the weights as GGUF rows, for mma_dq_launch (dequantized in the kernel)
    const void *w = nullptr, *w2 = nullptr;
    int wtype = -1;
};
// ws (optional, ws_floats floats): workspace for split-K partial sums, used
// when the output tiles would leave most SMs idle.
cudaError_t mma_gemm_launch(const MmaGemmSeg *segs, int nseg, const TensorMap *x_hi, const TensorMap *x_lo, int m,
                            int k, cudaStream_t st, float *ws = nullptr, size_t ws_floats = 0);
// Batched form: n independent GEMMs of the same shape (one segment) whose
// operands follow each other in the split buffers (a_stride / b_stride: the
// per-batch offset in 64-element box rows, i.e. rows64(rows) * k / 64); the
// output row of token tok of batch b is (rmod ? (tok % rmod) * rmul +
// (tok / rmod) * rdiv : tok) + b * rbatch.
struct MmaBatch {
    int n = 1;
    int a_stride = 0, b_stride = 0;
    int rmod = 0, rmul = 0, rdiv = 0, rbatch = 0;
    // causal attention (token tok is query row tok % cntok at position
    // cpos0 + tok % cntok, attending keys 0 .. that position): 1 -- the
    // weight rows are keys (S = Q.K^T), tiles whose keys are all masked are
    // skipped (their scores are never read); 2 -- K runs over keys (O = P.V),
    // each tile stops after its last attended key (P is zero beyond it)
    int causal = 0, cntok = 0, cpos0 = 0;
};
cudaError_t mma_gemm_batched_launch(const MmaGemmSeg *segs, int nseg, const TensorMap *x_hi, const TensorMap *x_lo,
                                    int m, int k, const MmaBatch &bt, cudaStream_t st, float *ws = nullptr,
                                    size_t ws_floats = 0);

// Tensor-core GEMM with the weights dequantized in shared memory (k_mma_dq.cu):
// the segments' w / w2 / wtype (one quantized type, or Q4_K with Q6_K), K a
// multiple of 256; otherwise as mma_gemm_launch.
bool dq_type(int t);
// defer_ks: when the launch splits K, leave the reduce to the caller and
// report the slice count (0: no split, the outputs are written).
cudaError_t mma_dq_launch(const MmaGemmSeg *segs, int nseg, const TensorMap *x_hi, const TensorMap *x_lo, int m, int k,
                          cudaStream_t st, float *ws = nullptr, size_t ws_floats = 0, int *defer_ks = nullptr);
// Split-K epilogue: y[tok][n] (epi)= bias[n] + the ks partial sums of ws, in order.
cudaError_t split_reduce_launch(const float *ws, int ks, int m, int n, float *y, int ldy, int epi, const float *bias,
                                const int32_t *yrow, cudaStream_t st);

// Prefill attention on the tensor cores: operand preparation (k_attn_split)
// and the softmax between S = Q.K^T and O = P.V (k_attn_softmax).
struct AttnMmaOps {
    const float *q, *kc, *vc;  // kc, vc: fp16 elements when kv_f16
    int kv_f16;
    const int32_t *page_row;
    int64_t layer_off;
    int page_size, kvd, ntok, L, Lp, G, nh, hd, nkv, pos0;
    int64_t rq;            // rows64(G * ntok)
    float scale;
    void *qh, *ql, *kh, *kl, *vh, *vl, *ph, *pl;
    const float *S;        // [nkv][G*ntok][Lp] scores
};
cudaError_t attn_split_launch(const AttnMmaOps &o, cudaStream_t st);
cudaError_t attn_softmax_launch(const AttnMmaOps &o, cudaStream_t st);

// Dequantize rows (exact): rows either consecutive (row_ids == nullptr) or
// gathered by id (embedding lookup, model.go:338-340).
cudaError_t dequant_launch(int type, const void *w, int64_t k, int64_t nrows, const int32_t *row_ids,
                           int64_t src_rows, float *out, int64_t ldo, cudaStream_t st);

// RMSNorm of m rows (model.go:213-222): y = x * scale * w.
cudaError_t rmsnorm_launch(const float *x, int ldx, const float *w, float *y, int ldy, int m, int n, float eps,
                           cudaStream_t st);

// Per-token metadata of a token batch.
struct TokMeta {
    const int32_t *seq;   // sequence slot of each token
    const int32_t *pos;   // position of each token
};

// Paged KV cache geometry.
struct KVDesc {
    float *k, *v;               // pools [layer][page][page_size][kvd]; fp16 elements when f16
    const int32_t *page_table;  // [max_seqs][max_pages]
    int max_pages;
    int page_size;              // positions per page (power of two)
    int64_t layer_stride;       // elements per layer in each pool
    int kvd;
    int f16;                    // 1: the pools hold IEEE half (reduced-precision cache), 0: fp32
};

// QK-norm + RoPE on q (in place) and k, then append k, v to the cache
// (model.go:362-382).
struct RopeDesc {
    float *q;          // [ntok][qd]
    const float *k, *v;// [ntok][kvd]
    const float *q_nw, *k_nw;  // optional per-head RMSNorm weights
    const float2 *tab; // [max_ctx][rope_dim/2] (cos, sin)
    int n_head, n_head_kv, head_dim, rope_dim, interleaved;
    float eps;
};
cudaError_t rope_append_launch(const RopeDesc &r, const KVDesc &kv, int layer, TokMeta tm, int ntok,
                               cudaStream_t st);

// Attention over the paged cache (model.go:384-408).
struct AttnDesc {
    const float *q;   // [ntok][qd]
    float *out;       // [ntok][qd]
    int n_head, n_head_kv, head_dim;
    float scale;
    float *part;      // split partials [ntok][n_head][nsplit][head_dim + 2]
    int nsplit;
    int *counter;     // [ntok][n_head] split-arrival counters (decode kernel), one per item head subset
    int min_items;    // decode kernel: smallest head subsets only while items < min_items (0: largest)
};
cudaError_t attention_launch(const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm, int ntok, int max_pos,
                             cudaStream_t st);
// Prefill attention for a batch of consecutive positions of one sequence
// (tiled over query tokens, two passes so the softmax weights are the
// reference's fastExp(s - max)).
cudaError_t attention_prefill_launch(const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm, int ntok,
                                     cudaStream_t st);
// Decode attention for a batch of tokens of distinct sequences with the
// QK-norm / RoPE / KV append of the new token fused in, and the split merge
// done by the last split of each (token, kv head).
cudaError_t attention_decode_launch(const RopeDesc &r, const AttnDesc &a, const KVDesc &kv, int layer, TokMeta tm,
                                    int ntok, int max_pos, cudaStream_t st);

// y = silu(g) * u elementwise (fallback when gate and up differ in type).
cudaError_t swiglu_launch(const float *g, const float *u, float *y, int64_t n, cudaStream_t st);

// Sampler (sampler.go:19-98) over logits rows.
struct SampleDesc {
    const float *logits;
    const int32_t *rows;     // logits row of token t (default t)
    int64_t ld;
    int vocab;
    const double *temp;      // per token
    const int32_t *top_k;
    const double *top_p;
    const uint64_t *seed;
    const uint64_t *step;
    int32_t *out;            // sampled ids [ntok]
    uint64_t *cand;          // scratch [ntok][nchunks][64]
    int nchunks;
};
cudaError_t sample_launch(const SampleDesc &s, int ntok, bool all_greedy, cudaStream_t st);

// After a decode step: next input = sampled id (or, when amax is given, the
// argmax the lm_head epilogue accumulated, which is then cleared), position
// + 1, step + 1, and the id recorded in hist[t][hist_col].
cudaError_t advance_launch(int32_t *tok, int32_t *pos, uint64_t *step, int32_t *out, unsigned long long *amax,
                           int32_t *hist, int hist_ld, int32_t *hist_col, int ntok, cudaStream_t st);


// Device error flag (timeouts in bounded waits).
int read_and_clear_dev_error();
// Polls a bounded mbarrier wait makes before it records a timeout (the
// device default is WAIT_LIMIT of common.cuh); applies to the current device.
cudaError_t set_wait_limit(uint32_t polls);
constexpr uint32_t WAIT_LIMIT_DEFAULT = 1u << 22;

// Batch-1 decode GEMV (k_gemv1.cu): activations in registers, lean CTAs.
bool gemv1_supported(int type, int64_t k);
cudaError_t gemv1_launch(const GemvSegDesc *segs, int nseg, const float *x, int64_t k, const float *norm_w,
                         float eps, int num_sms, cudaStream_t st, const L2Range *pf = nullptr, int npf = 0);
// Per-CTA timelines of batch-1 GEMV launches (profiling): launches planned
// while buf is set take consecutive slots of 160 CTAs x 8 stamps; null: off.
void gemv1_trace(unsigned long long *buf, int slots);
int gemv1_trace_used();

// Count of kernels this library has launched (graph replays add the kernels
// the graph holds); every launcher returns through launched().
extern std::atomic<unsigned long long> g_kernel_launches;
inline cudaError_t launched(int n) {
    g_kernel_launches += (unsigned long long)n;
    return cudaGetLastError();
}

}  // namespace acm
