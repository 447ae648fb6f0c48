/*
 * acm.h -- C ABI of libacmcuda.so, the B200 engine for auto-commit-msg's
 * token loop (load GGUF -> prefill -> decode with the top-k sampler).
 *
 * These are the entry points a cgo shim behind a `cuda` build tag in
 * internal/infer binds.  Each declaration names the reference interface it
 * replaces (paths are inside the auto-commit-msg tree).
 *
 * Conventions
 *  - Every call returns an int status (ACM_OK = 0).  On failure the message is
 *    available from acm_last_error(); the process is never aborted.
 *  - Host pointers are borrowed for the duration of the call only.
 *  - The library owns all device memory (weights, paged KV cache, activations,
 *    logits).  A model is driven by one host thread at a time; separate models
 *    (e.g. one per GPU) may be driven concurrently from separate threads.
 */
#ifndef ACM_H
#define ACM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ACM_API __attribute__((visibility("default")))

enum acm_status {
    ACM_OK = 0,
    ACM_ERR_INVALID = 1,          /* bad argument / state */
    ACM_ERR_CTX_EXCEEDED = 2,     /* model.go:320-321 "context length exceeded" */
    ACM_ERR_UNSUPPORTED_ARCH = 3, /* model.go:95 */
    ACM_ERR_UNSUPPORTED_TYPE = 4, /* gguf.go:164, tensor.go:79 */
    ACM_ERR_MISSING_TENSOR = 5,   /* model.go:136, :165, :198 */
    ACM_ERR_OOM = 6,
    ACM_ERR_CUDA = 7,
    ACM_ERR_TIMEOUT = 8,
    ACM_ERR_NO_SEQ = 9,
    ACM_ERR_IO = 10,
    ACM_ERR_FORMAT = 11            /* gguf.go:123-170 parse errors */
};

/* ggml tensor types accepted (gguf.go:31-40). */
enum acm_ggml_type {
    ACM_F32 = 0, ACM_F16 = 1, ACM_Q4_0 = 2, ACM_Q5_0 = 6, ACM_Q8_0 = 8,
    ACM_Q4_K = 12, ACM_Q5_K = 13, ACM_Q6_K = 14
};

enum acm_arch { ACM_ARCH_QWEN3 = 0, ACM_ARCH_QWEN2 = 1, ACM_ARCH_LLAMA = 2 };
enum acm_rope_scaling { ACM_ROPE_NONE = 0, ACM_ROPE_LINEAR = 1, ACM_ROPE_LLAMA3 = 2 };

/* Model hyper-parameters: infer.Config, internal/infer/model.go:14-40. */
typedef struct acm_config {
    int32_t arch;
    int32_t n_layers, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab, max_ctx, rope_dim;
    float rope_base;
    int32_t rope_interleaved;
    int32_t rope_scaling;
    float rope_factor, rope_lo_f, rope_hi_f, rope_orig_ctx;
    float rms_eps;
    int32_t bos, eos, eos2;
} acm_config;

/* infer.Sampler (sampler.go:12-17).  The reference draws from a time-seeded
 * PCG (internal/app/rand.go:10-13); here the uniform draw of decode step
 * `step` is Philox4x32-10 keyed by `seed`, so runs are reproducible. */
typedef struct acm_sampler {
    double temp;   /* <= 0: greedy */
    int32_t top_k; /* 0: 64 candidates */
    double top_p;  /* only applied when 0 < top_p < 1 */
    uint64_t seed;
} acm_sampler;

/* infer.Stats (sampler.go:101-106); durations in seconds. */
typedef struct acm_stats {
    int64_t prefill_toks;
    double prefill_s;
    int64_t decode_toks;
    double decode_s;
} acm_stats;

typedef struct acm_engine acm_engine; /* one CUDA device + stream */
typedef struct acm_model acm_model;   /* weights + paged KV + sequence slots */

/* Library version string. */
ACM_API const char *acm_version(void);

/* Open a device.  No reference counterpart (the reference is CPU-only). */
ACM_API int acm_open(int device, acm_engine **out);
ACM_API int acm_close(acm_engine *e);
ACM_API const char *acm_engine_error(acm_engine *e);

/* No counterpart in the reference (its cache is fp32, model.go:353-360).
 * Models created on this engine after the call keep their KV cache in IEEE
 * half instead of fp32 (enable != 0): half the cache's HBM bytes and traffic,
 * at the cost of rounding every cached key and value to 11 significant bits
 * (the appended position is rounded before its own step uses it, so a
 * position reads the same values in every step).  Logits then differ from
 * the reference's fp32 path by more than rounding order; the measured
 * deviation is stated with the tests that check it.  Default: fp32. */
ACM_API int acm_engine_set_kv_f16(acm_engine *e, int32_t enable);

/* Failure detection, no reference counterpart.  Every device-side wait of
 * the library's kernels (a weight stage landing, a pipeline slot freed) is
 * bounded: after `polls` unsuccessful tests it records a timeout, lets the
 * copies it started land, and returns, and the next call that synchronises
 * reports ACM_ERR_TIMEOUT ("a device-side wait timed out") instead of
 * hanging.  This sets the bound for the engine's device (polls < 0: the
 * default, ~2^22 polls, seconds; 0: every wait that does not find its data
 * already there gives up at once, which is how the tests make a wait run
 * out).  It applies to kernels launched after the call, on every engine of
 * that device. */
ACM_API int acm_engine_set_wait_limit(acm_engine *e, int64_t polls);

/* Create an empty model for `cfg`; replaces infer.Load's allocation part
 * (model.go:90-203).  max_seqs concurrent sequence slots, each up to
 * cfg->max_ctx positions. */
ACM_API int acm_model_create(acm_engine *e, const acm_config *cfg, int32_t max_seqs, acm_model **out);

/* Copy one GGUF tensor's bytes UNCHANGED to HBM (the blocks stay in ggml
 * layout: the decode matvecs read them as they are, and the tensor-core GEMM
 * of prefill dequantizes them in shared memory; only F16/F32 linear weights,
 * or quantized ones whose K is not a multiple of 256, get a bf16 hi/lo copy
 * built on first use).  dims[0] is the
 * innermost dimension as in gguf.Tensor.Dims (gguf.go:42-49).  host_bytes may
 * point into an mmap and is not retained. */
ACM_API int acm_model_add_tensor(acm_model *m, const char *name, uint32_t ggml_type, const uint64_t *dims,
                                 int32_t ndims, const void *host_bytes, size_t nbytes);

/* Bind tensors to layers and build the RoPE tables; the tensor checks of
 * infer.Load (model.go:161-201) with the same error texts. */
ACM_API int acm_model_finalize(acm_model *m);
ACM_API int acm_model_destroy(acm_model *m);
ACM_API const char *acm_last_error(acm_model *m);
ACM_API int acm_model_config(acm_model *m, acm_config *out);

/* Load a GGUF file (mmap, gguf.Parse gguf.go:121-174 and infer.Load
 * model.go:90-203) and upload it: the host path a C or Python caller uses.
 * max_ctx <= 0 or above the file's context_length selects the file's value. */
ACM_API int acm_model_load_gguf(acm_engine *e, const char *path, int32_t max_ctx, int32_t max_seqs,
                                acm_model **out);

/* acm_model_load_gguf over a GGUF image already in host memory (an mmap, or
 * bytes embedded in the binary as the reference's fat build does,
 * app/app.go:77-89): the same parse, rules and upload; `data` is not retained.
 * Replaces infer.Load(gguf.Parse(data), maxCtx) (model.go:90-203) for a host
 * that holds the file's bytes. */
ACM_API int acm_model_load_gguf_mem(acm_engine *e, const void *data, size_t nbytes, int32_t max_ctx,
                                    int32_t max_seqs, acm_model **out);

/* One model per engine from one mapping of the file (no reference
 * counterpart; the reference maps the file once per process,
 * app/model_unix.go:15-34): parsed once, every staging chunk filled once on
 * the host and copied to each engine's device (engines may share a device).
 * outs[i] is created on es[i]; on failure none is left and es[0] holds the
 * error.  1 <= n <= 64. */
ACM_API int acm_model_load_gguf_multi(acm_engine *const *es, int32_t n, const char *path, int32_t max_ctx,
                                      int32_t max_seqs, acm_model **outs);

/* Parse a GGUF file and derive its configuration without touching a device:
 * gguf.Parse (gguf.go:121-174) plus the metadata rules of infer.Load
 * (model.go:91-151).  err receives a message on failure. */
ACM_API int acm_load_config(const char *path, int32_t max_ctx, acm_config *out, char *err, int32_t errlen);
/* acm_load_config over a GGUF image in host memory. */
ACM_API int acm_load_config_mem(const void *data, size_t nbytes, int32_t max_ctx, acm_config *out, char *err,
                                int32_t errlen);

/* Sequence slots.  A slot is one infer.Model's sequence state (pos + KV). */
ACM_API int acm_seq_open(acm_model *m, int32_t *seq_out);
ACM_API int acm_seq_close(acm_model *m, int32_t seq);
/* Model.Reset, model.go:458-460: rewind to position 0 (KV pages are kept). */
ACM_API int acm_seq_reset(acm_model *m, int32_t seq);
/* Model.Pos, model.go:455-456. */
ACM_API int acm_seq_pos(acm_model *m, int32_t seq, int32_t *pos_out);

/* Model.Forward, model.go:315-442: evaluate n tokens at consecutive positions
 * of `seq`; the last token's logits stay on the device for acm_sample and are
 * copied to logits_out (vocab floats) when it is non-NULL. */
ACM_API int acm_forward(acm_model *m, int32_t seq, const int32_t *toks, int32_t n, float *logits_out);

/* Sampler.Sample, sampler.go:30-76, on the device-resident logits of `seq`
 * with the uniform draw of decode step `step`. */
ACM_API int acm_sample(acm_model *m, int32_t seq, const acm_sampler *s, uint64_t step, int32_t *tok_out);

/* One batched decode step for nseq independent sequences: Forward([in_tok[i]])
 * on seqs[i], then Sample on the new logits with samplers[i] at steps[i].
 * Writes the sampled ids to out_tok (and, when logits_out is non-NULL, the
 * nseq x vocab logits).  The batched form of the loop body in sampler.go:136-157. */
ACM_API int acm_decode_step(acm_model *m, int32_t nseq, const int32_t *seqs, const int32_t *in_tok,
                            const acm_sampler *samplers, const uint64_t *steps, int32_t *out_tok,
                            float *logits_out);

/* Model.Generate, sampler.go:108-157: prefill in chunks of <= 1024 then decode
 * until EOS/EOS2 (stop_on_eos != 0) or max_tok tokens.  out_ids needs max_tok
 * entries; *n_out receives the count.  stats may be NULL. */
ACM_API int acm_generate(acm_model *m, int32_t seq, const int32_t *prompt, int32_t n_prompt,
                         const acm_sampler *s, int32_t max_tok, int32_t stop_on_eos, int32_t *out_ids,
                         int32_t *n_out, acm_stats *stats);

/* One request of acm_serve: a prompt and its sampler; out_ids (max_tok
 * entries) receives the generated ids, n_out their count, status ACM_OK or
 * the request's own error (ACM_ERR_CTX_EXCEEDED, ACM_ERR_INVALID). */
typedef struct acm_request {
    const int32_t *prompt;
    int32_t n_prompt;
    acm_sampler sampler;
    int32_t max_tok;
    int32_t *out_ids;
    int32_t n_out;
    int32_t status;
} acm_request;

/* Continuous batching, no reference counterpart (the reference serves one
 * prompt per process): runs every request through Generate's loop
 * (sampler.go:108-157, the same draws as acm_generate) with up to max_batch
 * of them (<= the model's sequence slots) sharing each decode step; new
 * requests are prefilled into slots as others finish.  stats: prefill and
 * decode tokens and device seconds summed over all requests. */
ACM_API int acm_serve(acm_model *m, acm_request *reqs, int32_t n, int32_t max_batch, int32_t stop_on_eos,
                      acm_stats *stats);

/* MaxLogit, model.go:462-471 (host helper, first maximum wins). */
ACM_API int32_t acm_max_logit(const float *logits, int32_t n);

/* ---- kernel-level entry points (parity tests and the kernel bench) ---- */

/* Dequantize nrows rows of K elements with the device dequantizer
 * (dequantRowSlow, tensor.go:55-81); host buffers in and out. */
ACM_API int acm_dequant(acm_engine *e, uint32_t ggml_type, const void *host_bytes, int64_t nrows, int64_t k,
                        float *host_out);

/* matmul / matvec (tensor.go:253-303): y[m][n] = x[m][:] . W[n][:] with the
 * engine's kernels (fused dequant-GEMV for m <= 8, dequant-GEMM otherwise);
 * host buffers in and out. */
ACM_API int acm_matmul(acm_engine *e, uint32_t ggml_type, const void *host_w, int64_t n, int64_t k,
                       const float *host_x, int32_t m, float *host_y);

/* The same on device pointers, enqueued on the engine stream (no copies, no
 * synchronisation).  d_w must hold the tensor bytes at a 256-byte aligned
 * address followed by at least 16 readable bytes. */
ACM_API int acm_matmul_dev(acm_engine *e, uint32_t ggml_type, const void *d_w, int64_t n, int64_t k,
                           const float *d_x, int32_t m, float *d_y);

/* Kernel bench of acm_matmul_dev, the measurement of the reference's
 * matvec bench (internal/infer/mvbench_test.go:12-33; GB/s = weight bytes
 * over the time of one call, :30): `copies` copies of the weight tensor
 * lie at d_w + i * w_stride (w_stride a multiple of 256; the copies together
 * larger than L2, so that every call reads its weights from HBM).  One
 * untimed call per copy, then `reps` calls back to back on the engine stream,
 * call i on copy i % copies, timed with CUDA events around the sequence;
 * sec_per_call = mean device seconds per call.  Synchronises the stream. */
ACM_API int acm_bench_matmul(acm_engine *e, uint32_t ggml_type, const void *d_w, int64_t w_stride, int32_t copies,
                             int64_t n, int64_t k, const float *d_x, int32_t m, float *d_y, int32_t reps,
                             double *sec_per_call);

/* Sample from host logits with the device sampler (sampler parity tests). */
ACM_API int acm_sample_logits(acm_engine *e, const float *host_logits, int32_t n, const acm_sampler *s,
                              uint64_t step, int32_t *tok_out);

/* No counterpart in the reference (its sampler works on a Go slice).  The
 * sampler of acm_sample_logits on nrows device-resident logits rows (row r at
 * d_logits + r * ld, vocab floats), row r drawn with samplers[r] at step
 * steps[r] (samplers NULL: greedy; steps NULL: 0), ids written to the device
 * array d_out.  It allocates nothing: for callers that must not touch the
 * device allocator mid-decode (cudaMalloc / cudaFree synchronise the device,
 * and fail once the KV cache has taken the free HBM), the scratch is a fixed
 * 4 MiB buffer of the library image, one per device.  Limits: nrows <= 64,
 * vocab <= 262144; beyond them the call returns ACM_ERR_INVALID and says so.
 * Enqueued on the engine stream without waiting.  The buffer is shared by all
 * engines on a device, so calls must not overlap (one stream, or ordered by
 * the caller).  The first call on a device looks up the buffer's address
 * (cudaGetSymbolAddress); make it before beginning any stream capture. */
ACM_API int acm_sample_dev_noalloc(acm_engine *e, const float *d_logits, int64_t ld, int32_t nrows, int32_t vocab,
                                   const acm_sampler *samplers, const uint64_t *steps, int32_t *d_out);

/* Engine stream (cudaStream_t) and synchronisation, for callers that time
 * device work with their own events. */
ACM_API void *acm_engine_stream(acm_engine *e);
ACM_API int acm_engine_sync(acm_engine *e);

/* Device time in seconds of the last acm_forward / acm_generate phases,
 * measured with CUDA events on the model stream. */
ACM_API int acm_model_last_timing(acm_model *m, double *prefill_s, double *decode_s);

/* Number of kernels the library has launched in this process (a CUDA-graph
 * replay counts every kernel the graph holds).  No reference counterpart. */
ACM_API uint64_t acm_kernel_launches(void);

/* DebugLayer (model.go:231-233, called at :427-429 after each layer's
 * residual update): with enable != 0, every pass from now on (prefill chunks
 * and decode steps; decode graphs are rebuilt) copies the residual stream x
 * of its last token after each layer into a model buffer;
 * acm_model_debug_layers_read copies the last pass's [n_layers][n_embd]
 * values (after synchronising the model's stream).  The reference's hook
 * sees all nTok rows and is a Go callback; here the device keeps the last
 * row, the one the reference's layer_test.go inspects. */
ACM_API int acm_model_debug_layers(acm_model *m, int32_t enable);
ACM_API int acm_model_debug_layers_read(acm_model *m, float *out, int64_t cap);

/* Tracing of the batch-1 decode GEMV launches, no reference counterpart:
 * with slots > 0, decode graphs are rebuilt so that each batch-1 GEMV launch
 * of a step takes one slot (in launch order) of 160 CTAs x 8 values: the
 * %globaltimer ns at CTA entry, weights copy issued, dependency wait over,
 * activations staged, first weights landed, rows done, then the SM id;
 * slots = 0 turns it off.  acm_model_trace_gemv_read copies the slots the
 * last capture used ([used][160][8]). */
ACM_API int acm_model_trace_gemv(acm_model *m, int32_t slots);
ACM_API int acm_model_trace_gemv_read(acm_model *m, uint64_t *out, int64_t cap, int32_t *used);

/* Measurement helper, no reference counterpart: the tensor-core GEMM
 * launches of one ntok-token prefill (q/k/v, o, gate/up, down of every layer:
 * the matmul calls of model.go:346-348, :410, :418-419, :423) timed `reps`
 * times with CUDA events on the model stream (scratch activations; the
 * model's sequence state is untouched); seconds and useful flops
 * (2*ntok*weights) per pass, launches per pass. */
ACM_API int acm_model_bench_gemm(acm_model *m, int32_t ntok, int32_t reps, double *sec_per_pass,
                                 double *flops_per_pass, int32_t *launches_per_pass);

/* Measurement helper, no reference counterpart: replay the fused
 * dequant-GEMV launches of one batch-1 decode token on this model's weights
 * (q/k/v, o, gate/up, down of every layer, then lm_head -- the matvec calls of
 * model.go:346-348, :410, :418-419, :423, :440) `reps` times from a CUDA
 * graph and report the device seconds and algorithmic bytes (weight blocks +
 * activation reads + output writes) per pass and the launches per pass. */
ACM_API int acm_model_bench_gemv(acm_model *m, int32_t reps, double *sec_per_pass, double *bytes_per_pass,
                                 int32_t *launches_per_pass);

#ifdef __cplusplus
}
#endif
#endif /* ACM_H */
