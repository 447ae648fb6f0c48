// k_noalloc.cu -- the sampler (Sampler.Sample, sampler.go:30-76) on
// device-resident logits with every piece of scratch in a fixed buffer that
// belongs to this library's device image, so a call allocates nothing.
//
// Who needs it: a caller that already owns its logits and output buffers on
// the device and must not touch the device allocator while decoding --
// cudaMalloc / cudaFree synchronise the device (stalling other streams' work)
// and can fail once the paged KV cache has taken the free HBM.  The regular
// entry point (acm_sample_logits) stages through the engine's growable
// scratch, which may call cudaMalloc.
//
// Limits: nrows <= NA_ROWS_MAX, vocab <= NA_VOCAB_MAX.  The buffer is one per
// device and shared by every engine on that device, so calls must not
// overlap: issue them on one stream, or order them yourself.
#include <mutex>
#include <string>

#include "acm.h"
#include "common.cuh"
#include "kernels.h"

namespace acm {

namespace {

constexpr int NA_ROWS_MAX = 64;
constexpr int NA_VOCAB_MAX = 262144;
constexpr int NA_CHUNK = 2048;  // logits per top-k partial block (the sampler's chunk)
constexpr int NA_TOPK = 64;     // candidates kept per chunk
constexpr int NA_CHUNKS_MAX = NA_VOCAB_MAX / NA_CHUNK;

// Layout of the scratch buffer (in 8-byte words): per-row sampler
// parameters, then the per-chunk candidate keys [row][chunk][64].
constexpr size_t NA_TEMP = 0;
constexpr size_t NA_TOPP = NA_TEMP + NA_ROWS_MAX;
constexpr size_t NA_SEED = NA_TOPP + NA_ROWS_MAX;
constexpr size_t NA_STEP = NA_SEED + NA_ROWS_MAX;
constexpr size_t NA_TOPK_W = NA_STEP + NA_ROWS_MAX;          // int32 [64] in 32 words
constexpr size_t NA_CAND = 512;                              // 4 KiB offset
constexpr size_t NA_WORDS = NA_CAND + (size_t)NA_ROWS_MAX * NA_CHUNKS_MAX * NA_TOPK;  // 4 MiB + 4 KiB
static_assert(NA_TOPK_W + NA_ROWS_MAX / 2 <= NA_CAND, "parameter block overflows");

// Nothing here needs to start at zero: each call writes the parameter block
// for its rows and every candidate slot the final pass reads.
static __device__ __align__(256) uint64_t g_sample_scratch[NA_WORDS];

struct NoAllocParams {
    int nrows;
    int32_t top_k[NA_ROWS_MAX];
    double temp[NA_ROWS_MAX];
    double top_p[NA_ROWS_MAX];
    uint64_t seed[NA_ROWS_MAX];
    uint64_t step[NA_ROWS_MAX];
};
static_assert(sizeof(NoAllocParams) < 4000, "kernel parameter limit");

// Writes the by-value sampler parameters into the scratch buffer, so the
// sampler kernels read them from device memory without a host copy.
__global__ void k_noalloc_params(NoAllocParams p, uint64_t *scratch) {
    const int t = threadIdx.x;
    if (t >= p.nrows) return;
    reinterpret_cast<double *>(scratch + NA_TEMP)[t] = p.temp[t];
    reinterpret_cast<double *>(scratch + NA_TOPP)[t] = p.top_p[t];
    scratch[NA_SEED + t] = p.seed[t];
    scratch[NA_STEP + t] = p.step[t];
    reinterpret_cast<int32_t *>(scratch + NA_TOPK_W)[t] = p.top_k[t];
}

std::mutex g_na_mu;
uint64_t *g_na_ptr[64] = {};

// Device address of the scratch buffer for the current device.  The first
// call per device does the lookup (the driver places the buffer when the
// module is loaded on that device).
cudaError_t scratch_ptr(int dev, uint64_t **out) {
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_sample_scratch);
        if (e != cudaSuccess) return e;
        g_na_ptr[dev] = static_cast<uint64_t *>(p);
    }
    *out = g_na_ptr[dev];
    return cudaSuccess;
}

}  // namespace

// Returns 0, 1 (invalid argument) or 2 (CUDA error); *err gets the message.
int sample_noalloc(int dev, cudaStream_t st, const float *d_logits, int64_t ld, int nrows, int vocab,
                   const acm_sampler *samplers, const uint64_t *steps, int32_t *d_out, std::string *err) {
    if (nrows < 1 || nrows > NA_ROWS_MAX) {
        *err = "acm_sample_dev_noalloc: nrows " + std::to_string(nrows) + " outside 1.." +
               std::to_string(NA_ROWS_MAX) + " (the fixed scratch holds " + std::to_string(NA_ROWS_MAX) +
               " rows)";
        return 1;
    }
    if (vocab < 1 || vocab > NA_VOCAB_MAX) {
        *err = "acm_sample_dev_noalloc: vocab " + std::to_string(vocab) + " outside 1.." +
               std::to_string(NA_VOCAB_MAX) + " (the fixed scratch holds " + std::to_string(NA_VOCAB_MAX) +
               " logits per row)";
        return 1;
    }
    if (ld < vocab || !d_logits || !d_out) {
        *err = "acm_sample_dev_noalloc: null buffer or row stride below vocab";
        return 1;
    }
    uint64_t *s = nullptr;
    cudaError_t e = scratch_ptr(dev, &s);
    if (e != cudaSuccess) {
        *err = std::string("acm_sample_dev_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e);
        return 2;
    }
    NoAllocParams p = {};
    p.nrows = nrows;
    bool all_greedy = true;
    for (int i = 0; i < nrows; i++) {
        p.temp[i] = samplers ? samplers[i].temp : 0.0;
        p.top_k[i] = samplers ? samplers[i].top_k : 0;
        p.top_p[i] = samplers ? samplers[i].top_p : 0.0;
        p.seed[i] = samplers ? samplers[i].seed : 0;
        p.step[i] = steps ? steps[i] : 0;
        all_greedy = all_greedy && p.temp[i] <= 0.0;
    }
    k_noalloc_params<<<1, NA_ROWS_MAX, 0, st>>>(p, s);
    e = launched(1);
    if (e == cudaSuccess) {
        SampleDesc sd{d_logits,
                      nullptr,
                      ld,
                      vocab,
                      reinterpret_cast<const double *>(s + NA_TEMP),
                      reinterpret_cast<const int32_t *>(s + NA_TOPK_W),
                      reinterpret_cast<const double *>(s + NA_TOPP),
                      s + NA_SEED,
                      s + NA_STEP,
                      d_out,
                      s + NA_CAND,
                      (vocab + NA_CHUNK - 1) / NA_CHUNK};
        e = sample_launch(sd, nrows, all_greedy, st);
    }
    if (e != cudaSuccess) {
        *err = std::string("acm_sample_dev_noalloc: launch: ") + cudaGetErrorString(e);
        return 2;
    }
    return 0;
}

}  // namespace acm
