// attn_dev.cuh -- device helpers shared by the attention kernels and the
// persistent decode kernel: paged cache addressing and the per-head
// RMSNorm + RoPE of model.go:362-382.
#pragma once
#include "common.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace acm {

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

}  // namespace acm
