// common.cuh -- small device utilities shared by the kernels: mbarriers and
// the 1-D bulk copy engine (cp.async.bulk), bounded waits, reductions.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace acm {

// Set by a kernel whose bounded wait ran out; read and cleared by the host
// after each synchronisation (acm_status ACM_ERR_TIMEOUT).
extern __device__ int g_dev_error;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after `limit` polls, records the timeout and returns
// false so the caller can unwind instead of hanging the GPU.  mbar_wait uses
// the limit in g_wait_limit (default WAIT_LIMIT, ~2^22 polls: seconds; the
// host may lower it, see set_wait_limit).
constexpr uint32_t WAIT_LIMIT = 1u << 22;
extern __constant__ uint32_t g_wait_limit;
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t parity, uint32_t limit) {
    for (uint32_t it = 0; it < limit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(&g_dev_error, DEV_ERR_TIMEOUT);
    return false;
}
// The limit is read (constant cache) only when the phase has not completed
// at the first test; a zero limit makes every wait give up at once.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t limit = g_wait_limit;
    if (limit && mbar_try_wait(bar, parity)) return true;
    return mbar_wait_limit(bar, parity, limit);
}

// Order this thread's earlier generic-proxy accesses of shared memory before
// its later async-proxy (bulk copy) writes into the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Pull [p, p + bytes) into L2 (p 16-byte aligned, bytes a multiple of 16);
// completes on its own, nothing waits for it.
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the preceding kernel in the stream
// (all its memory operations visible), and allow the next one to start its
// CTAs early.  Both are no-ops when the launch did not opt in.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Order-preserving 64-bit key of (logit, index): descending key order is
// descending logit, and among equal logits ascending index -- the tie rule of
// greedy() and topK() (sampler.go:19-27, :80-98).  NaN ranks last.
__device__ __forceinline__ unsigned long long logit_key(float v, int idx) {
    const uint32_t b = __float_as_uint(v);
    uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    if (v != v) o = 0;
    return ((unsigned long long)o << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ float key_logit(unsigned long long k) {
    const uint32_t o = (uint32_t)(k >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}
__device__ __forceinline__ int key_index(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)k); }

// 16-byte asynchronous global -> shared copy (L2 only) and its wait.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Close the copies issued so far into a group; wait until at most N groups
// are still in flight.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Named barrier among `nthreads` threads (a subset of the CTA).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier that also ANDs a predicate over its `nthreads` threads, so
// that a group decides together (a bounded wait that gave up in one thread
// must not leave the others at a later barrier).
__device__ __forceinline__ bool named_and(int id, int nthreads, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\tbar.red.and.pred b, %2, %3, a;\n\t"
        "selp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// RMSNorm scale, model.go:213-222: ss is the fp32 sum of squares; the
// reference divides by n in fp32, adds eps and takes the square root in
// fp64, then inverts in fp32.
__device__ __forceinline__ float rms_scale(float ss, int n, float eps) {
    const float mean = __fdiv_rn(ss, (float)n);
    return __fdiv_rn(1.0f, (float)sqrt((double)mean + (double)eps));
}

}  // namespace acm
