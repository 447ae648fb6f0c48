// k_gemv.cu -- fused dequant-GEMV for decode (M = 1..8 tokens).
//
// The reference's matvec (internal/infer/tensor.go:253-303) dequantizes each
// weight row into an fp32 tile and dots it against the activations.  Decode
// is HBM-bound, so here the quantized GGUF bytes are streamed once, unchanged,
// and decoded in registers:
//   * one CTA per SM; each CTA owns a contiguous row range of one weight
//     matrix (several matrices -- q/k/v, gate/up -- share one launch);
//   * a producer warp moves whole rows into a ring of shared-memory stages
//     with the bulk-copy engine (cp.async.bulk + mbarrier).  It starts before
//     the kernel waits on its predecessor (programmatic dependent launch):
//     weights never depend on earlier kernels, so their HBM reads overlap the
//     previous kernel's tail;
//   * consumer warps decode the staged rows.  Unit path (small matrices): a
//     warp per row, lane l decodes 32-element units l, l+32, ... against the
//     activations permuted into unit order.  Wide path (large matrices such
//     as lm_head): `lpr` lanes per row, each decoding whole 256-element
//     super-blocks so block headers are read once per 256 weights;
//   * the row sum is a shuffle reduction; the epilogue stores, adds to the
//     residual stream, applies SwiGLU to a gate/up pair, or (lm_head under
//     greedy sampling) folds the row into a per-token argmax key.
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <vector>

#include "common.cuh"
#include "gemv_dev.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "quant.cuh"
#include "sbdot.cuh"

namespace acm {

__device__ int g_dev_error = 0;  // declared in common.cuh (relocatable device code)
__constant__ uint32_t g_wait_limit = WAIT_LIMIT;
bool g_pdl = [] {
    const char *e = getenv("ACM_PDL");
    return !(e && e[0] == '0');
}();

template <int MT, int TA, int TB>
__global__ void __launch_bounds__(Cfg<MT>::NT, 1) k_gemv(const __grid_constant__ GemvArgs a) {
    constexpr int NCW = Cfg<MT>::NCW;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    int sid = 0;
#pragma unroll 1
    for (int i = 1; i < a.nseg; i++)
        if ((int)blockIdx.x >= a.seg[i].cta0) sid = i;
    const GemvSeg &s = a.seg[sid];
    const int cta = (int)blockIdx.x - s.cta0;
    const int r0 = (int)((int64_t)s.n * cta / s.ncta), r1 = (int)((int64_t)s.n * (cta + 1) / s.ncta);
    const int K = a.k;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_NS_MAX;
    float *xs = reinterpret_cast<float *>(smem + 128);
    float *xsum = xs + x_area_floats(K, MT, a.lpr);
    float *red = xsum + 2 * MT * (K / 32);
    uint8_t *stg = smem + a.stage_off;
    if (tid == 0) {
        for (int i = 0; i < a.ns; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) pdl_trigger();
    if (r1 <= r0) {
        pdl_wait();
        return;
    }
    const int R = s.rows_per_stage, NS = a.ns;
    const int nst = (r1 - r0 + R - 1) / R;
    if (warp == NCW) {
        // producer: weights do not depend on earlier kernels -- stream them
        // before waiting on the predecessor
        if ((tid & 31) == 0) {
            int issued = 0;
            for (int i = 0; i < nst; i++) {
                const int slot = i % NS;
                if (i >= NS && !mbar_wait(&empty[slot], (uint32_t)(((i / NS) - 1) & 1))) break;
                const int ra = r0 + i * R, rbn = min(ra + R, r1);
                const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
                const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
                uint32_t total = (uint32_t)(a1 - a0);
                int64_t c0 = 0, c1 = 0;
                if (s.w2) {
                    c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
                    c1 = ((int64_t)rbn * s.rb2 + 15) & ~int64_t(15);
                    total += (uint32_t)(c1 - c0);
                }
                uint8_t *dst = stg + (size_t)slot * a.stage_bytes;
                mbar_arrive_expect_tx(&full[slot], total);
                bulk_g2s(dst, s.w + a0, (uint32_t)(a1 - a0), &full[slot]);
                if (s.w2) bulk_g2s(dst + (a1 - a0), s.w2 + c0, (uint32_t)(c1 - c0), &full[slot]);
                issued = i + 1;
            }
            // no copy may still be landing when the CTA exits (the consumers
            // leave early after a timed-out wait): wait, with the fixed bound,
            // for the last fill of every stage used
            for (int i = issued > NS ? issued - NS : 0; i < issued; i++)
                mbar_wait_limit(&full[i % NS], (uint32_t)((i / NS) & 1), WAIT_LIMIT);
            // this CTA's share of the next matvec's weights into L2
            for (int i = 0; i < a.npf; i++) {
                const int64_t bytes = a.pf[i].bytes;
                const int64_t chunk = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~int64_t(15);
                const int64_t off = (int64_t)blockIdx.x * chunk;
                if (off >= bytes) continue;
                const int64_t len = std::min<int64_t>(chunk, bytes - off) & ~int64_t(15);
                if (len > 0) prefetch_l2(static_cast<const uint8_t *>(a.pf[i].p) + off, (uint32_t)len);
            }
        }
        pdl_wait();
        return;
    }
    pdl_wait();
#define ACM_GEMV_BODY(T)                                                                               \
    prep_x<T, MT>(a, xs, xsum, red);                                                                   \
    if (a.lpr) consume_wide<T, MT>(a, s, r0, r1, full, empty, stg, xs, xsum);                          \
    else consume_unit<T, MT>(a, s, r0, r1, full, empty, stg, xs, reinterpret_cast<const float2 *>(xsum));
    if (s.type == TA) {
        ACM_GEMV_BODY(TA)
    } else if constexpr (TB != TA) {
        if (s.type == TB) {
            ACM_GEMV_BODY(TB)
        }
    }
#undef ACM_GEMV_BODY
}

static const int SMEM_MAX = 227 * 1024;

static int mt_of(int m) { return m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8; }

bool gemv_supported(int type, int64_t k, int m) {
    if (!type_ok(type) || m < 1 || m > 8 || k % 32 || k % blk_elems(type)) return false;
    const int mt = mt_of(m);
    const size_t xb = x_bytes(k, mt, 0);
    const int64_t rb = row_bytes(type, k);
    return xb + 2 * (size_t)(2 * rb + 64 + 128) + 16 <= (size_t)SMEM_MAX;
}

static bool sb_ok(int type) {
    return type == T_Q4_K || type == T_Q5_K || type == T_Q6_K || type == T_Q8_0 || type == T_F16;
}

template <int MT, int TA, int TB>
static cudaError_t launch_one(GemvArgs &a, int grid, size_t smem, cudaStream_t st) {
    static std::atomic<bool> attr_done[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv<MT, TA, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
        if (e != cudaSuccess) return e;
        attr_done[dev & 63] = true;
    }
    cudaError_t e = launch_pdl(k_gemv<MT, TA, TB>, dim3(grid), dim3(Cfg<MT>::NT), smem, st, a);
    if (e != cudaSuccess) return e;
    return launched(1);
}

template <int MT>
static cudaError_t launch_types(GemvArgs &a, int ta, int tb, int grid, size_t smem, cudaStream_t st) {
    if (ta == T_Q4_K && tb == T_Q6_K) return launch_one<MT, T_Q4_K, T_Q6_K>(a, grid, smem, st);
    switch (ta) {
        case T_Q4_K: return launch_one<MT, T_Q4_K, T_Q4_K>(a, grid, smem, st);
        case T_Q6_K: return launch_one<MT, T_Q6_K, T_Q6_K>(a, grid, smem, st);
        case T_Q8_0: return launch_one<MT, T_Q8_0, T_Q8_0>(a, grid, smem, st);
        case T_Q5_K: return launch_one<MT, T_Q5_K, T_Q5_K>(a, grid, smem, st);
        case T_Q4_0: return launch_one<MT, T_Q4_0, T_Q4_0>(a, grid, smem, st);
        case T_Q5_0: return launch_one<MT, T_Q5_0, T_Q5_0>(a, grid, smem, st);
        case T_F16: return launch_one<MT, T_F16, T_F16>(a, grid, smem, st);
        case T_F32: return launch_one<MT, T_F32, T_F32>(a, grid, smem, st);
    }
    return cudaErrorInvalidValue;
}

// CTAs per segment in proportion to its bytes, at least one and at most one
// per row, summing to at most num_sms (largest remainders get the rounding),
// so that a launch of one CTA per SM never spills into a second wave.
static void split_ctas(const GemvSegDesc *segs, int nseg, int64_t k, int num_sms, int *nc) {
    double total = 0, want[GEMV_MAX_SEG];
    for (int i = 0; i < nseg; i++) total += (double)row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1) * segs[i].n;
    int used = 0;
    for (int i = 0; i < nseg; i++) {
        want[i] = (double)row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1) * segs[i].n / total * num_sms;
        nc[i] = std::max(1, std::min<int>((int)want[i], (int)segs[i].n));
        used += nc[i];
    }
    while (used < num_sms) {
        int best = -1;
        double rem = -1.0;
        for (int i = 0; i < nseg; i++)
            if (nc[i] < segs[i].n && want[i] - nc[i] > rem) {
                rem = want[i] - nc[i];
                best = i;
            }
        if (best < 0 || rem <= 0.0) break;
        nc[best]++;
        used++;
    }
}

// One launch for segments whose types are {ta} or {ta, tb}.
static cudaError_t gemv_launch_group(const GemvSegDesc *segs, int nseg, int ta, int tb, const float *x, int ldx,
                                     int64_t k, int m, const float *norm_w, float eps, int num_sms, cudaStream_t st,
                                     const L2Range *pf, int npf) {
    const int mt = mt_of(m);
    GemvArgs a{};
    a.npf = 0;
    for (int i = 0; i < npf && a.npf < GEMV_MAX_PF; i++)
        if (pf[i].p && pf[i].bytes >= 16 && ((uintptr_t)pf[i].p & 15) == 0) a.pf[a.npf++] = pf[i];
    a.nseg = nseg;
    a.x = x;
    a.ldx = ldx;
    a.k = (int)k;
    a.m = m;
    a.norm_w = norm_w;
    a.eps = eps;
    int64_t maxrow = 0;
    for (int i = 0; i < nseg; i++) maxrow = std::max(maxrow, row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1));
    // wide path: a single large matrix whose format has a span decoder
    a.lpr = 0;
    if (nseg == 1 && sb_ok(segs[0].type) && k % 256 == 0 && segs[0].n / num_sms >= 128) {
        const int nsb = (int)(k / 256);
        int lpr = 1;
        while (lpr * 2 <= 4 && nsb % (lpr * 2) == 0) lpr *= 2;
        a.lpr = lpr;
    }
    const size_t xb = x_bytes(k, mt, a.lpr);
    // a stage holds R rows plus up to 60 bytes of 16-byte rounding (two
    // copies) and the 4-byte over-read of the unaligned word loader
    // enough rows per stage for every consumer warp to take a row (wide
    // path: a row group)
    const int ncw = mt <= 2 ? 16 : 8;
    int64_t sb = std::max<int64_t>(32 * 1024, (((int64_t)ncw * maxrow + 64 + 127) / 128) * 128);
    if (a.lpr) sb = std::max<int64_t>(sb, (((int64_t)ncw * (32 / a.lpr) * maxrow + 64 + 127) / 128) * 128);
    int ns = (int)std::min<int64_t>(6, ((int64_t)SMEM_MAX - (int64_t)xb - 16) / sb);
    if (ns < 2) {
        // long rows (F16 / Q8_0 at large K): two stages as large as shared
        // memory allows; a stage then feeds fewer warps, but the ring stays
        // double-buffered (one-row stages serialise the copies row by row)
        sb = (((int64_t)SMEM_MAX - (int64_t)xb - 16) / 2) & ~int64_t(127);
        ns = 2;
    }
    if (ns < 2 || sb < maxrow + 64) {
        sb = ((maxrow + 64 + 127) / 128) * 128;
        ns = (int)std::min<int64_t>(GEMV_NS_MAX, ((int64_t)SMEM_MAX - (int64_t)xb - 16) / sb);
        if (ns < 2) return cudaErrorInvalidValue;
    }
    // small matrices: shrink the ring to the stages a CTA actually needs, so
    // the kernel's shared memory leaves room for the next kernel's CTAs to
    // start early (programmatic dependent launch) and prefetch their weights
    int ncta[GEMV_MAX_SEG];
    split_ctas(segs, nseg, k, num_sms, ncta);
    {
        int64_t need_stages = 1, need_bytes = 0;
        for (int i = 0; i < nseg; i++) {
            const int64_t rbp = row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1);
            const int nc = ncta[i];
            const int64_t rows = (segs[i].n + nc - 1) / nc;
            const int64_t rps = (sb - 64) / rbp;
            need_stages = std::max<int64_t>(need_stages, (rows + rps - 1) / std::max<int64_t>(rps, 1));
            need_bytes = std::max<int64_t>(need_bytes, rows * rbp + 64);
        }
        if (need_stages == 1) {
            sb = std::min<int64_t>(sb, ((need_bytes + 127) / 128) * 128);
            ns = 1;
        } else {
            ns = (int)std::min<int64_t>(ns, need_stages);
        }
    }
    a.ns = ns;
    a.stage_bytes = (int)sb;
    a.stage_off = (int)xb;
    int grid = 0;
    for (int i = 0; i < nseg; i++) {
        GemvSeg &g = a.seg[i];
        const GemvSegDesc &d = segs[i];
        g.w = static_cast<const uint8_t *>(d.w);
        g.w2 = static_cast<const uint8_t *>(d.w2);
        g.type = d.type;
        g.rb = row_bytes(d.type, k);
        g.rb2 = d.w2 ? g.rb : 0;
        g.n = (int)d.n;
        g.epi = d.epi;
        g.y = d.y;
        g.ldy = d.ldy;
        g.bias = d.bias;
        g.yrow = d.yrow;
        g.amax = d.amax;
        const int nc = ncta[i];
        g.ncta = nc;
        g.cta0 = grid;
        grid += nc;
        g.rows_per_stage = (int)((sb - 64) / (g.rb + g.rb2));
        if (g.rows_per_stage < 1) return cudaErrorInvalidValue;
    }
    const size_t smem = xb + (size_t)ns * (size_t)sb + 16;
    switch (mt) {
        case 1: return launch_types<1>(a, ta, tb, grid, smem, st);
        case 2: return launch_types<2>(a, ta, tb, grid, smem, st);
        case 4: return launch_types<4>(a, ta, tb, grid, smem, st);
        default: return launch_types<8>(a, ta, tb, grid, smem, st);
    }
}

cudaError_t gemv_launch(const GemvSegDesc *segs, int nseg, const float *x, int ldx, int64_t k, int m,
                        const float *norm_w, float eps, int num_sms, cudaStream_t st, const L2Range *pf, int npf) {
    if (nseg < 1 || nseg > GEMV_MAX_SEG || m < 1 || m > 8) return cudaErrorInvalidValue;
    if (m == 1 && !((uintptr_t)x & 15) && !(norm_w && ((uintptr_t)norm_w & 15))) {
        // one token: the batch-1 kernel (activations in registers); matrices
        // of more than ~128 rows per SM (lm_head) stay on the wide path below,
        // whose lanes own whole super-blocks (Q4_K 1024 x 151936: 34.9 us
        // there, 49.8 us on the batch-1 kernel)
        bool ok = true;
        int64_t rows = 0;
        for (int i = 0; i < nseg; i++) {
            ok &= gemv1_supported(segs[i].type, k);
            rows += segs[i].n;
        }
        if (ok && rows < 128 * (int64_t)num_sms) return gemv1_launch(segs, nseg, x, k, norm_w, eps, num_sms, st, pf, npf);
    }
    // common instance: every type equal, or exactly {Q4_K, Q6_K}
    bool same = true, q46 = true;
    for (int i = 0; i < nseg; i++) {
        same &= segs[i].type == segs[0].type;
        q46 &= segs[i].type == T_Q4_K || segs[i].type == T_Q6_K;
    }
    if (same)
        return gemv_launch_group(segs, nseg, segs[0].type, segs[0].type, x, ldx, k, m, norm_w, eps, num_sms, st, pf, npf);
    if (q46) return gemv_launch_group(segs, nseg, T_Q4_K, T_Q6_K, x, ldx, k, m, norm_w, eps, num_sms, st, pf, npf);
    // otherwise one launch per distinct type (CTAs split by bytes)
    double tot = 0;
    for (int j = 0; j < nseg; j++) tot += (double)row_bytes(segs[j].type, k) * segs[j].n;
    for (int i = 0; i < nseg; i++) {
        bool first = true;
        for (int j = 0; j < i; j++) first &= segs[j].type != segs[i].type;
        if (!first) continue;
        std::vector<GemvSegDesc> grp;
        double frac = 0;
        for (int j = i; j < nseg; j++)
            if (segs[j].type == segs[i].type) {
                grp.push_back(segs[j]);
                frac += (double)row_bytes(segs[j].type, k) * segs[j].n;
            }
        const int sms = std::max(1, (int)(num_sms * frac / tot + 0.5));
        cudaError_t e = gemv_launch_group(grp.data(), (int)grp.size(), segs[i].type, segs[i].type, x, ldx, k, m,
                                          norm_w, eps, sms, st, pf, npf);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t set_wait_limit(uint32_t polls) {
    return cudaMemcpyToSymbol(g_wait_limit, &polls, sizeof(polls));
}

int read_and_clear_dev_error() {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
    if (v) cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
    return v;
}

}  // namespace acm
