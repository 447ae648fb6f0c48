// k_gemv1.cu -- batch-1 decode GEMV launches (device code in gemv1.cuh).
//
// Planning: CTAs are split over the launch's matrices in proportion to their
// bytes (one CTA per SM in all); a CTA's rows are split over its warps
// contiguously.  When every warp's rows fit one stage of a few KB (all the
// per-layer matvecs of the models served here), the warp moves them with one
// bulk copy before the dependency wait and the CTA stays small enough for
// the next kernels' CTAs to share the SM; larger matrices (lm_head) run 16
// warps, each double-buffering its rows through two stages.
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <atomic>
#include <vector>

#include "common.cuh"
#include "gemv1.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "quant.cuh"

namespace acm {

// The CTA's matvec in format T: team geometry, the weight copies and the L2
// prefetch before the dependency wait, then the activations and the rows.
template <int T>
__device__ __forceinline__ void gemv1_cta(const Gemv1Args &a, const GemvSeg &s, uint8_t *smem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const RowGeo geo = row_geo(T, a.k);
    const int TS = geo.ts, NT = (int)(blockDim.x >> 5) / TS;
    const int team = warp / TS, tw = warp - team * TS;
    const bool active = team < NT;
    const int cta = (int)blockIdx.x - s.cta0;
    const int r0 = (int)((int64_t)s.n * cta / s.ncta), r1 = (int)((int64_t)s.n * (cta + 1) / s.ncta);
    const int n = r1 - r0;
    const int tr0 = r0 + n * team / NT, tr1 = r0 + n * (team + 1) / NT;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem) + 2 * team;
    uint8_t *wbuf = smem + a.stage_off + (size_t)team * a.nstage * a.stage_bytes;
    float *part = reinterpret_cast<float *>(smem + a.part_off) + (size_t)team * (a.part_rows * 2 * TS + TS);
    float *red = part + a.part_rows * 2 * TS;
    const int R = s.rows_per_stage;
    const int nst = (active && tr1 > tr0) ? (tr1 - tr0 + R - 1) / R : 0;
    trace_stamp(a.trace, 0);
    if (a.trace && threadIdx.x == 0) {
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        a.trace[(size_t)blockIdx.x * 8 + 6] = smid;
    }
    if (tw == 0 && lane == 0 && nst > 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
        // weights do not depend on earlier kernels: stream them before the wait
        for (int i = 0; i < min(nst, a.nstage); i++) gemv1_issue(a, s, tr0, tr1, i, bar, wbuf);
    }
    if (threadIdx.x == 32) {
        // this CTA's share of the next matvecs' weights into L2
        for (int i = 0; i < a.npf; i++) {
            const int64_t bytes = a.pf[i].bytes;
            const int64_t chunk = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~int64_t(15);
            const int64_t off = (int64_t)blockIdx.x * chunk;
            if (off >= bytes) continue;
            const int64_t len = std::min<int64_t>(chunk, bytes - off) & ~int64_t(15);
            if (len > 0) prefetch_l2(static_cast<const uint8_t *>(a.pf[i].p) + off, (uint32_t)len);
        }
    }
    XStage xst;
    stage_x_pre(a.norm_w, a.k, xst, blockDim.x);
    trace_stamp(a.trace, 1);
    pdl_trigger();
    pdl_wait();
    trace_stamp(a.trace, 2);
    float *xs = reinterpret_cast<float *>(smem + GEMV1_BAR_BYTES);
    // every thread takes part (its barriers also order the mbarrier inits)
    stage_x<T>(a.x, a.norm_w, a.k, a.eps, xs, xs + a.k, xst, blockDim.x, 0);
    trace_stamp(a.trace, 3);
    if (nst > 0) gemv1_rows<T>(a, s, geo, tr0, tr1, bar, wbuf, nst, tw, 1 + team, part, red, xs);
}

// Up to 16 warps per CTA (12 in use, NWC), up to 128 registers a thread: one
// CTA per SM, and the block scheduler spreads the 148 CTAs over all SMs (CTAs
// that could share an SM were packed onto a third of them).
template <int TA, int TB>
__global__ void __launch_bounds__(512, 1) k_gemv1(const __grid_constant__ Gemv1Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    int sid = 0;
#pragma unroll 1
    for (int i = 1; i < a.nseg; i++)
        if ((int)blockIdx.x >= a.seg[i].cta0) sid = i;
    const GemvSeg &s = a.seg[sid];
    if (s.type == TA) {
        gemv1_cta<TA>(a, s, smem);
    } else if constexpr (TB != TA) {
        if (s.type == TB) gemv1_cta<TB>(a, s, smem);
    }
}

static const int SMEM_MAX1 = 227 * 1024;
static const int NWC = 12;  // warps per CTA

// Timeline tracing (profiling): launches planned while it is on take
// consecutive slots of the buffer.
static unsigned long long *g_trace_buf = nullptr;
static int g_trace_slots = 0, g_trace_next = 0;

void gemv1_trace(unsigned long long *buf, int slots) {
    g_trace_buf = buf;
    g_trace_slots = buf ? slots : 0;
    g_trace_next = 0;
}
int gemv1_trace_used() { return g_trace_next; }
// Largest single-stage footprint: a CTA whose teams' rows fit one stage each
// moves them with one copy per team.
static const int SMALL_SMEM = 128 * 1024;

bool gemv1_supported(int type, int64_t k) {
    return type_ok(type) && k >= 32 && k % 32 == 0 && k % blk_elems(type) == 0 && k % lane_elems_rt(type) == 0 &&
           row_geo(type, (int)k).ts <= NWC;
}

template <int TA, int TB>
static cudaError_t launch_inst(const Gemv1Args &a, int grid, int nthreads, size_t smem, cudaStream_t st) {
    static std::atomic<bool> attr_done[64] = {};  // per device: attributes set (host threads may race)
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_done[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv1<TA, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX1);
        if (e != cudaSuccess) return e;
        attr_done[dev & 63] = true;
    }
    cudaError_t e = launch_pdl(k_gemv1<TA, TB>, dim3(grid), dim3(nthreads), smem, st, a);
    if (e != cudaSuccess) return e;
    return launched(1);
}

static cudaError_t launch_types1(const Gemv1Args &a, int ta, int tb, int grid, int nthreads, size_t smem,
                                 cudaStream_t st) {
    if (ta == T_Q4_K && tb == T_Q6_K) return launch_inst<T_Q4_K, T_Q6_K>(a, grid, nthreads, smem, st);
    switch (ta) {
        case T_Q4_K: return launch_inst<T_Q4_K, T_Q4_K>(a, grid, nthreads, smem, st);
        case T_Q6_K: return launch_inst<T_Q6_K, T_Q6_K>(a, grid, nthreads, smem, st);
        case T_Q8_0: return launch_inst<T_Q8_0, T_Q8_0>(a, grid, nthreads, smem, st);
        case T_Q5_K: return launch_inst<T_Q5_K, T_Q5_K>(a, grid, nthreads, smem, st);
        case T_Q4_0: return launch_inst<T_Q4_0, T_Q4_0>(a, grid, nthreads, smem, st);
        case T_Q5_0: return launch_inst<T_Q5_0, T_Q5_0>(a, grid, nthreads, smem, st);
        case T_F16: return launch_inst<T_F16, T_F16>(a, grid, nthreads, smem, st);
        case T_F32: return launch_inst<T_F32, T_F32>(a, grid, nthreads, smem, st);
    }
    return cudaErrorInvalidValue;
}

// CTAs per matrix in proportion to its bytes, at least one and at most one
// per row, summing to at most num_sms (largest remainders get the rounding).
static void split_ctas1(const GemvSegDesc *segs, int nseg, int64_t k, int num_sms, int *nc) {
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

// One launch for matrices whose types are {ta} or {ta, tb}.
static cudaError_t gemv1_group(const GemvSegDesc *segs, int nseg, int ta, int tb, const float *x, int64_t k,
                               const float *norm_w, float eps, int num_sms, cudaStream_t st, const L2Range *pf,
                               int npf) {
    // teams per segment format: NWC warps, teams of row_geo().ts warps.  12
    // warps of up to 128 registers: one GEMV CTA per SM (two would need more
    // than the register file), with room left beside it for decode
    // attention CTAs; measured 1070 tok/s against 1045 at 16 warps and 990
    // at 8 (whose CTAs, two fitting per SM, were packed onto 106 SMs)
    int tsmax = 1, ntc[GEMV_MAX_SEG];
    for (int i = 0; i < nseg; i++) {
        const int ts = row_geo(segs[i].type, (int)k).ts;
        if (ts > GEMV1_MAX_TS || ts > NWC) return cudaErrorInvalidValue;
        tsmax = std::max(tsmax, ts);
        ntc[i] = NWC / ts;
    }
    int nc[GEMV_MAX_SEG];
    split_ctas1(segs, nseg, k, num_sms, nc);
    int64_t maxrow = 0;
    for (int i = 0; i < nseg; i++) maxrow = std::max(maxrow, row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1));
    // bytes of the largest per-team row range
    int64_t need = 0;
    for (int i = 0; i < nseg; i++) {
        const int64_t rows_cta = (segs[i].n + nc[i] - 1) / nc[i];
        const int64_t rows_t = (rows_cta + ntc[i] - 1) / ntc[i];
        need = std::max(need, rows_t * row_bytes(segs[i].type, k) * (segs[i].w2 ? 2 : 1));
    }
    need += 64;  // 16-byte rounding of up to two copies + the word loader's over-read
    // shared layout: [mbarriers][x: K floats + 32 of scratch][stages][team partials]
    const int xb = (int)(((k + 32) * 4 + 127) / 128 * 128);
    int nt = 1;  // stage slots: one per team of the format with the most teams
    for (int i = 0; i < nseg; i++) nt = std::max(nt, ntc[i]);
    int nstage = 1;
    int64_t sb = (need + 127) / 128 * 128;
    const int64_t part_cap = 64;  // rows per stage of a multi-warp team
    const int64_t part_bytes = tsmax > 1 ? (int64_t)nt * (part_cap * 2 * tsmax + tsmax) * 4 : 0;
    const int64_t room = SMEM_MAX1 - GEMV1_BAR_BYTES - xb - part_bytes;
    if ((int64_t)nt * sb > std::min<int64_t>(room, SMALL_SMEM)) {
        // large matrices: each team double-buffers its rows
        nstage = 2;
        sb = std::min<int64_t>(sb, (room / (nt * nstage)) & ~int64_t(127));
        if (sb < maxrow + 64) return cudaErrorInvalidValue;
    }
    Gemv1Args a{};
    a.nseg = nseg;
    a.x = x;
    a.k = (int)k;
    a.norm_w = norm_w;
    a.eps = eps;
    a.nstage = nstage;
    a.stage_bytes = (int)sb;
    a.trace = nullptr;
    a.npf = 0;
    for (int i = 0; i < npf && a.npf < GEMV_MAX_PF; i++)
        if (pf[i].p && pf[i].bytes >= 16 && ((uintptr_t)pf[i].p & 15) == 0) a.pf[a.npf++] = pf[i];
    if (g_trace_buf && g_trace_next < g_trace_slots)
        a.trace = g_trace_buf + (size_t)(g_trace_next++) * GEMV1_TRACE_CTAS * 8;
    int grid = 0, part_rows = 1;
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
        g.ncta = nc[i];
        g.cta0 = grid;
        grid += nc[i];
        int64_t rps = (sb - 64) / (g.rb + g.rb2);
        if (tsmax > 1) rps = std::min(rps, part_cap);
        g.rows_per_stage = (int)rps;
        if (g.rows_per_stage < 1) return cudaErrorInvalidValue;
        part_rows = std::max(part_rows, g.rows_per_stage);
    }
    a.part_rows = part_rows;
    a.stage_off = GEMV1_BAR_BYTES + xb;
    a.part_off = (int)(a.stage_off + (size_t)nt * nstage * sb);
    const size_t smem = (size_t)a.part_off + (tsmax > 1 ? (size_t)nt * (part_rows * 2 * tsmax + tsmax) * 4 : 0);
    if (smem > (size_t)SMEM_MAX1) return cudaErrorInvalidValue;
    return launch_types1(a, ta, tb, grid, NWC * 32, smem, st);
}

cudaError_t gemv1_launch(const GemvSegDesc *segs, int nseg, const float *x, int64_t k, const float *norm_w,
                         float eps, int num_sms, cudaStream_t st, const L2Range *pf, int npf) {
    if (nseg < 1 || nseg > GEMV_MAX_SEG || ((uintptr_t)x & 15) || (norm_w && ((uintptr_t)norm_w & 15)))
        return cudaErrorInvalidValue;
    bool same = true, q46 = true;
    for (int i = 0; i < nseg; i++) {
        if (!gemv1_supported(segs[i].type, k)) return cudaErrorInvalidValue;
        same &= segs[i].type == segs[0].type;
        q46 &= segs[i].type == T_Q4_K || segs[i].type == T_Q6_K;
    }
    if (same) return gemv1_group(segs, nseg, segs[0].type, segs[0].type, x, k, norm_w, eps, num_sms, st, pf, npf);
    if (q46) return gemv1_group(segs, nseg, T_Q4_K, T_Q6_K, x, k, norm_w, eps, num_sms, st, pf, npf);
    // otherwise one launch per distinct type (SMs split by bytes)
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
        cudaError_t e = gemv1_group(grp.data(), (int)grp.size(), segs[i].type, segs[i].type, x, k, norm_w, eps, sms,
                                    st, pf, npf);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace acm
