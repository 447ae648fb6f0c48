// k_decode.cu -- persistent decode kernel: one cooperative launch runs a whole
// decode step (every layer of model.go:342-430 plus the lm_head matvec of
// model.go:433-441) for a batch of tokens of distinct sequences.
//
// A decode step at batch 1 is a chain of ~140 small dependent operations; as
// separate kernels each pays a launch and a ramp/drain of several
// microseconds while moving only a few MB.  Here one CTA per SM stays
// resident for the whole step:
//   * phases: per layer  q/k/v GEMV | attention | o GEMV (+residual) |
//     gate/up GEMV (SwiGLU) | down GEMV (+residual); then lm_head.  A grid
//     barrier separates consecutive phases;
//   * every CTA owns a fixed row range of every GEMV phase (a per-CTA phase
//     table built on the host), and its producer warp streams those rows of
//     upcoming phases into the shared-memory ring without waiting for the
//     barriers -- weights do not depend on activations -- so weight traffic
//     overlaps barrier latency and the attention phases;
//   * attention items (token, kv head, 16-position chunk) are spread over four
//     4-warp groups per CTA; the last chunk to finish merges the partials;
//   * activations written by other CTAs are read with L2-only loads.
// Greedy sampling: the lm_head epilogue folds rows into per-token argmax keys
// and CTA 0 advances the token/position/step state after the last barrier.
#include <float.h>
#include <stdio.h>

#include <algorithm>
#include <vector>

#include "attn_dev.cuh"
#include "common.cuh"
#include "gemv1.cuh"
#include "gemv_dev.cuh"
#include "kernels.h"
#include "quant.cuh"

namespace acm {

constexpr int DCH = DEC_CHUNK;  // attention chunk (positions)
constexpr int DGROUPS = 3;    // attention groups per CTA (4 warps each)
constexpr int DNCW = 15;      // consumer warps (16 warps in all: 128 registers a thread)
constexpr int DNT = DNCW * 32 + 32;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Grid barrier among the consumer warps of all CTAs; bounded wait.  With a
// trace buffer, records when this CTA arrives (slot arrive) and leaves.
// Trace slots per (CTA, phase): 0 barrier left (phase start), 1 activations
// staged, 2 first weights stage ready, 3 barrier arrival (phase end).
__device__ __forceinline__ bool grid_sync(unsigned *bar, unsigned target, int *abort_flag,
                                          unsigned long long *arrive = nullptr, unsigned long long *leave = nullptr) {
    named_sync(1, DNCW * 32);
    if (threadIdx.x == 0) {
        if (arrive) *arrive = gtimer();
        __threadfence();
        atomicAdd(bar, 1u);
        uint32_t it = 0;
        while (ld_acquire_u32(bar) < target) {
            if (++it > (1u << 24) || *(volatile int *)&g_dev_error) {
                atomicExch(&g_dev_error, DEV_ERR_TIMEOUT);
                *abort_flag = 1;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
        if (leave) *leave = gtimer();
    }
    named_sync(1, DNCW * 32);
    return *(volatile int *)abort_flag == 0;
}

// A group's attention items are the same in every layer of a step (they
// depend only on the tokens' positions), so the first attention phase
// enumerates them and caches their cache offsets in shared memory.
constexpr int DMETA = 4;  // cached items per group
struct AttnMeta {
    int t, g, c, pos, h0, hn;
    int64_t base, newo;
};
struct AttnMetaGroup {
    AttnMeta it[DMETA];
    int n, pad_[3];
};

template <int HD>
__device__ void attn_phase(const DecArgs &A, const DecPhase &P, float *area, AttnMetaGroup *meta) {
    const int tid = threadIdx.x, grp = tid >> 7, gtid = tid & 127, bid = 2 + grp;
    if (grp >= DGROUPS) return;  // the last consumer warps sit attention out
    const int nkv = A.a.n_head_kv;
    float *sm = area + grp * A.attn_group_floats;
    AttnMetaGroup &mg = meta[grp];
    if (P.layer > 0 && mg.n <= DMETA) {
        for (int k = 0; k < mg.n; k++) {
            const AttnMeta m = mg.it[k];
            decode_attn_item<HD, DCH>(A.r, P.q_nw, P.k_nw, A.a, A.kv, P.layer, m.t, m.pos, m.g, m.c, m.base, m.newo,
                                      sm, gtid, bid, m.h0, m.hn);
        }
        return;
    }
    // items enumerated token by token: (t, g, j, c) with c < ceil(L_t / DCH)
    // and j a subset of hn_t query heads of kv head g
    const int G = A.a.n_head / nkv, slots = (int)gridDim.x * DGROUPS;
    int total = 0;
    for (int t = 0; t < A.ntok; t++) {
        const int nch = (A.tm.pos[t] + DCH) / DCH;
        total += nkv * (G / dec_heads_per_item(G, nch, nkv, HD, DCH, slots)) * nch;
    }
    int k = 0;
    for (int item = blockIdx.x * DGROUPS + grp; item < total; item += gridDim.x * DGROUPS, k++) {
        int t = 0, rem = item, nch = 0, hn = 1;
        while (true) {
            nch = (A.tm.pos[t] + DCH) / DCH;
            hn = dec_heads_per_item(G, nch, nkv, HD, DCH, slots);
            const int cnt = nkv * (G / hn) * nch;
            if (rem < cnt) break;
            rem -= cnt;
            t++;
        }
        const int pos = A.tm.pos[t];
        const int gj = rem / nch, c = rem % nch, g = gj / (G / hn), h0 = (gj % (G / hn)) * hn;
        int64_t base, newo;
        dec_item_offsets(A.kv, A.tm.seq[t], pos, g, c * DCH, HD, base, newo);
        if (k < DMETA && gtid == 0) mg.it[k] = AttnMeta{t, g, c, pos, h0, hn, base, newo};
        decode_attn_item<HD, DCH>(A.r, P.q_nw, P.k_nw, A.a, A.kv, P.layer, t, pos, g, c, base, newo, sm, gtid, bid,
                                  h0, hn);
    }
    if (P.layer == 0 && gtid == 0) mg.n = k;
}

// A GEMV phase: the activations staged once (RMSNorm-ed when the phase has a
// norm weight) and held in registers, the rows consumed from the ring by warp
// teams (gemv1_ring); the lm_head phase (lanes per row: P.lpr) keeps the wide
// span decoder.  Returns false on abort.
template <int T>
__device__ __forceinline__ bool gemv_phase(const DecArgs &A, const DecPhase &P, uint64_t *full, uint64_t *empty,
                                           const uint8_t *stg, float *area, uint32_t cur, XStage &xst,
                                           int *abort_flag, unsigned long long *tp) {
    if (P.lpr) {
        GemvArgs a{};
        a.nseg = 1;
        a.x = P.x;
        a.ldx = P.ldx;
        a.k = P.k;
        a.m = A.ntok;
        a.norm_w = P.norm_w;
        a.eps = A.eps;
        a.ns = A.ns;
        a.stage_bytes = A.sb;
        a.lpr = P.lpr;
        float *xs = area;
        float *xsum = xs + x_area_floats(P.k, 1, P.lpr);
        float *red = xsum + 2 * (P.k / 32);
        prep_x<T, 1, DNCW>(a, xs, xsum, red);
        consume_wide<T, 1, DNCW>(a, P.seg, P.r0, P.r1, full, empty, stg, xs, xsum, cur);
        return true;
    }
    float *xs = area, *red = xs + P.k, *part = red + 32;
    stage_x<T>(P.x, P.norm_w, P.k, A.eps, xs, red, xst, DNCW * 32, 1);
    if (tp && threadIdx.x == 0) tp[1] = gtimer();
    return gemv1_ring<T>(P.seg, P.r0, P.r1, P.k, full, empty, stg, A.ns, A.sb, cur, xs, part, A.part_rows, DNCW,
                         abort_flag, tp);
}

template <int T, int... Ts>
__device__ __forceinline__ bool gemv_dispatch(int type, const DecArgs &A, const DecPhase &P, uint64_t *full,
                                              uint64_t *empty, const uint8_t *stg, float *area, uint32_t cur,
                                              XStage &xst, int *abort_flag, unsigned long long *tp) {
    if (type == T) return gemv_phase<T>(A, P, full, empty, stg, area, cur, xst, abort_flag, tp);
    if constexpr (sizeof...(Ts) > 0)
        return gemv_dispatch<Ts...>(type, A, P, full, empty, stg, area, cur, xst, abort_flag, tp);
    return true;
}

template <int HD, int... Ts>
__global__ void __launch_bounds__(DNT, 1) k_decode(const __grid_constant__ DecArgs A) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + GEMV_NS_MAX;
    int *abort_flag = reinterpret_cast<int *>(smem + 2 * GEMV_NS_MAX * 8);
    DecPhase *ph = reinterpret_cast<DecPhase *>(smem + 256);
    float *area = reinterpret_cast<float *>(smem + A.area_off);
    AttnMetaGroup *meta = reinterpret_cast<AttnMetaGroup *>(smem + A.meta_off);
    uint8_t *stg = smem + A.ring_off;
    // this CTA's phase table into shared memory
    const DecPhase *src = A.ph + (int64_t)blockIdx.x * A.nph;
    for (int i = tid; i < A.nph * (int)(sizeof(DecPhase) / 4); i += DNT)
        reinterpret_cast<uint32_t *>(ph)[i] = reinterpret_cast<const uint32_t *>(src)[i];
    if (tid == 0) {
        for (int i = 0; i < A.ns; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], DNCW);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == DNCW) {
        // producer: stream this CTA's rows of every GEMV phase, in order
        if ((tid & 31) == 0) {
            uint32_t cur = 0;
            bool stop = false;
            for (int p = 0; p < A.nph && !stop; p++) {
                const DecPhase &P = ph[p];
                if (P.kind != DPH_GEMV || P.r1 <= P.r0) continue;
                const GemvSeg &s = P.seg;
                const int R = s.rows_per_stage, nst = (P.r1 - P.r0 + R - 1) / R;
                for (int i = 0; i < nst; i++) {
                    const uint32_t ring = cur;  // stages issued so far
                    const int slot = (int)(ring % (uint32_t)A.ns);
                    if (ring >= (uint32_t)A.ns &&
                        !mbar_wait(&empty[slot], ((ring / (uint32_t)A.ns) - 1u) & 1u)) {
                        stop = true;
                        break;
                    }
                    const int ra = P.r0 + i * R, rbn = min(ra + R, P.r1);
                    const int64_t a0 = ((int64_t)ra * s.rb) & ~int64_t(15);
                    const int64_t a1 = ((int64_t)rbn * s.rb + 15) & ~int64_t(15);
                    uint32_t total = (uint32_t)(a1 - a0);
                    int64_t c0 = 0, c1 = 0;
                    if (s.w2) {
                        c0 = ((int64_t)ra * s.rb2) & ~int64_t(15);
                        c1 = ((int64_t)rbn * s.rb2 + 15) & ~int64_t(15);
                        total += (uint32_t)(c1 - c0);
                    }
                    uint8_t *dst = stg + (size_t)slot * A.sb;
                    mbar_arrive_expect_tx(&full[slot], total);
                    bulk_g2s(dst, s.w + a0, (uint32_t)(a1 - a0), &full[slot]);
                    if (s.w2) bulk_g2s(dst + (a1 - a0), s.w2 + c0, (uint32_t)(c1 - c0), &full[slot]);
                    ++cur;
                }
            }
            // no copy may still be landing when the CTA exits: wait, with the
            // fixed bound, for the last fill of every ring slot used
            for (uint32_t r = cur > (uint32_t)A.ns ? cur - (uint32_t)A.ns : 0u; r < cur; r++)
                mbar_wait_limit(&full[r % (uint32_t)A.ns], (r / (uint32_t)A.ns) & 1u, WAIT_LIMIT);
        }
        return;
    }
    uint32_t cur = 0;
    unsigned long long *tr = A.trace ? A.trace + (size_t)blockIdx.x * A.nph * 4 : nullptr;
    if (tr && tid == 0) tr[0] = gtimer();
    for (int p = 0; p < A.nph; p++) {
        const DecPhase &P = ph[p];
        XStage xst;
        // the phase's norm weights never change: load them before the barrier
        if (P.kind == DPH_GEMV && !P.lpr) stage_x_pre(P.norm_w, P.k, xst, DNCW * 32);
        if (p > 0 && !grid_sync(A.bar, (unsigned)p * gridDim.x, abort_flag, tr ? tr + 4 * (p - 1) + 3 : nullptr,
                                tr ? tr + 4 * p : nullptr))
            return;
        if (P.kind == DPH_GEMV) {
            if (P.r1 > P.r0) {
                if (!gemv_dispatch<Ts...>(P.seg.type, A, P, full, empty, stg, area, cur, xst, abort_flag,
                                          tr ? tr + 4 * p : nullptr))
                    return;
                const int R = P.seg.rows_per_stage;
                cur += (uint32_t)((P.r1 - P.r0 + R - 1) / R);
            }
        } else {
            attn_phase<HD>(A, P, area, meta);
        }
    }
    if (A.amax == nullptr) {
        if (tr) {
            named_sync(1, DNCW * 32);
            if (tid == 0) tr[4 * (A.nph - 1) + 3] = gtimer();
        }
        return;
    }
    if (!grid_sync(A.bar, (unsigned)A.nph * gridDim.x, abort_flag, tr ? tr + 4 * (A.nph - 1) + 3 : nullptr)) return;
    if (blockIdx.x == 0 && tid < A.ntok) {
        // greedy: the argmax keys of the lm_head phase -> next input token
        const int t = tid;
        const unsigned long long key = atomicAdd(&A.amax[t], 0ull);
        const int32_t id = key_index(key);
        A.amax[t] = 0ull;
        A.out[t] = id;
        A.tok[t] = id;
        A.pos[t] += 1;
        A.step[t] += 1;
        const int col = *A.hist_col;
        if (A.hist && col >= 0 && col < A.hist_ld) A.hist[(int64_t)t * A.hist_ld + col] = id;
    }
    if (blockIdx.x == 0) {
        named_sync(1, DNCW * 32);
        if (tid == 0) *A.hist_col += 1;
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static const int DSMEM_MAX = 227 * 1024;

// Launch one decode step; with A == nullptr only check that a CTA of this
// instance (DNT threads, its registers, `smem` bytes) fits on an SM, which
// the cooperative launch of one CTA per SM needs.
template <int HD, int... Ts>
static cudaError_t launch_decode(const DecArgs *Ap, size_t smem, int grid, cudaStream_t st) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_decode<HD, Ts...>, cudaFuncAttributeMaxDynamicSharedMemorySize, DSMEM_MAX);
        if (e != cudaSuccess) return e;
        attr[dev & 63] = true;
    }
    if (!Ap) {
        int nb = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_decode<HD, Ts...>, DNT, smem);
        if (e != cudaSuccess) return e;
        return nb >= 1 ? cudaSuccess : cudaErrorLaunchOutOfResources;
    }
    const DecArgs &A = *Ap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_decode<HD, Ts...>, A);
    if (e != cudaSuccess) return e;
    return launched(1);
}

// Type set of the model's linear weights -> compiled instance.
static int type_mask(int t) { return 1 << t; }
enum : int {
    MASK_Q4K_Q6K = (1 << T_Q4_K) | (1 << T_Q6_K),
    MASK_Q80 = 1 << T_Q8_0,
    MASK_F16 = 1 << T_F16,
    MASK_Q5 = (1 << T_Q5_K) | (1 << T_Q5_0) | (1 << T_F16),
    MASK_ALL = (1 << T_F32) | (1 << T_F16) | (1 << T_Q4_0) | (1 << T_Q5_0) | (1 << T_Q8_0) | (1 << T_Q4_K) |
               (1 << T_Q5_K) | (1 << T_Q6_K),
};

bool decode_plan(DecPlan &plan, const DecLayerDesc *layers, int n_layers, const DecLmDesc &lm, int n_embd,
                 int n_head, int n_head_kv, int head_dim, int n_ff, int num_sms, int ntok) {
    plan = DecPlan();
    if (ntok != 1) return false;
    const int E = n_embd, hd = head_dim, qd = n_head * hd, kvd = n_head_kv * hd, F = n_ff;
    const int G = n_head / n_head_kv;
    if ((hd != 64 && hd != 128) || G > 8) return false;
    int mask = type_mask(lm.type);
    for (int l = 0; l < n_layers; l++) {
        const DecLayerDesc &L = layers[l];
        mask |= type_mask(L.tq) | type_mask(L.tk) | type_mask(L.tv) | type_mask(L.to) | type_mask(L.tg) |
                type_mask(L.tu) | type_mask(L.td);
        if (L.tg != L.tu) return false;
    }
    if ((mask & ~MASK_ALL) != 0) return false;
    plan.inst = (mask & ~MASK_Q4K_Q6K) == 0 ? 1 : (mask & ~MASK_Q80) == 0 ? 2 : (mask & ~MASK_F16) == 0 ? 3
              : (mask & ~MASK_Q5) == 0 ? 4 : 5;
    plan.grid = num_sms;
    const int grid = num_sms;
    // ring: three 40 KB stages (plus 64 bytes of rounding slack per stage)
    plan.ns = 3;
    int64_t maxrow = row_bytes(lm.type, E);
    for (int l = 0; l < n_layers; l++) {
        const DecLayerDesc &L = layers[l];
        maxrow = std::max<int64_t>(maxrow, row_bytes(L.tq, E));
        maxrow = std::max<int64_t>(maxrow, row_bytes(L.tv, E));
        maxrow = std::max<int64_t>(maxrow, row_bytes(L.to, qd));
        maxrow = std::max<int64_t>(maxrow, 2 * row_bytes(L.tg, E));
        maxrow = std::max<int64_t>(maxrow, row_bytes(L.td, F));
    }
    plan.sb = (int)std::max<int64_t>(40 * 1024, ((maxrow + 64 + 127) / 128) * 128);
    // phases
    std::vector<DecPhase> proto;  // one prototype per phase (segments resolved per CTA below)
    struct Seg {
        GemvSegDesc d;
        int64_t rb;
    };
    std::vector<std::vector<Seg>> segs;
    auto add_gemv = [&](std::vector<Seg> s, const float *x, int ldx, int k, const float *norm_w) {
        DecPhase P{};
        P.kind = DPH_GEMV;
        P.x = x;
        P.ldx = ldx;
        P.k = k;
        P.norm_w = norm_w;
        proto.push_back(P);
        segs.push_back(std::move(s));
    };
    for (int l = 0; l < n_layers; l++) {
        const DecLayerDesc &L = layers[l];
        add_gemv({{{L.q, nullptr, L.tq, qd, EPI_STORE, L.q_out, qd, L.q_b, nullptr, nullptr}, row_bytes(L.tq, E)},
                  {{L.k, nullptr, L.tk, kvd, EPI_STORE, L.k_out, kvd, L.k_b, nullptr, nullptr}, row_bytes(L.tk, E)},
                  {{L.v, nullptr, L.tv, kvd, EPI_STORE, L.v_out, kvd, L.v_b, nullptr, nullptr}, row_bytes(L.tv, E)}},
                 L.x, E, E, L.attn_nw);
        DecPhase A{};
        A.kind = DPH_ATTN;
        A.layer = l;
        A.q_nw = L.q_nw;
        A.k_nw = L.k_nw;
        proto.push_back(A);
        segs.push_back({});
        add_gemv({{{L.o, nullptr, L.to, E, EPI_ADD, L.x, E, nullptr, nullptr, nullptr}, row_bytes(L.to, qd)}}, L.att,
                 qd, qd, nullptr);
        add_gemv({{{L.gate, L.up, L.tg, F, EPI_SWIGLU, L.hb, F, nullptr, nullptr, nullptr}, 2 * row_bytes(L.tg, E)}},
                 L.x, E, E, L.ffn_nw);
        add_gemv({{{L.down, nullptr, L.td, E, EPI_ADD, L.x, E, nullptr, nullptr, nullptr}, row_bytes(L.td, F)}}, L.hb,
                 F, F, nullptr);
    }
    add_gemv({{{lm.w, nullptr, lm.type, lm.rows, EPI_STORE, lm.logits, lm.ldy, nullptr, lm.yrow, lm.amax},
               row_bytes(lm.type, E)}},
             lm.x, E, E, lm.norm_w);
    const int nph = (int)proto.size();
    plan.nph = nph;
    plan.table.assign((size_t)grid * nph, DecPhase());
    size_t area = 0;
    for (int p = 0; p < nph; p++) {
        DecPhase P = proto[p];
        if (P.kind != DPH_GEMV) {
            for (int b = 0; b < grid; b++) plan.table[(size_t)b * nph + p] = P;
            continue;
        }
        const std::vector<Seg> &sg = segs[p];
        double total = 0;
        for (const Seg &s : sg) total += (double)s.rb * s.d.n;
        // wide path for a single large matrix with a span decoder
        int lpr = 0;
        const int t0 = sg[0].d.type;
        if (sg.size() == 1 && (t0 == T_Q4_K || t0 == T_Q5_K || t0 == T_Q6_K || t0 == T_Q8_0 || t0 == T_F16) &&
            P.k % 256 == 0 && sg[0].d.n / grid >= 128) {
            const int nsb = P.k / 256;
            lpr = 1;
            while (lpr * 2 <= 4 && nsb % (lpr * 2) == 0) lpr *= 2;
        }
        P.lpr = lpr;
        if (lpr) {
            area = std::max(area, x_bytes(P.k, 1, lpr) - 128);
        } else {
            // staged activations + 32 floats of scratch + team partial sums
            for (const Seg &sgi : sg) {
                const int ts = row_geo(sgi.d.type, P.k).ts, nt = DNCW / ts;
                if (nt < 1) return false;
                const int64_t rmax = (plan.sb - 64) / (row_bytes(sgi.d.type, P.k) * (sgi.d.w2 ? 2 : 1));
                const int prow = ts > 1 ? (int)((rmax + nt - 1) / nt) : 1;
                plan.part_rows = std::max(plan.part_rows, prow);
                area = std::max(area, ((size_t)P.k + 32 + (size_t)nt * (prow * 2 * ts + ts)) * 4);
            }
        }
        int cta0 = 0;
        for (size_t i = 0; i < sg.size(); i++) {
            int nc = (int)((double)sg[i].rb * sg[i].d.n / total * grid + 0.5);
            if (i + 1 == sg.size()) nc = grid - cta0;  // every CTA gets a segment
            nc = std::max(1, std::min<int>(nc, (int)sg[i].d.n));
            GemvSeg g{};
            const GemvSegDesc &d = sg[i].d;
            g.w = static_cast<const uint8_t *>(d.w);
            g.w2 = static_cast<const uint8_t *>(d.w2);
            g.type = d.type;
            g.rb = row_bytes(d.type, P.k);
            g.rb2 = d.w2 ? g.rb : 0;
            g.n = (int)d.n;
            g.epi = d.epi;
            g.y = d.y;
            g.ldy = d.ldy;
            g.bias = d.bias;
            g.yrow = d.yrow;
            g.amax = d.amax;
            g.rows_per_stage = (int)((plan.sb - 64) / (g.rb + g.rb2));
            if (g.rows_per_stage < 1) return false;
            g.cta0 = cta0;
            g.ncta = nc;
            for (int c = 0; c < nc && cta0 + c < grid; c++) {
                DecPhase Q = P;
                Q.seg = g;
                Q.r0 = (int)((int64_t)d.n * c / nc);
                Q.r1 = (int)((int64_t)d.n * (c + 1) / nc);
                plan.table[(size_t)(cta0 + c) * nph + p] = Q;
            }
            cta0 += nc;
            if (cta0 >= grid) break;
        }
        for (int b = cta0; b < grid; b++) {  // CTAs without rows this phase
            DecPhase Q = P;
            Q.seg = GemvSeg{};
            Q.seg.type = t0;
            Q.seg.rows_per_stage = 1;
            Q.r0 = Q.r1 = 0;
            plan.table[(size_t)b * nph + p] = Q;
        }
    }
    const int attn_floats = dec_item_floats(hd, DCH, G);
    plan.attn_group_floats = (attn_floats + 31) & ~31;
    area = std::max(area, (size_t)plan.attn_group_floats * DGROUPS * 4);
    plan.meta_off = (int)((256 + (size_t)nph * sizeof(DecPhase) + 15) & ~size_t(15));
    plan.area_off = (int)((plan.meta_off + DGROUPS * sizeof(AttnMetaGroup) + 1023) & ~size_t(1023));
    plan.ring_off = (int)((plan.area_off + area + 1023) & ~size_t(1023));
    plan.smem = (size_t)plan.ring_off + (size_t)plan.ns * plan.sb + 16;
    while (plan.smem > (size_t)DSMEM_MAX && plan.ns > 2) {
        plan.ns--;
        plan.smem = (size_t)plan.ring_off + (size_t)plan.ns * plan.sb + 16;
    }
    return plan.smem <= (size_t)DSMEM_MAX;
}

cudaError_t decode_launch(const DecPlan &plan, const DecArgs *A, int head_dim, cudaStream_t st) {
    const bool h128 = head_dim == 128;
    switch (plan.inst) {
        case 1: return h128 ? launch_decode<128, T_Q4_K, T_Q6_K>(A, plan.smem, plan.grid, st)
                            : launch_decode<64, T_Q4_K, T_Q6_K>(A, plan.smem, plan.grid, st);
        case 2: return h128 ? launch_decode<128, T_Q8_0>(A, plan.smem, plan.grid, st)
                            : launch_decode<64, T_Q8_0>(A, plan.smem, plan.grid, st);
        case 3: return h128 ? launch_decode<128, T_F16>(A, plan.smem, plan.grid, st)
                            : launch_decode<64, T_F16>(A, plan.smem, plan.grid, st);
        case 4: return h128 ? launch_decode<128, T_Q5_K, T_Q5_0, T_F16>(A, plan.smem, plan.grid, st)
                            : launch_decode<64, T_Q5_K, T_Q5_0, T_F16>(A, plan.smem, plan.grid, st);
        default:
            return h128 ? launch_decode<128, T_Q4_K, T_Q6_K, T_Q8_0, T_F16, T_Q5_K, T_Q5_0, T_Q4_0, T_F32>(
                              A, plan.smem, plan.grid, st)
                        : launch_decode<64, T_Q4_K, T_Q6_K, T_Q8_0, T_F16, T_Q5_K, T_Q5_0, T_Q4_0, T_F32>(
                              A, plan.smem, plan.grid, st);
    }
}

}  // namespace acm
