#!/usr/bin/env python
"""Token-loop benchmark: decode & prefill tok/s of a Qwen3-0.6B-shape Q4_K_M
model (28 layers, hidden 1024, 16/8 heads, head_dim 128, FFN 3072, vocab
151936, Q4_K with Q6_K attn_v/ffn_down, random-init N(0, 0.02) weights),
389-token seeded prompt, 64 greedy decode tokens, ctx 2048, batch 1 -- the
workload the reference's README quotes (200 / 21 tok/s on a 12-core CPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one full Generate (prefill + 64 decode tokens, EOS stopping off so
every step decodes exactly 64 tokens).  Multi-GPU: one process per GPU
(torchrun), each rank serves its own independent sequence (weak scaling, no
collective on the data path; a gloo group carries only the barrier and the
max-over-ranks timing).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

PROMPT_LEN, GEN_TOKENS, CTX = 389, 64, 2048
METRIC = "decode & prefill tok/s, Qwen3-0.6B-shape Q4_K_M, 1/2/4/8 B200; % HBM roofline"
WORKLOAD = "qwen3-0.6b-shape Q4_K_M (Q4_K + Q6_K attn_v/ffn_down), prompt 389, 64 greedy tokens, ctx 2048, batch 1"
MODEL_DIR = os.environ.get("ACM_BENCH_DIR", os.path.join(tempfile.gettempdir(), "acm_bench"))


def dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as td
        td.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as td
        td.barrier()


def allreduce(vals, world, op="max"):
    if world == 1:
        return list(vals)
    import torch
    import torch.distributed as td
    t = torch.tensor(vals, dtype=torch.float64)
    td.all_reduce(t, op=td.ReduceOp.MAX if op == "max" else td.ReduceOp.SUM)
    return t.tolist()


# The model shapes of the parity workloads: (synth builder, file name, prompt
# length, prompt seed, vocab).  qwen3 is the benchmark's own workload.
MODELS = {
    "qwen3": ("qwen3_06b", "qwen3-0.6b-q4km-seed0.gguf", PROMPT_LEN, 1, 151936),
    "qwen2": ("qwen2_15b", "qwen2-1.5b-q8_0-seed0.gguf", 944, 3, 151936),
    "llama_f16": ("llama32_1b_f16", "llama3.2-1b-f16-seed0.gguf", 1500, 4, 128256),
    "llama_q5": ("llama32_1b_q5", "llama3.2-1b-q5-seed0.gguf", 1500, 4, 128256),
}


def model_path(rank, world, name="qwen3"):
    synth = importlib.import_module("auto-commit-msg_b200.synth")
    fn, fname, plen, pseed, vocab = MODELS[name]
    path = os.path.join(MODEL_DIR, fname)
    if rank == 0 and not os.path.exists(path):
        os.makedirs(MODEL_DIR, exist_ok=True)
        tmp = path + f".tmp{os.getpid()}"
        synth.build_model(getattr(synth, fn)(), tmp, seed=0)
        os.replace(tmp, path)
    barrier(world)
    return path, synth.prompt_ids(plen, vocab, seed=pseed)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the burst figure (kernels timed alone)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def bench_gemm(acm, m, ntok=PROMPT_LEN, reps=5):
    """The prefill's tensor-core GEMM launches (q/k/v, o, gate/up, down x 28
    layers at ntok tokens) timed with CUDA events: (s, useful flops, launches)
    per pass, or None when the model has no tensor-core path."""
    import ctypes as C
    sec, fl, nl = C.c_double(), C.c_double(), C.c_int32()
    if acm.lib().acm_model_bench_gemm(m.handle, ntok, reps, C.byref(sec), C.byref(fl), C.byref(nl)):
        return None
    return sec.value, fl.value, nl.value


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if "Active" in v and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_model():
    """Host CPU model name and core count (recorded beside every CPU figure)."""
    name = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    name = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return name, os.cpu_count()


def cpu_baseline(path, prompt, nthreads=0, decode_tokens=GEN_TOKENS):
    """The oracle (a C restatement of the reference's AVX2 CPU path) on the
    host cores: one Generate of the workload (prefill of the 389-token prompt
    + `decode_tokens` greedy steps).  Also returns its ids, the parity check
    of the device's output."""
    import oracle as O
    O.set_threads(nthreads)
    m = O.Model(path, CTX)
    r = m.generate(prompt, max_tok=decode_tokens, stop_on_eos=False)
    st = r["stats"]
    m.close()
    return {"decode_tok_s": st["decode_toks"] / st["decode_s"], "prefill_tok_s": st["prefill_toks"] / st["prefill_s"],
            "cores": O.threads(), "seconds": st["decode_s"] + st["prefill_s"], "ids": [int(i) for i in r["ids"]]}


# The reference arm times a bounded number of full Generates (each ~6 s of
# CPU work on 16 cores): the whole --steps/--warmup run stays within a minute.
REF_STEPS, REF_WARMUP = 4, 1


def run_reference(args, rank, world):
    if rank != 0:
        return
    path, prompt = model_path(0, 1)
    import oracle as O
    O.set_threads(0)
    m = O.Model(path, CTX)
    steps, warmup = min(args.steps, REF_STEPS), min(args.warmup, REF_WARMUP)
    dec_tok, dec_s, pre_tok, pre_s = 0, 0.0, 0, 0.0
    for i in range(warmup + steps):
        m.reset()
        r = m.generate(prompt, max_tok=GEN_TOKENS, stop_on_eos=False)
        if i >= warmup:
            dec_tok += r["stats"]["decode_toks"]
            dec_s += r["stats"]["decode_s"]
            pre_tok += r["stats"]["prefill_toks"]
            pre_s += r["stats"]["prefill_s"]
    v = dec_tok / dec_s
    cpu, ncpu = cpu_model()
    sample = (f"{steps} timed Generates after {warmup} warm-up (of --steps {args.steps} / --warmup {args.warmup}), "
              f"each the full workload: prefill {PROMPT_LEN} tokens + {GEN_TOKENS} greedy decode tokens")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * (dec_s + pre_s) / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "prefill_tok_s": round(pre_tok / pre_s, 3),
        "config": {"workload": WORKLOAD, "impl": "CPU restatement of the reference's AVX2 path (oracle/)"},
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": O.threads(), "kind": "port",
                         "cpu": cpu, "nproc": ncpu, "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args, rank, world, local):
    import torch
    acm = importlib.import_module("auto-commit-msg_b200")
    path, prompt = model_path(rank, world)
    torch.cuda.set_device(local)
    eng = acm.Engine(local)
    m = acm.Load(path, CTX, engine=eng)
    greedy = acm.Sampler(0.0)
    for _ in range(args.warmup):
        m.Generate(prompt, greedy, GEN_TOKENS, stop_on_eos=False)
        m.Reset()
    stream = torch.cuda.ExternalStream(eng.stream(), device=local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    eng.sync()
    clocks = Clocks(local)
    n0 = acm.lib().acm_kernel_launches()
    w0 = time.perf_counter()
    ev0.record(stream)
    dec_s = pre_s = 0.0
    first = None
    for _ in range(args.steps):
        ids = m.Generate(prompt, greedy, GEN_TOKENS, stop_on_eos=False)
        first = first or ids
        dec_s += m.Stats.Decode
        pre_s += m.Stats.Prefill
        m.Reset()
    ev1.record(stream)
    eng.sync()
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    launches = acm.lib().acm_kernel_launches() - n0
    barrier(world)
    ck = clocks.stop()
    dev = ev0.elapsed_time(ev1) * 1e-3
    mx = allreduce([dec_s, pre_s, dev, wall], world, "max")
    tot_launches = int(allreduce([float(launches)], world, "sum")[0])
    dec_max, pre_max, dev_max, wall_max = mx
    value = world * args.steps * GEN_TOKENS / dec_max
    # dominant kernel: the fused dequant-GEMV launches of one decode token
    sec, nbytes, nl = bench_gemv(acm, m)
    peak, peak_kind = peaks()
    achieved = nbytes / sec / 1e9
    traffic = prefill_traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            tj = json.load(f)
        traffic = tj.get("k_gemv_decode_pass_bytes")
        prefill_traffic = tj.get("k_mma_dq_prefill_pass_bytes")
    except Exception:
        pass
    # prefill: the tensor-core GEMM launches of one 389-token prefill
    prefill_roof = None
    g = bench_gemm(acm, m)
    if g:
        gsec, gfl, gnl = g
        tpk, tpk_kind = tensor_peak()
        pipe = 3 * gfl / gsec / 1e12  # three bf16 products per K step on the tensor pipe
        prefill_roof = {"bound": "tensor", "kernel": "k_mma_dq (all GEMM launches of one 389-token prefill)",
                        "achieved": round(pipe, 1), "peak": tpk, "unit": "TFLOP/s", "frac": round(pipe / tpk, 4),
                        "peak_kind": tpk_kind, "useful_tflops": round(gfl / gsec / 1e12, 1),
                        "note": "achieved counts the 3 bf16 products of the hi/lo split (3 x 2*M*N*K per GEMM)",
                        "ms_per_pass": round(gsec * 1e3, 3), "launches_per_pass": gnl, "traffic": prefill_traffic,
                        "traffic_source": "profiles/traffic.json (DRAM bytes of one layer's four launches, one ncu "
                                          "capture with warm caches, x 28 layers)"}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * dev_max / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (random-init weights, seeded prompt)",
        "prefill_tok_s": round(world * args.steps * PROMPT_LEN / pre_max, 1),
        "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": PROMPT_LEN + GEN_TOKENS,
                   "parallelism": f"dp{world} (independent sequences)",
                   "value": "decode tok/s (64 tokens per step / device time of the decode Forward calls)",
                   "l2": "no flush: every decode token streams 366 MB of weights, > 126 MB L2"},
        "e2e": {"value": round(world * args.steps * GEN_TOKENS / wall_max, 2), "unit": "tok/s",
                "h2d_bytes_per_step": PROMPT_LEN * 4 + 128, "d2h_bytes_per_step": GEN_TOKENS * 4,
                "note": "acm_generate through the C ABI: host prompt in, host ids out, prefill included"},
        "roofline": {"bound": "hbm", "kernel": "k_gemv1 + k_gemv (all 113 matvec launches of one decode token)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "bytes_per_pass": int(nbytes), "launches_per_pass": nl, "traffic": traffic,
                     "traffic_source": "profiles/traffic.json (DRAM bytes with warm caches: one layer's four k_gemv1 "
                                       "launches x 28 + the lm_head launch, ncu captures)"},
        "prefill_roofline": prefill_roof,
        "gpu_launches": tot_launches,
        "clocks": ck,
    }
    if world == 1 and rank == 0 and not args.no_cpu:
        cb = cpu_baseline(path, prompt)
        cpu, ncpu = cpu_model()
        line["cpu_baseline"] = {"value": round(cb["decode_tok_s"], 3), "unit": "tok/s", "cores": cb["cores"],
                                "kind": "port", "prefill_tok_s": round(cb["prefill_tok_s"], 2), "cpu": cpu,
                                "nproc": ncpu,
                                "sample": f"one Generate: prefill {PROMPT_LEN} tokens + {GEN_TOKENS} greedy decode "
                                          "tokens, oracle/ on all host threads"}
        # parity of what was timed: the first timed Generate's ids against the oracle's
        line["parity"] = {"ids_equal": first == cb["ids"], "steps": GEN_TOKENS,
                          "first_diff": next((i for i, (a, b) in enumerate(zip(first, cb["ids"])) if a != b), None)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    m.close()
    eng.close()


def bench_gemv(acm, m, reps=20):
    import ctypes as C
    sec, b, nl = C.c_double(), C.c_double(), C.c_int32()
    rc = acm.lib().acm_model_bench_gemv(m.handle, reps, C.byref(sec), C.byref(b), C.byref(nl))
    if rc:
        raise RuntimeError(acm.lib().acm_last_error(m.handle).decode())
    return sec.value, b.value, nl.value


SERVE_N, SERVE_GEN, SERVE_BATCH, SERVE_CTX = 512, 48, 64, 1152


def serve_requests():
    """The many-request workload: 512 prompts of U[300, 1000] uniform ids
    (seed 5), per-request sampler seed 1000 + i, top-k 40, T 0.7, top-p off,
    48 decode tokens each."""
    import numpy as np
    rng = np.random.default_rng(5)
    lens = rng.integers(300, 1001, SERVE_N)
    return [(rng.integers(0, 151936, int(n)).astype(np.int32), 1000 + i) for i, n in enumerate(lens)]


def partition(reqs, world):
    """Longest-prompt-first greedy balancing of (prompt + decode) work."""
    load = [0] * world
    parts = [[] for _ in range(world)]
    for i in sorted(range(len(reqs)), key=lambda i: -len(reqs[i][0])):
        r = min(range(world), key=lambda j: load[j])
        parts[r].append(i)
        load[r] += len(reqs[i][0]) + SERVE_GEN
    return parts


def run_serve(args, rank, world, local):
    """512 independent requests, <= 64 sharing each decode step per GPU
    (acm_serve), data parallel over the ranks; prints prefill and decode
    aggregate tok/s (device time, max over ranks) and the wall-clock rate."""
    import torch
    acm = importlib.import_module("auto-commit-msg_b200")
    path, _ = model_path(rank, world)
    torch.cuda.set_device(local)
    eng = acm.Engine(local)
    m = acm.Load(path, SERVE_CTX, engine=eng, max_seqs=SERVE_BATCH + 1, kv_f16=args.kv_f16)
    reqs = serve_requests()
    mine = [reqs[i] for i in partition(reqs, world)[rank]]
    batch = [(p, acm.Sampler(0.7, 40, 0.0, Seed=seed), SERVE_GEN) for p, seed in mine]
    m.Serve(batch[: min(len(batch), 2 * SERVE_BATCH)], max_batch=SERVE_BATCH, stop_on_eos=False)  # warm-up
    barrier(world)
    torch.cuda.synchronize()
    w0 = time.perf_counter()
    res = m.Serve(batch, max_batch=SERVE_BATCH, stop_on_eos=False)
    wall = time.perf_counter() - w0
    st = m.Stats
    bad = sum(1 for ids, status in res if status != 0 or len(ids) != SERVE_GEN)
    tot = allreduce([float(st.PrefillToks), float(st.DecodeToks), float(bad)], world, "sum")
    mx = allreduce([st.Prefill, st.Decode, wall], world, "max")
    if rank == 0:
        print(json.dumps({
            "metric": "many-request serving: prefill & decode aggregate tok/s (Qwen3-0.6B-shape Q4_K_M)",
            "value": round(tot[1] / mx[1], 1), "unit": "decode tok/s", "prefill_tok_s": round(tot[0] / mx[0], 1),
            "n_gpus": world, "higher_is_better": True, "scaling": "strong",
            "wall_tok_s": round(tot[1] / mx[2], 1), "wall_s": round(mx[2], 3), "failed_requests": int(tot[2]),
            "config": {"workload": f"{SERVE_N} requests, prompts U[300,1000] (seed 5), {SERVE_GEN} decode tokens, "
                                   f"top-k 40, T 0.7, seed 1000+i, <= {SERVE_BATCH} concurrent per GPU, "
                                   "longest-prompt-first partition over GPUs",
                       "kv_cache": "f16" if args.kv_f16 else "f32",
                       "prefill_tokens": int(tot[0]), "decode_tokens": int(tot[1])},
            "data": "synthetic (random-init weights, seeded prompts)"}), flush=True)
    m.close()
    eng.close()


KB_TYPES = {"q4_0": 2, "q5_0": 6, "q8_0": 8, "q4_k": 12, "q5_k": 13, "q6_k": 14}
KB_SHAPES = [(1024, 2048), (2048, 1024), (1024, 3072), (3072, 1024), (1024, 151936)]  # [K x N]
KB_M = (1, 389, 944)
L2_BYTES = 126 * 2**20


def kb_weights(synth, typ, k, n, seed, uniq=509):
    """[N rows of K] weight bytes: `uniq` distinct quantized N(0, 0.02) rows
    repeated over all N rows (quantizing 155M elements per type would take
    longer than the bench itself; the kernels' time does not depend on the
    values)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    one = np.frombuffer(synth.quantize(typ, rng.standard_normal((uniq, k)).astype(np.float32) * 0.02), np.uint8)
    return np.tile(one, -(-n // uniq))[: n * synth.row_bytes(typ, k)]


def run_kernels(args, rank, world, local):
    """The kernel microbench: acm_matmul_dev for every quantized type x
    [K x N] weight shape of the decode/prefill linears and the lm_head, at
    M = 1 (fused dequant-GEMV) and M = 389 / 944 (tensor-core GEMM, the call
    including the dequant + bf16 split of W and x).  L2 is defeated by
    rotating weight copies totalling more than 2 x L2.  GB/s = weight bytes
    per call / time (the reference's matvec bench definition)."""
    import numpy as np
    import torch
    acm = importlib.import_module("auto-commit-msg_b200")
    synth = importlib.import_module("auto-commit-msg_b200.synth")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    eng = acm.Engine(local)
    peak, peak_kind = peaks()
    tpk, tpk_kind = tensor_peak()
    gen = torch.Generator(device=dev).manual_seed(2)
    rows = []
    n0 = acm.lib().acm_kernel_launches()
    for tname, typ in KB_TYPES.items():
        for k, n in KB_SHAPES:
            w = kb_weights(synth, typ, k, n, seed=typ * 1000 + k + n)
            wbytes = w.size
            stride = (wbytes + 16 + 255) // 256 * 256
            copies = max(8, -(-2 * L2_BYTES // wbytes) + 1)
            buf = torch.empty(copies * stride, dtype=torch.uint8, device=dev)
            wt = torch.from_numpy(w).to(dev)
            for c in range(copies):
                buf[c * stride: c * stride + wbytes].copy_(wt)
            buf_view = buf.view(copies, stride)
            buf_view[:, wbytes:].zero_()
            del wt
            for m in KB_M:
                x = torch.randn(m, k, device=dev, generator=gen)
                y = torch.empty(m, n, device=dev)
                reps = max(2 * copies, 64) if m == 1 else max(copies, 8)
                torch.cuda.synchronize()
                sec = eng.bench_matmul(typ, buf.data_ptr(), stride, copies, n, k, x.data_ptr(), m, y.data_ptr(), reps)
                r = {"type": tname, "K": k, "N": n, "M": m, "us": round(sec * 1e6, 2),
                     "weight_GBs": round(wbytes / sec / 1e9, 1), "copies": copies}
                if m == 1:
                    r["hbm_frac"] = round(wbytes / sec / 1e9 / peak, 4)
                else:
                    r["useful_TFLOPs"] = round(2.0 * m * n * k / sec / 1e12, 2)
                rows.append(r)
                del x, y
            del buf, buf_view
            torch.cuda.empty_cache()
    launches = acm.lib().acm_kernel_launches() - n0
    if rank == 0:
        print(json.dumps({
            "metric": "kernel microbench: matmul weight GB/s (mvbench_test.go:30) and GEMM TFLOP/s, L2 defeated",
            "unit": "GB/s", "higher_is_better": True, "n_gpus": 1, "rows": rows,
            "peak": {"hbm_gbs": peak, "kind": peak_kind, "bf16_tflops": tpk, "bf16_kind": tpk_kind},
            "config": {"workload": "6 quantized types x [K x N] in {1024x2048, 2048x1024, 1024x3072, 3072x1024, "
                                   "1024x151936} x M in {1, 389, 944}",
                       "l2": "rotating weight copies totalling > 2 x 126 MB L2",
                       "gemm": "M > 8 calls include the dequant + bf16 hi/lo split of W (the model caches it)"},
            "gpu_launches": int(launches), "data": "synthetic (509 distinct quantized rows, repeated)"}), flush=True)
    eng.close()


def run_profile(args):
    """Short workloads for the profiler (no JSON line): `prefill` runs three
    389-token prefills; `decode` one prefill + `--tokens` greedy decode tokens."""
    import ctypes as C

    import numpy as np

    acm = importlib.import_module("auto-commit-msg_b200")
    lib = acm.lib()
    if args.profile == "gemv":
        # the lm_head-shape matvec ([K x N] = 1024 x 151936, M = 1) of one
        # weight type, 6 calls over 4 weight copies (the first 3 warm up)
        import torch
        synth = importlib.import_module("auto-commit-msg_b200.synth")
        typ = KB_TYPES[args.type]
        k, n = 1024, 151936
        w = kb_weights(synth, typ, k, n, seed=typ)
        stride = (w.size + 16 + 255) // 256 * 256
        buf = torch.zeros(4 * stride, dtype=torch.uint8, device="cuda:0")
        wt = torch.from_numpy(w).cuda()
        for c in range(4):
            buf[c * stride: c * stride + w.size].copy_(wt)
        x, y = torch.randn(1, k, device="cuda:0"), torch.empty(1, n, device="cuda:0")
        eng = acm.Engine(0)
        torch.cuda.synchronize()
        for i in range(6):
            eng.matmul_dev(typ, buf.data_ptr() + (i % 4) * stride, n, k, x.data_ptr(), 1, y.data_ptr())
        eng.sync()
        sec = eng.bench_matmul(typ, buf.data_ptr(), stride, 4, n, k, x.data_ptr(), 1, y.data_ptr(), 64)
        print(f"gemv {args.type} {k}x{n}: {sec * 1e6:.2f} us, {w.size / sec / 1e9:.1f} GB/s", flush=True)
        eng.close()
        return
    path, prompt = model_path(0, 1, args.model)
    eng = acm.Engine(0)
    if args.profile == "serve":
        # the first 64 requests of the many-request workload, `--tokens` decode
        # tokens each: one prefill per request, then 64-token decode steps
        m = acm.Load(path, SERVE_CTX, engine=eng, max_seqs=SERVE_BATCH + 1, kv_f16=args.kv_f16)
        reqs = [(p, acm.Sampler(0.7, 40, 0.0, Seed=seed), args.tokens) for p, seed in serve_requests()[:SERVE_BATCH]]
        m.Serve(reqs, max_batch=SERVE_BATCH, stop_on_eos=False)
        st = m.Stats
        print(f"serve {len(reqs)} requests: decode {st.DecodeToks / st.Decode:.1f} tok/s, "
              f"prefill {st.PrefillToks / st.Prefill:.1f} tok/s", flush=True)
        m.close()
        eng.close()
        return
    if args.profile == "load":
        for i in range(3):  # GGUF parse + upload of every tensor + finalize, wall clock
            t0 = time.perf_counter()
            m = acm.Load(path, CTX, engine=eng)
            eng.sync()
            print(f"load {i}: {1e3 * (time.perf_counter() - t0):.1f} ms ({os.path.getsize(path) / 2**20:.0f} MiB file)",
                  flush=True)
            m.close()
        eng.close()
        return
    m = acm.Load(path, CTX, engine=eng)
    if args.profile == "gtrace":
        # per-CTA timelines of the batch-1 GEMV launches of the last decode token
        slots = 400
        if lib.acm_model_trace_gemv(m.handle, slots):
            raise RuntimeError(lib.acm_last_error(m.handle).decode())
        m.Generate(prompt, acm.Sampler(0.0), args.tokens, stop_on_eos=False)
        print(f"decode {args.tokens} tokens: {args.tokens / m.Stats.Decode:.1f} tok/s", flush=True)
        buf = (C.c_uint64 * (slots * 160 * 8))()
        used = C.c_int32()
        if lib.acm_model_trace_gemv_read(m.handle, buf, slots * 160 * 8, C.byref(used)):
            raise RuntimeError(lib.acm_last_error(m.handle).decode())
        t = np.frombuffer(buf, dtype=np.uint64)[: used.value * 160 * 8].reshape(used.value, 160, 8).astype(np.int64)
        per_tok = 4 * m.Cfg.n_layers + 1
        t = t[used.value - per_tok: used.value]
        valid = t[:, :, 0] > 0
        base = t[:, :, 0][valid].min()
        names = ["qkv", "o", "gateup", "down"] * m.Cfg.n_layers + ["lm_head"]
        prev_end = None
        for i in range(per_tok):
            v = valid[i]
            r = t[i][v]
            st = lambda c: (r[:, c] - base) / 1e3
            sm = np.bincount(r[:, 6].astype(np.int64), minlength=148)
            end = st(5).max()
            print(f"{i:3d} {names[i]:8s} ctas {v.sum():3d} sms {np.count_nonzero(sm):3d} max/sm {sm.max()}  "
                  f"entry {st(0).min():8.2f}..{st(0).max():8.2f}  wait_over {st(2).min():8.2f}..{st(2).max():8.2f}  "
                  f"x {st(3).max():8.2f}  w {st(4).min():8.2f}..{st(4).max():8.2f}  done {st(5).min():8.2f}..{end:8.2f}"
                  + (f"  gap {st(2).min() - prev_end:6.2f}" if prev_end is not None else ""))
            prev_end = end
        lib.acm_model_trace_gemv(m.handle, 0)
        m.close()
        eng.close()
        return
    if args.profile == "prefill":
        for i in range(3):
            m.Forward(prompt)
            eng.sync()
            print(f"prefill {i}: {1e3 * m.last_timing()[0]:.3f} ms", flush=True)
            m.Reset()
    else:
        ids = m.Generate(prompt, acm.Sampler(0.0), args.tokens, stop_on_eos=False)
        print(f"decode {args.tokens} tokens: {args.tokens / m.Stats.Decode:.1f} tok/s", flush=True)
    m.close()
    eng.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--profile", choices=["prefill", "decode", "gtrace", "load", "gemv", "serve"],
                    help="run a short workload for the profiler instead of the benchmark")
    ap.add_argument("--tokens", type=int, default=8, help="decode tokens of --profile decode/gtrace")
    ap.add_argument("--type", choices=list(KB_TYPES), default="q4_k", help="weight type of --profile gemv")
    ap.add_argument("--kv-f16", action="store_true",
                    help="--workload serve / --profile serve with the reduced-precision (IEEE half) KV cache")
    ap.add_argument("--model", choices=list(MODELS), default="qwen3",
                    help="model shape of --profile prefill/decode/gtrace/load (qwen3: the benchmark's own)")
    ap.add_argument("--workload", choices=["single", "serve", "kernels"], default="single",
                    help="single: the batch-1 Generate benchmark (default); serve: 512 requests through acm_serve; "
                         "kernels: the matmul microbench over every quantized type and weight shape")
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
        return
    rank, world, local = dist()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.workload == "serve":
            run_serve(args, rank, world, local)
        elif args.workload == "kernels":
            run_kernels(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as td
            td.destroy_process_group()


if __name__ == "__main__":
    main()
