"""Parity of the benchmarked workload at full size: the Qwen3-0.6B-shape
Q4_K_M model (28 layers, hidden 1024, 16/8 heads, head_dim 128, FFN 3072,
vocab 151936, Q4_K with Q6_K attn_v / ffn_down, seed 0) with the default
fp32 KV cache at ctx 2048, the 389-token seed-1 prompt, then 64
teacher-forced decode steps -- the shape, positions and kernels bench.py
times (batch-1 decode GEMVs, decode attention over positions 389-452, the
151936-row lm_head).

Gates (the parity bar of this workload): every step's logits within 1e-3 relative L2 of the
oracle's fp32 path (internal/infer/model.go:317-442), and at least 99%
greedy top-1 agreement.  A step whose oracle top-1 / top-2 margin is below
twice the step's largest absolute logit difference counts as a tie: within
the tolerance either id is the reference's choice.  Then the greedy token
loop itself (sampler.go:111-157, acm_generate's CUDA graph with the argmax
folded into the lm_head) must produce the oracle's 64 ids.
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

GATE = 1e-3
PROMPT, STEPS = 389, 64


@pytest.fixture(scope="module")
def bench_model(tmp_path_factory, synth):
    d = tmp_path_factory.mktemp("bench")
    return synth.build_model(synth.qwen3_06b(ctx=2048), str(d / "qwen3-0.6b.gguf"), seed=0)


def test_qwen3_06b_teacher_forced(acm, oracle, synth, bench_model):
    oracle.set_threads(0)
    m = acm.Load(bench_model, 2048, device=0)
    o = oracle.Model(bench_model, 2048)
    p = synth.prompt_ids(PROMPT, m.Cfg.vocab, 1)
    lg, lo = m.Forward(p), o.forward(p)
    errs, margins, ties, mism = [], [], 0, 0
    for step in range(STEPS + 1):
        if step:
            lg, lo = m.Forward([tok]), o.forward([tok])
        e = rel_l2(lg, lo)
        errs.append(e)
        srt = np.sort(lo.astype(np.float64))
        margin = float(srt[-1] - srt[-2])
        margins.append(margin)
        if int(np.argmax(lg)) != int(np.argmax(lo)):
            if margin < 2.0 * float(np.max(np.abs(lg.astype(np.float64) - lo))):
                ties += 1
            else:
                mism += 1
        tok = int(np.argmax(lo))  # teacher forcing: the oracle's greedy id
    assert m.Pos() == o.pos == PROMPT + STEPS
    print(f"\nqwen3-0.6b teacher-forced: {STEPS + 1} steps, max rel L2 {max(errs):.3e}, "
          f"mean {np.mean(errs):.3e}, min top-1 margin {min(margins):.3e}, ties {ties}, mismatches {mism}")
    assert max(errs) < GATE, errs
    assert (STEPS + 1 - mism) / (STEPS + 1) >= 0.99 and mism == 0
    m.close()
    o.close()


def test_qwen3_06b_greedy_generate(acm, oracle, synth, bench_model):
    oracle.set_threads(0)
    m = acm.Load(bench_model, 2048, device=0)
    o = oracle.Model(bench_model, 2048)
    p = synth.prompt_ids(PROMPT, m.Cfg.vocab, 1)
    ids = m.Generate(p, acm.Sampler(0.0), STEPS, stop_on_eos=False)
    want = o.generate(p, max_tok=STEPS, stop_on_eos=False)["ids"].tolist()
    assert ids == want
    m.close()
    o.close()
