"""Full-size parity: the Qwen2-1.5B-shape (all Q8_0, q/k/v biases, 12/2 heads)
and Llama-3.2-1B-shape (F16; Q5_K attention + Q5_0 FFN; 32/8 heads,
head_dim 64, interleaved rope, llama3 scaling) models with seeded random-init
weights, at the prompt lengths of their workloads: 944 tokens, and 1500
tokens (prefill chunks 1024 + 476, sampler.go:116).

Gate: logits within 1e-3 relative L2 of the oracle's fp32 path
and greedy top-1 agreement, on the prefill and on teacher-forced decode
steps.  Decoding the Llama model to its full 2048-position context is
checked through size-independent properties: every step succeeds, the
position ends at 2048, and one more step fails with the reference's
"context length exceeded".
"""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

GATE = 1e-3


@pytest.fixture(scope="module")
def eng(acm):
    e = acm.Engine(0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def full_models(tmp_path_factory, synth):
    d = tmp_path_factory.mktemp("full")
    return {
        "qwen2_1.5b_q8_0": synth.build_model(synth.qwen2_15b(ctx=2048), str(d / "q2.gguf"), seed=21),
        "llama3.2_1b_f16": synth.build_model(synth.llama32_1b_f16(ctx=2048), str(d / "lf.gguf"), seed=22),
        "llama3.2_1b_q5": synth.build_model(synth.llama32_1b_q5(ctx=2048), str(d / "lq.gguf"), seed=23),
    }


@pytest.mark.parametrize("name,plen,seed", [("qwen2_1.5b_q8_0", 944, 3), ("llama3.2_1b_f16", 1500, 4),
                                            ("llama3.2_1b_q5", 1500, 4)])
def test_fullsize_prefill_and_decode(acm, eng, oracle, synth, full_models, name, plen, seed):
    oracle.set_threads(0)
    path = full_models[name]
    m = acm.Load(path, 2048, engine=eng)
    o = oracle.Model(path, 2048)
    p = synth.prompt_ids(plen, m.Cfg.vocab, seed)
    lg, lo = m.Forward(p), o.forward(p)
    assert rel_l2(lg, lo) < GATE
    assert int(np.argmax(lg)) == int(np.argmax(lo))
    tok = int(np.argmax(lo))
    for _ in range(4):  # teacher-forced decode steps
        lg, lo = m.Forward([tok]), o.forward([tok])
        assert rel_l2(lg, lo) < GATE
        assert int(np.argmax(lg)) == int(np.argmax(lo))
        tok = int(np.argmax(lo))
    assert m.Pos() == o.pos == plen + 4
    m.close()


def test_fullsize_decode_to_context_end(acm, eng, synth, full_models):
    """Llama shape: prefill 1500, then greedy decode until the 2048-position
    context is full (the KV cache grows across pages the whole way)."""
    m = acm.Load(full_models["llama3.2_1b_q5"], 2048, engine=eng)
    p = synth.prompt_ids(1500, m.Cfg.vocab, 4)
    ids = m.Generate(p, acm.Sampler(0.0), 548, stop_on_eos=False)
    assert len(ids) == 548 and m.Pos() == 2048
    assert all(0 <= i < m.Cfg.vocab for i in ids)
    with pytest.raises(acm.AcmError) as e:
        m.Forward([ids[-1]])
    assert "context length exceeded" in str(e.value)
    m.close()
