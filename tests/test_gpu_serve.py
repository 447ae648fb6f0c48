"""Continuous batching (acm_serve) through the C ABI.

Each request must follow Generate's loop (sampler.go:108-157) exactly as a
single-sequence run does: greedy ids equal the oracle's; with top-k sampling
the ids do not depend on which other requests share a decode step (batches of
up to 8 tokens take the same per-token arithmetic), so two different batch
limits give identical ids.  Batches above 8 tokens run the linear layers on
the tensor-core GEMM; greedy ids there are checked against the oracle too.
"""
import pytest

pytestmark = pytest.mark.gpu


def _requests(synth, vocab, sampler, n=10, seed=0):
    import numpy as np

    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        plen = int(rng.integers(3, 70))
        out.append((synth.prompt_ids(plen, vocab, 100 + seed * 31 + i), sampler(i), int(rng.integers(1, 26))))
    return out


@pytest.fixture(scope="module")
def eng(acm):
    e = acm.Engine(0)
    yield e
    e.close()


@pytest.mark.parametrize("max_batch", [4, 12, 24])
def test_serve_greedy_matches_oracle(acm, eng, oracle, synth, tiny_models, max_batch):
    path = tiny_models["qwen3"]
    m = acm.Load(path, 0, engine=eng, max_seqs=max_batch + 1)
    reqs = _requests(synth, m.Cfg.vocab, lambda i: acm.Sampler(0.0), n=max(14, max_batch + 6), seed=max_batch)
    res = m.Serve(reqs, max_batch=max_batch, stop_on_eos=False)
    assert m.Stats.PrefillToks == sum(len(p) for p, _, _ in reqs)
    assert m.Stats.DecodeToks == sum(t for _, _, t in reqs)
    o = oracle.Model(path, 0)
    for (p, _, t), (ids, status) in zip(reqs, res):
        assert status == 0
        o.reset()
        assert ids == o.generate(p, max_tok=t, stop_on_eos=False)["ids"].tolist()
    m.close()


def test_serve_topk_batch_invariant(acm, eng, synth, tiny_models):
    """cfg4's sampler (top-k 40, T 0.7, per-request seed 1000+i): the same
    ids whatever the batch limit, and equal to one-at-a-time Generate runs."""
    path = tiny_models["llama_q5"]
    m = acm.Load(path, 0, engine=eng, max_seqs=7)
    reqs = _requests(synth, m.Cfg.vocab, lambda i: acm.Sampler(0.7, 40, 0.0, Seed=1000 + i), n=12, seed=5)
    a = m.Serve(reqs, max_batch=3, stop_on_eos=False)
    b = m.Serve(reqs, max_batch=6, stop_on_eos=False)
    assert a == b
    assert all(st == 0 and len(ids) == t for (ids, st), (_, _, t) in zip(a, reqs))
    m.close()


def test_serve_stops_on_eos(acm, eng, oracle, synth, tiny_models):
    path = tiny_models["qwen3"]
    m = acm.Load(path, 0, engine=eng, max_seqs=5)
    reqs = _requests(synth, m.Cfg.vocab, lambda i: acm.Sampler(0.0), n=8, seed=9)
    res = m.Serve(reqs, max_batch=4, stop_on_eos=True)
    o = oracle.Model(path, 0)
    for (p, _, t), (ids, status) in zip(reqs, res):
        o.reset()
        assert status == 0 and ids == o.generate(p, max_tok=t, stop_on_eos=True)["ids"].tolist()
    m.close()


def test_serve_request_errors(acm, eng, synth, tiny_models):
    """A request that does not fit the context fails alone (the reference's
    "context length exceeded"); an empty request yields nothing; the others
    complete."""
    path = tiny_models["qwen3"]
    m = acm.Load(path, 0, engine=eng, max_seqs=4)
    ctx = m.Cfg.max_ctx
    v = m.Cfg.vocab
    reqs = [(synth.prompt_ids(10, v, 1), acm.Sampler(0.0), 5),
            (synth.prompt_ids(ctx + 5, v, 2), acm.Sampler(0.0), 5),
            (synth.prompt_ids(12, v, 3), acm.Sampler(0.0), 0),
            (synth.prompt_ids(ctx - 3, v, 4), acm.Sampler(0.0), 10),
            (synth.prompt_ids(7, v, 5), acm.Sampler(0.0), 6)]
    res = m.Serve(reqs, max_batch=3, stop_on_eos=False)
    assert res[0][1] == 0 and len(res[0][0]) == 5
    assert res[1][1] == 2 and res[1][0] == []          # ACM_ERR_CTX_EXCEEDED at prefill
    assert res[2] == ([], 0)
    assert res[3][1] == 2 and len(res[3][0]) == 4      # positions ctx-3 .. ctx-1 forwarded, then no room
    assert res[4][1] == 0 and len(res[4][0]) == 6
    m.close()
