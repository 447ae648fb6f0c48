"""Token-loop parity on the GPU: Load / Forward / Generate / Reset / decode
steps through the C ABI against the CPU oracle on the same seeded models.

Gate (per step): logits within 1e-3 relative L2 of the oracle's fp32 path,
greedy top-1 agreement under teacher forcing; the tiny models sit orders of
magnitude inside it (the measured error is asserted at 1e-4)."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

ARCHS = ["qwen3", "qwen2", "llama_f16", "llama_q5", "qwen3_f32"]


@pytest.fixture(scope="module")
def eng(acm):
    e = acm.Engine(0)
    yield e
    e.close()


@pytest.mark.parametrize("name", ARCHS)
def test_forward_and_teacher_forced_decode(acm, eng, oracle, synth, tiny_models, name):
    m = acm.Load(tiny_models[name], 0, engine=eng)
    o = oracle.Model(tiny_models[name], 0)
    assert m.Cfg.vocab == o.cfg.vocab and m.Cfg.eos2 == o.cfg.eos2
    p = synth.prompt_ids(50, m.Cfg.vocab, 7)
    lg, lo = m.Forward(p), o.forward(p)
    assert rel_l2(lg, lo) < 1e-4
    assert int(np.argmax(lg)) == int(np.argmax(lo))
    tok = int(np.argmax(lo))
    for _ in range(12):  # decode steps on the oracle's tokens
        lg, lo = m.Forward([tok]), o.forward([tok])
        assert rel_l2(lg, lo) < 1e-4
        assert int(np.argmax(lg)) == int(np.argmax(lo))
        tok = int(np.argmax(lo))
    assert m.Pos() == o.pos == 62
    m.close()


@pytest.mark.parametrize("name", ["qwen3", "qwen2", "llama_f16"])
def test_prefill_continues_context(acm, eng, oracle, synth, tiny_models, name):
    """A prefill that continues earlier context (Forward of 70 tokens, then of
    130 more at positions 70..199): the second chunk's attention reads keys
    written by the first (the tensor-core attention's pos0 > 0 path, key
    blocks that straddle the chunks, G query heads per kv head)."""
    m = acm.Load(tiny_models[name], 0, engine=eng)
    o = oracle.Model(tiny_models[name], 0)
    p1 = synth.prompt_ids(70, m.Cfg.vocab, 17)
    p2 = synth.prompt_ids(130, m.Cfg.vocab, 18)
    assert rel_l2(m.Forward(p1), o.forward(p1)) < 1e-4
    lg, lo = m.Forward(p2), o.forward(p2)
    assert rel_l2(lg, lo) < 1e-4
    assert int(np.argmax(lg)) == int(np.argmax(lo))
    assert m.Pos() == o.pos == 200
    m.close()


@pytest.mark.parametrize("name", ARCHS)
def test_generate_greedy_matches_oracle(acm, eng, oracle, synth, tiny_models, name):
    m = acm.Load(tiny_models[name], 0, engine=eng)
    o = oracle.Model(tiny_models[name], 0)
    p = synth.prompt_ids(33, m.Cfg.vocab, 3)
    got = m.Generate(p, acm.Sampler(0.0), 40, stop_on_eos=False)
    want = o.generate(p, max_tok=40, stop_on_eos=False)["ids"].tolist()
    assert got == want
    assert m.Stats.PrefillToks == 33 and m.Stats.DecodeToks == 40 and m.Pos() == 73
    # Reset keeps the cache; a second run is identical (model.go:458-460)
    m.Reset()
    assert m.Generate(p, acm.Sampler(0.0), 40, stop_on_eos=False) == got
    m.close()


@pytest.mark.parametrize("name", ["qwen3", "llama_q5"])
def test_forward_sample_topk(acm, eng, oracle, synth, tiny_models, name):
    """Host-driven loop (acm_forward + acm_sample per step, top-k 40, T 0.7,
    teacher-forced on the oracle's tokens).  Two gated properties per step:
    the logits are within 1e-3 relative L2 of the oracle's, and the device
    sampler returns exactly what the reference's Sample (sampler.go:30-76)
    returns on the device's own logits with the same draw.  The ids
    themselves agree except where two candidates tie to within fp32 noise
    (the reference's cumulative walk is order-sensitive); such steps are
    counted and must be rare."""
    m = acm.Load(tiny_models[name], 0, engine=eng)
    o = oracle.Model(tiny_models[name], 0)
    p = synth.prompt_ids(20, m.Cfg.vocab, 11)
    s = acm.Sampler(0.7, 40, 0.0, Seed=77)
    lg, lo = m.Forward(p), o.forward(p)
    differ = 0
    for step in range(40):
        assert rel_l2(lg, lo) < 1e-3
        u = oracle.uniform(77, step)
        g = m.Sample(s, step)
        assert g == oracle.sample(lg, 0.7, 40, 0.0, u)
        w = oracle.sample(lo, 0.7, 40, 0.0, u)
        differ += g != w
        lg, lo = m.Forward([w]), o.forward([w])
    assert differ <= 2
    m.close()


def reachable(oracle, lg, temp, top_k, top_p, u, eps=3e-5, trials=64, seed=0):
    """Ids the reference sampler can return on logits within +-eps of lg
    (fp32 noise of a different summation order)."""
    rng = np.random.default_rng(seed)
    out = {oracle.sample(lg, temp, top_k, top_p, u)}
    for _ in range(trials):
        j = (lg + rng.uniform(-eps, eps, lg.shape)).astype(np.float32)
        out.add(oracle.sample(j, temp, top_k, top_p, u))
    return out


@pytest.mark.parametrize("name", ["qwen3", "llama_q5"])
def test_generate_topk_matches_oracle(acm, eng, oracle, synth, tiny_models, name):
    """Device-side loop (acm_generate) with top-k sampling: ids equal the
    oracle's up to the first step where the oracle's own choice is not
    unique under fp32 noise of the logits (an order tie); that step's device
    choice must be one the reference sampler reaches within that noise."""
    m = acm.Load(tiny_models[name], 0, engine=eng)
    o = oracle.Model(tiny_models[name], 0)
    p = synth.prompt_ids(20, m.Cfg.vocab, 11)
    s = acm.Sampler(0.7, 40, 0.0, Seed=77)
    got = m.Generate(p, s, 30, stop_on_eos=False)
    r = o.generate(p, temp=0.7, top_k=40, seed=77, max_tok=30, stop_on_eos=False, keep_logits=True)
    want = r["ids"].tolist()
    m.close()
    j = next((i for i, (a, b) in enumerate(zip(got, want)) if a != b), None)
    if j is not None:
        ok = reachable(oracle, r["logits"][j], 0.7, 40, 0.0, oracle.uniform(77, j))
        assert len(ok) > 1 and got[j] in ok, (j, got[j], want[j], ok)


def test_generate_stops_on_eos(acm, eng, oracle, synth, tiny_models):
    """Stop on EOS or EOS2 (sampler.go:140): find a prompt whose greedy
    continuation hits a stop id by forcing it through the oracle's loop."""
    m = acm.Load(tiny_models["qwen3"], 0, engine=eng)
    o = oracle.Model(tiny_models["qwen3"], 0)
    p = synth.prompt_ids(25, m.Cfg.vocab, 2)
    free = o.generate(p, max_tok=30, stop_on_eos=False)["ids"].tolist()
    # choose the token at position 9 as a pseudo stop id by reloading with eos patched is not
    # possible; instead check the stop rule by comparing with the oracle with stopping enabled
    o.reset()
    want = o.generate(p, max_tok=30, stop_on_eos=True)["ids"].tolist()
    got = m.Generate(p, acm.Sampler(0.0), 30, stop_on_eos=True)
    assert got == want
    assert got == free[:len(got)]
    m.close()


def test_batched_decode_matches_single(acm, eng, oracle, synth, tiny_models):
    """acm_decode_step over several sequence slots equals per-sequence oracle
    runs (independent sequences, each at its own position)."""
    path = tiny_models["qwen3"]
    m = acm.Load(path, 0, engine=eng, max_seqs=4)
    seqs = [m.seq, m.open_seq(), m.open_seq()]
    prompts = [synth.prompt_ids(n, m.Cfg.vocab, 20 + n) for n in (5, 17, 40)]
    oracles = [oracle.Model(path, 0) for _ in seqs]
    toks = []
    for s, p, o in zip(seqs, prompts, oracles):
        lg = m.Forward(p, seq=s)
        lo = o.forward(p)
        assert rel_l2(lg, lo) < 1e-4
        toks.append(int(np.argmax(lo)))
    samplers = [acm.Sampler(0.0)] * 3
    for step in range(10):
        out, lgs = m.decode_step(seqs, toks, samplers, [step + 1] * 3, want_logits=True)
        for i, o in enumerate(oracles):
            lo = o.forward([toks[i]])
            assert rel_l2(lgs[i], lo) < 1e-4
            assert out[i] == int(np.argmax(lo))
        toks = [int(t) for t in out]
    assert [m.Pos(s) for s in seqs] == [15, 27, 50]
    m.close()


@pytest.mark.parametrize("name,nseq,kv_f16", [("qwen3", 24, False), ("qwen2", 40, False), ("llama_q5", 24, False),
                                              ("qwen3", 24, True)])
def test_batched_decode_streaming_attention(acm, eng, oracle, synth, tiny_models, name, nseq, kv_f16):
    """Enough (token, kv head) pairs in one decode step that attention takes
    the streaming kernel (32-position tiles, running softmax, a few splits per
    pair): every slot's logits against its own oracle run, over contexts of
    1 to 7 tiles (GQA groups of 2 and 4, head dims 128 and 64; fp32 and half
    caches -- the half cache against the fp32 oracle within its stated
    deviation)."""
    tol = 1e-3 if kv_f16 else 1e-4
    path = tiny_models[name]
    m = acm.Load(path, 0, engine=eng, max_seqs=nseq, kv_f16=kv_f16)
    seqs = [m.seq] + [m.open_seq() for _ in range(nseq - 1)]
    rng = np.random.default_rng(nseq)
    lens = [int(n) for n in rng.integers(1, 220, nseq)]
    oracles = [oracle.Model(path, 0) for _ in seqs]
    toks = []
    for s, n, o in zip(seqs, lens, oracles):
        p = synth.prompt_ids(n, m.Cfg.vocab, 900 + n)
        lg, lo = m.Forward(p, seq=s), o.forward(p)
        toks.append(int(np.argmax(lo)))
    samplers = [acm.Sampler(0.0)] * nseq
    for step in range(4):
        out, lgs = m.decode_step(seqs, toks, samplers, [step + 1] * nseq, want_logits=True)
        nxt = []
        for i, o in enumerate(oracles):
            lo = o.forward([toks[i]])
            assert rel_l2(lgs[i], lo) < tol, (i, lens[i], step)
            nxt.append(int(np.argmax(lo)))  # teacher forcing
        toks = nxt
    assert [m.Pos(s) for s in seqs] == [n + 4 for n in lens]
    m.close()


def test_add_tensor_boundary(acm, eng, oracle, synth, tiny_models):
    """The low-level boundary a cgo shim uses: create + add_tensor per GGUF
    tensor (bytes unchanged) + finalize gives the same logits as Load."""
    path = tiny_models["llama_q5"]
    L = acm.lib()
    cfg = acm.LoadConfig(path, 0)
    h = C.c_void_p()
    assert L.acm_model_create(eng.handle, C.byref(cfg), 1, C.byref(h)) == 0
    g = oracle.GGUF(path)
    for t in g.tensors():
        data = g.tensor_bytes(t["name"])
        dims = (C.c_uint64 * len(t["dims"]))(*t["dims"])
        rc = L.acm_model_add_tensor(h, t["name"].encode(), t["type"], dims, len(t["dims"]), data, len(data))
        assert rc == 0, L.acm_last_error(h)
    assert L.acm_model_finalize(h) == 0, L.acm_last_error(h)
    m = acm.Model(eng, h, False)
    ref = acm.Load(path, 0, engine=eng)
    p = synth.prompt_ids(12, cfg.vocab, 1)
    assert np.array_equal(m.Forward(p), ref.Forward(p))
    m.close()
    ref.close()


def test_errors(acm, eng, synth, tiny_models, tmp_path):
    m = acm.Load(tiny_models["qwen3"], 32, engine=eng)
    assert m.Cfg.max_ctx == 32
    m.Forward(list(range(30)))
    with pytest.raises(acm.AcmError, match=r"context length exceeded \(33 > 32\)") as ei:
        m.Forward([1, 2, 3])
    assert ei.value.code == 2
    assert m.Pos() == 30
    with pytest.raises(acm.AcmError, match="out of range"):
        m.Forward([m.Cfg.vocab + 5])
    m.close()
    # a layer tensor missing (model.go:196-199)
    s = synth.ModelShape("qwen3", 2, 256, 4, 2, 128, 512, 300, ctx=64)
    path = synth.build_model(s, str(tmp_path / "x.gguf"))
    import oracle as O
    g = O.GGUF(path)
    L = acm.lib()
    cfg = acm.LoadConfig(path, 0)
    h = C.c_void_p()
    assert L.acm_model_create(eng.handle, C.byref(cfg), 1, C.byref(h)) == 0
    for t in g.tensors():
        if t["name"] == "blk.1.ffn_up.weight":
            continue
        data = g.tensor_bytes(t["name"])
        dims = (C.c_uint64 * len(t["dims"]))(*t["dims"])
        assert L.acm_model_add_tensor(h, t["name"].encode(), t["type"], dims, len(t["dims"]), data, len(data)) == 0
    assert L.acm_model_finalize(h) == 5
    assert L.acm_last_error(h) == b"layer 1: missing tensors"
    L.acm_model_destroy(h)
    # unsupported type at the boundary
    h = C.c_void_p()
    assert L.acm_model_create(eng.handle, C.byref(cfg), 1, C.byref(h)) == 0
    dims = (C.c_uint64 * 1)(32)
    assert L.acm_model_add_tensor(h, b"w", 3, dims, 1, b"\0" * 20, 20) == 4
    L.acm_model_destroy(h)
