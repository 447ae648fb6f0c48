"""The CPU oracle pinned against independent implementations (CPU only).

* dequant: bit-identical to gguf-py's decoder of the same ggml formats
  (tests/golden/dequant_golden.npz), the pin the reference's own
  TestDequantAsmMatchesScalar (internal/infer/dequant_asm_test.go:15-44) and
  TestAsmVsScalarLogits (cmp_test.go:15-41) express as self-consistency;
* Forward: against a float64 numpy restatement (tests/np_ref.py);
* sampler: Random123's published Philox4x32-10 known-answer vectors and the
  reference's tie rules (sampler.go:19-98).
"""
import os

import numpy as np
import pytest

from conftest import rel_l2, same_bits

GOLD = os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz")
TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q5_0": 6, "q8_0": 8, "q4_k": 12, "q5_k": 13, "q6_k": 14}


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("kind", ["quant", "random"])
def test_dequant_matches_golden(oracle, name, kind):
    g = np.load(GOLD)
    rows, k = int(g["rows"]), int(g["k"])
    raw = g[f"{name}_{kind}_in"]
    want = g[f"{name}_{kind}_out"]
    got = oracle.dequant(TYPES[name], raw.tobytes(), rows, k)
    assert same_bits(got, want).all()


def test_dequant_quantizers_round_trip(oracle, synth):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((8, 1024)).astype(np.float32) * 0.02
    tol = {synth.Q4_0: 0.02, synth.Q5_0: 0.01, synth.Q8_0: 1e-3, synth.Q4_K: 0.01, synth.Q5_K: 6e-3,
           synth.Q6_K: 4e-3, synth.F16: 1e-4, synth.F32: 0.0}
    for t, tl in tol.items():
        back = oracle.dequant(t, synth.quantize(t, w), 8, 1024)
        assert np.abs(back - w).max() <= tl, synth.TYPE_NAMES[t]


@pytest.mark.parametrize("typ", [0, 1, 2, 6, 8, 12, 13, 14])
@pytest.mark.parametrize("m", [1, 3, 4, 9])
def test_matmul_semantics(oracle, synth, typ, m):
    """matmul (tensor.go:253-298): dst[j][i] = x[j] . W[i] with the tile/dot4
    structure; compared with dequant + float64 matmul."""
    rng = np.random.default_rng(typ * 7 + m)
    n, k = 70, 512
    w = synth.quantize(typ, rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    x = rng.standard_normal((m, k)).astype(np.float32)
    got = oracle.matmul(typ, w, n, k, x)
    want = x.astype(np.float64) @ oracle.dequant(typ, w, n, k).astype(np.float64).T
    assert rel_l2(got, want) < 1e-6


def test_philox_known_answers(oracle):
    """Random123 kat_vectors for philox4x32_10."""
    import ctypes as C
    L = oracle.lib()
    L.or_philox4x32_10.argtypes = [C.POINTER(C.c_uint32), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]
    cases = [((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
             ((0xffffffff,) * 4, (0xffffffff, 0xffffffff), (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
             ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
              (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]
    for ctr, key, want in cases:
        c = (C.c_uint32 * 4)(*ctr)
        k = (C.c_uint32 * 2)(*key)
        o = (C.c_uint32 * 4)()
        L.or_philox4x32_10(c, k, o)
        assert tuple(o) == want


def test_uniform_range_and_spread(oracle):
    u = np.array([oracle.uniform(123, s) for s in range(4000)])
    assert (u >= 0).all() and (u < 1).all()
    assert abs(u.mean() - 0.5) < 0.02
    assert len(set(u.tolist())) == len(u)


def test_fast_exp(oracle):
    """fastExp (model.go:282-295), 0 below -87.  Its degree-5 polynomial is
    accurate to ~9e-5 relative (at f -> 1 it gives 1.99983 for 2^f), not the
    1e-6 its comment states; the engine restates the same polynomial."""
    xs = np.linspace(-86.9, 0, 2001, dtype=np.float32)
    got = np.array([oracle.fast_exp(float(x)) for x in xs])
    assert np.max(np.abs(got / np.exp(xs.astype(np.float64)) - 1)) < 1e-4
    assert oracle.fast_exp(-87.5) == 0.0


def test_greedy_and_topk_ties(oracle):
    lg = np.array([0.5, 2.0, 2.0, -1.0, 2.0, 1.0], dtype=np.float32)
    # greedy: first maximum (sampler.go:19-27)
    assert oracle.sample(lg, 0.0, 0, 0.0, 0.3) == 1
    # topK: descending, equal logits keep index order (sampler.go:80-98)
    assert oracle.topk(lg, 4).tolist() == [1, 2, 4, 5]
    assert oracle.topk(lg, 2).tolist() == [1, 2]
    assert oracle.topk(lg, 10).tolist() == [1, 2, 4, 5, 0, 3]


def test_sample_draw_rules(oracle):
    lg = np.array([0.0, 1.0, 3.0, 2.0], dtype=np.float32)
    # top-k 1 at any temperature is argmax
    for u in (0.0, 0.5, 0.999):
        assert oracle.sample(lg, 0.7, 1, 0.0, u) == 2
    # r = u*sum walks candidates in descending order (sampler.go:71-76)
    p = np.exp((np.array([3.0, 2.0, 1.0, 0.0]) - 3.0) / 1.0)
    c = np.cumsum(p) / p.sum()
    assert oracle.sample(lg, 1.0, 0, 0.0, c[0] * 0.999) == 2
    assert oracle.sample(lg, 1.0, 0, 0.0, (c[0] + c[1]) / 2) == 3
    assert oracle.sample(lg, 1.0, 0, 0.0, 0.9999999) == 0
    # top-p cut: first prefix whose mass reaches top_p (sampler.go:52-69)
    assert oracle.sample(lg, 1.0, 0, 0.5, 0.999) == 2


@pytest.mark.parametrize("name", ["qwen3", "qwen2", "llama_f16", "llama_q5", "qwen3_f32"])
def test_forward_vs_float64_restatement(oracle, tiny_models, name):
    import np_ref
    m = oracle.Model(tiny_models[name], 0)
    cfg = {f: getattr(m.cfg, f) for f, _ in m.cfg._fields_}
    ref = np_ref.RefModel(np_ref.load_weights(m.file, oracle), cfg)
    rng = np.random.default_rng(5)
    p = rng.integers(0, cfg["vocab"], 40).astype(np.int32)
    assert rel_l2(m.forward(p), ref.forward(p)) < 1e-4
    for t in (7, 11, 3):  # decode steps reuse the cache
        assert rel_l2(m.forward([t]), ref.forward([t])) < 1e-4
    assert m.pos == 43


def test_generate_stop_rules(oracle, tiny_models, synth):
    m = oracle.Model(tiny_models["qwen3"], 0)
    p = synth.prompt_ids(20, m.cfg.vocab, 9)
    r = m.generate(p, max_tok=12, stop_on_eos=False, keep_logits=True)
    assert len(r["ids"]) == 12 and r["stats"]["decode_toks"] == 12 and r["stats"]["prefill_toks"] == 20
    # greedy: every id is the argmax of the logits it was sampled from
    for i, t in enumerate(r["ids"]):
        assert t == int(np.argmax(r["logits"][i]))
    assert m.pos == 32
    m.reset()
    assert m.pos == 0
    # the sampled sequence is reproducible after Reset (sampler.go:111, model.go:458-460)
    r2 = m.generate(p, max_tok=12, stop_on_eos=False)
    assert r2["ids"].tolist() == r["ids"].tolist()


def test_prefill_chunking(oracle, synth, tmp_path):
    """Generate prefills in chunks of <= 1024 (sampler.go:116-129); the
    chunked result equals one Forward over the whole prompt."""
    shape = synth.ModelShape("qwen3", 1, 256, 2, 1, 128, 256, 500, ctx=1400)
    path = synth.build_model(shape, str(tmp_path / "c.gguf"), seed=2)
    m = oracle.Model(path, 0)
    p = synth.prompt_ids(1100, 500, 4)
    r = m.generate(p, max_tok=1, stop_on_eos=False, keep_logits=True)
    m2 = oracle.Model(path, 0)
    lg = m2.forward(p)
    assert rel_l2(r["logits"][0], lg) < 1e-5


def test_context_exceeded(oracle, tiny_models):
    m = oracle.Model(tiny_models["qwen3"], 64)
    assert m.cfg.max_ctx == 64
    m.forward(list(range(60)))
    with pytest.raises(ValueError, match=r"context length exceeded \(65 > 64\)"):
        m.forward(list(range(5)))
