"""C ABI and host logic without a GPU: the library loads, exports every symbol
include/acm.h declares, and its GGUF parser + config rules (gguf.go:121-174,
model.go:91-151) agree with the oracle's."""
import ctypes as C
import os
import re
import struct

import numpy as np

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "acm.h")).read()
    return sorted(set(re.findall(r"ACM_API[^;(]*?\b(acm_\w+)\s*\(", src)))


def test_library_exports_header(acm):
    L = C.CDLL(acm._lib.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(acm._lib.SIGNATURES), "ctypes table out of sync with include/acm.h"


def test_version(acm):
    assert b"sm_100a" in acm.lib().acm_version()


CFG_FIELDS = ["arch", "n_layers", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff", "vocab", "max_ctx",
              "rope_dim", "rope_base", "rope_interleaved", "rope_scaling", "rope_factor", "rope_lo_f", "rope_hi_f",
              "rope_orig_ctx", "rms_eps", "bos", "eos", "eos2"]


@pytest.mark.parametrize("name", ["qwen3", "qwen2", "llama_f16", "llama_q5", "qwen3_f32"])
@pytest.mark.parametrize("ctx", [0, 100, 100000])
def test_config_matches_oracle(acm, oracle, tiny_models, name, ctx):
    c = acm.LoadConfig(tiny_models[name], ctx)
    o = oracle.Model(tiny_models[name], ctx).cfg
    for f in CFG_FIELDS:
        assert getattr(c, f) == getattr(o, f), f


@pytest.mark.parametrize("name", ["qwen3", "llama_q5"])
def test_config_from_bytes(acm, tiny_models, name):
    """acm_load_config_mem over the file's bytes equals the path entry."""
    with open(tiny_models[name], "rb") as f:
        data = f.read()
    for ctx in (0, 100):
        a, b = acm.LoadConfig(tiny_models[name], ctx), acm.LoadConfigBytes(data, ctx)
        for f in CFG_FIELDS:
            assert getattr(a, f) == getattr(b, f), f
    with pytest.raises(acm.AcmError, match="truncated"):
        acm.LoadConfigBytes(data[:40])


def test_config_rules(acm, synth, tmp_path):
    # llama with freq_base >= 5e5 and no scaling keys gets llama3 defaults (model.go:126-134)
    s = synth.ModelShape("llama", 1, 256, 4, 2, 64, 256, 300, ctx=512, rope_base=5e5)
    c = acm.LoadConfig(synth.build_model(s, str(tmp_path / "a.gguf")))
    assert (c.rope_scaling, c.rope_factor, c.rope_lo_f, c.rope_hi_f, c.rope_orig_ctx) == (2, 32, 1, 4, 8192)
    assert c.rope_interleaved == 1
    # EOS2 is the stop token that is not eos (model.go:142-151)
    assert c.eos == 299 and c.eos2 == 298
    # explicit linear scaling keys are honoured
    s2 = synth.ModelShape("qwen2", 1, 256, 4, 2, 64, 256, 300, ctx=512,
                          extra_kv=[("qwen2.rope.scaling.type", "linear"), ("qwen2.rope.scaling.factor", 4.0)])
    c2 = acm.LoadConfig(synth.build_model(s2, str(tmp_path / "b.gguf")))
    assert (c2.rope_scaling, c2.rope_factor, c2.rope_interleaved) == (1, 4.0, 0)


def _raw_gguf(version=3, arch="qwen3", nt=0, extra=b""):
    def s(x):
        e = x.encode()
        return struct.pack("<Q", len(e)) + e
    kv = s("general.architecture") + struct.pack("<I", 8) + s(arch)
    return b"GGUF" + struct.pack("<IQQ", version, nt, 1) + kv + extra


def test_parse_errors(acm, tmp_path):
    cases = {
        b"NOPE" + b"\0" * 40: ("not a GGUF file", 11),
        _raw_gguf(version=4): ("unsupported GGUF version 4", 11),
        _raw_gguf()[:30]: ("truncated", 11),
        _raw_gguf(arch="gpt2"): ('unsupported architecture "gpt2"', 3),
        _raw_gguf(arch="qwen3"): ("missing required metadata for arch qwen3", 1),
    }
    for i, (blob, (msg, code)) in enumerate(cases.items()):
        p = tmp_path / f"e{i}.gguf"
        p.write_bytes(blob)
        with pytest.raises(acm.AcmError) as ei:
            acm.LoadConfig(str(p))
        assert msg in str(ei.value) and ei.value.code == code
        with pytest.raises(acm.AcmError) as ei:
            acm.LoadConfigBytes(blob)
        assert msg in str(ei.value) and ei.value.code == code


def test_parse_tensor_errors(acm, synth, tmp_path):
    def s(x):
        e = x.encode()
        return struct.pack("<Q", len(e)) + e
    head = b"GGUF" + struct.pack("<IQQ", 3, 1, 1) + s("general.architecture") + struct.pack("<I", 8) + s("qwen3")
    # unsupported tensor type (gguf.go:163-165)
    bad_type = head + s("w") + struct.pack("<IQIQ", 1, 32, 3, 0)
    p = tmp_path / "t.gguf"
    p.write_bytes(bad_type + b"\0" * 256)
    with pytest.raises(acm.AcmError, match="tensor w: unsupported type 3"):
        acm.LoadConfig(str(p))
    # data past the end (gguf.go:166-170)
    oob = head + s("w") + struct.pack("<IQIQ", 1, 1024, 0, 0)
    p.write_bytes(oob + b"\0" * 64)
    with pytest.raises(acm.AcmError, match="tensor w: out of bounds"):
        acm.LoadConfig(str(p))


def test_max_logit_first_max(acm):
    """MaxLogit (model.go:462-471): the first of equal maxima wins; a host
    function of the library, no device involved."""
    rng = np.random.default_rng(3)
    for n in (1, 7, 1000, 151936):
        lg = rng.standard_normal(n).astype(np.float32)
        assert acm.MaxLogit(lg) == int(np.argmax(lg))
    lg = np.array([0.5, 2.0, -1.0, 2.0, 2.0], dtype=np.float32)
    assert acm.MaxLogit(lg) == 1
    lg = np.full(64, -3.0, dtype=np.float32)
    assert acm.MaxLogit(lg) == 0
