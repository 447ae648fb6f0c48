"""GGUF upload entry points beside the path one (acm_model_load_gguf):

* acm_model_load_gguf_mem -- infer.Load(gguf.Parse(data), maxCtx)
  (model.go:90-203) over the file's bytes in host memory, which is what the
  reference's host holds after readModel (app/model_unix.go:15-34) or for its
  embedded model (app/app.go:77-89);
* acm_model_load_gguf_multi -- one mapping, parsed once, each staging chunk
  read once and copied to every engine's device (engines may share a device,
  so the test runs on one GPU as well as on several).

Each model must compute exactly what the path-loaded model computes, and a
failing load must leave no model behind and report the reference's error."""
import numpy as np
import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["qwen3", "qwen2", "llama_q5"])
def test_load_bytes_matches_path(acm, oracle, synth, tiny_models, name):
    path = tiny_models[name]
    with open(path, "rb") as f:
        data = f.read()
    a = acm.Load(path, 0)
    b = acm.LoadBytes(data, 0)
    for fld in ("n_layers", "n_embd", "vocab", "max_ctx", "eos", "eos2"):
        assert getattr(a.Cfg, fld) == getattr(b.Cfg, fld)
    p = synth.prompt_ids(12, a.Cfg.vocab, 3)
    la, lb = a.Forward(p), b.Forward(p)
    assert np.array_equal(la, lb)
    o = oracle.Model(path, 0)
    assert rel_l2(lb, o.forward(p)) < 1e-4
    ids_a = a.Generate([int(np.argmax(la))], acm.Sampler(0.0), 6, stop_on_eos=False)
    ids_b = b.Generate([int(np.argmax(lb))], acm.Sampler(0.0), 6, stop_on_eos=False)
    assert ids_a == ids_b
    a.close()
    b.close()
    o.close()


def test_load_bytes_errors(acm, tiny_models):
    with open(tiny_models["qwen3"], "rb") as f:
        data = f.read()
    # the header parses; the tensors reach past the end (gguf.go:166-170)
    with pytest.raises(acm.AcmError, match="out of bounds"):
        acm.LoadBytes(data[: len(data) // 2], 0)
    with pytest.raises(acm.AcmError, match="truncated"):
        acm.LoadBytes(data[:40], 0)
    with pytest.raises(acm.AcmError, match="not a GGUF file"):
        acm.LoadBytes(b"NOPE" + bytes(60), 0)


def test_load_multi_fan_out(acm, synth, tiny_models):
    path = tiny_models["qwen3"]
    ndev = torch.cuda.device_count()
    n = min(max(2, ndev), 4)
    engines = [acm.Engine(i % ndev) for i in range(n)]
    ms = acm.LoadMulti(path, engines, 0)
    assert len(ms) == n
    ref = acm.Load(path, 0)
    p = synth.prompt_ids(20, ref.Cfg.vocab, 5)
    want = ref.Forward(p)
    for m in ms:
        assert np.array_equal(m.Forward(p), want)
    want_ids = ref.Generate([int(np.argmax(want))], acm.Sampler(0.0), 8, stop_on_eos=False)
    for m in ms:
        m.Reset()
        m.Forward(p)
        assert m.Generate([int(np.argmax(want))], acm.Sampler(0.0), 8, stop_on_eos=False) == want_ids
    for m in ms:
        m.close()
    ref.close()
    # a failing load leaves no model and names the reference's error
    with pytest.raises(acm.AcmError, match="open"):
        acm.LoadMulti(path + ".missing", engines, 0)
    for e in engines:
        e.close()
