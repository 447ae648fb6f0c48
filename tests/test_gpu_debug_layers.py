"""DebugLayer (internal/infer/model.go:231-233, called at :427-429) and
MaxLogit (model.go:462-471).

With the per-layer dump on, the residual stream after every layer of the
device's pass must match the oracle's, layer by layer -- the way the
reference's layer_test.go follows a forward through the stack, and what
bisects a logits mismatch to the first layer that diverges.  Checked on a
prefill and on a decode step (whose dump comes from the captured decode
graph)."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["qwen3", "qwen2", "llama_q5"])
def test_debug_layers_match_oracle(acm, oracle, synth, tiny_models, name):
    path = tiny_models[name]
    m = acm.Load(path, 0, device=0)
    o = oracle.Model(path, 0)
    m.DebugLayer(True)
    o.debug_layers(True)
    p = synth.prompt_ids(21, m.Cfg.vocab, 5)
    m.Forward(p)
    o.forward(p)
    got, want = m.DebugLayers(), o.layers.copy()
    for li in range(m.Cfg.n_layers):
        assert rel_l2(got[li], want[li]) < 1e-5, (li, rel_l2(got[li], want[li]))
    # a decode step through Generate's graph: the dump is the last step's
    ids = m.Generate([int(p[-1])], acm.Sampler(0.0), 3, stop_on_eos=False)
    o.generate([int(p[-1])], max_tok=3, stop_on_eos=False)
    got = m.DebugLayers()
    for li in range(m.Cfg.n_layers):
        assert rel_l2(got[li], o.layers[li]) < 1e-4, (li, rel_l2(got[li], o.layers[li]))
    assert len(ids) == 3
    m.DebugLayer(False)
    m.close()
    o.close()
