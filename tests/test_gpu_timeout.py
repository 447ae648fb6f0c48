"""Failure detection without a GPU fault: every device-side wait of the
library's kernels is bounded, and a wait that runs out is reported as a
status instead of a hang (the reference has no device code; its failures are
returned errors, internal/infer/model.go:320-321).  The test lowers the bound
to zero polls, so the first wait of the next decode step that does not find
its weights already landed gives up at once: the kernel records the
timeout, lets the copies it started land, and returns.  The call must fail
with ACM_ERR_TIMEOUT and "a device-side wait timed out"; with the default
bound back, a fresh engine and model decode normally and match the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ACM_ERR_TIMEOUT = 8


def test_device_wait_timeout_is_reported(acm, oracle, synth, tiny_models):
    path = tiny_models["qwen3"]
    eng = acm.Engine(0)
    lib = acm.lib()
    m = acm.Load(path, 0, engine=eng)
    p = synth.prompt_ids(12, m.Cfg.vocab, 7)
    m.Forward(p)
    try:
        assert lib.acm_engine_set_wait_limit(eng.handle, 0) == 0
        with pytest.raises(acm.AcmError) as e:
            for _ in range(4):  # a one-token step: batch-1 matvecs and the lm_head pipeline
                m.Forward([int(p[-1])])
        assert e.value.code == ACM_ERR_TIMEOUT
        assert "a device-side wait timed out" in str(e.value)
    finally:
        assert lib.acm_engine_set_wait_limit(eng.handle, -1) == 0
    m.close()
    eng.close()
    # the device is usable and correct again: a fresh engine and model
    eng2 = acm.Engine(0)
    m2 = acm.Load(path, 0, engine=eng2)
    o = oracle.Model(path, 0)
    lg, lo = m2.Forward(p), o.forward(p)
    assert float(np.linalg.norm(lg - lo) / np.linalg.norm(lo)) < 1e-4
    ids = m2.Generate([int(np.argmax(lo))], acm.Sampler(0.0), 6, stop_on_eos=False)
    want = o.generate([int(np.argmax(lo))], max_tok=6, stop_on_eos=False)["ids"].tolist()
    assert ids == want
    m2.close()
    eng2.close()
