"""acm_sample_dev_noalloc -- the sampler with its scratch in a fixed buffer
of the library image -- against acm_sample_logits, the entry point that
stages through the engine's allocator.  Both run the same sampler
(Sampler.Sample, sampler.go:30-76) on the same logits, so the token ids must
be identical (tolerance: none), on two calls in a row.

Collected last on purpose (file name), so it also runs after every other GPU
test has used the engine's own scratch.
"""
import ctypes as C
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ACM_ERR_INVALID = 1


@pytest.fixture(scope="module")
def env(acm):
    import torch

    lib = importlib.import_module("auto-commit-msg_b200._lib")
    e = acm.Engine(0)
    yield e, lib, torch
    e.close()


def _noalloc(env, d_lg, ld, rows, vocab, samplers, steps, d_out):
    e, lib, _ = env
    arr = (lib.CSampler * rows)(*[s.c() for s in samplers]) if samplers is not None else None
    st = (C.c_uint64 * rows)(*steps) if steps is not None else None
    return lib.lib().acm_sample_dev_noalloc(e.handle, C.c_void_p(d_lg), ld, rows, vocab,
                                            C.cast(arr, C.c_void_p) if arr is not None else None,
                                            C.cast(st, C.c_void_p) if st is not None else None,
                                            C.c_void_p(d_out))


def _check(env, acm, lg, ld, samplers, steps):
    e, lib, torch = env
    rows, vocab = lg.shape[0], lg.shape[1]
    host = np.zeros((rows, ld), dtype=np.float32)
    host[:, :vocab] = lg
    d_lg = torch.from_numpy(host).to("cuda:0")
    d_out = torch.empty(rows, dtype=torch.int32, device="cuda:0")
    want = [e.sample_logits(np.ascontiguousarray(lg[r]), samplers[r] if samplers else acm.Sampler(0.0),
                            steps[r] if steps else 0) for r in range(rows)]
    for _ in range(2):  # two calls in a row on the same scratch
        d_out.fill_(-1)
        torch.cuda.synchronize()
        rc = _noalloc(env, d_lg.data_ptr(), ld, rows, vocab, samplers, steps, d_out.data_ptr())
        assert rc == 0, lib.lib().acm_engine_error(e.handle).decode()
        e.sync()
        assert d_out.cpu().numpy().tolist() == want


def test_noalloc_sampler_mixed_rows(env, acm):
    rng = np.random.default_rng(7)
    rows, vocab = 6, 151936
    lg = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    lg[1, 500] = lg[1, 70000] = lg[1].max() + 1.0  # greedy tie: lower index wins
    S = acm.Sampler
    samplers = [S(0.0), S(0.0), S(0.7, 40, 0.0, 11), S(0.7, 40, 0.9, 12), S(1.3, 0, 0.0, 13), S(0.5, 5, 0.5, 14)]
    steps = [3, 4, 17, 5, 1 << 40, 0]
    _check(env, acm, lg, vocab, samplers, steps)


def test_noalloc_sampler_greedy_strided(env, acm):
    rng = np.random.default_rng(8)
    rows, vocab, ld = 64, 32000, 32768  # the row limit, padded row stride, all greedy
    lg = rng.standard_normal((rows, vocab)).astype(np.float32)
    _check(env, acm, lg, ld, None, None)


def test_noalloc_sampler_largest_vocab(env, acm):
    rng = np.random.default_rng(9)
    rows, vocab = 2, 262144
    lg = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    S = acm.Sampler
    _check(env, acm, lg, vocab, [S(0.8, 64, 0.95, 21), S(0.0)], [7, 8])


@pytest.mark.parametrize("rows,vocab", [(65, 1000), (0, 1000), (1, 262145)])
def test_noalloc_sampler_limits(env, rows, vocab):
    e, lib, torch = env
    d = torch.zeros(16, dtype=torch.float32, device="cuda:0")
    rc = _noalloc(env, d.data_ptr(), vocab, rows, vocab, None, None, d.data_ptr())
    assert rc == ACM_ERR_INVALID
    msg = lib.lib().acm_engine_error(e.handle).decode()
    assert "acm_sample_dev_noalloc" in msg and "fixed scratch" in msg
