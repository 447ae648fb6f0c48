"""Kernel parity on the GPU through the C ABI (acm_dequant / acm_matmul /
acm_sample_logits) against the CPU oracle.

Tolerances: dequant bit-exact (tensor.go:55-226 is exact in fp32; the
reference pins asm vs scalar at 0 difference, cmp_test.go:37-40); matvec
(m <= 8, CUDA-core fp32) relative L2 <= 2e-6 against a float64 product of the
exact dequantized weights (fp32 accumulation in a different order); GEMM
(m > 8, K a multiple of 64) on the tensor cores with bf16 hi/lo split
operands (hi.hi + hi.lo + lo.hi, fp32 accumulation) relative L2 <= 3e-5;
GEMM with K not a multiple of 64 (CUDA-core fp32) 2e-6; sampler ids identical.
"""

MMA_TOL = 3e-5  # tensor-core GEMM: bf16 split operands (three products)
import os

import numpy as np
import pytest

from conftest import rel_l2, same_bits

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz")
TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q5_0": 6, "q8_0": 8, "q4_k": 12, "q5_k": 13, "q6_k": 14}
QTYPES = [2, 6, 8, 12, 13, 14]


@pytest.fixture(scope="module")
def eng(acm):
    e = acm.Engine(0)
    yield e
    e.close()


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("kind", ["quant", "random"])
def test_dequant_golden(eng, name, kind):
    g = np.load(GOLD)
    rows, k = int(g["rows"]), int(g["k"])
    got = eng.dequant(TYPES[name], g[f"{name}_{kind}_in"].tobytes(), rows, k)
    assert same_bits(got, g[f"{name}_{kind}_out"]).all()


@pytest.mark.parametrize("typ", list(TYPES.values()))
@pytest.mark.parametrize("rows,k", [(37, 1024), (5, 3072), (3, 2048)])
def test_dequant_random_blocks(eng, oracle, synth, typ, rows, k):
    data = synth.random_blocks(typ, rows, k, seed=typ * 31 + rows)
    assert same_bits(eng.dequant(typ, data, rows, k), oracle.dequant(typ, data, rows, k)).all()


def _check_matmul(eng, oracle, synth, typ, n, k, m, seed, tol=2e-6):
    rng = np.random.default_rng(seed)
    w = synth.quantize(typ, rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    x = rng.standard_normal((m, k)).astype(np.float32)
    got = eng.matmul(typ, w, n, k, x)
    want = x.astype(np.float64) @ oracle.dequant(typ, w, n, k).astype(np.float64).T
    assert got.shape == (m, n)
    assert rel_l2(got, want) < tol
    for j in range(m):  # every token row individually
        assert rel_l2(got[j], want[j]) < 5 * tol


@pytest.mark.parametrize("typ", list(TYPES.values()))
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
def test_gemv(eng, oracle, synth, typ, m):
    _check_matmul(eng, oracle, synth, typ, 300, 1024, m, seed=typ + 10 * m)


@pytest.mark.parametrize("typ", list(TYPES.values()))
@pytest.mark.parametrize("n,k", [(77, 3072), (1000, 256), (64, 8192)])
def test_gemv_shapes(eng, oracle, synth, typ, n, k):
    _check_matmul(eng, oracle, synth, typ, n, k, 1, seed=n + k + typ)


@pytest.mark.parametrize("typ", list(TYPES.values()))
@pytest.mark.parametrize("m", [9, 64, 130])
def test_gemm(eng, oracle, synth, typ, m):
    _check_matmul(eng, oracle, synth, typ, 200, 512, m, seed=typ * 3 + m, tol=MMA_TOL)


@pytest.mark.parametrize("typ", [12, 14])
@pytest.mark.parametrize("shape", [(1024, 2048), (2048, 1024), (1024, 3072), (3072, 1024)])
def test_gemm_prefill_shapes(eng, oracle, synth, typ, shape):
    """The prefill GEMMs of the Qwen3-0.6B shape at a 389-token prompt
    (ragged last token tile) on the tensor cores."""
    k, n = shape
    _check_matmul(eng, oracle, synth, typ, n, k, 389, seed=k + n + typ, tol=MMA_TOL)


@pytest.mark.parametrize("typ", [8, 12, 14])
@pytest.mark.parametrize("m", [150, 389])
def test_gemm_wide_token_tiles(eng, oracle, synth, typ, m):
    """8192 rows: 64 row tiles, so the in-kernel dequant GEMM widens its token
    tiles to 2 or 3 blocks of 64 tokens (uneven: 1+2 blocks at 150 tokens,
    3+2+2 at 389; Q8_0's wider rows limit it to 2 blocks)."""
    _check_matmul(eng, oracle, synth, typ, 8192, 512, m, seed=typ + m, tol=MMA_TOL)


@pytest.mark.parametrize("typ", [0, 1, 2, 6, 8])
def test_gemm_k_not_64(eng, oracle, synth, typ):
    """K = 1056 (a multiple of 32, not of 64): the CUDA-core GEMM."""
    _check_matmul(eng, oracle, synth, typ, 150, 1056, 40, seed=typ + 77)


@pytest.mark.parametrize("typ", QTYPES)
@pytest.mark.parametrize("shape", [(1024, 2048), (2048, 1024), (1024, 3072), (3072, 1024)])
def test_microbench_shapes(eng, oracle, synth, typ, shape):
    """The kernel-microbench weight shapes [K x N] at activation batch 1."""
    k, n = shape
    _check_matmul(eng, oracle, synth, typ, n, k, 1, seed=k * 7 + n + typ)


@pytest.mark.parametrize("typ", QTYPES)
def test_microbench_lm_head_shape(eng, oracle, synth, typ):
    """[K x N] = 1024 x 151936 (the tied lm_head) at batch 1: 509 distinct
    quantized rows repeated over all 151936 rows (a prime period, so a row
    index off by anything but a multiple of 509 shows)."""
    k, n, u = 1024, 151936, 509
    rng = np.random.default_rng(typ + 77)
    one = synth.quantize(typ, rng.standard_normal((u, k)).astype(np.float32) * 0.02)
    reps = -(-n // u)
    w = (one * reps)[: n * synth.row_bytes(typ, k)]
    x = rng.standard_normal((1, k)).astype(np.float32)
    got = eng.matmul(typ, w, n, k, x)
    yu = x.astype(np.float64) @ oracle.dequant(typ, one, u, k).astype(np.float64).T
    want = np.tile(yu, (1, reps))[:, :n]
    assert rel_l2(got, want) < 2e-6


@pytest.mark.parametrize("typ,m", [(12, 1), (14, 1), (8, 389)])
def test_bench_matmul_rotates_copies(eng, oracle, synth, typ, m):
    """acm_bench_matmul: every call reads its own weight copy; the last call's
    output is the product with copy (reps - 1) % copies."""
    import torch
    k, n, copies, reps = 1024, 300, 3, 5
    rng = np.random.default_rng(typ + m)
    ws = [synth.quantize(typ, rng.standard_normal((n, k)).astype(np.float32) * 0.02) for _ in range(copies)]
    wb = len(ws[0])
    stride = (wb + 16 + 255) // 256 * 256
    buf = torch.zeros(copies * stride, dtype=torch.uint8, device="cuda:0")
    for c, w in enumerate(ws):
        buf[c * stride: c * stride + wb].copy_(torch.from_numpy(np.frombuffer(w, np.uint8).copy()))
    x = rng.standard_normal((m, k)).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(m, n, device="cuda:0")
    torch.cuda.synchronize()
    sec = eng.bench_matmul(typ, buf.data_ptr(), stride, copies, n, k, dx.data_ptr(), m, dy.data_ptr(), reps)
    assert sec > 0
    last = ws[(reps - 1) % copies]
    want = x.astype(np.float64) @ oracle.dequant(typ, last, n, k).astype(np.float64).T
    assert rel_l2(dy.cpu().numpy(), want) < (MMA_TOL if m > 8 else 2e-6)
    with pytest.raises(Exception):  # overlapping copies are refused
        eng.bench_matmul(typ, buf.data_ptr(), 256, copies, n, k, dx.data_ptr(), m, dy.data_ptr(), reps)


def _logits(v, seed, ties=True):
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal(v).astype(np.float32) * 2
    if ties:  # repeated maxima and repeated values across chunk boundaries
        top = lg.max() + 1
        lg[[5, 4000 % v, 150000 % v, v - 1]] = top
        lg[rng.integers(0, v, 200)] = np.float32(1.25)
    return lg


@pytest.mark.parametrize("v", [1000, 151936, 128256])
def test_sampler_greedy(eng, oracle, acm, v):
    for seed in range(3):
        lg = _logits(v, seed)
        assert eng.sample_logits(lg, acm.Sampler(0.0), 0) == oracle.sample(lg, 0.0, 0, 0.0, 0.5)


@pytest.mark.parametrize("v", [1000, 151936])
@pytest.mark.parametrize("temp,top_k,top_p", [(0.7, 40, 0.0), (1.0, 0, 0.9), (0.5, 64, 0.0), (1.3, 5, 0.5)])
def test_sampler_topk(eng, oracle, acm, v, temp, top_k, top_p):
    for step in range(20):
        lg = _logits(v, 100 + step, ties=step % 2 == 0)
        s = acm.Sampler(temp, top_k, top_p, Seed=1000 + step)
        want = oracle.sample(lg, temp, top_k, top_p, oracle.uniform(1000 + step, step))
        assert eng.sample_logits(lg, s, step) == want
