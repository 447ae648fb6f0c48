import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: full-size workloads")


@pytest.fixture(scope="session")
def acm():
    return importlib.import_module("auto-commit-msg_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("auto-commit-msg_b200.synth")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


def tiny_shapes(S):
    """Small models of every architecture and quant mix the engine serves:
    fast for the CPU oracle, same code paths as the full-size shapes."""
    return {
        # Qwen3 layout (QK-norm, NeoX rope), Q4_K / Q6_K mix, head_dim 128
        "qwen3": S.ModelShape("qwen3", 2, 256, 4, 2, 128, 512, 1000, ctx=256),
        # Qwen2 layout (q/k/v biases), all Q8_0, 4 query heads per kv head
        "qwen2": S.ModelShape("qwen2", 2, 256, 4, 1, 64, 512, 1000, ctx=256, t_embd=S.Q8_0, t_q=S.Q8_0,
                              t_k=S.Q8_0, t_v=S.Q8_0, t_o=S.Q8_0, t_gate=S.Q8_0, t_up=S.Q8_0, t_down=S.Q8_0),
        # Llama layout (interleaved rope, llama3 scaling from freq_base), F16
        "llama_f16": S.ModelShape("llama", 2, 256, 4, 2, 64, 768, 1000, ctx=256, rope_base=5e5, eps=1e-5,
                                  t_embd=S.F16, t_q=S.F16, t_k=S.F16, t_v=S.F16, t_o=S.F16, t_gate=S.F16,
                                  t_up=S.F16, t_down=S.F16),
        # Llama layout, Q5_K attention + Q5_0 FFN, untied Q4_0 output
        "llama_q5": S.ModelShape("llama", 2, 256, 4, 2, 64, 768, 1000, ctx=256, rope_base=5e5, eps=1e-5,
                                 t_embd=S.F16, t_q=S.Q5_K, t_k=S.Q5_K, t_v=S.Q5_K, t_o=S.Q5_K, t_gate=S.Q5_0,
                                 t_up=S.Q5_0, t_down=S.Q5_0, tied=False, t_out=S.Q4_0),
        # F32 weights and an untied Q8_0 output, Qwen3 layout
        "qwen3_f32": S.ModelShape("qwen3", 1, 256, 2, 2, 128, 256, 600, ctx=128, t_embd=S.F32, t_q=S.F32,
                                  t_k=S.F32, t_v=S.F32, t_o=S.F32, t_gate=S.F32, t_up=S.F32, t_down=S.F32,
                                  tied=False, t_out=S.Q8_0),
    }


@pytest.fixture(scope="session")
def tiny_models(tmp_path_factory, synth):
    d = tmp_path_factory.mktemp("models")
    out = {}
    for i, (name, shape) in enumerate(tiny_shapes(synth).items()):
        out[name] = synth.build_model(shape, str(d / f"{name}.gguf"), seed=10 + i)
    return out


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def same_bits(a, b):
    """Bit-identical float arrays, treating any NaN as equal to any NaN."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
