"""Generate tests/golden/dequant_golden.npz.

Inputs: for every ggml type the reference decodes (internal/gguf/gguf.go:31-40)
two row sets -- N(0, 0.02) weights quantized by acm_b200.synth, and uniformly
random block bytes (every fp16 scale pattern, incl. NaN/Inf/subnormal).
Expected outputs: the dequantization of an independent implementation of the
same ggml block formats, gguf-py 0.19.0 (`gguf.quants.dequantize`), which the
oracle must reproduce bit for bit.  Run in a container where gguf-py is
importable:

    python tests/golden/make_golden.py
"""
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
S = importlib.import_module("auto-commit-msg_b200.synth")

from gguf import GGMLQuantizationType as G  # noqa: E402
from gguf import quants  # noqa: E402

TMAP = {S.F32: G.F32, S.F16: G.F16, S.Q4_0: G.Q4_0, S.Q5_0: G.Q5_0, S.Q8_0: G.Q8_0, S.Q4_K: G.Q4_K,
        S.Q5_K: G.Q5_K, S.Q6_K: G.Q6_K}
ROWS, K = 6, 512


def main():
    out = {}
    for t, gt in TMAP.items():
        name = S.TYPE_NAMES[t]
        rng = np.random.default_rng(100 + t)
        w = (rng.standard_normal((ROWS, K)).astype(np.float32) * 0.02)
        for kind, data in (("quant", S.quantize(t, w)), ("random", S.random_blocks(t, ROWS, K, 200 + t))):
            raw = np.frombuffer(data, dtype=np.uint8).reshape(ROWS, -1)
            with np.errstate(all="ignore"):
                ref = quants.dequantize(raw, gt).astype(np.float32).reshape(ROWS, K)
            out[f"{name}_{kind}_in"] = raw.copy()
            out[f"{name}_{kind}_out"] = ref
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), rows=ROWS, k=K, **out)
    print("wrote", os.path.join(HERE, "dequant_golden.npz"))


if __name__ == "__main__":
    main()
