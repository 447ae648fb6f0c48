"""ctypes binding of libacmcuda.so (C ABI declared in include/acm.h).

The library is built in-tree (build.py).  There is no CPU fallback: if the
library is missing or no CUDA device is present, the calls fail loudly.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libacmcuda.so")

ACM_OK = 0
STATUS = {0: "OK", 1: "INVALID", 2: "CTX_EXCEEDED", 3: "UNSUPPORTED_ARCH", 4: "UNSUPPORTED_TYPE",
          5: "MISSING_TENSOR", 6: "OOM", 7: "CUDA", 8: "TIMEOUT", 9: "NO_SEQ", 10: "IO", 11: "FORMAT"}


class AcmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code
        self.status = STATUS.get(code, str(code))


class Config(C.Structure):
    """infer.Config (internal/infer/model.go:14-40)."""
    _fields_ = [("arch", C.c_int32), ("n_layers", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("head_dim", C.c_int32), ("n_ff", C.c_int32), ("vocab", C.c_int32),
                ("max_ctx", C.c_int32), ("rope_dim", C.c_int32), ("rope_base", C.c_float),
                ("rope_interleaved", C.c_int32), ("rope_scaling", C.c_int32), ("rope_factor", C.c_float),
                ("rope_lo_f", C.c_float), ("rope_hi_f", C.c_float), ("rope_orig_ctx", C.c_float),
                ("rms_eps", C.c_float), ("bos", C.c_int32), ("eos", C.c_int32), ("eos2", C.c_int32)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


class CSampler(C.Structure):
    _fields_ = [("temp", C.c_double), ("top_k", C.c_int32), ("top_p", C.c_double), ("seed", C.c_uint64)]


class CStats(C.Structure):
    _fields_ = [("prefill_toks", C.c_int64), ("prefill_s", C.c_double), ("decode_toks", C.c_int64),
                ("decode_s", C.c_double)]


class CRequest(C.Structure):
    _fields_ = [("prompt", C.c_void_p), ("n_prompt", C.c_int32), ("sampler", CSampler), ("max_tok", C.c_int32),
                ("out_ids", C.c_void_p), ("n_out", C.c_int32), ("status", C.c_int32)]


# name -> (restype, argtypes); every symbol of include/acm.h
P = C.c_void_p
SIGNATURES = {
    "acm_version": (C.c_char_p, []),
    "acm_open": (C.c_int, [C.c_int, C.POINTER(P)]),
    "acm_close": (C.c_int, [P]),
    "acm_engine_error": (C.c_char_p, [P]),
    "acm_model_create": (C.c_int, [P, C.POINTER(Config), C.c_int32, C.POINTER(P)]),
    "acm_model_add_tensor": (C.c_int, [P, C.c_char_p, C.c_uint32, C.POINTER(C.c_uint64), C.c_int32, P, C.c_size_t]),
    "acm_model_finalize": (C.c_int, [P]),
    "acm_model_destroy": (C.c_int, [P]),
    "acm_last_error": (C.c_char_p, [P]),
    "acm_model_config": (C.c_int, [P, C.POINTER(Config)]),
    "acm_model_load_gguf": (C.c_int, [P, C.c_char_p, C.c_int32, C.c_int32, C.POINTER(P)]),
    "acm_load_config": (C.c_int, [C.c_char_p, C.c_int32, C.POINTER(Config), C.c_char_p, C.c_int32]),
    "acm_model_load_gguf_mem": (C.c_int, [P, C.c_void_p, C.c_size_t, C.c_int32, C.c_int32, C.POINTER(P)]),
    "acm_model_load_gguf_multi": (C.c_int, [C.POINTER(P), C.c_int32, C.c_char_p, C.c_int32, C.c_int32, C.POINTER(P)]),
    "acm_load_config_mem": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int32, C.POINTER(Config), C.c_char_p, C.c_int32]),
    "acm_seq_open": (C.c_int, [P, C.POINTER(C.c_int32)]),
    "acm_seq_close": (C.c_int, [P, C.c_int32]),
    "acm_seq_reset": (C.c_int, [P, C.c_int32]),
    "acm_seq_pos": (C.c_int, [P, C.c_int32, C.POINTER(C.c_int32)]),
    "acm_forward": (C.c_int, [P, C.c_int32, P, C.c_int32, P]),
    "acm_sample": (C.c_int, [P, C.c_int32, C.POINTER(CSampler), C.c_uint64, C.POINTER(C.c_int32)]),
    "acm_decode_step": (C.c_int, [P, C.c_int32, P, P, P, P, P, P]),
    "acm_generate": (C.c_int, [P, C.c_int32, P, C.c_int32, C.POINTER(CSampler), C.c_int32, C.c_int32, P,
                               C.POINTER(C.c_int32), C.POINTER(CStats)]),
    "acm_max_logit": (C.c_int32, [P, C.c_int32]),
    "acm_dequant": (C.c_int, [P, C.c_uint32, P, C.c_int64, C.c_int64, P]),
    "acm_matmul": (C.c_int, [P, C.c_uint32, P, C.c_int64, C.c_int64, P, C.c_int32, P]),
    "acm_matmul_dev": (C.c_int, [P, C.c_uint32, P, C.c_int64, C.c_int64, P, C.c_int32, P]),
    "acm_bench_matmul": (C.c_int, [P, C.c_uint32, P, C.c_int64, C.c_int32, C.c_int64, C.c_int64, P, C.c_int32, P,
                                   C.c_int32, C.POINTER(C.c_double)]),
    "acm_sample_logits": (C.c_int, [P, P, C.c_int32, C.POINTER(CSampler), C.c_uint64, C.POINTER(C.c_int32)]),
    "acm_sample_dev_noalloc": (C.c_int, [P, P, C.c_int64, C.c_int32, C.c_int32, P, P, P]),
    "acm_engine_stream": (P, [P]),
    "acm_engine_sync": (C.c_int, [P]),
    "acm_engine_set_kv_f16": (C.c_int, [P, C.c_int32]),
    "acm_engine_set_wait_limit": (C.c_int, [P, C.c_int64]),
    "acm_model_last_timing": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "acm_kernel_launches": (C.c_uint64, []),
    "acm_model_bench_gemm": (C.c_int, [P, C.c_int32, C.c_int32, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                       C.POINTER(C.c_int32)]),
    "acm_serve": (C.c_int, [P, C.POINTER(CRequest), C.c_int32, C.c_int32, C.c_int32, C.POINTER(CStats)]),
    "acm_model_debug_layers": (C.c_int, [P, C.c_int32]),
    "acm_model_debug_layers_read": (C.c_int, [P, P, C.c_int64]),
    "acm_model_trace_gemv": (C.c_int, [P, C.c_int32]),
    "acm_model_trace_gemv_read": (C.c_int, [P, P, C.c_int64, C.POINTER(C.c_int32)]),
    "acm_model_bench_gemv": (C.c_int, [P, C.c_int32, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                       C.POINTER(C.c_int32)]),
}

_lib = None


def lib():
    """Load libacmcuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"CUDA engine library not built: {LIB_PATH} (run build.py)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib
