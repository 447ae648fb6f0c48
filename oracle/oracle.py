"""ctypes binding of the CPU oracle (oracle/acm_oracle.c).

Test infrastructure only: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs load this; the engine never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
SRC_PATH = os.path.join(HERE, "acm_oracle.c")


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (AVX2/FMA, pthreads)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC_PATH):
        cmd = ["gcc", "-O3", "-mavx2", "-mfma", "-fPIC", "-shared", "-Wall", "-o", LIB_PATH + ".tmp",
               SRC_PATH, "-lpthread", "-lm"]
        subprocess.check_call(cmd)
        os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


class Config(C.Structure):
    _fields_ = [("arch", C.c_int), ("n_layers", C.c_int), ("n_embd", C.c_int), ("n_head", C.c_int),
                ("n_head_kv", C.c_int), ("head_dim", C.c_int), ("n_ff", C.c_int), ("vocab", C.c_int),
                ("max_ctx", C.c_int), ("rope_dim", C.c_int), ("rope_base", C.c_float),
                ("rope_interleaved", C.c_int), ("rope_scaling", C.c_int), ("rope_factor", C.c_float),
                ("rope_lo_f", C.c_float), ("rope_hi_f", C.c_float), ("rope_orig_ctx", C.c_float),
                ("rms_eps", C.c_float), ("bos", C.c_int), ("eos", C.c_int), ("eos2", C.c_int)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ndims", C.c_uint32), ("dims", C.c_uint64 * 4), ("type", C.c_uint32),
                ("offset", C.c_uint64), ("numel", C.c_int64), ("data", C.c_void_p), ("nbytes", C.c_uint64)]


class Sampler(C.Structure):
    _fields_ = [("temp", C.c_double), ("top_k", C.c_int32), ("top_p", C.c_double), ("seed", C.c_uint64)]


class Stats(C.Structure):
    _fields_ = [("prefill_toks", C.c_int64), ("prefill_s", C.c_double), ("decode_toks", C.c_int64),
                ("decode_s", C.c_double)]


_lib = None
# DebugLayer callback: (layer, x, ntok, embd, ctx)
_DEBUG_FN = C.CFUNCTYPE(None, C.c_int, C.POINTER(C.c_float), C.c_int, C.c_int, C.c_void_p)


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        L.or_dequant_rows.argtypes = [C.c_uint32, P, C.c_int64, C.c_int64, P]
        L.or_dequant_row.argtypes = [C.c_uint32, P, P, C.c_int64]
        L.or_matmul.argtypes = [P, C.c_uint32, P, C.c_int64, C.c_int64, P, C.c_int]
        L.or_f16.argtypes = [C.c_uint16]
        L.or_f16.restype = C.c_float
        L.or_fast_exp.argtypes = [C.c_float]
        L.or_fast_exp.restype = C.c_float
        L.or_gguf_open.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
        L.or_gguf_open.restype = P
        L.or_gguf_close.argtypes = [P]
        L.or_gguf_str.argtypes = [P, C.c_char_p]
        L.or_gguf_str.restype = C.c_char_p
        L.or_gguf_u64.argtypes = [P, C.c_char_p, C.c_uint64]
        L.or_gguf_u64.restype = C.c_uint64
        L.or_gguf_f32.argtypes = [P, C.c_char_p, C.c_float]
        L.or_gguf_f32.restype = C.c_float
        L.or_gguf_strs_len.argtypes = [P, C.c_char_p]
        L.or_gguf_strs_len.restype = C.c_int64
        L.or_gguf_tensor_count.argtypes = [P]
        L.or_gguf_tensor_at.argtypes = [P, C.c_int]
        L.or_gguf_tensor_at.restype = C.POINTER(Tensor)
        L.or_gguf_tensor.argtypes = [P, C.c_char_p]
        L.or_gguf_tensor.restype = C.POINTER(Tensor)
        L.or_load.argtypes = [P, C.c_int, C.c_char_p, C.c_int]
        L.or_load.restype = P
        L.or_model_free.argtypes = [P]
        L.or_model_config.argtypes = [P]
        L.or_model_config.restype = C.POINTER(Config)
        L.or_model_pos.argtypes = [P]
        L.or_model_set_debug.argtypes = [P, _DEBUG_FN, C.c_void_p]
        L.or_model_set_debug.restype = None
        L.or_model_reset.argtypes = [P]
        L.or_model_freqs.argtypes = [P]
        L.or_model_freqs.restype = C.POINTER(C.c_float)
        L.or_forward.argtypes = [P, P, C.c_int, C.c_char_p, C.c_int]
        L.or_forward.restype = C.POINTER(C.c_float)
        L.or_topk.argtypes = [P, C.c_int, C.c_int, P]
        L.or_greedy.argtypes = [P, C.c_int]
        L.or_sample_u.argtypes = [C.POINTER(Sampler), P, C.c_int, C.c_double]
        L.or_sample.argtypes = [C.POINTER(Sampler), P, C.c_int, C.c_uint64]
        L.or_uniform.argtypes = [C.c_uint64, C.c_uint64]
        L.or_uniform.restype = C.c_double
        L.or_generate.argtypes = [P, P, C.c_int, C.POINTER(Sampler), C.c_int, C.c_int, P, P, C.POINTER(Stats),
                                  C.c_char_p, C.c_int]
        L.or_set_threads.argtypes = [C.c_int]
        L.or_get_threads.restype = C.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def dequant(typ: int, data: bytes, rows: int, k: int) -> np.ndarray:
    buf = np.frombuffer(data, dtype=np.uint8)
    out = np.empty((rows, k), dtype=np.float32)
    if not lib().or_dequant_rows(typ, _ptr(buf), rows, k, _ptr(out)):
        raise ValueError(f"unsupported type {typ}")
    return out


def matmul(typ: int, w: bytes, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """dst[m][n] = x[m][k] . W[n][k] with the reference's matmul algorithm."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    buf = np.frombuffer(w, dtype=np.uint8)
    out = np.empty((x.shape[0], n), dtype=np.float32)
    lib().or_matmul(_ptr(out), typ, _ptr(buf), n, k, _ptr(x), x.shape[0])
    return out


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


def threads() -> int:
    return lib().or_get_threads()


class GGUF:
    def __init__(self, path: str):
        err = C.create_string_buffer(256)
        self.h = lib().or_gguf_open(path.encode(), err, 256)
        if not self.h:
            raise ValueError(err.value.decode())

    def close(self):
        if self.h:
            lib().or_gguf_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def str(self, key):
        return lib().or_gguf_str(self.h, key.encode()).decode()

    def u64(self, key, default=0):
        return lib().or_gguf_u64(self.h, key.encode(), default)

    def f32(self, key, default=0.0):
        return lib().or_gguf_f32(self.h, key.encode(), default)

    def tensors(self):
        out = []
        for i in range(lib().or_gguf_tensor_count(self.h)):
            t = lib().or_gguf_tensor_at(self.h, i).contents
            out.append(dict(name=t.name.decode(), dims=tuple(t.dims[j] for j in range(t.ndims)), type=t.type,
                            offset=t.offset, numel=t.numel, nbytes=t.nbytes, data=t.data))
        return out

    def tensor_bytes(self, name: str) -> bytes:
        p = lib().or_gguf_tensor(self.h, name.encode())
        if not p:
            raise KeyError(name)
        t = p.contents
        return C.string_at(t.data, t.nbytes)


class Model:
    """The oracle's Model (model.go:51-64): Load / Forward / Generate / Reset."""

    def __init__(self, path: str, max_ctx: int = 0):
        self.file = GGUF(path)
        err = C.create_string_buffer(256)
        self.h = lib().or_load(self.file.h, max_ctx, err, 256)
        if not self.h:
            raise ValueError(err.value.decode())
        self.cfg = Config.from_buffer_copy(lib().or_model_config(self.h).contents)

    def close(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None
        if getattr(self, "file", None):
            self.file.close()

    def __del__(self):
        self.close()

    @property
    def pos(self) -> int:
        return lib().or_model_pos(self.h)

    def reset(self):
        lib().or_model_reset(self.h)

    def freqs(self) -> np.ndarray:
        p = lib().or_model_freqs(self.h)
        return np.ctypeslib.as_array(p, shape=(self.cfg.rope_dim // 2,)).copy()

    def debug_layers(self, enable: bool = True) -> None:
        """Record the residual stream of the last token after each layer
        (the DebugLayer hook, model.go:427-429) on the following forwards."""
        if not enable:
            lib().or_model_set_debug(self.h, _DEBUG_FN(0), None)
            self._dbg_cb = None
            return
        self.layers = np.zeros((self.cfg.n_layers, self.cfg.n_embd), dtype=np.float32)

        def cb(li, x, ntok, embd, ctx):
            row = np.ctypeslib.as_array(x, shape=(ntok * embd,))[(ntok - 1) * embd:]
            self.layers[li] = row
        self._dbg_cb = _DEBUG_FN(cb)
        lib().or_model_set_debug(self.h, self._dbg_cb, None)

    def forward(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        err = C.create_string_buffer(256)
        p = lib().or_forward(self.h, _ptr(t), len(t), err, 256)
        if not p:
            raise ValueError(err.value.decode())
        return np.ctypeslib.as_array(p, shape=(self.cfg.vocab,)).copy()

    def generate(self, prompt, temp=0.0, top_k=0, top_p=0.0, seed=0, max_tok=64, stop_on_eos=True,
                 keep_logits=False):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_tok, 1), dtype=np.int32)
        lg = np.zeros((max_tok + 1, self.cfg.vocab), dtype=np.float32) if keep_logits else None
        st = Stats()
        err = C.create_string_buffer(256)
        s = Sampler(temp, top_k, top_p, seed)
        n = lib().or_generate(self.h, _ptr(p), len(p), C.byref(s), max_tok, int(stop_on_eos), _ptr(out),
                              _ptr(lg) if lg is not None else None, C.byref(st), err, 256)
        if n < 0:
            raise ValueError(err.value.decode())
        res = dict(ids=out[:n].copy(), stats=dict(prefill_toks=st.prefill_toks, prefill_s=st.prefill_s,
                                                   decode_toks=st.decode_toks, decode_s=st.decode_s))
        if lg is not None:
            res["logits"] = lg[:n + (1 if n < max_tok else 0)] if n else lg[:1]
        return res


def sample(logits: np.ndarray, temp: float, top_k: int, top_p: float, u: float) -> int:
    s = Sampler(temp, top_k, top_p, 0)
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return lib().or_sample_u(C.byref(s), _ptr(lg), len(lg), u)


def topk(logits: np.ndarray, k: int) -> np.ndarray:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    idx = np.zeros(k, dtype=np.int32)
    n = lib().or_topk(_ptr(lg), len(lg), k, _ptr(idx))
    return idx[:n]


def uniform(seed: int, step: int) -> float:
    return lib().or_uniform(seed, step)


def fast_exp(x: float) -> float:
    return lib().or_fast_exp(x)
