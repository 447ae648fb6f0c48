"""Python mirror of the reference's engine API (internal/infer) over the C ABI.

Names follow the Go package so tests read like the reference's own:
``Load`` (model.go:90), ``Model.Forward`` (model.go:317), ``Model.Generate``
(sampler.go:111), ``Model.Reset`` / ``Model.Pos`` (model.go:455-460),
``Model.Cfg``, ``Model.Stats`` (sampler.go:101-106), ``Sampler``
(sampler.go:12-17) and ``MaxLogit`` (model.go:462-471).  Every call goes
through libacmcuda.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import AcmError, Config, CSampler, CStats


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


@dataclass
class Sampler:
    """infer.Sampler.  The reference draws from a time-seeded PCG; here the
    draw of sample call `step` is Philox4x32-10 keyed by Seed."""
    Temp: float = 0.0
    TopK: int = 0
    TopP: float = 0.0
    Seed: int = 0

    def c(self) -> CSampler:
        return CSampler(float(self.Temp), int(self.TopK), float(self.TopP), int(self.Seed) & ((1 << 64) - 1))


@dataclass
class Stats:
    """infer.Stats; durations in seconds (device time from CUDA events)."""
    PrefillToks: int = 0
    Prefill: float = 0.0
    DecodeToks: int = 0
    Decode: float = 0.0


class Engine:
    """One CUDA device and its stream."""

    def __init__(self, device: int = 0):
        self._h = C.c_void_p()
        rc = _lib.lib().acm_open(device, C.byref(self._h))
        if rc:
            raise AcmError(rc, f"acm_open({device}) failed (status {_lib.STATUS.get(rc, rc)})")
        self.device = device

    @property
    def handle(self):
        return self._h

    def _check(self, rc: int):
        if rc:
            raise AcmError(rc, _lib.lib().acm_engine_error(self._h).decode())

    def close(self):
        if self._h:
            _lib.lib().acm_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- kernel-level entry points --
    def dequant(self, typ: int, data: bytes, rows: int, k: int) -> np.ndarray:
        buf = np.frombuffer(data, dtype=np.uint8)
        out = np.empty((rows, k), dtype=np.float32)
        self._check(_lib.lib().acm_dequant(self._h, typ, _ptr(buf), rows, k, _ptr(out)))
        return out

    def matmul(self, typ: int, w: bytes, n: int, k: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
        buf = np.frombuffer(w, dtype=np.uint8)
        out = np.empty((x.shape[0], n), dtype=np.float32)
        self._check(_lib.lib().acm_matmul(self._h, typ, _ptr(buf), n, k, _ptr(x), x.shape[0], _ptr(out)))
        return out

    def matmul_dev(self, typ: int, d_w: int, n: int, k: int, d_x: int, m: int, d_y: int) -> None:
        self._check(_lib.lib().acm_matmul_dev(self._h, typ, C.c_void_p(d_w), n, k, C.c_void_p(d_x), m,
                                              C.c_void_p(d_y)))

    def bench_matmul(self, typ: int, d_w: int, w_stride: int, copies: int, n: int, k: int, d_x: int, m: int,
                     d_y: int, reps: int) -> float:
        """Mean device seconds of one matmul_dev call over `reps` back-to-back
        calls cycling through `copies` weight copies (acm_bench_matmul)."""
        sec = C.c_double()
        self._check(_lib.lib().acm_bench_matmul(self._h, typ, C.c_void_p(d_w), w_stride, copies, n, k,
                                                C.c_void_p(d_x), m, C.c_void_p(d_y), reps, C.byref(sec)))
        return sec.value

    def sample_logits(self, logits: np.ndarray, s: Sampler, step: int) -> int:
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        out = C.c_int32(-1)
        cs = s.c()
        self._check(_lib.lib().acm_sample_logits(self._h, _ptr(lg), len(lg), C.byref(cs), step, C.byref(out)))
        return out.value

    def stream(self) -> int:
        return _lib.lib().acm_engine_stream(self._h) or 0

    def sync(self):
        self._check(_lib.lib().acm_engine_sync(self._h))


class Model:
    """A loaded model with `max_seqs` sequence slots.  Slot 0 is this object's
    own sequence (the reference Model holds exactly one); the others serve
    batched decode (scheduler.py)."""

    def __init__(self, engine: Engine, handle: C.c_void_p, own_engine: bool):
        self._e = engine
        self._h = handle
        self._own_engine = own_engine
        cfg = Config()
        self._check(_lib.lib().acm_model_config(self._h, C.byref(cfg)))
        self.Cfg = cfg
        self.Stats = Stats()
        s = C.c_int32(-1)
        self._check(_lib.lib().acm_seq_open(self._h, C.byref(s)))
        self.seq = s.value

    @property
    def engine(self) -> Engine:
        return self._e

    @property
    def handle(self):
        return self._h

    def _check(self, rc: int):
        if rc:
            raise AcmError(rc, _lib.lib().acm_last_error(self._h).decode())

    def close(self):
        if self._h:
            _lib.lib().acm_model_destroy(self._h)
            self._h = C.c_void_p()
        if self._own_engine and self._e is not None:
            self._e.close()
            self._e = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- model.go --
    def Pos(self, seq: Optional[int] = None) -> int:
        p = C.c_int32()
        self._check(_lib.lib().acm_seq_pos(self._h, self.seq if seq is None else seq, C.byref(p)))
        return p.value

    def Reset(self, seq: Optional[int] = None) -> None:
        self._check(_lib.lib().acm_seq_reset(self._h, self.seq if seq is None else seq))

    def Forward(self, tokens: Sequence[int], seq: Optional[int] = None, want_logits: bool = True):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.Cfg.vocab, dtype=np.float32) if want_logits else None
        self._check(_lib.lib().acm_forward(self._h, self.seq if seq is None else seq, _ptr(t), len(t), _ptr(out)))
        return out

    def Sample(self, s: Sampler, step: int, seq: Optional[int] = None) -> int:
        out = C.c_int32(-1)
        cs = s.c()
        self._check(_lib.lib().acm_sample(self._h, self.seq if seq is None else seq, C.byref(cs), step,
                                          C.byref(out)))
        return out.value

    # -- sampler.go --
    def Generate(self, prompt: Sequence[int], s: Optional[Sampler] = None, maxTok: int = 64,
                 onToken: Optional[Callable[[int], None]] = None, stop_on_eos: bool = True,
                 seq: Optional[int] = None) -> list:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(maxTok, 1), dtype=np.int32)
        n = C.c_int32(0)
        st = CStats()
        cs = (s or Sampler()).c()
        self._check(_lib.lib().acm_generate(self._h, self.seq if seq is None else seq, _ptr(p), len(p), C.byref(cs),
                                            maxTok, int(stop_on_eos), _ptr(out), C.byref(n), C.byref(st)))
        self.Stats = Stats(st.prefill_toks, st.prefill_s, st.decode_toks, st.decode_s)
        ids = [int(v) for v in out[:n.value]]
        if onToken is not None:
            for i in ids:
                onToken(i)
        return ids

    def Serve(self, requests: Sequence[tuple], max_batch: int = 0, stop_on_eos: bool = True):
        """Continuous batching over independent requests (acm_serve): each
        request is (prompt, Sampler, maxTok) and runs Generate's loop with the
        same draws as Generate; up to max_batch (0: all free slots) share each
        decode step.  Returns [(ids, status)] in request order; Stats holds
        the summed prefill / decode tokens and device seconds."""
        keep, reqs = [], (_lib.CRequest * max(len(requests), 1))()
        for i, (prompt, s, max_tok) in enumerate(requests):
            p = np.ascontiguousarray(prompt, dtype=np.int32)
            out = np.zeros(max(int(max_tok), 1), dtype=np.int32)
            keep.append((p, out))
            reqs[i].prompt = p.ctypes.data
            reqs[i].n_prompt = len(p)
            reqs[i].sampler = (s or Sampler()).c()
            reqs[i].max_tok = int(max_tok)
            reqs[i].out_ids = out.ctypes.data
        st = CStats()
        self._check(_lib.lib().acm_serve(self._h, reqs, len(requests), int(max_batch), int(stop_on_eos),
                                         C.byref(st)))
        self.Stats = Stats(st.prefill_toks, st.prefill_s, st.decode_toks, st.decode_s)
        return [([int(v) for v in keep[i][1][:reqs[i].n_out]], int(reqs[i].status)) for i in range(len(requests))]

    # -- batched decode (several sequence slots) --
    def open_seq(self) -> int:
        s = C.c_int32(-1)
        self._check(_lib.lib().acm_seq_open(self._h, C.byref(s)))
        return s.value

    def close_seq(self, seq: int) -> None:
        self._check(_lib.lib().acm_seq_close(self._h, seq))

    def decode_step(self, seqs: Sequence[int], in_tok: Sequence[int], samplers: Sequence[Sampler],
                    steps: Sequence[int], want_logits: bool = False):
        n = len(seqs)
        sq = np.ascontiguousarray(seqs, dtype=np.int32)
        it = np.ascontiguousarray(in_tok, dtype=np.int32)
        arr = (CSampler * n)(*[s.c() for s in samplers])
        stp = np.ascontiguousarray(steps, dtype=np.uint64)
        out = np.zeros(n, dtype=np.int32)
        lg = np.empty((n, self.Cfg.vocab), dtype=np.float32) if want_logits else None
        self._check(_lib.lib().acm_decode_step(self._h, n, _ptr(sq), _ptr(it), C.cast(arr, C.c_void_p), _ptr(stp),
                                               _ptr(out), _ptr(lg)))
        return (out, lg) if want_logits else out

    def DebugLayer(self, enable: bool = True) -> None:
        """Turn the per-layer residual dump on or off (DebugLayer,
        model.go:231-233, :427-429); see DebugLayers."""
        self._check(_lib.lib().acm_model_debug_layers(self._h, 1 if enable else 0))

    def DebugLayers(self) -> np.ndarray:
        """Residual stream of the last pass's last token after each layer,
        [n_layers][n_embd] (DebugLayer must be on)."""
        out = np.zeros((self.Cfg.n_layers, self.Cfg.n_embd), dtype=np.float32)
        self._check(_lib.lib().acm_model_debug_layers_read(self._h, _ptr(out), out.size))
        return out

    def last_timing(self):
        a, b = C.c_double(), C.c_double()
        self._check(_lib.lib().acm_model_last_timing(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value


def Load(path: str, maxCtx: int = 0, engine: Optional[Engine] = None, max_seqs: int = 1,
         device: int = 0, kv_f16: bool = False) -> Model:
    """infer.Load (model.go:90-203) on a GGUF file path: parse, derive the
    config, upload the blocks unchanged and build the device state.  kv_f16:
    keep the KV cache in IEEE half (acm_engine_set_kv_f16; no reference
    counterpart)."""
    own = engine is None
    e = engine or Engine(device)
    h = C.c_void_p()
    _lib.lib().acm_engine_set_kv_f16(e.handle, 1 if kv_f16 else 0)
    rc = _lib.lib().acm_model_load_gguf(e.handle, path.encode(), maxCtx, max_seqs, C.byref(h))
    _lib.lib().acm_engine_set_kv_f16(e.handle, 0)
    if rc:
        msg = _lib.lib().acm_engine_error(e.handle).decode()
        if own:
            e.close()
        raise AcmError(rc, msg)
    return Model(e, h, own)


def LoadBytes(data, maxCtx: int = 0, engine: Optional[Engine] = None, max_seqs: int = 1,
              device: int = 0) -> Model:
    """infer.Load(gguf.Parse(data), maxCtx) (model.go:90-203, gguf.go:121-174)
    over a GGUF image in host memory (bytes, a bytearray, an mmap or a numpy
    uint8 array): what the reference's host holds after readModel or for its
    embedded model (app/app.go:77-89)."""
    buf = np.frombuffer(data, dtype=np.uint8)
    own = engine is None
    e = engine or Engine(device)
    h = C.c_void_p()
    rc = _lib.lib().acm_model_load_gguf_mem(e.handle, buf.ctypes.data_as(C.c_void_p), buf.nbytes, maxCtx,
                                            max_seqs, C.byref(h))
    if rc:
        msg = _lib.lib().acm_engine_error(e.handle).decode()
        if own:
            e.close()
        raise AcmError(rc, msg)
    return Model(e, h, own)


def LoadMulti(path: str, engines: Sequence[Engine], maxCtx: int = 0, max_seqs: int = 1) -> List[Model]:
    """One model per engine from one mapping of the file: parsed once, each
    staging chunk read from the mapping once and copied to every engine's
    device (no reference counterpart; app/model_unix.go:15-34 maps it once per
    process).  The engines stay the caller's."""
    n = len(engines)
    es = (C.c_void_p * n)(*[e.handle for e in engines])
    hs = (C.c_void_p * n)()
    rc = _lib.lib().acm_model_load_gguf_multi(es, n, path.encode(), maxCtx, max_seqs, hs)
    if rc:
        raise AcmError(rc, _lib.lib().acm_engine_error(engines[0].handle).decode())
    return [Model(engines[i], C.c_void_p(hs[i]), False) for i in range(n)]


def LoadConfigBytes(data, maxCtx: int = 0) -> Config:
    """LoadConfig over a GGUF image in host memory."""
    buf = np.frombuffer(data, dtype=np.uint8)
    cfg = Config()
    err = C.create_string_buffer(512)
    rc = _lib.lib().acm_load_config_mem(buf.ctypes.data_as(C.c_void_p), buf.nbytes, maxCtx, C.byref(cfg), err, 512)
    if rc:
        raise AcmError(rc, err.value.decode())
    return cfg


def LoadConfig(path: str, maxCtx: int = 0) -> Config:
    """Parse a GGUF file and apply infer.Load's metadata rules (model.go:91-151)
    on the host only (no device)."""
    cfg = Config()
    err = C.create_string_buffer(512)
    rc = _lib.lib().acm_load_config(path.encode(), maxCtx, C.byref(cfg), err, 512)
    if rc:
        raise AcmError(rc, err.value.decode())
    return cfg


def MaxLogit(logits) -> int:
    """MaxLogit (model.go:462-471): first maximum wins."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return int(_lib.lib().acm_max_logit(_ptr(lg), len(lg)))
