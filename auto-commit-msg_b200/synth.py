"""Seeded synthetic GGUF models and weight matrices.

No model checkpoint exists offline, so every workload runs on random-init
weights of the named architecture, written as a GGUF v3 file with the metadata
keys the reference's loader reads (internal/infer/model.go:98-135) and the
ggml block layouts its dequantizers decode (internal/infer/tensor.go:83-226).

The quantizers here are this project's own simple per-block min/max (or
max-abs) schemes.  They only have to produce valid blocks of each layout; they
are not llama.cpp's optimising quantizers.
"""
from __future__ import annotations

import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np

# ggml tensor types, internal/gguf/gguf.go:31-40
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 6, 8, 12, 13, 14
TYPE_NAMES = {F32: "f32", F16: "f16", Q4_0: "q4_0", Q5_0: "q5_0", Q8_0: "q8_0",
              Q4_K: "q4_k", Q5_K: "q5_k", Q6_K: "q6_k"}
# (elements per block, bytes per block), gguf.go:70-90
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34),
         Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


def row_bytes(typ: int, k: int) -> int:
    bs, ts = BLOCK[typ]
    return k // bs * ts


def _f16(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def _safe_div(a, b):
    out = np.zeros_like(a, dtype=np.float32)
    np.divide(a, b, out=out, where=b != 0)
    return out


def _pack_k4_scales(sc: np.ndarray, mq: np.ndarray) -> np.ndarray:
    """Inverse of scaleMinK4 (tensor.go:124-130): 8 six-bit (scale, min)
    pairs -> 12 bytes."""
    nb = sc.shape[0]
    out = np.zeros((nb, 12), dtype=np.uint8)
    sc = sc.astype(np.uint8)
    mq = mq.astype(np.uint8)
    for j in range(4):
        out[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        out[:, j + 4] = (mq[:, j] & 63) | ((mq[:, j + 4] >> 4) << 6)
    for j in range(4, 8):
        out[:, j + 4] = (sc[:, j] & 0x0F) | ((mq[:, j] & 0x0F) << 4)
    return out


def _q_k_minmax(x: np.ndarray, levels: int):
    """Shared part of Q4_K / Q5_K: per-32 scale/min quantized to 6 bits
    against fp16 super-block d/dmin."""
    nb = x.shape[0]
    sub = x.reshape(nb, 8, 32)
    mn = np.minimum(sub.min(-1), 0.0)
    mx = sub.max(-1)
    scale = (mx - mn) / levels
    mneg = -mn
    d16 = _f16(scale.max(-1) / 63.0)
    dm16 = _f16(mneg.max(-1) / 63.0)
    d = d16.astype(np.float32)[:, None]
    dm = dm16.astype(np.float32)[:, None]
    sc = np.clip(np.rint(_safe_div(scale, np.broadcast_to(d, scale.shape))), 0, 63)
    mq = np.clip(np.rint(_safe_div(mneg, np.broadcast_to(dm, mneg.shape))), 0, 63)
    eff_s = (d * sc).astype(np.float32)
    eff_m = (dm * mq).astype(np.float32)
    q = np.clip(np.rint(_safe_div(sub + eff_m[..., None], np.broadcast_to(eff_s[..., None], sub.shape))), 0, levels)
    return d16, dm16, sc, mq, q.astype(np.uint8)


def quant_q4_k(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d16, dm16, sc, mq, q = _q_k_minmax(x, 15)
    out = np.zeros((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_k4_scales(sc, mq)
    for j in range(4):
        out[:, 16 + 32 * j:16 + 32 * j + 32] = q[:, 2 * j] | (q[:, 2 * j + 1] << 4)
    return out


def quant_q5_k(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d16, dm16, sc, mq, q = _q_k_minmax(x, 31)
    out = np.zeros((nb, 176), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_k4_scales(sc, mq)
    qh = np.zeros((nb, 32), dtype=np.uint8)
    for j in range(4):
        lo, hi = q[:, 2 * j], q[:, 2 * j + 1]
        qh |= ((lo >> 4) & 1) << (2 * j)
        qh |= ((hi >> 4) & 1) << (2 * j + 1)
        out[:, 48 + 32 * j:48 + 32 * j + 32] = (lo & 15) | ((hi & 15) << 4)
    out[:, 16:48] = qh
    return out


def _signed_maxabs(g: np.ndarray) -> np.ndarray:
    idx = np.abs(g).argmax(-1)
    return np.take_along_axis(g, idx[..., None], -1)[..., 0]


def quant_q6_k(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    g = x.reshape(nb, 16, 16)
    scale = _signed_maxabs(g) / -32.0
    d16 = _f16(np.abs(scale).max(-1) / 127.0)
    d = d16.astype(np.float32)[:, None]
    sc = np.clip(np.rint(_safe_div(scale, np.broadcast_to(d, scale.shape))), -128, 127)
    eff = (d * sc).astype(np.float32)
    q = np.clip(np.rint(_safe_div(g, np.broadcast_to(eff[..., None], g.shape))), -32, 31) + 32
    q = q.astype(np.uint8).reshape(nb, 256)
    out = np.zeros((nb, 210), dtype=np.uint8)
    for h in range(2):
        b = 128 * h
        q0, q1, q2, q3 = q[:, b:b + 32], q[:, b + 32:b + 64], q[:, b + 64:b + 96], q[:, b + 96:b + 128]
        out[:, 64 * h:64 * h + 32] = (q0 & 15) | ((q2 & 15) << 4)
        out[:, 64 * h + 32:64 * h + 64] = (q1 & 15) | ((q3 & 15) << 4)
        out[:, 128 + 32 * h:128 + 32 * h + 32] = (q0 >> 4) | ((q1 >> 4) << 2) | ((q2 >> 4) << 4) | ((q3 >> 4) << 6)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(nb, 2)
    return out


def quant_q8_0(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d16 = _f16(np.abs(x).max(-1) / 127.0)
    d = d16.astype(np.float32)[:, None]
    q = np.clip(np.rint(_safe_div(x, np.broadcast_to(d, x.shape))), -127, 127).astype(np.int8)
    out = np.zeros((nb, 34), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:34] = q.view(np.uint8)
    return out


def quant_q4_0(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d16 = _f16(_signed_maxabs(x) / -8.0)
    d = d16.astype(np.float32)[:, None]
    q = (np.clip(np.rint(_safe_div(x, np.broadcast_to(d, x.shape))) + 8, 0, 15)).astype(np.uint8)
    out = np.zeros((nb, 18), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:18] = q[:, :16] | (q[:, 16:] << 4)
    return out


def quant_q5_0(x: np.ndarray) -> np.ndarray:
    nb = x.shape[0]
    d16 = _f16(_signed_maxabs(x) / -16.0)
    d = d16.astype(np.float32)[:, None]
    q = (np.clip(np.rint(_safe_div(x, np.broadcast_to(d, x.shape))) + 16, 0, 31)).astype(np.uint32)
    qh = ((q >> 4) & 1) << np.arange(32, dtype=np.uint32)[None, :]
    qh = qh.sum(-1, dtype=np.uint64).astype(np.uint32)
    out = np.zeros((nb, 22), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:6] = qh.astype("<u4").view(np.uint8).reshape(nb, 4)
    q8 = q.astype(np.uint8)
    out[:, 6:22] = (q8[:, :16] & 15) | ((q8[:, 16:] & 15) << 4)
    return out


_QUANT = {Q4_K: quant_q4_k, Q5_K: quant_q5_k, Q6_K: quant_q6_k, Q8_0: quant_q8_0,
          Q4_0: quant_q4_0, Q5_0: quant_q5_0}


def quantize(typ: int, w: np.ndarray) -> bytes:
    """Quantize a [rows, K] float32 matrix row by row into the ggml layout."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if typ == F32:
        return w.astype("<f4").tobytes()
    if typ == F16:
        return w.astype("<f2").tobytes()
    bs, ts = BLOCK[typ]
    rows, k = w.shape
    assert k % bs == 0, (k, bs)
    flat = w.reshape(-1, bs)
    nblk = flat.shape[0]
    fn = _QUANT[typ]
    step = 1 << 16
    if nblk <= step:
        return fn(flat).tobytes()
    parts = [(i, min(i + step, nblk)) for i in range(0, nblk, step)]
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        outs = list(ex.map(lambda p: fn(flat[p[0]:p[1]]), parts))
    return b"".join(o.tobytes() for o in outs)


def random_blocks(typ: int, rows: int, k: int, seed: int) -> bytes:
    """Uniformly random block bytes (every bit pattern of every field,
    including fp16 NaN/Inf/subnormal scales): the stress input for the
    bit-exact dequant checks."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=rows * row_bytes(typ, k), dtype=np.uint8).tobytes()


# ----------------------------------------------------------------------
# GGUF v3 writer (the inverse of internal/gguf/gguf.go:121-174)
# ----------------------------------------------------------------------
_VT_U8, _VT_I8, _VT_U16, _VT_I16, _VT_U32, _VT_I32, _VT_F32, _VT_BOOL, _VT_STR, _VT_ARR, _VT_U64, _VT_I64, _VT_F64 = range(13)


def _s(b: str) -> bytes:
    e = b.encode()
    return struct.pack("<Q", len(e)) + e


def _kv_bytes(key: str, val) -> bytes:
    out = _s(key)
    if isinstance(val, tuple) and val[0] == "u32":
        return out + struct.pack("<II", _VT_U32, val[1])
    if isinstance(val, tuple) and val[0] == "u64":
        return out + struct.pack("<IQ", _VT_U64, val[1])
    if isinstance(val, tuple) and val[0] == "i32":
        return out + struct.pack("<Ii", _VT_I32, val[1])
    if isinstance(val, tuple) and val[0] == "f64":
        return out + struct.pack("<Id", _VT_F64, val[1])
    if isinstance(val, bool):
        return out + struct.pack("<IB", _VT_BOOL, int(val))
    if isinstance(val, int):
        return out + struct.pack("<II", _VT_U32, val)
    if isinstance(val, float):
        return out + struct.pack("<If", _VT_F32, val)
    if isinstance(val, str):
        return out + struct.pack("<I", _VT_STR) + _s(val)
    if isinstance(val, list):
        if all(isinstance(v, str) for v in val):
            return out + struct.pack("<IIQ", _VT_ARR, _VT_STR, len(val)) + b"".join(_s(v) for v in val)
        if all(isinstance(v, int) for v in val):
            return out + struct.pack("<IIQ", _VT_ARR, _VT_I32, len(val)) + struct.pack(f"<{len(val)}i", *val)
    raise TypeError(f"unsupported metadata value for {key}: {type(val)}")


@dataclass
class TensorSpec:
    name: str
    dims: tuple          # dims[0] innermost (K), as GGUF stores them
    typ: int
    data: bytes


def write_gguf(path: str, kv: list, tensors: list, alignment: int = 32) -> None:
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    head += b"".join(_kv_bytes(k, v) for k, v in kv)
    off = 0
    infos, offs = [], []
    for t in tensors:
        off = (off + alignment - 1) // alignment * alignment
        offs.append(off)
        infos.append(_s(t.name) + struct.pack("<I", len(t.dims)) +
                     b"".join(struct.pack("<Q", d) for d in t.dims) + struct.pack("<IQ", t.typ, off))
        off += len(t.data)
    head += b"".join(infos)
    pad = (-len(head)) % alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for t, o in zip(tensors, offs):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            f.write(t.data)
            pos += len(t.data)


# ----------------------------------------------------------------------
# Architectures (the shapes the workloads name)
# ----------------------------------------------------------------------
@dataclass
class ModelShape:
    arch: str            # qwen3 | qwen2 | llama
    n_layers: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_ff: int
    vocab: int
    ctx: int = 2048
    rope_base: float = 1e6
    eps: float = 1e-6
    tied: bool = True
    # per-tensor quant types
    t_embd: int = Q4_K
    t_q: int = Q4_K
    t_k: int = Q4_K
    t_v: int = Q6_K
    t_o: int = Q4_K
    t_gate: int = Q4_K
    t_up: int = Q4_K
    t_down: int = Q6_K
    t_out: int = Q6_K
    write_rope_scaling: bool = False
    extra_kv: list = field(default_factory=list)


def qwen3_06b(**kw) -> ModelShape:
    """Qwen3-0.6B shape, Q4_K_M-style mix (Q6_K for attn_v and ffn_down)."""
    return ModelShape("qwen3", 28, 1024, 16, 8, 128, 3072, 151936, **kw)


def qwen2_15b(**kw) -> ModelShape:
    """Qwen2-1.5B shape, every linear weight (and the tied embedding) Q8_0."""
    d = dict(t_embd=Q8_0, t_q=Q8_0, t_k=Q8_0, t_v=Q8_0, t_o=Q8_0, t_gate=Q8_0, t_up=Q8_0, t_down=Q8_0)
    d.update(kw)
    return ModelShape("qwen2", 28, 1536, 12, 2, 128, 8960, 151936, **d)


def llama32_1b_f16(**kw) -> ModelShape:
    d = dict(rope_base=5e5, eps=1e-5, t_embd=F16, t_q=F16, t_k=F16, t_v=F16, t_o=F16, t_gate=F16, t_up=F16, t_down=F16)
    d.update(kw)
    return ModelShape("llama", 16, 2048, 32, 8, 64, 8192, 128256, **d)


def llama32_1b_q5(**kw) -> ModelShape:
    """Q5_K attention, Q5_0 FFN, F16 embedding."""
    d = dict(rope_base=5e5, eps=1e-5, t_embd=F16, t_q=Q5_K, t_k=Q5_K, t_v=Q5_K, t_o=Q5_K,
             t_gate=Q5_0, t_up=Q5_0, t_down=Q5_0)
    d.update(kw)
    return ModelShape("llama", 16, 2048, 32, 8, 64, 8192, 128256, **d)


def vocab_tokens(shape: ModelShape):
    """Token strings with the special tokens the loader scans for EOS2
    (model.go:142-151) at their usual ids; returns (tokens, bos, eos)."""
    v = shape.vocab
    toks = [f"t{i}" for i in range(v)]
    if shape.arch == "llama":
        bos, eot, eos = (128000, 128001, 128009) if v > 128009 else (v - 3, v - 2, v - 1)
        toks[bos], toks[eot], toks[eos] = "<|begin_of_text|>", "<|end_of_text|>", "<|eot_id|>"
        return toks, bos, eos
    bos, eos = (151643, 151645) if v > 151645 else (v - 3, v - 1)
    toks[bos], toks[eos] = "<|endoftext|>", "<|im_end|>"
    return toks, bos, eos


def build_model(shape: ModelShape, path: str, seed: int = 0) -> str:
    """Write a random-init model of `shape`: linear weights N(0, 0.02),
    norm weights 1 + N(0, 0.02), biases N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    s = shape
    qd, kvd = s.n_head * s.head_dim, s.n_head_kv * s.head_dim

    def normal(rows, k, sd=0.02):
        return (rng.standard_normal((rows, k), dtype=np.float32) * np.float32(sd))

    def lin(name, k, n, typ):
        return TensorSpec(name, (k, n), typ, quantize(typ, normal(n, k)))

    def vec(name, n, base=0.0):
        v = (np.float32(base) + normal(1, n)[0]).astype(np.float32)
        return TensorSpec(name, (n,), F32, v.tobytes())

    toks, bos, eos = vocab_tokens(s)
    a = s.arch
    kv = [("general.architecture", a), ("general.alignment", 32), ("general.name", f"synthetic-{a}"),
          (f"{a}.block_count", s.n_layers), (f"{a}.embedding_length", s.n_embd),
          (f"{a}.attention.head_count", s.n_head), (f"{a}.attention.head_count_kv", s.n_head_kv),
          (f"{a}.feed_forward_length", s.n_ff), (f"{a}.context_length", s.ctx),
          (f"{a}.rope.freq_base", float(s.rope_base)),
          (f"{a}.attention.layer_norm_rms_epsilon", float(s.eps)),
          (f"{a}.attention.key_length", s.head_dim), (f"{a}.attention.value_length", s.head_dim),
          ("tokenizer.ggml.model", "gpt2"), ("tokenizer.ggml.tokens", toks),
          ("tokenizer.ggml.bos_token_id", bos), ("tokenizer.ggml.eos_token_id", eos)]
    if s.write_rope_scaling:
        kv += [(f"{a}.rope.scaling.type", "llama3"), (f"{a}.rope.scaling.factor", 32.0),
               (f"{a}.rope.scaling.low_freq_factor", 1.0), (f"{a}.rope.scaling.high_freq_factor", 4.0),
               (f"{a}.rope.scaling.original_context_length", 8192.0)]
    kv += list(s.extra_kv)
    ts = [lin("token_embd.weight", s.n_embd, s.vocab, s.t_embd), vec("output_norm.weight", s.n_embd, 1.0)]
    if not s.tied:
        ts.append(lin("output.weight", s.n_embd, s.vocab, s.t_out))
    for i in range(s.n_layers):
        b = f"blk.{i}."
        ts.append(vec(b + "attn_norm.weight", s.n_embd, 1.0))
        ts.append(lin(b + "attn_q.weight", s.n_embd, qd, s.t_q))
        ts.append(lin(b + "attn_k.weight", s.n_embd, kvd, s.t_k))
        ts.append(lin(b + "attn_v.weight", s.n_embd, kvd, s.t_v))
        if a == "qwen2":
            ts.append(vec(b + "attn_q.bias", qd))
            ts.append(vec(b + "attn_k.bias", kvd))
            ts.append(vec(b + "attn_v.bias", kvd))
        if a == "qwen3":
            ts.append(vec(b + "attn_q_norm.weight", s.head_dim, 1.0))
            ts.append(vec(b + "attn_k_norm.weight", s.head_dim, 1.0))
        ts.append(lin(b + "attn_output.weight", qd, s.n_embd, s.t_o))
        ts.append(vec(b + "ffn_norm.weight", s.n_embd, 1.0))
        ts.append(lin(b + "ffn_gate.weight", s.n_embd, s.n_ff, s.t_gate))
        ts.append(lin(b + "ffn_up.weight", s.n_embd, s.n_ff, s.t_up))
        ts.append(lin(b + "ffn_down.weight", s.n_ff, s.n_embd, s.t_down))
    write_gguf(path, kv, ts)
    return path


def prompt_ids(n: int, vocab: int, seed: int) -> np.ndarray:
    """Prompt of n token ids uniform in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)
