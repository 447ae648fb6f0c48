"""A second, independent restatement of the reference Forward in numpy
float64 (test infrastructure): used to check the C oracle, which in turn checks
the CUDA engine.  Follows internal/infer/model.go:317-442 with exact exp and
float64 arithmetic throughout, so it differs from the reference only by fp32
rounding."""
import numpy as np


def load_weights(g, oracle):
    """Dequantize every tensor of a GGUF (oracle.GGUF) to float64."""
    out = {}
    for t in g.tensors():
        k = t["dims"][0]
        n = t["numel"] // k
        out[t["name"]] = oracle.dequant(t["type"], g.tensor_bytes(t["name"]), n, k).astype(np.float64)
    return out


def rope_freqs(c):
    """ropeFreqs, model.go:253-280 (float32 results as the reference)."""
    half = c["rope_dim"] // 2
    f = np.array([np.float32(1.0 / np.float32(c["rope_base"] ** (2 * i / c["rope_dim"])))
                  for i in range(half)], dtype=np.float32)
    if c["rope_scaling"] == 1:
        f = (f / np.float32(c["rope_factor"])).astype(np.float32)
    elif c["rope_scaling"] == 2:
        lo = np.float32(c["rope_orig_ctx"]) / np.float32(c["rope_lo_f"])
        hi = np.float32(c["rope_orig_ctx"]) / np.float32(c["rope_hi_f"])
        for i in range(half):
            wl = 2 * np.pi / float(f[i])
            if wl < hi:
                pass
            elif wl > lo:
                f[i] = np.float32(f[i] / np.float32(c["rope_factor"]))
            else:
                sm = (np.float32(c["rope_orig_ctx"]) / np.float32(wl) - np.float32(c["rope_lo_f"])) / \
                     (np.float32(c["rope_hi_f"]) - np.float32(c["rope_lo_f"]))
                f[i] = np.float32((1 - sm) * f[i] / np.float32(c["rope_factor"]) + sm * f[i])
    return f


class RefModel:
    def __init__(self, weights, cfg):
        self.w = weights
        self.c = cfg
        self.freqs = rope_freqs(cfg)
        self.kc = [np.zeros((0, cfg["n_head_kv"] * cfg["head_dim"])) for _ in range(cfg["n_layers"])]
        self.vc = [np.zeros((0, cfg["n_head_kv"] * cfg["head_dim"])) for _ in range(cfg["n_layers"])]
        self.pos = 0

    def _rms(self, x, w):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + self.c["rms_eps"]) * w

    def _rope(self, x, pos):
        c = self.c
        half = c["rope_dim"] // 2
        ang = (np.float32(pos) * self.freqs).astype(np.float32).astype(np.float64)
        cs, sn = np.cos(ang), np.sin(ang)
        x = x.copy()
        if c["rope_interleaved"]:
            a, b = x[..., 0:2 * half:2].copy(), x[..., 1:2 * half:2].copy()
            x[..., 0:2 * half:2] = a * cs - b * sn
            x[..., 1:2 * half:2] = a * sn + b * cs
        else:
            a, b = x[..., :half].copy(), x[..., half:2 * half].copy()
            x[..., :half] = a * cs - b * sn
            x[..., half:2 * half] = a * sn + b * cs
        return x

    def forward(self, toks):
        c, w = self.c, self.w
        n = len(toks)
        nh, nkv, hd = c["n_head"], c["n_head_kv"], c["head_dim"]
        x = w["token_embd.weight"][np.asarray(toks)].copy()
        for li in range(c["n_layers"]):
            b = f"blk.{li}."
            h = self._rms(x, w[b + "attn_norm.weight"][0])
            q = h @ w[b + "attn_q.weight"].T
            k = h @ w[b + "attn_k.weight"].T
            v = h @ w[b + "attn_v.weight"].T
            if b + "attn_q.bias" in w:
                q += w[b + "attn_q.bias"][0]
                k += w[b + "attn_k.bias"][0]
                v += w[b + "attn_v.bias"][0]
            q = q.reshape(n, nh, hd)
            k = k.reshape(n, nkv, hd)
            if b + "attn_q_norm.weight" in w:
                q = self._rms(q, w[b + "attn_q_norm.weight"][0])
                k = self._rms(k, w[b + "attn_k_norm.weight"][0])
            for j in range(n):
                q[j] = self._rope(q[j], self.pos + j)
                k[j] = self._rope(k[j], self.pos + j)
            self.kc[li] = np.concatenate([self.kc[li][:self.pos], k.reshape(n, -1)])
            self.vc[li] = np.concatenate([self.vc[li][:self.pos], v])
            kc = self.kc[li].reshape(-1, nkv, hd)
            vc = self.vc[li].reshape(-1, nkv, hd)
            att = np.zeros((n, nh, hd))
            for j in range(n):
                L = self.pos + j + 1
                for hh in range(nh):
                    g = hh // (nh // nkv)
                    s = kc[:L, g, :] @ q[j, hh] / np.sqrt(hd)
                    p = np.exp(s - s.max())
                    p /= p.sum()
                    att[j, hh] = p @ vc[:L, g, :]
            x = x + att.reshape(n, -1) @ w[b + "attn_output.weight"].T
            h = self._rms(x, w[b + "ffn_norm.weight"][0])
            g = h @ w[b + "ffn_gate.weight"].T
            u = h @ w[b + "ffn_up.weight"].T
            x = x + (g / (1 + np.exp(-g)) * u) @ w[b + "ffn_down.weight"].T
        self.pos += n
        hf = self._rms(x[-1], w["output_norm.weight"][0])
        out = w.get("output.weight", w["token_embd.weight"])
        return hf @ out.T
