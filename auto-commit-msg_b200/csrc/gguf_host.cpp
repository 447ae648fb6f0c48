// gguf_host.cpp -- see gguf_host.h.
#include "gguf_host.h"

#include <string.h>

namespace acm {
namespace gguf {

namespace {

// BlockSize, gguf.go:70-90
bool block_size(uint32_t t, int &bs, int &ts) {
    switch (t) {
        case 0: bs = 1; ts = 4; return true;
        case 1: bs = 1; ts = 2; return true;
        case 2: bs = 32; ts = 18; return true;
        case 6: bs = 32; ts = 22; return true;
        case 8: bs = 32; ts = 34; return true;
        case 12: bs = 256; ts = 144; return true;
        case 13: bs = 256; ts = 176; return true;
        case 14: bs = 256; ts = 210; return true;
    }
    bs = ts = 0;
    return false;
}

struct Reader {
    const uint8_t *b;
    size_t len, pos = 0;
    bool bad = false;
    const uint8_t *take(size_t n) {
        if (bad || n > len - pos) {
            bad = true;
            return nullptr;
        }
        const uint8_t *p = b + pos;
        pos += n;
        return p;
    }
    uint64_t le(size_t n) {
        const uint8_t *p = take(n);
        uint64_t v = 0;
        if (p)
            for (size_t i = 0; i < n; i++) v |= (uint64_t)p[i] << (8 * i);
        return v;
    }
    std::string str() {
        uint64_t n = le(8);
        if (bad || n > len - pos) {
            bad = true;
            return std::string();
        }
        const uint8_t *p = take((size_t)n);
        return p ? std::string(reinterpret_cast<const char *>(p), (size_t)n) : std::string();
    }
    // valueTyped, gguf.go:318-347 (scalar part)
    bool scalar(int t, uint64_t &u, double &f, std::string &s) {
        switch (t) {
            case V_U8: u = le(1); return !bad;
            case V_I8: u = (uint64_t)(int64_t)(int8_t)le(1); return !bad;
            case V_U16: u = le(2); return !bad;
            case V_I16: u = (uint64_t)(int64_t)(int16_t)le(2); return !bad;
            case V_U32: u = le(4); return !bad;
            case V_I32: u = (uint64_t)(int64_t)(int32_t)le(4); return !bad;
            case V_U64:
            case V_I64: u = le(8); return !bad;
            case V_F32: {
                uint32_t b = (uint32_t)le(4);
                float x;
                memcpy(&x, &b, 4);
                f = x;
                return !bad;
            }
            case V_F64: {
                uint64_t b = le(8);
                memcpy(&f, &b, 8);
                return !bad;
            }
            case V_BOOL: u = le(1) != 0; return !bad;
            case V_STR: s = str(); return !bad;
        }
        return false;
    }
};

bool is_int(int t) {
    return t == V_U8 || t == V_I8 || t == V_U16 || t == V_I16 || t == V_U32 || t == V_I32 || t == V_U64 || t == V_I64;
}

}  // namespace

std::string File::Str(const std::string &key) const {
    auto it = kv.find(key);
    return (it != kv.end() && it->second.type == V_STR) ? it->second.s : std::string();
}
// U64 / toU64, gguf.go:176-212: non-integer values read as 0.
uint64_t File::U64(const std::string &key, uint64_t def) const {
    auto it = kv.find(key);
    if (it == kv.end()) return def;
    return is_int(it->second.type) ? it->second.u : 0;
}
float File::F32(const std::string &key, float def) const {
    auto it = kv.find(key);
    if (it != kv.end() && (it->second.type == V_F32 || it->second.type == V_F64)) return (float)it->second.f;
    return def;
}
std::vector<std::string> File::Strs(const std::string &key) const {
    auto it = kv.find(key);
    if (it == kv.end() || it->second.type != V_ARR) return {};
    if (it->second.etype == V_STR) return it->second.astr;
    return std::vector<std::string>(it->second.aint.size() + it->second.afl.size());
}
const Tensor *File::T(const std::string &name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
}

// Parse, gguf.go:121-174
int parse(const uint8_t *data, size_t len, File &f, std::string &err) {
    Reader r{data, len};
    const uint8_t *magic = r.take(4);
    if (!magic || memcmp(magic, "GGUF", 4) != 0) {
        err = "not a GGUF file";
        return ACM_ERR_FORMAT;
    }
    f.version = (uint32_t)r.le(4);
    if (f.version != 3 && f.version != 2) {
        err = "unsupported GGUF version " + std::to_string(f.version);
        return ACM_ERR_FORMAT;
    }
    const uint64_t nt = r.le(8), nkv = r.le(8);
    if (r.bad || nkv > len || nt > len) {
        err = "truncated GGUF header";
        return ACM_ERR_FORMAT;
    }
    for (uint64_t i = 0; i < nkv && !r.bad; i++) {
        std::string k = r.str();
        Value v;
        v.type = (int)r.le(4);
        if (v.type == V_ARR) {
            v.etype = (int)r.le(4);
            const uint64_t n = r.le(8);
            if (r.bad || n > len) {
                r.bad = true;
                break;
            }
            for (uint64_t a = 0; a < n && !r.bad; a++) {
                uint64_t u = 0;
                double fl = 0;
                std::string s;
                if (!r.scalar(v.etype, u, fl, s)) {
                    r.bad = true;
                    break;
                }
                if (v.etype == V_STR) v.astr.push_back(std::move(s));
                else if (v.etype == V_F32 || v.etype == V_F64) v.afl.push_back(fl);
                else v.aint.push_back(u);
            }
        } else if (!r.scalar(v.type, v.u, v.f, v.s)) {
            r.bad = true;
        }
        if (!r.bad) f.kv[k] = std::move(v);
    }
    if (r.bad) {
        err = "truncated GGUF metadata";
        return ACM_ERR_FORMAT;
    }
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        Tensor t;
        t.name = r.str();
        const uint32_t nd = (uint32_t)r.le(4);
        if (nd > 8) {
            r.bad = true;
            break;
        }
        t.numel = 1;
        for (uint32_t j = 0; j < nd; j++) {
            t.dims.push_back(r.le(8));
            t.numel *= (int64_t)t.dims.back();
        }
        t.type = (uint32_t)r.le(4);
        t.offset = r.le(8);
        if (!r.bad) {
            f.order.push_back(t.name);
            f.tensors[t.name] = std::move(t);
        }
    }
    if (r.bad) {
        err = "truncated GGUF tensor index";
        return ACM_ERR_FORMAT;
    }
    uint64_t align = 32;
    auto it = f.kv.find("general.alignment");
    if (it != f.kv.end()) align = is_int(it->second.type) ? it->second.u : 0;
    if (align == 0) align = 32;
    const uint64_t start = ((uint64_t)r.pos + align - 1) / align * align;
    for (const std::string &name : f.order) {
        Tensor &t = f.tensors[name];
        int bs, ts;
        if (!block_size(t.type, bs, ts)) {
            err = "tensor " + name + ": unsupported type " + std::to_string(t.type);
            return ACM_ERR_UNSUPPORTED_TYPE;
        }
        const uint64_t size = (uint64_t)(t.numel / bs) * (uint64_t)ts;
        const uint64_t abs_ = start + t.offset;
        if (abs_ + size > len || abs_ + size < abs_) {
            err = "tensor " + name + ": out of bounds";
            return ACM_ERR_FORMAT;
        }
        t.data = data + abs_;
        t.nbytes = size;
    }
    return ACM_OK;
}

// Load, model.go:91-151
int load_config(const File &f, int max_ctx, acm_config &c, std::string &err) {
    const std::string arch = f.Str("general.architecture");
    memset(&c, 0, sizeof c);
    if (arch == "qwen3") c.arch = ACM_ARCH_QWEN3;
    else if (arch == "qwen2") c.arch = ACM_ARCH_QWEN2;
    else if (arch == "llama") c.arch = ACM_ARCH_LLAMA;
    else {
        err = "unsupported architecture \"" + arch + "\" (want qwen2, qwen3, or llama)";
        return ACM_ERR_UNSUPPORTED_ARCH;
    }
    const std::string p = arch + ".";
    c.n_layers = (int)f.U64(p + "block_count", 0);
    c.n_embd = (int)f.U64(p + "embedding_length", 0);
    c.n_head = (int)f.U64(p + "attention.head_count", 0);
    c.n_head_kv = (int)f.U64(p + "attention.head_count_kv", 0);
    c.n_ff = (int)f.U64(p + "feed_forward_length", 0);
    c.max_ctx = (int)f.U64(p + "context_length", 0);
    c.rope_base = f.F32(p + "rope.freq_base", 10000.0f);
    c.rms_eps = f.F32(p + "attention.layer_norm_rms_epsilon", 1e-6f);
    const std::vector<std::string> toks = f.Strs("tokenizer.ggml.tokens");
    c.vocab = (int)toks.size();
    c.bos = (int)f.U64("tokenizer.ggml.bos_token_id", 0);
    c.eos = (int)f.U64("tokenizer.ggml.eos_token_id", 0);
    const int kl = (int)f.U64(p + "attention.key_length", 0);
    const Tensor *tq = f.T("blk.0.attn_q.weight");
    if (kl > 0) c.head_dim = kl;
    else if (tq && tq->dims.size() > 1 && c.n_head) c.head_dim = (int)tq->dims[1] / c.n_head;
    else c.head_dim = c.n_head ? c.n_embd / c.n_head : 0;
    c.rope_interleaved = arch == "llama";
    c.rope_dim = (int)f.U64(p + "rope.dimension_count", (uint64_t)c.head_dim);
    const std::string sc = f.Str(p + "rope.scaling.type");
    c.rope_scaling = sc == "linear" ? ACM_ROPE_LINEAR : sc == "llama3" ? ACM_ROPE_LLAMA3 : ACM_ROPE_NONE;
    c.rope_factor = f.F32(p + "rope.scaling.factor", 0);
    c.rope_lo_f = f.F32(p + "rope.scaling.low_freq_factor", 0);
    c.rope_hi_f = f.F32(p + "rope.scaling.high_freq_factor", 0);
    c.rope_orig_ctx = f.F32(p + "rope.scaling.original_context_length", 0);
    if (arch == "llama" && sc.empty() && c.rope_base >= 500000) {
        // legacy Llama-3.x GGUFs omit the scaling keys (model.go:126-134)
        c.rope_scaling = ACM_ROPE_LLAMA3;
        c.rope_factor = 32;
        c.rope_lo_f = 1;
        c.rope_hi_f = 4;
        c.rope_orig_ctx = 8192;
    }
    const int hkv = c.n_head_kv ? c.n_head_kv : c.n_head;  // HeadKV, model.go:205-210
    if (hkv == 0 || c.n_embd == 0 || c.n_layers == 0) {
        err = "missing required metadata for arch " + arch;
        return ACM_ERR_INVALID;
    }
    c.n_head_kv = hkv;
    if (max_ctx <= 0 || max_ctx > c.max_ctx) max_ctx = c.max_ctx;
    c.max_ctx = max_ctx;
    c.eos2 = -1;
    for (size_t i = 0; i < toks.size(); i++) {
        const std::string &t = toks[i];
        if ((t == "<|endoftext|>" || t == "<|eot_id|>" || t == "<|end_of_text|>") && (int)i != c.eos)
            c.eos2 = (int)i;
    }
    return ACM_OK;
}

}  // namespace gguf
}  // namespace acm
