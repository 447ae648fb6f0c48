// gguf_host.h -- GGUF v2/v3 parser (internal/gguf/gguf.go:121-258) and the
// configuration rules of infer.Load (internal/infer/model.go:90-151), on the
// host side of the C ABI.
#pragma once
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "acm.h"

namespace acm {
namespace gguf {

// Metadata value types, gguf.go:14-28.
enum { V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64 };

struct Value {
    int type = -1;
    int etype = -1;  // element type of an array
    uint64_t u = 0;  // integer / bool payload
    double f = 0;    // float payload
    std::string s;
    std::vector<std::string> astr;
    std::vector<uint64_t> aint;
    std::vector<double> afl;
};

struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;  // dims[0] innermost
    uint32_t type = 0;
    uint64_t offset = 0;
    int64_t numel = 0;
    const uint8_t *data = nullptr;
    uint64_t nbytes = 0;
};

struct File {
    uint32_t version = 0;
    std::map<std::string, Value> kv;
    std::map<std::string, Tensor> tensors;
    std::vector<std::string> order;

    std::string Str(const std::string &key) const;
    uint64_t U64(const std::string &key, uint64_t def) const;
    float F32(const std::string &key, float def) const;
    std::vector<std::string> Strs(const std::string &key) const;
    const Tensor *T(const std::string &name) const;
};

// Parse; returns ACM_OK or ACM_ERR_FORMAT / ACM_ERR_UNSUPPORTED_TYPE with err.
int parse(const uint8_t *data, size_t len, File &f, std::string &err);

// infer.Load's metadata rules (model.go:91-151) -> acm_config.
int load_config(const File &f, int max_ctx, acm_config &c, std::string &err);

}  // namespace gguf
}  // namespace acm
