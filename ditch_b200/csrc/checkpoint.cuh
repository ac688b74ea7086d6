// Checkpoint files on the host: the structures the loader
// (checkpoint.cu) and the export (export.cu) share. A Hugging Face directory
// (config.json plus safetensors shards) or a GGUF file is memory-mapped and
// described tensor by tensor as stored.
#pragma once

#include <sys/mman.h>

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "model.cuh"

namespace ditch {
namespace ckpt {

#define CK_REQUIRE(cond, ...)          \
    do {                               \
        if (!(cond)) {                 \
            set_error(__VA_ARGS__);    \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)

// ---- a small JSON reader (config.json, safetensors headers) ----------------
struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal *get(const std::string &k) const {
        if (kind != Obj) return nullptr;
        for (const auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
    double number(const std::string &k, double dflt) const {
        const JVal *v = get(k);
        return v && v->kind == Num ? v->num : v && v->kind == Bool ? (v->b ? 1.0 : 0.0) : dflt;
    }
    std::string string(const std::string &k, const std::string &dflt = "") const {
        const JVal *v = get(k);
        return v && v->kind == Str ? v->str : dflt;
    }
};

bool parse_json(const char *s, size_t n, JVal &out);
bool read_text(const std::string &path, std::string &out);

// ---- read-only file mappings -----------------------------------------------
struct Mapping {
    void *base = nullptr;
    size_t size = 0;
    ~Mapping() {
        if (base && base != MAP_FAILED) munmap(base, size);
    }
};

// ---- the tensors of a checkpoint, as stored -------------------------------
struct RawTensor {
    std::string dtype;            // safetensors dtype ("BF16", "F8_E4M3", ...) or "GGML_Q8_0" / "GGML_Q4_K"
    std::vector<int64_t> shape;   // rows first (GGUF dims reversed)
    const uint8_t *data = nullptr;
    size_t bytes = 0;
};

struct Checkpoint {
    std::vector<std::unique_ptr<Mapping>> maps;
    std::map<std::string, RawTensor> t;
    JVal config;                        // config.json, or the GGUF metadata
    JVal embedded;                      // a GGUF file's embedded Hugging Face config, if any
    bool gguf = false;
    std::vector<std::vector<uint8_t>> owned;  // stacked experts, split or un-permuted rows

    const RawTensor *find(const std::string &n) const {
        auto it = t.find(n);
        return it == t.end() ? nullptr : &it->second;
    }
    uint8_t *alloc(size_t n) {
        owned.emplace_back(n);
        return owned.back().data();
    }
};

size_t dtype_size(const std::string &d);

// The model config and tensor table built from a checkpoint.
struct Built {
    ditch_cuda_model_config cfg{};
    std::vector<uint8_t> moe_layers;
    std::vector<float> rope_factors;  // per-frequency RoPE divisors (rope_scaling 4)
    std::vector<ditch_cuda_tensor> tensors;
    std::vector<std::unique_ptr<std::string>> names;
    bool tied = false;
    std::string family;          // model_type of the device path
    int br = 0, bc = 0;          // FP8 weight blocks
    int int_bits = 0, int_group = 0;
};

int read_hf_dir(const std::string &dir, Checkpoint &ck);
int read_gguf(const std::string &path, Checkpoint &ck);
int build_config(Checkpoint &ck, Built &b);
// read + config + tensor table (a directory: Hugging Face; a file: GGUF)
int open_checkpoint(const char *path, Checkpoint &ck, Built &b);

}  // namespace ckpt
}  // namespace ditch
