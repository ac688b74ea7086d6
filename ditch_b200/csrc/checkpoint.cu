// Checkpoint loading on the host: a Hugging Face directory (config.json plus
// safetensors shards) or a GGUF file, turned into the tensor table of
// ditch_cuda_model_load with the quantised groups kept raw (FP8 codes and
// block scales, pack-quantized INT words, ggml blocks). This is the part of
// ditch's loaders the device path needs (src/safetensors.zig,
// src/dequant.zig:783-1187 for the formats, src/gguf_model.zig, and the
// expert layouts of src/moe.zig:83-92, 728-770); tokenizers and the exotic
// families stay with ditch.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "checkpoint.cuh"

namespace ditch {
namespace ckpt {

using namespace ditch;

struct JParser {
    const char *p, *end;
    bool ok = true;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
    }
    bool lit(const char *s) {
        const size_t n = strlen(s);
        if ((size_t)(end - p) < n || memcmp(p, s, n) != 0) return false;
        p += n;
        return true;
    }
    std::string str() {
        std::string out;
        if (p >= end || *p != '"') {
            ok = false;
            return out;
        }
        p++;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\' && p < end) {
                const char e = *p++;
                switch (e) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {  // \uXXXX: kept as UTF-8 (basic plane; names and config values are ASCII)
                    if (end - p < 4) {
                        ok = false;
                        return out;
                    }
                    const unsigned cp = (unsigned)strtoul(std::string(p, 4).c_str(), nullptr, 16);
                    p += 4;
                    if (cp < 0x80) out += (char)cp;
                    else if (cp < 0x800) out += (char)(0xc0 | (cp >> 6)), out += (char)(0x80 | (cp & 0x3f));
                    else out += (char)(0xe0 | (cp >> 12)), out += (char)(0x80 | ((cp >> 6) & 0x3f)),
                        out += (char)(0x80 | (cp & 0x3f));
                    break;
                }
                default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (p >= end) ok = false;
        else p++;
        return out;
    }
    JVal value(int depth = 0) {
        JVal v;
        ws();
        if (p >= end || depth > 64) {
            ok = false;
            return v;
        }
        if (*p == '{') {
            v.kind = JVal::Obj;
            p++;
            ws();
            if (p < end && *p == '}') {
                p++;
                return v;
            }
            while (ok) {
                ws();
                std::string k = str();
                ws();
                if (p >= end || *p != ':') {
                    ok = false;
                    break;
                }
                p++;
                v.obj.emplace_back(std::move(k), value(depth + 1));
                ws();
                if (p < end && *p == ',') {
                    p++;
                    continue;
                }
                if (p < end && *p == '}') {
                    p++;
                    break;
                }
                ok = false;
            }
        } else if (*p == '[') {
            v.kind = JVal::Arr;
            p++;
            ws();
            if (p < end && *p == ']') {
                p++;
                return v;
            }
            while (ok) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (p < end && *p == ',') {
                    p++;
                    continue;
                }
                if (p < end && *p == ']') {
                    p++;
                    break;
                }
                ok = false;
            }
        } else if (*p == '"') {
            v.kind = JVal::Str;
            v.str = str();
        } else if (lit("true")) {
            v.kind = JVal::Bool;
            v.b = true;
        } else if (lit("false")) {
            v.kind = JVal::Bool;
        } else if (lit("null")) {
            v.kind = JVal::Null;
        } else {
            const char *q = p;
            while (q < end && (isdigit((unsigned char)*q) || *q == '-' || *q == '+' || *q == '.' || *q == 'e' ||
                               *q == 'E'))
                q++;
            const std::string num(p, q);
            char *e = nullptr;
            v.kind = JVal::Num;
            v.num = strtod(num.c_str(), &e);
            if (num.empty() || e != num.c_str() + num.size()) ok = false;
            p = q;
        }
        return v;
    }
};

bool parse_json(const char *s, size_t n, JVal &out) {
    JParser jp{s, s + n};
    out = jp.value();
    return jp.ok;
}

// ---- read-only file mappings -----------------------------------------------
int map_file(const std::string &path, std::unique_ptr<Mapping> &out) {
    const int fd = open(path.c_str(), O_RDONLY);
    CK_REQUIRE(fd >= 0, "cannot open %s", path.c_str());
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        set_error("cannot read %s", path.c_str());
        return DITCH_CUDA_INVALID;
    }
    auto m = std::make_unique<Mapping>();
    m->size = (size_t)st.st_size;
    m->base = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    CK_REQUIRE(m->base != MAP_FAILED, "cannot map %s", path.c_str());
    out = std::move(m);
    return DITCH_CUDA_OK;
}

bool read_text(const std::string &path, std::string &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[1 << 16];
    size_t n;
    out.clear();
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
    fclose(f);
    return true;
}

}  // namespace ckpt
}  // namespace ditch

namespace ditch {
namespace ckpt {

// ---- the tensors of a checkpoint, as stored -------------------------------
size_t dtype_size(const std::string &d) {
    if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    if (d == "F8_E4M3" || d == "U8" || d == "I8" || d == "BOOL") return 1;
    return 0;
}

int read_safetensors(const std::string &path, Checkpoint &ck) {
    std::unique_ptr<Mapping> m;
    int s;
    if ((s = map_file(path, m))) return s;
    const uint8_t *base = static_cast<const uint8_t *>(m->base);
    CK_REQUIRE(m->size >= 8, "%s: too short for a safetensors file", path.c_str());
    uint64_t n;
    memcpy(&n, base, 8);
    CK_REQUIRE(n <= m->size - 8, "%s: bad header length", path.c_str());
    JVal h;
    CK_REQUIRE(parse_json(reinterpret_cast<const char *>(base + 8), n, h) && h.kind == JVal::Obj,
               "%s: bad safetensors header", path.c_str());
    const size_t data0 = 8 + n;
    for (const auto &kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal &e = kv.second;
        const JVal *shp = e.get("shape"), *off = e.get("data_offsets");
        CK_REQUIRE(shp && off && off->arr.size() == 2, "%s: tensor %s has no shape / offsets", path.c_str(),
                   kv.first.c_str());
        RawTensor r;
        r.dtype = e.string("dtype");
        for (const JVal &d : shp->arr) r.shape.push_back((int64_t)d.num);
        const size_t b = (size_t)off->arr[0].num, en = (size_t)off->arr[1].num;
        CK_REQUIRE(b <= en && data0 + en <= m->size, "%s: tensor %s outside the file", path.c_str(), kv.first.c_str());
        r.data = base + data0 + b;
        r.bytes = en - b;
        if (const size_t es = dtype_size(r.dtype)) {
            size_t elems = 1;
            for (int64_t d : r.shape) {
                CK_REQUIRE(d >= 0, "%s: tensor %s has a negative dimension", path.c_str(), kv.first.c_str());
                elems *= (size_t)d;
            }
            CK_REQUIRE(elems * es == r.bytes, "%s: tensor %s holds %zu bytes, its %s shape needs %zu", path.c_str(),
                       kv.first.c_str(), r.bytes, r.dtype.c_str(), elems * es);
        }
        ck.t[kv.first] = r;
    }
    ck.maps.push_back(std::move(m));
    return DITCH_CUDA_OK;
}

int read_hf_dir(const std::string &dir, Checkpoint &ck) {
    // an export that did not finish leaves its marker (src/model.zig:866-869)
    CK_REQUIRE(access((dir + "/.incomplete").c_str(), F_OK) != 0,
               "%s contains .incomplete: the export did not finish; refusing to load it", dir.c_str());
    std::string text;
    CK_REQUIRE(read_text(dir + "/config.json", text), "%s: no config.json", dir.c_str());
    CK_REQUIRE(parse_json(text.data(), text.size(), ck.config) && ck.config.kind == JVal::Obj,
               "%s: bad config.json", dir.c_str());
    std::vector<std::string> files;
    if (DIR *d = opendir(dir.c_str())) {
        while (dirent *e = readdir(d)) {
            const std::string n = e->d_name;
            if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(dir + "/" + n);
        }
        closedir(d);
    }
    CK_REQUIRE(!files.empty(), "%s: no .safetensors files", dir.c_str());
    std::sort(files.begin(), files.end());
    int s;
    for (const std::string &f : files)
        if ((s = read_safetensors(f, ck))) return s;
    return DITCH_CUDA_OK;
}

// ---- GGUF (v2 / v3) ---------------------------------------------------------
struct GgufReader {
    const uint8_t *p, *end;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if ((size_t)(end - p) < sizeof(T)) {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string gstr() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t)(end - p) < n) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char *>(p), n);
        p += n;
        return s;
    }
    // one metadata value of type `ty` as JSON (numbers, strings, arrays of them)
    JVal value(uint32_t ty, int depth = 0) {
        JVal v;
        if (depth > 4) {
            ok = false;
            return v;
        }
        v.kind = JVal::Num;
        switch (ty) {
        case 0: v.num = get<uint8_t>(); break;
        case 1: v.num = get<int8_t>(); break;
        case 2: v.num = get<uint16_t>(); break;
        case 3: v.num = get<int16_t>(); break;
        case 4: v.num = get<uint32_t>(); break;
        case 5: v.num = get<int32_t>(); break;
        case 6: v.num = get<float>(); break;
        case 7: v.kind = JVal::Bool, v.b = get<uint8_t>() != 0; break;
        case 8: v.kind = JVal::Str, v.str = gstr(); break;
        case 9: {
            v.kind = JVal::Arr;
            const uint32_t et = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            // long arrays (the vocabulary) are skipped, not kept
            const bool keep = n <= 4096;
            for (uint64_t i = 0; i < n && ok; i++) {
                JVal e = value(et, depth + 1);
                if (keep) v.arr.push_back(std::move(e));
            }
            break;
        }
        case 10: v.num = (double)get<uint64_t>(); break;
        case 11: v.num = (double)get<int64_t>(); break;
        case 12: v.num = get<double>(); break;
        default: ok = false;
        }
        return v;
    }
};

int read_gguf(const std::string &path, Checkpoint &ck) {
    std::unique_ptr<Mapping> m;
    int s;
    if ((s = map_file(path, m))) return s;
    const uint8_t *base = static_cast<const uint8_t *>(m->base);
    GgufReader r{base, base + m->size};
    CK_REQUIRE(m->size > 24 && memcmp(base, "GGUF", 4) == 0, "%s: not a GGUF file", path.c_str());
    r.p += 4;
    const uint32_t version = r.get<uint32_t>();
    CK_REQUIRE(version == 2 || version == 3, "%s: GGUF version %u", path.c_str(), version);
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    JVal meta;
    meta.kind = JVal::Obj;
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        std::string key = r.gstr();
        const uint32_t ty = r.get<uint32_t>();
        meta.obj.emplace_back(std::move(key), r.value(ty));
    }
    CK_REQUIRE(r.ok, "%s: bad GGUF metadata", path.c_str());
    struct Info {
        std::string name;
        std::vector<uint64_t> dims;
        uint32_t type;
        uint64_t offset;
    };
    std::vector<Info> infos;
    for (uint64_t i = 0; i < n_tensors && r.ok; i++) {
        Info in;
        in.name = r.gstr();
        const uint32_t nd = r.get<uint32_t>();
        CK_REQUIRE(nd >= 1 && nd <= 4, "%s: tensor with %u dims", path.c_str(), nd);
        for (uint32_t d = 0; d < nd; d++) in.dims.push_back(r.get<uint64_t>());
        in.type = r.get<uint32_t>();
        in.offset = r.get<uint64_t>();
        infos.push_back(std::move(in));
    }
    CK_REQUIRE(r.ok, "%s: bad GGUF tensor table", path.c_str());
    const uint64_t align = (uint64_t)meta.number("general.alignment", 32);
    CK_REQUIRE(align > 0 && (align & (align - 1)) == 0, "%s: alignment %llu", path.c_str(), (unsigned long long)align);
    const uint64_t data0 = ((uint64_t)(r.p - base) + align - 1) / align * align;
    for (const Info &in : infos) {
        RawTensor t;
        uint64_t elems = 1;
        for (uint64_t d : in.dims) elems *= d;
        size_t bytes = 0;
        switch (in.type) {
        case 0: t.dtype = "F32", bytes = elems * 4; break;
        case 1: t.dtype = "F16", bytes = elems * 2; break;
        case 30: t.dtype = "BF16", bytes = elems * 2; break;
        case 8: t.dtype = "GGML_Q8_0", bytes = elems / 32 * 34; break;
        case 12: t.dtype = "GGML_Q4_K", bytes = elems / 256 * 144; break;
        default:
            set_error("%s: tensor %s has ggml type %u (F32, F16, BF16, Q8_0 and Q4_K are taken)", path.c_str(),
                      in.name.c_str(), in.type);
            return DITCH_CUDA_UNSUPPORTED;
        }
        for (size_t d = in.dims.size(); d-- > 0;) t.shape.push_back((int64_t)in.dims[d]);  // rows first
        CK_REQUIRE(data0 + in.offset + bytes <= m->size, "%s: tensor %s outside the file", path.c_str(),
                   in.name.c_str());
        t.data = base + data0 + in.offset;
        t.bytes = bytes;
        ck.t[in.name] = t;
    }
    ck.config = std::move(meta);
    ck.gguf = true;
    ck.maps.push_back(std::move(m));
    return DITCH_CUDA_OK;
}

}  // namespace ckpt
}  // namespace ditch

namespace ditch {
namespace ckpt {

// ---- the model config ------------------------------------------------------
const JVal *path_get(const JVal &v, std::initializer_list<const char *> keys) {
    const JVal *cur = &v;
    for (const char *k : keys) {
        cur = cur ? cur->get(k) : nullptr;
        if (!cur) return nullptr;
    }
    return cur;
}

// The Hugging Face config.json fields of src/model.zig's parseConfig for the
// families of the device path (llama, mistral, qwen2, qwen3, qwen3_moe,
// mixtral), with the fp8 / compressed-tensors quantization_config of
// src/dequant.zig:108-233.
// parseRopeScaling (src/arch.zig:1646-1720): the rope_scaling dictionary
// `rs` of config `j` into the device config's RoPE fields. Values are read
// as f32, as the reference stores them.
int rope_scaling_config(const JVal &j, const JVal &rs, ditch_cuda_model_config &c, Built &b) {
    auto f32 = [](double v) { return (double)(float)v; };
    const std::string ty = rs.string("rope_type", rs.string("type"));
    const int half = c.head_dim / 2;
    if (ty == "llama3") {
        c.rope_scaling = 1;
        c.rope_factor = f32(rs.number("factor", 8.0));
        c.rope_low_ff = f32(rs.number("low_freq_factor", 1.0));
        c.rope_high_ff = f32(rs.number("high_freq_factor", 4.0));
        c.rope_orig_max = f32(rs.number("original_max_position_embeddings", 8192));
    } else if (ty == "linear") {
        c.rope_scaling = 2;
        c.rope_factor = f32(rs.number("factor", 1.0));
    } else if (ty == "yarn") {
        const double factor = f32(rs.number("factor", 1.0));
        const double mscale = f32(rs.number("mscale", 1.0)), all_dim = f32(rs.number("mscale_all_dim", 0.0));
        // yarnMscale (src/arch.zig:1722-1725), in f32
        auto ms = [&](double m) { return factor <= 1 ? 1.0 : f32(f32(0.1 * m * std::log((float)factor)) + 1.0); };
        const JVal *af = rs.get("attention_factor");
        c.rope_scaling = 3;
        c.rope_factor = factor;
        c.rope_attention_factor = af && af->kind == JVal::Num ? f32(af->num)
                                  : (mscale != 0 && all_dim != 0) ? f32(ms(mscale) / ms(all_dim))
                                                                  : ms(1.0);
        c.rope_orig_max = f32(rs.number("original_max_position_embeddings",
                                        j.number("original_max_position_embeddings", 4096)));
        c.rope_beta_fast = f32(rs.number("beta_fast", 32));
        c.rope_beta_slow = f32(rs.number("beta_slow", 1));
        c.rope_truncate = rs.number("truncate", 1) != 0;
    } else if (ty == "longrope") {
        // the short factors for every position, as the reference does
        const double max_pos = j.number("max_position_embeddings", 4096);
        const double orig = f32(j.number("original_max_position_embeddings",
                                         rs.number("original_max_position_embeddings", max_pos)));
        b.rope_factors.assign(half, 1.0f);
        if (const JVal *sf = rs.get("short_factor"))
            for (size_t i = 0; i < sf->arr.size() && (int)i < half; i++)
                if (sf->arr[i].kind == JVal::Num) b.rope_factors[i] = (float)sf->arr[i].num;
        const JVal *fv = rs.get("factor");
        const double factor = fv && fv->kind == JVal::Num ? f32(fv->num) : f32(max_pos / orig);
        const JVal *af = rs.get("attention_factor");
        c.rope_scaling = 4;
        c.rope_attention_factor = af && af->kind == JVal::Num ? f32(af->num)
                                  : factor <= 1 ? 1.0
                                                : f32(std::sqrt(1.0f + std::log((float)factor) / std::log((float)orig)));
    } else if (ty == "ditch_factors") {
        // per-frequency divisors written by ditch's GGUF config (src/gguf_model.zig:326-335)
        b.rope_factors.clear();
        if (const JVal *fa = rs.get("factors"))
            for (const JVal &v : fa->arr) b.rope_factors.push_back(v.kind == JVal::Num ? (float)v.num : 1.0f);
        if (!b.rope_factors.empty()) c.rope_scaling = 4;
    } else if (ty == "proportional") {
        // a factor divides the frequencies like linear scaling
        const double factor = f32(rs.number("factor", 1.0));
        if (factor != 1) c.rope_scaling = 2, c.rope_factor = factor;
    }
    // anything else (dynamic NTK, mrope over text positions, default, types
    // the reference does not know) is plain RoPE, as the reference reads it
    (void)j;
    return DITCH_CUDA_OK;
}

int hf_config(const JVal &j, Built &b) {
    ditch_cuda_model_config &c = b.cfg;
    const std::string mt = j.string("model_type");
    if (mt != "llama" && mt != "mistral" && mt != "qwen2" && mt != "qwen3" && mt != "qwen3_moe" && mt != "mixtral") {
        set_error("model_type '%s' is not taken by the device path", mt.c_str());
        return DITCH_CUDA_UNSUPPORTED;
    }
    b.family = mt;
    c.n_layers = (int)j.number("num_hidden_layers", 0);
    c.hidden = (int)j.number("hidden_size", 0);
    c.heads = (int)j.number("num_attention_heads", 0);
    c.kv_heads = (int)j.number("num_key_value_heads", c.heads);
    const JVal *hd = j.get("head_dim");
    c.head_dim = hd && hd->kind == JVal::Num ? (int)hd->num : (c.heads ? c.hidden / c.heads : 0);
    c.inter = (int)j.number("intermediate_size", 0);
    c.vocab = (int)j.number("vocab_size", 0);
    c.eps = (float)j.number("rms_norm_eps", 1e-6);
    c.rope_theta = j.number("rope_theta", 10000.0);
    c.qk_norm = mt == "qwen3" || mt == "qwen3_moe";
    b.tied = j.number("tie_word_embeddings", 0) != 0;
    const JVal *rs = j.get("rope_scaling");
    if (!rs || rs->kind != JVal::Obj) {
        // rope_parameters (newer configs): the full-attention entry when split
        const JVal *rp = j.get("rope_parameters");
        rs = rp && rp->kind == JVal::Obj ? (rp->get("full_attention") ? rp->get("full_attention") : rp) : nullptr;
        if (rs && rs->kind != JVal::Obj) rs = nullptr;
        if (rs && !j.get("rope_theta")) c.rope_theta = rs->number("rope_theta", c.rope_theta);
    }
    if (rs)
        if (const int st = rope_scaling_config(j, *rs, c, b)) return st;
    if (mt == "qwen3_moe") {
        c.n_experts = (int)j.number("num_experts", 0);
        c.top_k = (int)j.number("num_experts_per_tok", 0);
        c.moe_inter = (int)j.number("moe_intermediate_size", 0);
        c.norm_topk = j.number("norm_topk_prob", 1) != 0;
        const int step = std::max(1, (int)j.number("decoder_sparse_step", 1));
        std::vector<int> only;
        if (const JVal *o = j.get("mlp_only_layers"))
            for (const JVal &e : o->arr) only.push_back((int)e.num);
        b.moe_layers.assign(std::max(c.n_layers, 0), 0);
        for (int i = 0; i < c.n_layers; i++)
            b.moe_layers[i] = std::find(only.begin(), only.end(), i) == only.end() && (i + 1) % step == 0;
    } else if (mt == "mixtral") {
        c.n_experts = (int)j.number("num_local_experts", 0);
        c.top_k = (int)j.number("num_experts_per_tok", 0);
        c.moe_inter = c.inter;
        c.norm_topk = 1;
        b.moe_layers.assign(std::max(c.n_layers, 0), 1);
    }
    if (const JVal *q = j.get("quantization_config")) {
        const std::string qm = q->string("quant_method");
        if (qm == "fp8") {
            const JVal *bs = q->get("weight_block_size");
            CK_REQUIRE(bs && bs->arr.size() == 2, "fp8 quantization_config without weight_block_size");
            b.br = (int)bs->arr[0].num;
            b.bc = (int)bs->arr[1].num;
        } else if (qm == "compressed-tensors") {
            const JVal *w = path_get(*q, {"config_groups", "group_0", "weights"});
            CK_REQUIRE(w, "compressed-tensors config without config_groups.group_0.weights");
            b.int_bits = (int)w->number("num_bits", 4);
            b.int_group = (int)w->number("group_size", 128);
        } else {
            set_error("quant_method '%s' is not taken", qm.c_str());
            return DITCH_CUDA_UNSUPPORTED;
        }
    }
    return DITCH_CUDA_OK;
}

// The config ditch builds from GGUF metadata (src/gguf_model.zig:114-129
// for the family, 282-372 for the fields): general.architecture as llama.cpp
// names it, `llama` with experts being Mixtral; layers with no
// ffn_gate_exps tensor are the dense ones.
int gguf_config(const Checkpoint &ck, Built &b) {
    ditch_cuda_model_config &c = b.cfg;
    const JVal &j = ck.config;
    const std::string arch = j.string("general.architecture");
    const std::string a = arch + ".";
    const int n_exp = (int)j.number(a + "expert_count", 0);
    if (arch == "llama") b.family = n_exp > 0 ? "mixtral" : "llama";
    else if (arch == "qwen2" || arch == "qwen3") b.family = arch;
    else if (arch == "qwen3moe") b.family = "qwen3_moe";
    else {
        set_error("GGUF architecture '%s' is not taken (llama, qwen2, qwen3 and qwen3moe are)", arch.c_str());
        return DITCH_CUDA_UNSUPPORTED;
    }
    CK_REQUIRE(n_exp == 0 || b.family == "mixtral" || b.family == "qwen3_moe", "GGUF %s with %d experts", arch.c_str(),
               n_exp);
    c.n_layers = (int)j.number(a + "block_count", 0);
    c.hidden = (int)j.number(a + "embedding_length", 0);
    c.heads = (int)j.number(a + "attention.head_count", 0);
    c.kv_heads = (int)j.number(a + "attention.head_count_kv", c.heads);
    c.head_dim = c.heads ? (int)j.number(a + "attention.key_length", c.hidden / c.heads) : 0;
    c.inter = (int)j.number(a + "feed_forward_length", 4.0 * c.hidden);
    c.eps = (float)j.number(a + "attention.layer_norm_rms_epsilon", 1e-6);
    c.rope_theta = j.number(a + "rope.freq_base", 10000.0);
    c.qk_norm = b.family == "qwen3" || b.family == "qwen3_moe";
    // rope.scaling.type linear (src/gguf_model.zig:305-309); other types read
    // as plain RoPE, and rope_freqs.weight is read below when none is set
    if (j.string(a + "rope.scaling.type") == "linear") {
        c.rope_scaling = 2;
        c.rope_factor = (double)(float)j.number(a + "rope.scaling.factor", 1.0);
    }
    const RawTensor *emb = ck.find("token_embd.weight");
    CK_REQUIRE(emb && emb->shape.size() == 2, "GGUF without a 2-D token_embd.weight");
    c.vocab = (int)emb->shape[0];
    b.tied = ck.find("output.weight") == nullptr;
    if (n_exp > 0) {
        c.n_experts = n_exp;
        c.top_k = (int)j.number(a + "expert_used_count", 2);
        c.moe_inter = (int)j.number(a + "expert_feed_forward_length", c.inter);
        c.norm_topk = 1;  // qwen3_moe and mixtral
        b.moe_layers.assign(std::max(c.n_layers, 0), 0);
        for (int i = 0; i < c.n_layers; i++)
            b.moe_layers[i] = ck.find("blk." + std::to_string(i) + ".ffn_gate_exps.weight") != nullptr;
    }
    return DITCH_CUDA_OK;
}

// llama.cpp's per-frequency factors of a llama3 rope scaling, recomputed the
// way ditch does to recognise the standard Llama 3 settings in a GGUF file's
// rope_freqs.weight (src/gguf_model.zig:150-170, 301-325): low_freq_factor 1,
// high_freq_factor 4, 8192 original positions, factor = the largest factor.
bool llama3_factors_match(const float *f, size_t n, float theta, int head_dim, float factor) {
    if ((size_t)head_dim / 2 != n) return false;
    const float orig = 8192.f, low_ff = 1.f, high_ff = 4.f;
    const float low_wavelen = orig / low_ff, high_wavelen = orig / high_ff;
    for (size_t i = 0; i < n; i++) {
        const double exponent = (double)(2 * i) / (double)head_dim;
        const double freq = 1.0 / std::pow((double)theta, exponent);
        const float wavelen = (float)(2.0 * M_PI / freq);
        float e;
        if (wavelen < high_wavelen) e = 1.f;
        else if (wavelen > low_wavelen) e = factor;
        else {
            const float smooth = (orig / wavelen - low_ff) / (high_ff - low_ff);
            e = 1.f / ((1.f - smooth) / factor + smooth);
        }
        if (std::fabs(e - f[i]) > 1e-4f * std::max(1.f, std::fabs(e))) return false;
    }
    return true;
}

int build_config(Checkpoint &ck, Built &b) {
    ditch_cuda_model_config &c = b.cfg;
    int s;
    if (ck.gguf) {
        // a GGUF file written by ditch's export carries the Hugging Face
        // config itself (src/gguf_model.zig:25, 222-227)
        const JVal *e = ck.config.get("ditch.hf.config_json");
        if (e && e->kind == JVal::Str) {
            CK_REQUIRE(parse_json(e->str.data(), e->str.size(), ck.embedded) && ck.embedded.kind == JVal::Obj,
                       "GGUF: bad ditch.hf.config_json");
            s = hf_config(ck.embedded, b);
        } else {
            s = gguf_config(ck, b);
        }
        if (s) return s;
        if (const RawTensor *rf = ck.find("rope_freqs.weight"); rf && !c.rope_scaling) {
            CK_REQUIRE(rf->dtype == "F32", "GGUF rope_freqs.weight of type %s", rf->dtype.c_str());
            const float *f = reinterpret_cast<const float *>(rf->data);
            const size_t n = rf->bytes / 4;
            float factor = 1.f;
            for (size_t i = 0; i < n; i++) factor = std::max(factor, f[i]);
            if (llama3_factors_match(f, n, (float)c.rope_theta, c.head_dim, factor)) {
                c.rope_scaling = 1;
                c.rope_factor = factor;
                c.rope_low_ff = 1.0;
                c.rope_high_ff = 4.0;
                c.rope_orig_max = 8192.0;
            } else {
                // other factors: the divisors themselves (src/gguf_model.zig:227-228, 326-335)
                b.rope_factors.assign(f, f + n);
                c.rope_scaling = 4;
            }
        }
    } else if ((s = hf_config(ck.config, b))) {
        return s;
    }
    CK_REQUIRE(c.n_layers > 0 && c.hidden > 0 && c.heads > 0 && c.kv_heads > 0 && c.vocab > 0,
               "incomplete model config (layers %d, hidden %d, heads %d / %d, vocab %d)", c.n_layers, c.hidden, c.heads,
               c.kv_heads, c.vocab);
    c.moe_layers = b.moe_layers.empty() ? nullptr : b.moe_layers.data();
    c.rope_factors = b.rope_factors.empty() ? nullptr : b.rope_factors.data();
    c.n_rope_factors = b.rope_factors.size();
    return DITCH_CUDA_OK;
}

}  // namespace ckpt
}  // namespace ditch

namespace ditch {
namespace ckpt {

// ---- the tensor table --------------------------------------------------------
struct Table {
    Checkpoint &ck;
    Built &b;

    const char *keep(const std::string &n) {
        b.names.push_back(std::make_unique<std::string>(n));
        return b.names.back()->c_str();
    }
    static void dims(const RawTensor &r, size_t &rows, size_t &cols) {
        rows = r.shape.empty() ? 1 : (size_t)r.shape[r.shape.size() >= 2 ? r.shape.size() - 2 : 0];
        cols = r.shape.size() >= 2 ? (size_t)r.shape.back() : 1;
    }

    // One stored tensor (or `slabs` stacked ones in `r`) as a table entry.
    int entry(const std::string &canon, const std::string &hf, const RawTensor &r, size_t slabs,
              const RawTensor *scales) {
        ditch_cuda_tensor t{};
        t.name = keep(canon);
        t.slabs = slabs;
        dims(r, t.rows, t.cols);
        t.data = r.data;
        t.data_bytes = r.bytes;
        if (r.dtype == "BF16") t.format = DITCH_FMT_BF16;
        else if (r.dtype == "F16") t.format = DITCH_FMT_F16;
        else if (r.dtype == "F32") t.format = DITCH_FMT_F32;
        else if (r.dtype == "GGML_Q8_0") t.format = DITCH_FMT_Q8_0;
        else if (r.dtype == "GGML_Q4_K") t.format = DITCH_FMT_Q4_K;
        else if (r.dtype == "F8_E4M3") {
            CK_REQUIRE(scales && scales->dtype == "F32", "%s: FP8 weight without f32 %s_scale_inv", hf.c_str(),
                       hf.c_str());
            CK_REQUIRE(b.br > 0 && b.bc > 0, "%s: FP8 weight without weight_block_size in the config", hf.c_str());
            t.format = DITCH_FMT_FP8_BLOCK;
            t.scales = scales->data;
            t.scales_bytes = scales->bytes;
            t.scales_dtype = DITCH_SCALE_F32;
            t.block_rows = b.br;
            t.block_cols = b.bc;
        } else {
            set_error("%s: dtype %s is not taken", hf.c_str(), r.dtype.c_str());
            return DITCH_CUDA_UNSUPPORTED;
        }
        b.tensors.push_back(t);
        return DITCH_CUDA_OK;
    }

    // The compressed-tensors pack-quantized form of `base` (weight_packed,
    // weight_scale, optional weight_zero_point, weight_shape).
    int packed(const std::string &canon, const std::string &base, size_t slabs, const RawTensor &pk,
               const RawTensor &sc, const RawTensor *zp, size_t rows, size_t cols) {
        CK_REQUIRE(b.int_bits > 0, "%s: packed weight without a compressed-tensors config", base.c_str());
        if (ck.find(base + ".weight_g_idx")) {
            set_error("%s: activation-ordered groups (weight_g_idx) are not taken", base.c_str());
            return DITCH_CUDA_UNSUPPORTED;
        }
        ditch_cuda_tensor t{};
        t.name = keep(canon);
        t.format = DITCH_FMT_INT_PACKED;
        t.slabs = slabs;
        t.rows = rows;
        t.cols = cols;
        t.data = pk.data;
        t.data_bytes = pk.bytes;
        t.scales = sc.data;
        t.scales_bytes = sc.bytes;
        CK_REQUIRE(sc.dtype == "BF16" || sc.dtype == "F32", "%s: weight_scale dtype %s", base.c_str(), sc.dtype.c_str());
        t.scales_dtype = sc.dtype == "BF16" ? DITCH_SCALE_BF16 : DITCH_SCALE_F32;
        if (zp) {
            t.zeros = zp->data;
            t.zeros_bytes = zp->bytes;
        }
        t.block_cols = b.int_group;
        t.bits = b.int_bits;
        b.tensors.push_back(t);
        return DITCH_CUDA_OK;
    }

    static bool shape_of(const RawTensor &r, size_t &rows, size_t &cols) {
        int64_t v[2] = {0, 0};
        if (r.dtype == "I64" && r.bytes >= 16) memcpy(v, r.data, 16);
        else if (r.dtype == "I32" && r.bytes >= 8) {
            int32_t w[2];
            memcpy(w, r.data, 8);
            v[0] = w[0], v[1] = w[1];
        } else
            return false;
        rows = (size_t)v[0], cols = (size_t)v[1];
        return true;
    }

    // A dense weight by HF name (absent: skipped unless required).
    int dense(const std::string &canon, const std::string &hf, bool required) {
        if (const RawTensor *r = ck.find(hf)) return entry(canon, hf, *r, 1, ck.find(hf + "_scale_inv"));
        const std::string base = hf.size() > 7 && hf.compare(hf.size() - 7, 7, ".weight") == 0 ? hf.substr(0, hf.size() - 7)
                                                                                                 : hf;
        const RawTensor *pk = ck.find(base + ".weight_packed");
        if (pk) {
            const RawTensor *sc = ck.find(base + ".weight_scale"), *shp = ck.find(base + ".weight_shape");
            size_t rows = 0, cols = 0;
            CK_REQUIRE(sc && shp && shape_of(*shp, rows, cols), "%s: packed weight without scale / shape", base.c_str());
            return packed(canon, base, 1, *pk, *sc, ck.find(base + ".weight_zero_point"), rows, cols);
        }
        CK_REQUIRE(!required, "tensor %s is missing", hf.c_str());
        return DITCH_CUDA_OK;
    }

    // Per-expert tensors of one projection, stacked [E][rows][cols] (their
    // FP8 scales, packed words, scales and zero points stacked alike).
    int stack(const std::string &canon, const std::vector<std::string> &hf) {
        std::vector<const RawTensor *> rs;
        for (const std::string &n : hf) {
            const RawTensor *r = ck.find(n);
            if (!r) break;
            rs.push_back(r);
        }
        if (rs.size() != hf.size()) {  // the pack-quantized form
            const std::string base0 = hf[0].substr(0, hf[0].size() - 7);
            CK_REQUIRE(ck.find(base0 + ".weight_packed"), "tensor %s is missing", hf[0].c_str());
            std::vector<const RawTensor *> pk, sc, zp;
            size_t rows = 0, cols = 0;
            for (const std::string &n : hf) {
                const std::string base = n.substr(0, n.size() - 7);
                const RawTensor *p = ck.find(base + ".weight_packed"), *s = ck.find(base + ".weight_scale"),
                                *z = ck.find(base + ".weight_zero_point"), *sh = ck.find(base + ".weight_shape");
                size_t r2 = 0, c2 = 0;
                CK_REQUIRE(p && s && sh && shape_of(*sh, r2, c2), "%s: packed expert incomplete", base.c_str());
                CK_REQUIRE(pk.empty() || (r2 == rows && c2 == cols && p->bytes == pk[0]->bytes), "%s: experts differ",
                           base.c_str());
                rows = r2, cols = c2;
                pk.push_back(p), sc.push_back(s), zp.push_back(z);
            }
            RawTensor P = concat(pk), S = concat(sc);
            RawTensor Z;
            const bool has_z = zp[0] != nullptr;
            if (has_z) {
                for (const RawTensor *z : zp) CK_REQUIRE(z, "%s: zero points on some experts only", base0.c_str());
                Z = concat(zp);
            }
            return packed(canon, base0, hf.size(), P, S, has_z ? &Z : nullptr, rows, cols);
        }
        for (const RawTensor *r : rs)
            CK_REQUIRE(r->dtype == rs[0]->dtype && r->shape == rs[0]->shape, "%s: experts differ", hf[0].c_str());
        RawTensor all = concat(rs);
        all.shape = rs[0]->shape;
        if (rs[0]->dtype == "F8_E4M3") {
            std::vector<const RawTensor *> ss;
            for (const std::string &n : hf) {
                const RawTensor *s = ck.find(n + "_scale_inv");
                CK_REQUIRE(s, "%s_scale_inv is missing", n.c_str());
                ss.push_back(s);
            }
            RawTensor S = concat(ss);
            S.dtype = ss[0]->dtype;
            return entry(canon, hf[0], all, hf.size(), &S);
        }
        return entry(canon, hf[0], all, hf.size(), nullptr);
    }

    RawTensor concat(const std::vector<const RawTensor *> &rs) {
        size_t n = 0;
        for (const RawTensor *r : rs) n += r->bytes;
        uint8_t *dst = ck.alloc(n);
        size_t o = 0;
        for (const RawTensor *r : rs) {
            memcpy(dst + o, r->data, r->bytes);
            o += r->bytes;
        }
        RawTensor out;
        out.dtype = rs[0]->dtype;
        out.shape = rs[0]->shape;
        out.data = dst;
        out.bytes = n;
        return out;
    }
};

}  // namespace ckpt
}  // namespace ditch

namespace ditch {
namespace ckpt {

// Rows of a llama GGUF q / k weight back in the Hugging Face order: the
// converter stores head h's rows as (i, half) pairs, ditch's model reads
// (half, i) (llama.cpp's permute of q and k; n = the heads of the tensor).
RawTensor unpermute_rows(Checkpoint &ck, const RawTensor &r, int n) {
    const size_t rows = (size_t)r.shape[0], rb = r.bytes / rows, d = rows / n;
    uint8_t *dst = ck.alloc(r.bytes);
    for (size_t h = 0; h < (size_t)n; h++)
        for (size_t half = 0; half < 2; half++)
            for (size_t i = 0; i < d / 2; i++)
                memcpy(dst + (h * d + half * (d / 2) + i) * rb, r.data + (h * d + 2 * i + half) * rb, rb);
    RawTensor out = r;
    out.data = dst;
    return out;
}

// A fused expert tensor [E][a][b] split into per-expert row blocks (and
// transposed per expert when `transpose`), as separate tensors of `ck`.
int split_fused(Checkpoint &ck, const RawTensor &r, bool transpose, int row0, int nrows, const std::string &prefix,
                std::vector<std::string> &names) {
    const size_t es = dtype_size(r.dtype);
    CK_REQUIRE(r.shape.size() == 3 && (r.dtype == "BF16" || r.dtype == "F16" || r.dtype == "F32"),
               "fused experts %s: 3-D bf16 / f16 / f32 expected", prefix.c_str());
    const size_t E = (size_t)r.shape[0], A = (size_t)r.shape[1], B = (size_t)r.shape[2];
    // per expert the logical matrix is [A][B] (or [B][A] transposed); rows [row0, row0 + nrows) of it
    const size_t R = transpose ? B : A, Cn = transpose ? A : B;
    CK_REQUIRE((size_t)(row0 + nrows) <= R, "fused experts %s: rows out of range", prefix.c_str());
    for (size_t e = 0; e < E; e++) {
        uint8_t *dst = ck.alloc((size_t)nrows * Cn * es);
        const uint8_t *src = r.data + e * A * B * es;
        for (int i = 0; i < nrows; i++)
            for (size_t j = 0; j < Cn; j++) {
                const size_t si = transpose ? (j * B + (row0 + i)) : ((row0 + i) * B + j);
                memcpy(dst + ((size_t)i * Cn + j) * es, src + si * es, es);
            }
        RawTensor t;
        t.dtype = r.dtype;
        t.shape = {(int64_t)nrows, (int64_t)Cn};
        t.data = dst;
        t.bytes = (size_t)nrows * Cn * es;
        const std::string name = prefix + std::to_string(e) + ".weight";
        ck.t[name] = t;
        names.push_back(name);
    }
    return DITCH_CUDA_OK;
}

int build_tensors(Checkpoint &ck, Built &b) {
    const ditch_cuda_model_config &c = b.cfg;
    Table tb{ck, b};
    int s;
    if (ck.gguf) {
        // llama.cpp names; q / k rows (and biases) of the llama family stored
        // permuted (src/gguf_model.zig:141-143, 700-800)
        const bool permuted = b.family == "llama" || b.family == "mistral" || b.family == "mixtral";
        if ((s = tb.dense("embed", "token_embd.weight", true))) return s;
        if ((s = tb.dense("final_norm", "output_norm.weight", true))) return s;
        if ((s = tb.dense("lm_head", b.tied ? "token_embd.weight" : "output.weight", true))) return s;
        for (int i = 0; i < c.n_layers; i++) {
            const std::string p = "blk." + std::to_string(i) + ".", L = "L" + std::to_string(i) + ".";
            const char *map[][2] = {{"input_norm", "attn_norm.weight"}, {"post_norm", "ffn_norm.weight"},
                                    {"v", "attn_v.weight"}, {"o", "attn_output.weight"}};
            for (auto &m : map)
                if ((s = tb.dense(L + m[0], p + m[1], true))) return s;
            for (const char *qk : {"q", "k"})
                for (const char *kind : {"weight", "bias"}) {
                    const std::string hf = p + "attn_" + qk + "." + kind;
                    const RawTensor *r = ck.find(hf);
                    const bool weight = kind[0] == 'w';
                    CK_REQUIRE(r || !weight, "tensor %s is missing", hf.c_str());
                    if (!r) continue;
                    if (permuted) ck.t[hf] = unpermute_rows(ck, *r, qk[0] == 'q' ? c.heads : c.kv_heads);
                    if ((s = tb.dense(L + qk + (weight ? "" : "b"), hf, true))) return s;
                }
            if ((s = tb.dense(L + "vb", p + "attn_v.bias", false))) return s;
            if (c.qk_norm) {
                if ((s = tb.dense(L + "q_norm", p + "attn_q_norm.weight", true))) return s;
                if ((s = tb.dense(L + "k_norm", p + "attn_k_norm.weight", true))) return s;
            }
            if (!b.moe_layers.empty() && b.moe_layers[i]) {
                // experts stacked [E][rows][cols] in one tensor, the device's slab layout
                if ((s = tb.dense(L + "router", p + "ffn_gate_inp.weight", true))) return s;
                for (const char *e : {"gate", "up", "down"}) {
                    const std::string hf = p + "ffn_" + e + "_exps.weight";
                    const RawTensor *r = ck.find(hf);
                    CK_REQUIRE(r && r->shape.size() == 3 && r->shape[0] == c.n_experts,
                               "%s: 3-D [%d experts][rows][cols] expected", hf.c_str(), c.n_experts);
                    if ((s = tb.entry(L + "e_" + e, hf, *r, (size_t)c.n_experts, nullptr))) return s;
                }
                continue;
            }
            for (const char *m : {"gate", "up", "down"})
                if ((s = tb.dense(L + m, p + "ffn_" + m + ".weight", true))) return s;
        }
        return DITCH_CUDA_OK;
    }
    const std::string mt = ck.config.string("model_type");
    if ((s = tb.dense("embed", "model.embed_tokens.weight", true))) return s;
    if ((s = tb.dense("final_norm", "model.norm.weight", true))) return s;
    if ((s = tb.dense("lm_head", b.tied ? "model.embed_tokens.weight" : "lm_head.weight", true))) return s;
    for (int i = 0; i < c.n_layers; i++) {
        const std::string p = "model.layers." + std::to_string(i) + ".", L = "L" + std::to_string(i) + ".";
        if ((s = tb.dense(L + "input_norm", p + "input_layernorm.weight", true))) return s;
        if ((s = tb.dense(L + "post_norm", p + "post_attention_layernorm.weight", true))) return s;
        for (const char *a : {"q", "k", "v", "o"})
            if ((s = tb.dense(L + a, p + "self_attn." + a + "_proj.weight", true))) return s;
        for (const char *a : {"q", "k", "v"})
            if ((s = tb.dense(L + a + "b", p + "self_attn." + a + "_proj.bias", false))) return s;
        if (c.qk_norm) {
            if ((s = tb.dense(L + "q_norm", p + "self_attn.q_norm.weight", true))) return s;
            if ((s = tb.dense(L + "k_norm", p + "self_attn.k_norm.weight", true))) return s;
        }
        const bool moe = !b.moe_layers.empty() && b.moe_layers[i];
        if (!moe) {
            for (const char *a : {"gate", "up", "down"})
                if ((s = tb.dense(L + a, p + "mlp." + a + "_proj.weight", true))) return s;
            continue;
        }
        // routed experts: one tensor per expert and projection (src/moe.zig:83-92)
        std::vector<std::string> g, u, d;
        if (mt == "mixtral") {
            if ((s = tb.dense(L + "router", p + "block_sparse_moe.gate.weight", true))) return s;
            for (int e = 0; e < c.n_experts; e++) {
                const std::string x = p + "block_sparse_moe.experts." + std::to_string(e) + ".";
                g.push_back(x + "w1.weight"), u.push_back(x + "w3.weight"), d.push_back(x + "w2.weight");
            }
        } else {
            if ((s = tb.dense(L + "router", p + "mlp.gate.weight", true))) return s;
            const RawTensor *gu = ck.find(p + "mlp.experts.gate_up_proj"), *dn = ck.find(p + "mlp.experts.down_proj");
            if (gu && dn) {
                // fused [E, 2I, H] / [E, H, I], or transposed [E, H, 2I] / [E, I, H] (src/moe.zig:728-770)
                const bool tr = gu->shape.size() == 3 && gu->shape[1] == c.hidden && gu->shape[2] != c.hidden;
                const int I2 = (int)(tr ? gu->shape[2] : gu->shape[1]);
                const std::string x = p + "mlp.experts.split.";
                const RawTensor gu_c = *gu, dn_c = *dn;
                if ((s = split_fused(ck, gu_c, tr, 0, I2 / 2, x + "gate.", g))) return s;
                if ((s = split_fused(ck, gu_c, tr, I2 / 2, I2 / 2, x + "up.", u))) return s;
                if ((s = split_fused(ck, dn_c, tr, 0, c.hidden, x + "down.", d))) return s;
            } else {
                for (int e = 0; e < c.n_experts; e++) {
                    const std::string x = p + "mlp.experts." + std::to_string(e) + ".";
                    g.push_back(x + "gate_proj.weight"), u.push_back(x + "up_proj.weight"),
                        d.push_back(x + "down_proj.weight");
                }
            }
        }
        if ((s = tb.stack(L + "e_gate", g))) return s;
        if ((s = tb.stack(L + "e_up", u))) return s;
        if ((s = tb.stack(L + "e_down", d))) return s;
    }
    return DITCH_CUDA_OK;
}

int open_checkpoint(const char *path, Checkpoint &ck, Built &b) {
    const std::string p = path;
    struct stat st;
    CK_REQUIRE(stat(path, &st) == 0, "%s does not exist", path);
    int s = S_ISDIR(st.st_mode) ? read_hf_dir(p, ck) : read_gguf(p, ck);
    if (s) return s;
    if ((s = build_config(ck, b))) return s;
    return build_tensors(ck, b);
}

}  // namespace ckpt
}  // namespace ditch

using namespace ditch::ckpt;

extern "C" {

int ditch_cuda_checkpoint_inspect(const char *path, ditch_cuda_model_config *cfg, size_t *n_tensors,
                                  uint8_t *moe_layers, size_t moe_layers_len, float *rope_factors,
                                  size_t rope_factors_len) {
    clear_error();
    CK_REQUIRE(path && cfg && n_tensors, "null argument");
    Checkpoint ck;
    Built b;
    int s;
    if ((s = open_checkpoint(path, ck, b))) return s;
    *cfg = b.cfg;
    cfg->moe_layers = nullptr;
    cfg->rope_factors = nullptr;
    if (moe_layers)
        for (size_t i = 0; i < moe_layers_len && i < b.moe_layers.size(); i++) moe_layers[i] = b.moe_layers[i];
    if (rope_factors)
        for (size_t i = 0; i < rope_factors_len && i < b.rope_factors.size(); i++) rope_factors[i] = b.rope_factors[i];
    *n_tensors = b.tensors.size();
    return DITCH_CUDA_OK;
}

int ditch_cuda_model_load_checkpoint(ditch_cuda_device *dev, const char *path, int max_seq, ditch_cuda_model **out) {
    clear_error();
    CK_REQUIRE(dev && path && out, "null argument");
    Checkpoint ck;
    Built b;
    int s;
    if ((s = open_checkpoint(path, ck, b))) return s;
    b.cfg.max_seq = max_seq > 0 ? max_seq : 4096;
    return ditch_cuda_model_load(dev, &b.cfg, b.tensors.data(), b.tensors.size(), out);
}

}  // extern "C"
