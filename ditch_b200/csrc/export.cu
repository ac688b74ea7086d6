// Export of an edited model (src/export.zig): every tensor of the Hugging
// Face checkpoint the model was loaded from is written again as safetensors,
// with the model's abliteration deltas merged into the weights they edit.
// The merge runs on the device over the deltas already resident there:
// a tensor that changes (an edited one, a quantised group decoded to bf16, a
// dtype conversion) goes up once, is decoded to f32, merged, rounded to its
// output dtype and comes back; a tensor that does not change is copied from
// the mapped file as it is.
//
//   edited [out][in] weight   W' = W + B A, each term added in rank order
//                             (src/export.zig:88-131, tensor.axpy)
//   fused expert down tensor  per expert slice, [hidden][inter] like the
//                             above, [inter][hidden] with the rank terms
//                             summed first (src/moe.zig:368-390)
//   FP8 / pack-quantized      decoded to bf16 as at load; config.json loses
//                             quantization_config (src/dequant.zig:1195-1219)
//   output dtype              the source's own for float tensors, bf16 for
//                             decoded groups, or the requested one (config.json
//                             then names it, src/export.zig:239-283)
//
// Files: `.incomplete` first, the shards (model.safetensors, or
// model-0000i-of-0000n.safetensors plus model.safetensors.index.json once
// the tensors pass max_shard_bytes), config.json, the tokenizer and side
// files, then `.incomplete` removed (src/export.zig:353-440).
#include <dirent.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "checkpoint.cuh"
#include "kernels.cuh"

namespace ditch {
namespace {

using namespace ckpt;

constexpr int kExportThreads = 256;

int export_blocks(long long n) {
    long long b = (n + kExportThreads - 1) / kExportThreads;
    return (int)std::max(1LL, std::min(b, 148LL * 16));
}

// IEEE binary16 round to nearest even (Zig's @floatCast, src/tensor.zig:437);
// a NaN keeps the top of its payload with the quiet bit set.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float v) {
    const uint32_t x = __float_as_uint(v);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // 65520 and up round to infinity
    if (ax < 0x38800000u) {                                      // below 2^-14: subnormal or zero
        if (ax <= 0x33000000u) return (uint16_t)sign;            // up to 2^-25 (a tie) rounds to zero
        const uint32_t e = ax >> 23, mant = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;                         // 14..23: units of 2^-24
        uint32_t q = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t r = ax - 0x38000000u;  // exponent rebased from 127 to 15
    r += 0xfffu + ((r >> 13) & 1u);
    return (uint16_t)(sign | (r >> 13));
}

// w[r][c] += b[r][k] * a[k][c] for k = 0 .. rank-1, each product rounded and
// then added, in k order (tensor.axpy per rank term: no fused multiply-add).
__global__ void k_merge_rows(float *w, long long rows, int cols, const float *a, const float *b, int rank) {
    const long long n = rows * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / cols;
        const int c = (int)(i - r * cols);
        float y = w[i];
        for (int k = 0; k < rank; k++) y = __fadd_rn(y, __fmul_rn(b[r * rank + k], a[(long long)k * cols + c]));
        w[i] = y;
    }
}

// The transposed form: w[j][i] += sum_k b[i][k] * a[k][j], the rank terms
// summed first (rows j: the delta's input side, columns i: its output side).
__global__ void k_merge_cols(float *w, int rows, int cols, const float *a, const float *b, int rank) {
    const long long n = (long long)rows * cols;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < n; t += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(t / cols), i = (int)(t - (long long)j * cols);
        float acc = 0.0f;
        for (int k = 0; k < rank; k++) acc = __fadd_rn(acc, __fmul_rn(b[(long long)i * rank + k], a[(long long)k * rows + j]));
        w[t] = __fadd_rn(w[t], acc);
    }
}

__global__ void k_f32_to_bf16_out(const float *src, uint16_t *dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = f32_to_bf16_bits(src[i]);
}

__global__ void k_f32_to_f16_out(const float *src, uint16_t *dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = f32_to_f16_bits(src[i]);
}

// ---- config.json text (edited in place, the source's formatting kept) ------

size_t string_end(const std::string &t, size_t i) {  // just past the string opening at t[i]
    for (size_t j = i + 1; j < t.size(); j++) {
        if (t[j] == '\\') j++;
        else if (t[j] == '"') return j + 1;
    }
    return std::string::npos;
}

size_t skip_ws(const std::string &t, size_t j) {
    while (j < t.size() && (t[j] == ' ' || t[j] == '\n' || t[j] == '\r' || t[j] == '\t')) j++;
    return j;
}

size_t value_end(const std::string &t, size_t i) {
    if (i >= t.size()) return std::string::npos;
    if (t[i] == '"') return string_end(t, i);
    if (t[i] == '{' || t[i] == '[') {
        int depth = 0;
        for (size_t j = i; j < t.size(); j++) {
            if (t[j] == '"') {
                const size_t e = string_end(t, j);
                if (e == std::string::npos) return e;
                j = e - 1;
            } else if (t[j] == '{' || t[j] == '[') {
                depth++;
            } else if (t[j] == '}' || t[j] == ']') {
                if (--depth == 0) return j + 1;
            }
        }
        return std::string::npos;
    }
    size_t j = i;
    while (j < t.size() && t[j] != ',' && t[j] != '}' && t[j] != ']' && t[j] != ' ' && t[j] != '\n' && t[j] != '\r' &&
           t[j] != '\t')
        j++;
    return j;
}

// The first `"key": value` at any depth: [start of the key, end of the value).
bool find_key(const std::string &t, const std::string &key, size_t &start, size_t &end) {
    for (size_t i = 0; i < t.size(); i++) {
        if (t[i] != '"') continue;
        const size_t s_end = string_end(t, i);
        if (s_end == std::string::npos) return false;
        const size_t j = skip_ws(t, s_end);
        if (j < t.size() && t[j] == ':' && t.compare(i + 1, s_end - i - 2, key) == 0 && s_end - i - 2 == key.size()) {
            const size_t v = skip_ws(t, j + 1), ve = value_end(t, v);
            if (ve == std::string::npos) return false;
            start = i, end = ve;
            return true;
        }
        i = s_end - 1;  // a string is skipped whole; other values are scanned (nested objects may hold the key)
    }
    return false;
}

// Every "quantization_config" and "expert_dtype" entry removed with one of its
// separating commas (the following one, else the preceding one).
std::string strip_quantization(std::string t) {
    for (const char *key : {"quantization_config", "expert_dtype"}) {
        size_t s, e;
        while (find_key(t, key, s, e)) {
            const size_t j = skip_ws(t, e);
            if (j < t.size() && t[j] == ',') {
                e = skip_ws(t, j + 1);
            } else {
                size_t i = s;
                while (i > 0 && (t[i - 1] == ' ' || t[i - 1] == '\n' || t[i - 1] == '\r' || t[i - 1] == '\t')) i--;
                if (i > 0 && t[i - 1] == ',') s = i - 1;
            }
            t = t.substr(0, s) + t.substr(e);
        }
    }
    return t;
}

// Every "dtype" / "torch_dtype" whose value is float32, float16 or bfloat16
// renamed to the export's dtype, at any depth.
std::string with_config_dtype(const std::string &t, const char *name) {
    std::string out;
    size_t i = 0;
    while (i < t.size()) {
        const size_t at = t.find('"', i);
        if (at == std::string::npos) break;
        const size_t key_end = string_end(t, at);
        if (key_end == std::string::npos) break;
        const std::string key = t.substr(at + 1, key_end - at - 2);
        size_t j = skip_ws(t, key_end);
        if (j < t.size() && t[j] == ':' && (key == "dtype" || key == "torch_dtype")) {
            j = skip_ws(t, j + 1);
            if (j < t.size() && t[j] == '"') {
                const size_t v_end = string_end(t, j);
                if (v_end == std::string::npos) break;
                const std::string v = t.substr(j + 1, v_end - j - 2);
                if (v == "float32" || v == "float16" || v == "bfloat16") {
                    out.append(t, i, j + 1 - i);
                    out += name;
                    out += '"';
                } else {
                    out.append(t, i, v_end - i);
                }
                i = v_end;
                continue;
            }
        }
        out.append(t, i, key_end - i);  // a key or a string value, copied through
        i = key_end;
    }
    out.append(t, i, std::string::npos);
    return out;
}

const char *dtype_config_name(int dtype) {
    return dtype == DITCH_DTYPE_F32 ? "float32" : dtype == DITCH_DTYPE_F16 ? "float16" : dtype == DITCH_DTYPE_BF16 ? "bfloat16" : nullptr;
}

}  // namespace
}  // namespace ditch

namespace ditch {
namespace {

using namespace ckpt;

// One tensor of the export.
struct OutTensor {
    enum Kind { Copy, Float, Fp8, Packed };
    enum Edit { None, O, Down, Expert, Fused };
    std::string name, dtype;          // as written
    std::vector<int64_t> shape;
    size_t bytes = 0;
    Kind kind = Copy;
    const RawTensor *src = nullptr, *scales = nullptr, *zeros = nullptr;
    size_t rows = 0, cols = 0;        // the 2-D view of the source values
    Edit edit = None;
    int layer = -1, expert = 0;
    bool fused_t = false;             // fused expert tensor stored [E][inter][hidden]
};

bool ends_with(const std::string &s, const char *suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// "model.layers.<i>.<rest>"
bool layer_name(const std::string &n, int &layer, std::string &rest) {
    static const char pre[] = "model.layers.";
    if (n.compare(0, sizeof pre - 1, pre) != 0) return false;
    size_t i = sizeof pre - 1, j = i;
    while (j < n.size() && n[j] >= '0' && n[j] <= '9') j++;
    if (j == i || j >= n.size() || n[j] != '.') return false;
    layer = atoi(n.c_str() + i);
    rest = n.substr(j + 1);
    return true;
}

// "<pre><e><post>" -> e
bool expert_name(const std::string &rest, const char *pre, const char *post, int &e) {
    const size_t np = strlen(pre), nq = strlen(post);
    if (rest.size() <= np + nq || rest.compare(0, np, pre) != 0 || !ends_with(rest, post)) return false;
    const std::string mid = rest.substr(np, rest.size() - np - nq);
    if (mid.empty() || mid.find_first_not_of("0123456789") != std::string::npos) return false;
    e = atoi(mid.c_str());
    return true;
}

const char *out_float_dtype(int dtype, const std::string &own) {
    return dtype == DITCH_DTYPE_F32 ? "F32" : dtype == DITCH_DTYPE_F16 ? "F16" : dtype == DITCH_DTYPE_BF16 ? "BF16" : own.c_str();
}

// Which delta of the model edits tensor `o` (src/model.zig:2315-2340 for the
// families of the device path).
void find_edit(const ditch_cuda_model *m, const Checkpoint &ck, OutTensor &o) {
    int li;
    std::string rest;
    if (!layer_name(o.name, li, rest) || li >= (int)m->layers.size()) return;
    const Layer &L = m->layers[li];
    int e;
    if (rest == "self_attn.o_proj.weight") {
        if (L.o_edit) o.edit = OutTensor::O;
    } else if (!L.moe) {
        if (rest == "mlp.down_proj.weight" && L.down_edit) o.edit = OutTensor::Down;
    } else if (expert_name(rest, "mlp.experts.", ".down_proj.weight", e) ||
               expert_name(rest, "block_sparse_moe.experts.", ".w2.weight", e)) {
        if (e < (int)L.e_edit.size() && L.e_edit[e]) o.edit = OutTensor::Expert, o.expert = e;
    } else if (rest == "mlp.experts.down_proj") {
        if (std::find(L.e_edit.begin(), L.e_edit.end(), 1) == L.e_edit.end()) return;
        o.edit = OutTensor::Fused;
        // the loader's rule: gate_up [E][hidden][2 inter] is the transposed form
        const RawTensor *gu = ck.find("model.layers." + std::to_string(li) + ".mlp.experts.gate_up_proj");
        o.fused_t = gu && gu->shape.size() == 3 && gu->shape[1] == m->cfg.hidden && gu->shape[2] != m->cfg.hidden;
    }
    if (o.edit != OutTensor::None) o.layer = li;
}

int plan_export(const ditch_cuda_model *m, const Checkpoint &ck, int dtype, std::vector<OutTensor> &plan,
                bool &decoded) {
    decoded = false;
    for (const auto &kv : ck.t) {
        const std::string &n = kv.first;
        const RawTensor &r = kv.second;
        // companions of a quantised group go with it
        if (ends_with(n, "_scale_inv")) {
            const RawTensor *w = ck.find(n.substr(0, n.size() - 10));
            if (w && w->dtype == "F8_E4M3") continue;
        }
        bool companion = false;
        for (const char *suf : {".weight_scale", ".weight_zero_point", ".weight_shape", ".weight_g_idx"})
            if (ends_with(n, suf) && ck.find(n.substr(0, n.size() - strlen(suf)) + ".weight_packed")) companion = true;
        if (companion) continue;
        OutTensor o;
        o.src = &r;
        size_t elems = 1;
        if (r.dtype == "F8_E4M3") {
            CK_REQUIRE(r.shape.size() == 2, "%s: FP8 weights of %zu dims are not exported", n.c_str(), r.shape.size());
            o.scales = ck.find(n + "_scale_inv");
            CK_REQUIRE(o.scales && o.scales->dtype == "F32", "%s: f32 %s_scale_inv missing", n.c_str(), n.c_str());
            o.kind = OutTensor::Fp8;
            o.name = n;
            o.shape = r.shape;
            o.dtype = out_float_dtype(dtype, "BF16");
            decoded = true;
        } else if (ends_with(n, ".weight_packed")) {
            const std::string base = n.substr(0, n.size() - 14);
            CK_REQUIRE(!ck.find(base + ".weight_g_idx"), "%s: activation-ordered groups are not exported", base.c_str());
            const RawTensor *shp = ck.find(base + ".weight_shape");
            o.scales = ck.find(base + ".weight_scale");
            o.zeros = ck.find(base + ".weight_zero_point");
            int64_t v[2] = {0, 0};
            if (shp && shp->dtype == "I64" && shp->bytes >= 16) memcpy(v, shp->data, 16);
            else if (shp && shp->dtype == "I32" && shp->bytes >= 8) {
                int32_t w[2];
                memcpy(w, shp->data, 8);
                v[0] = w[0], v[1] = w[1];
            }
            CK_REQUIRE(o.scales && v[0] > 0 && v[1] > 0, "%s: packed weight without scale / shape", base.c_str());
            o.kind = OutTensor::Packed;
            o.name = base + ".weight";
            o.shape = {v[0], v[1]};
            o.dtype = out_float_dtype(dtype, "BF16");
            decoded = true;
        } else if (r.dtype == "BF16" || r.dtype == "F16" || r.dtype == "F32") {
            o.name = n;
            o.shape = r.shape;
            o.dtype = out_float_dtype(dtype, r.dtype);
            o.kind = o.dtype == r.dtype ? OutTensor::Copy : OutTensor::Float;
        } else if (r.dtype == "I32") {  // integer tables, never converted (src/model.zig:2086-2092)
            o.name = n;
            o.shape = r.shape;
            o.dtype = r.dtype;
        } else if (r.dtype == "F8_E5M2" || r.dtype == "U8") {
            set_error("%s: %s tensors are not exported by the device path", n.c_str(), r.dtype.c_str());
            return DITCH_CUDA_UNSUPPORTED;
        } else {
            continue;  // other dtypes are skipped, as ditch skips them at load
        }
        for (int64_t d : o.shape) elems *= (size_t)d;
        o.rows = o.shape.empty() ? 1 : (size_t)o.shape[0];
        o.cols = o.shape.empty() ? 1 : elems / o.rows;
        o.bytes = elems * dtype_size(o.dtype);
        find_edit(m, ck, o);
        if (o.edit != OutTensor::None && o.kind == OutTensor::Copy) o.kind = OutTensor::Float;
        plan.push_back(std::move(o));
    }
    return DITCH_CUDA_OK;
}

// Device and pinned host buffers of one export, grown as needed.
struct Work {
    ditch_cuda_model *m;
    DevBuf raw, sc, zr, bf, f, out;
    void *host = nullptr;
    size_t host_bytes = 0;
    ~Work() {
        if (host) cudaFreeHost(host);
    }
    cudaError_t host_reserve(size_t n) {
        if (n <= host_bytes) return cudaSuccess;
        if (host) cudaFreeHost(host);
        host = nullptr, host_bytes = 0;
        cudaError_t e = cudaHostAlloc(&host, n, cudaHostAllocDefault);
        if (e == cudaSuccess) host_bytes = n;
        return e;
    }
};

int upload(Work &w, DevBuf &dst, const RawTensor &r) {
    DITCH_CUDA(dst.reserve(r.bytes));
    DITCH_CUDA(cudaMemcpyAsync(dst.ptr, r.data, r.bytes, cudaMemcpyHostToDevice, w.m->dev->stream));
    return DITCH_CUDA_OK;
}

// The merge of o's delta into the f32 values in w.f.
int merge(Work &w, const OutTensor &o) {
    ditch_cuda_model *m = w.m;
    ditch_cuda_device *dev = m->dev;
    const Layer &L = m->layers[o.layer];
    const int H = m->cfg.hidden, mi = m->cfg.moe_inter;
    float *v = w.f.as<float>();
    const long long n = (long long)o.rows * o.cols;
    switch (o.edit) {
    case OutTensor::O:
    case OutTensor::Down: {
        const bool is_o = o.edit == OutTensor::O;
        const size_t want_cols = is_o ? (size_t)m->cfg.heads * m->cfg.head_dim : (size_t)m->cfg.inter;
        CK_REQUIRE(o.rows == (size_t)H && o.cols == want_cols, "%s: [%zu][%zu] is not the model's [%d][%zu]",
                   o.name.c_str(), o.rows, o.cols, H, want_cols);
        k_merge_rows<<<export_blocks(n), kExportThreads, 0, dev->stream>>>(
            v, (long long)o.rows, (int)o.cols, (is_o ? L.o_a : L.down_a).as<float>(), (is_o ? L.o_b : L.down_b).as<float>(),
            is_o ? L.o_rank : L.down_rank);
        DITCH_LAUNCH(dev, cudaGetLastError());
        break;
    }
    case OutTensor::Expert:
        CK_REQUIRE(o.rows == (size_t)H && o.cols == (size_t)mi, "%s: [%zu][%zu] is not the model's [%d][%d]",
                   o.name.c_str(), o.rows, o.cols, H, mi);
        k_merge_rows<<<export_blocks(n), kExportThreads, 0, dev->stream>>>(
            v, H, mi, L.e_a.as<float>() + (size_t)o.expert * L.e_rank * mi,
            L.e_b.as<float>() + (size_t)o.expert * H * L.e_rank, L.e_rank);
        DITCH_LAUNCH(dev, cudaGetLastError());
        break;
    case OutTensor::Fused: {
        const int E = (int)L.e_edit.size();
        CK_REQUIRE(o.shape.size() == 3 && o.shape[0] == E && (size_t)o.shape[1] * o.shape[2] == (size_t)H * mi,
                   "%s: not the model's [%d] experts of [%d][%d]", o.name.c_str(), E, H, mi);
        for (int e = 0; e < E; e++) {
            if (!L.e_edit[e]) continue;
            float *blk = v + (size_t)e * H * mi;
            const int r = L.e_rank;
            const float *a = L.e_a.as<float>() + (size_t)e * r * mi, *b = L.e_b.as<float>() + (size_t)e * H * r;
            if (o.fused_t) k_merge_cols<<<export_blocks((long long)H * mi), kExportThreads, 0, dev->stream>>>(blk, mi, H, a, b, r);
            else k_merge_rows<<<export_blocks((long long)H * mi), kExportThreads, 0, dev->stream>>>(blk, H, mi, a, b, r);
            DITCH_LAUNCH(dev, cudaGetLastError());
        }
        break;
    }
    case OutTensor::None:
        break;
    }
    return DITCH_CUDA_OK;
}

// The bytes of tensor o as written, into w.host.
int produce(Work &w, const Built &b, const OutTensor &o) {
    ditch_cuda_device *dev = w.m->dev;
    cudaStream_t st = dev->stream;
    const long long n = (long long)o.rows * o.cols;
    DITCH_CUDA(w.host_reserve(o.bytes));
    const void *result = nullptr;  // device bytes of the output
    bool have_f32 = false;
    if (o.kind == OutTensor::Fp8 || o.kind == OutTensor::Packed) {
        int s;
        if ((s = upload(w, w.raw, *o.src))) return s;
        DITCH_CUDA(w.bf.reserve((size_t)n * 2));
        uint16_t *bf = w.bf.as<uint16_t>();
        if (o.kind == OutTensor::Fp8) {
            if ((s = upload(w, w.sc, *o.scales))) return s;
            DITCH_LAUNCH(dev, dequant_fp8_bf16(w.raw.as<uint8_t>(), w.sc.as<float>(), (int)o.rows, (int)o.cols, b.br, b.bc,
                                               bf, st));
        } else {
            CK_REQUIRE(b.int_bits > 0 && b.int_group > 0, "%s: packed weight without a compressed-tensors config",
                       o.name.c_str());
            const int groups = (int)((o.cols + b.int_group - 1) / b.int_group);
            DITCH_CUDA(w.sc.reserve((size_t)o.rows * groups * 4));
            if (o.scales->dtype == "BF16") {
                DevBuf s16;
                DITCH_CUDA(s16.reserve(o.scales->bytes));
                DITCH_CUDA(cudaMemcpyAsync(s16.ptr, o.scales->data, o.scales->bytes, cudaMemcpyHostToDevice, st));
                DITCH_LAUNCH(dev, bf16_to_f32(s16.as<uint16_t>(), w.sc.as<float>(), (long long)o.rows * groups, st));
                DITCH_CUDA(cudaStreamSynchronize(st));
            } else {
                CK_REQUIRE(o.scales->dtype == "F32", "%s: weight_scale dtype %s", o.name.c_str(), o.scales->dtype.c_str());
                DITCH_CUDA(cudaMemcpyAsync(w.sc.ptr, o.scales->data, o.scales->bytes, cudaMemcpyHostToDevice, st));
            }
            if (o.zeros && (s = upload(w, w.zr, *o.zeros))) return s;
            const long long wpr = ((long long)o.cols * b.int_bits + 31) / 32;
            DITCH_LAUNCH(dev, dequant_int_bf16(w.raw.as<uint32_t>(), wpr, w.sc.as<float>(),
                                               o.zeros ? w.zr.as<uint32_t>() : nullptr, nullptr, groups, (int)o.rows,
                                               (int)o.cols, b.int_bits, b.int_group, bf, st));
        }
        if (o.edit == OutTensor::None && o.dtype == "BF16") {
            result = bf;
        } else {
            DITCH_CUDA(w.f.reserve((size_t)n * 4));
            DITCH_LAUNCH(dev, bf16_to_f32(bf, w.f.as<float>(), n, st));
            have_f32 = true;
        }
    } else {  // Float: bf16 / f16 / f32 values
        int s;
        if ((s = upload(w, w.raw, *o.src))) return s;
        DITCH_CUDA(w.f.reserve((size_t)n * 4));
        if (o.src->dtype == "BF16") DITCH_LAUNCH(dev, bf16_to_f32(w.raw.as<uint16_t>(), w.f.as<float>(), n, st));
        else if (o.src->dtype == "F16") DITCH_LAUNCH(dev, f16_to_f32(w.raw.as<uint16_t>(), w.f.as<float>(), n, st));
        else DITCH_CUDA(cudaMemcpyAsync(w.f.ptr, w.raw.ptr, (size_t)n * 4, cudaMemcpyDeviceToDevice, st));
        have_f32 = true;
    }
    if (have_f32) {
        int s;
        if (o.edit != OutTensor::None && (s = merge(w, o))) return s;
        if (o.dtype == "F32") {
            result = w.f.ptr;
        } else {
            DITCH_CUDA(w.out.reserve((size_t)n * 2));
            if (o.dtype == "BF16")
                k_f32_to_bf16_out<<<export_blocks(n), kExportThreads, 0, st>>>(w.f.as<float>(), w.out.as<uint16_t>(), n);
            else
                k_f32_to_f16_out<<<export_blocks(n), kExportThreads, 0, st>>>(w.f.as<float>(), w.out.as<uint16_t>(), n);
            DITCH_LAUNCH(dev, cudaGetLastError());
            result = w.out.ptr;
        }
    }
    DITCH_CUDA(cudaMemcpyAsync(w.host, result, o.bytes, cudaMemcpyDeviceToHost, st));
    DITCH_CUDA(cudaStreamSynchronize(st));
    return DITCH_CUDA_OK;
}

}  // namespace
}  // namespace ditch

namespace ditch {
namespace {

using namespace ckpt;

std::string json_string(const std::string &s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        if (c == '"' || c == '\\') o += '\\', o += (char)c;
        else if (c < 0x20) {
            char buf[8];
            snprintf(buf, sizeof buf, "\\u%04x", c);
            o += buf;
        } else o += (char)c;
    }
    return o + "\"";
}

bool write_all(FILE *f, const void *p, size_t n) { return n == 0 || fwrite(p, 1, n, f) == n; }

int write_text(const std::string &path, const std::string &text) {
    FILE *f = fopen(path.c_str(), "wb");
    CK_REQUIRE(f, "cannot create %s", path.c_str());
    const bool ok = write_all(f, text.data(), text.size());
    CK_REQUIRE(fclose(f) == 0 && ok, "cannot write %s", path.c_str());
    return DITCH_CUDA_OK;
}

int copy_file(const std::string &from, const std::string &to) {
    std::string text;
    if (!read_text(from, text)) return DITCH_CUDA_OK;  // absent: nothing to copy
    return write_text(to, text);
}

// One shard: the header (metadata first, 8-byte aligned with spaces), then
// every tensor's bytes in order (src/export.zig:133-168).
int write_shard(Work &w, const Built &b, const std::string &path, const std::vector<const OutTensor *> &ts) {
    std::string h = "{\"__metadata__\":{\"format\":\"pt\",\"producer\":\"ditch\"}";
    size_t off = 0;
    for (const OutTensor *o : ts) {
        h += "," + json_string(o->name) + ":{\"dtype\":\"" + o->dtype + "\",\"shape\":[";
        for (size_t i = 0; i < o->shape.size(); i++) h += (i ? "," : "") + std::to_string(o->shape[i]);
        h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + o->bytes) + "]}";
        off += o->bytes;
    }
    h += "}";
    while (h.size() % 8) h += ' ';
    FILE *f = fopen(path.c_str(), "wb");
    CK_REQUIRE(f, "cannot create %s", path.c_str());
    const uint64_t hn = h.size();
    bool ok = write_all(f, &hn, 8) && write_all(f, h.data(), h.size());
    for (const OutTensor *o : ts) {
        if (!ok) break;
        if (o->kind == OutTensor::Copy) {
            ok = write_all(f, o->src->data, o->bytes);
            continue;
        }
        const int s = produce(w, b, *o);
        if (s) {
            fclose(f);
            return s;
        }
        ok = write_all(f, w.host, o->bytes);
    }
    CK_REQUIRE(fclose(f) == 0 && ok, "cannot write %s", path.c_str());
    return DITCH_CUDA_OK;
}

int export_checkpoint(ditch_cuda_model *m, const char *src, const char *out_dir, int dtype, uint64_t max_shard) {
    CK_REQUIRE(m && src && out_dir, "null argument");
    CK_REQUIRE(dtype < 0 || dtype_config_name(dtype), "export dtype %d is not f32, f16 or bf16", dtype);
    if (m->cfg.tp_world > 1 || m->cfg.ep_world > 1) {
        set_error("a tensor- or expert-parallel model holds part of the weights: export from a single-device model");
        return DITCH_CUDA_UNSUPPORTED;
    }
    struct stat st;
    CK_REQUIRE(stat(src, &st) == 0, "%s does not exist", src);
    if (!S_ISDIR(st.st_mode)) {
        set_error("%s: only Hugging Face directories are exported by the device path (not GGUF)", src);
        return DITCH_CUDA_UNSUPPORTED;
    }
    Checkpoint ck;
    Built b;
    int s;
    if ((s = read_hf_dir(src, ck)) || (s = build_config(ck, b))) return s;
    const Config &c = m->cfg;
    CK_REQUIRE(b.cfg.n_layers == c.n_layers && b.cfg.hidden == c.hidden && b.cfg.vocab == c.vocab &&
                   b.cfg.n_experts == c.n_experts,
               "%s does not hold the model's checkpoint (layers %d / %d, hidden %d / %d, vocab %d / %d)", src,
               b.cfg.n_layers, c.n_layers, b.cfg.hidden, c.hidden, b.cfg.vocab, c.vocab);
    std::vector<OutTensor> plan;
    bool decoded = false;
    if ((s = plan_export(m, ck, dtype, plan, decoded))) return s;

    const std::string dir = out_dir;
    mkdir(dir.c_str(), 0755);
    CK_REQUIRE(stat(dir.c_str(), &st) == 0 && S_ISDIR(st.st_mode), "cannot create %s", out_dir);
    const std::string marker = dir + "/.incomplete";
    if ((s = write_text(marker, "export in progress\n"))) return s;

    // shards: a new one when the next tensor would pass max_shard (src/export.zig:387-397)
    const uint64_t limit = max_shard ? max_shard : (5ull << 30);
    std::vector<std::vector<const OutTensor *>> shards(1);
    uint64_t acc = 0, total = 0;
    for (const OutTensor &o : plan) {
        if (!shards.back().empty() && acc + o.bytes > limit) shards.emplace_back(), acc = 0;
        shards.back().push_back(&o);
        acc += o.bytes;
        total += o.bytes;
    }
    Work w{m};
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    if (shards.size() == 1) {
        if ((s = write_shard(w, b, dir + "/model.safetensors", shards[0]))) return s;
    } else {
        std::string index = "{\n  \"metadata\": {\n    \"total_size\": " + std::to_string(total) + "\n  },\n  \"weight_map\": {\n";
        bool first = true;
        for (size_t i = 0; i < shards.size(); i++) {
            char name[64];
            snprintf(name, sizeof name, "model-%05zu-of-%05zu.safetensors", i + 1, shards.size());
            if ((s = write_shard(w, b, dir + "/" + name, shards[i]))) return s;
            for (const OutTensor *o : shards[i]) {
                index += (first ? "    " : ",\n    ") + json_string(o->name) + ": \"" + name + "\"";
                first = false;
            }
        }
        index += "\n  }\n}\n";
        if ((s = write_text(dir + "/model.safetensors.index.json", index))) return s;
    }

    // config.json: without quantization_config when groups were decoded,
    // naming the export dtype when one was asked for
    std::string config;
    CK_REQUIRE(read_text(std::string(src) + "/config.json", config), "%s: no config.json", src);
    if (decoded) config = strip_quantization(config);
    if (dtype >= 0) config = with_config_dtype(config, dtype_config_name(dtype));
    if ((s = write_text(dir + "/config.json", config))) return s;
    // tokenizer and side files (src/export.zig:170-200, 428-436)
    for (const char *f : {"tokenizer.json", "tokenizer_config.json", "generation_config.json", "special_tokens_map.json",
                          "chat_template.jinja", "chat_template.json", "added_tokens.json", "preprocessor_config.json"})
        if ((s = copy_file(std::string(src) + "/" + f, dir + "/" + f))) return s;
    if (access((std::string(src) + "/tokenizer.json").c_str(), F_OK) != 0)  // a tiktoken vocabulary
        for (const char *f : {"tiktoken.model", "tokenizer.model"})
            if ((s = copy_file(std::string(src) + "/" + f, dir + "/" + f))) return s;
    if (DIR *d = opendir(src)) {
        while (dirent *e = readdir(d)) {
            const std::string n = e->d_name;
            if (ends_with(n, ".py") && (s = copy_file(std::string(src) + "/" + n, dir + "/" + n))) {
                closedir(d);
                return s;
            }
        }
        closedir(d);
    }
    CK_REQUIRE(unlink(marker.c_str()) == 0, "cannot remove %s", marker.c_str());
    return DITCH_CUDA_OK;
}

}  // namespace
}  // namespace ditch

using namespace ditch;

extern "C" {

int ditch_cuda_export_checkpoint(ditch_cuda_model *m, const char *src_dir, const char *out_dir, int dtype,
                                 uint64_t max_shard_bytes) {
    clear_error();
    return export_checkpoint(m, src_dir, out_dir, dtype, max_shard_bytes);
}

int ditch_cuda_export_config(const char *json, size_t len, int dtype, int strip_quantization_config, char *out,
                             size_t cap, size_t *out_len) {
    clear_error();
    CK_REQUIRE(json && out_len, "null argument");
    CK_REQUIRE(dtype < 0 || dtype_config_name(dtype), "export dtype %d is not f32, f16 or bf16", dtype);
    std::string t(json, len);
    if (strip_quantization_config) t = strip_quantization(t);
    if (dtype >= 0) t = with_config_dtype(t, dtype_config_name(dtype));
    *out_len = t.size();
    if (out && cap) {
        const size_t n = std::min(cap, t.size());
        memcpy(out, t.data(), n);
    }
    return DITCH_CUDA_OK;
}

int ditch_cuda_model_delta(ditch_cuda_model *m, size_t layer, int which, size_t expert, float *a, float *b,
                           size_t max_rank, size_t *rank) {
    clear_error();
    CK_REQUIRE(m && rank, "null argument");
    CK_REQUIRE(layer < m->layers.size(), "layer %zu out of range", layer);
    const Layer &L = m->layers[layer];
    const Config &c = m->cfg;
    const float *da = nullptr, *db = nullptr;
    size_t r = 0, cols = 0, rows = (size_t)c.hidden;
    if (which == 0 && L.o_edit) da = L.o_a.as<float>(), db = L.o_b.as<float>(), r = L.o_rank, cols = (size_t)c.heads * c.head_dim;
    else if (which == 1 && !L.moe && L.down_edit) da = L.down_a.as<float>(), db = L.down_b.as<float>(), r = L.down_rank, cols = c.inter;
    else if (which == 2) {
        CK_REQUIRE(L.moe && expert < L.e_edit.size(), "layer %zu has no routed expert %zu", layer, expert);
        if (L.e_edit[expert]) {
            r = (size_t)L.e_rank, cols = c.moe_inter;
            da = L.e_a.as<float>() + expert * r * c.moe_inter, db = L.e_b.as<float>() + expert * c.hidden * r;
        }
    } else CK_REQUIRE(which >= 0 && which <= 2, "component %d: 0 attention output, 1 MLP down, 2 expert down", which);
    *rank = r;
    if (!r) return DITCH_CUDA_OK;
    CK_REQUIRE(r <= max_rank && a && b, "the delta has rank %zu", r);
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    DITCH_CUDA(cudaMemcpyAsync(a, da, r * cols * 4, cudaMemcpyDeviceToHost, m->dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(b, db, rows * r * 4, cudaMemcpyDeviceToHost, m->dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(m->dev->stream));
    return DITCH_CUDA_OK;
}

int ditch_cuda_round_f32(ditch_cuda_device *dev, const float *src, size_t n, int dtype, uint16_t *dst) {
    clear_error();
    CK_REQUIRE(dev && (src && dst || !n), "null argument");
    CK_REQUIRE(dtype == DITCH_DTYPE_BF16 || dtype == DITCH_DTYPE_F16, "dtype %d is not bf16 or f16", dtype);
    if (!n) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DevBuf s, d;
    DITCH_CUDA(s.reserve(n * 4));
    DITCH_CUDA(d.reserve(n * 2));
    DITCH_CUDA(cudaMemcpyAsync(s.ptr, src, n * 4, cudaMemcpyHostToDevice, dev->stream));
    if (dtype == DITCH_DTYPE_BF16)
        k_f32_to_bf16_out<<<export_blocks((long long)n), kExportThreads, 0, dev->stream>>>(s.as<float>(), d.as<uint16_t>(), (long long)n);
    else
        k_f32_to_f16_out<<<export_blocks((long long)n), kExportThreads, 0, dev->stream>>>(s.as<float>(), d.as<uint16_t>(), (long long)n);
    DITCH_LAUNCH(dev, cudaGetLastError());
    DITCH_CUDA(cudaMemcpyAsync(dst, d.ptr, n * 2, cudaMemcpyDeviceToHost, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    return DITCH_CUDA_OK;
}

}  // extern "C"
