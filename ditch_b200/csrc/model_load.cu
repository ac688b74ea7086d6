// Resident-model loading: canonical tensors -> GEMM-ready storage in HBM.
// Quantised groups stay quantised where the GEMM decodes the format inside
// its operand load (FP8 blocks, MXFP4, INT4 groups of 64k); other formats are
// decoded once at load to bf16 (the reference's mapped-mode materialisation,
// src/dequant.zig:449-456).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>

#include "model.cuh"

using namespace ditch;

namespace {

#define REQUIRE(cond, ...)             \
    do {                               \
        if (!(cond)) {                 \
            set_error(__VA_ARGS__);    \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)

struct Seg {
    const ditch_cuda_tensor *t;
    int slab;
};

size_t slab_bytes(size_t total, size_t slabs) { return slabs ? total / slabs : total; }

cudaMemcpyKind kind_of(const ditch_cuda_tensor *t) {
    return t->on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
}

// Copies `bytes` of segment data (at byte offset `off` of the tensor's slab).
cudaError_t copy_in(ditch_cuda_model *m, void *dst, const void *src_base, size_t off, size_t bytes,
                    const ditch_cuda_tensor *t) {
    if (!bytes) return cudaSuccess;
    return cudaMemcpyAsync(dst, static_cast<const uint8_t *>(src_base) + off, bytes, kind_of(t), m->dev->stream);
}

// Decodes one segment to bf16 rows at `dst` (rows x cols), through a device
// staging copy of its raw bytes.
int decode_seg_bf16(ditch_cuda_model *m, const Seg &s, uint16_t *dst) {
    const ditch_cuda_tensor *t = s.t;
    ditch_cuda_device *dev = m->dev;
    const size_t rows = t->rows, cols = t->cols, n = rows * cols;
    const size_t db = slab_bytes(t->data_bytes, t->slabs), sb = slab_bytes(t->scales_bytes, t->slabs);
    const size_t zb = slab_bytes(t->zeros_bytes, t->slabs);
    DevBuf raw, sc, zr, f32buf;
    DITCH_CUDA(raw.reserve(db));
    DITCH_CUDA(copy_in(m, raw.ptr, t->data, db * s.slab, db, t));
    switch (t->format) {
    case DITCH_FMT_BF16:
        DITCH_CUDA(cudaMemcpyAsync(dst, raw.ptr, n * 2, cudaMemcpyDeviceToDevice, dev->stream));
        break;
    case DITCH_FMT_F32:
        DITCH_LAUNCH(dev, f32_to_bf16(raw.as<float>(), dst, (long long)n, dev->stream));
        break;
    case DITCH_FMT_F16:
        DITCH_CUDA(f32buf.reserve(n * 4));
        DITCH_LAUNCH(dev, f16_to_f32(raw.as<uint16_t>(), f32buf.as<float>(), (long long)n, dev->stream));
        DITCH_LAUNCH(dev, f32_to_bf16(f32buf.as<float>(), dst, (long long)n, dev->stream));
        break;
    case DITCH_FMT_FP8_BLOCK: {
        REQUIRE(t->block_rows > 0 && t->block_cols > 0, "%s: FP8 block shape missing", t->name);
        REQUIRE(t->scales_dtype == DITCH_SCALE_F32, "%s: FP8 scales must be f32", t->name);
        DITCH_CUDA(sc.reserve(sb));
        DITCH_CUDA(copy_in(m, sc.ptr, t->scales, sb * s.slab, sb, t));
        DITCH_LAUNCH(dev, dequant_fp8_bf16(raw.as<uint8_t>(), sc.as<float>(), (int)rows, (int)cols, t->block_rows,
                                           t->block_cols, dst, dev->stream));
        break;
    }
    case DITCH_FMT_INT_PACKED: {
        REQUIRE(t->bits >= 1 && t->bits <= 8 && t->block_cols > 0, "%s: INT bits / group missing", t->name);
        const int groups = (int)((cols + t->block_cols - 1) / t->block_cols);
        DITCH_CUDA(sc.reserve(rows * groups * 4));
        if (t->scales_dtype == DITCH_SCALE_BF16) {
            DevBuf s16;
            DITCH_CUDA(s16.reserve(sb));
            DITCH_CUDA(copy_in(m, s16.ptr, t->scales, sb * s.slab, sb, t));
            DITCH_LAUNCH(dev, bf16_to_f32(s16.as<uint16_t>(), sc.as<float>(), (long long)rows * groups, dev->stream));
            DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        } else {
            DITCH_CUDA(copy_in(m, sc.ptr, t->scales, sb * s.slab, sb, t));
        }
        if (t->zeros) {
            DITCH_CUDA(zr.reserve(zb));
            DITCH_CUDA(copy_in(m, zr.ptr, t->zeros, zb * s.slab, zb, t));
        }
        const long long wpr = (long long)(cols * t->bits + 31) / 32;
        DITCH_LAUNCH(dev, dequant_int_bf16(raw.as<uint32_t>(), wpr, sc.as<float>(), t->zeros ? zr.as<uint32_t>() : nullptr,
                                           nullptr, groups, (int)rows, (int)cols, t->bits, t->block_cols, dst,
                                           dev->stream));
        break;
    }
    case DITCH_FMT_MXFP4:
        DITCH_CUDA(sc.reserve(sb));
        DITCH_CUDA(copy_in(m, sc.ptr, t->scales, sb * s.slab, sb, t));
        DITCH_LAUNCH(dev, dequant_mxfp4_bf16(raw.as<uint8_t>(), sc.as<uint8_t>(), (int)rows, (int)cols, dst,
                                             dev->stream));
        break;
    case DITCH_FMT_Q8_0:
        DITCH_LAUNCH(dev, dequant_ggml_bf16(DITCH_DTYPE_Q8_0, raw.as<uint8_t>(), (long long)n, dst, dev->stream));
        break;
    case DITCH_FMT_Q4_K:
        DITCH_LAUNCH(dev, dequant_ggml_bf16(DITCH_DTYPE_Q4_K, raw.as<uint8_t>(), (long long)n, dst, dev->stream));
        break;
    default:
        set_error("%s: unknown format %d", t->name, t->format);
        return DITCH_CUDA_INVALID;
    }
    // The staging buffers are freed on return: finish their readers first.
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    return DITCH_CUDA_OK;
}

// Decodes one segment to f32 rows at `dst` (rows x cols): f32 / f16 / bf16
// values as stored, ggml blocks to f32 as src/quant.zig decodes them, the
// other quantised formats to their bf16 values (src/dequant.zig's output).
int decode_seg_f32(ditch_cuda_model *m, const Seg &s, float *dst) {
    const ditch_cuda_tensor *t = s.t;
    ditch_cuda_device *dev = m->dev;
    const size_t n = t->rows * t->cols;
    const size_t db = slab_bytes(t->data_bytes, t->slabs);
    switch (t->format) {
    case DITCH_FMT_F32:
        DITCH_CUDA(copy_in(m, dst, t->data, db * s.slab, n * 4, t));
        return DITCH_CUDA_OK;
    case DITCH_FMT_F16:
    case DITCH_FMT_Q8_0:
    case DITCH_FMT_Q4_K: {
        DevBuf raw;
        DITCH_CUDA(raw.reserve(db));
        DITCH_CUDA(copy_in(m, raw.ptr, t->data, db * s.slab, db, t));
        if (t->format == DITCH_FMT_F16)
            DITCH_LAUNCH(dev, f16_to_f32(raw.as<uint16_t>(), dst, (long long)n, dev->stream));
        else
            DITCH_LAUNCH(dev, dequant_ggml_f32(t->format == DITCH_FMT_Q8_0 ? DITCH_DTYPE_Q8_0 : DITCH_DTYPE_Q4_K,
                                               raw.as<uint8_t>(), (long long)n, dst, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));  // raw is freed on return
        return DITCH_CUDA_OK;
    }
    default: {
        DevBuf b16;
        DITCH_CUDA(b16.reserve(n * 2));
        int st = decode_seg_bf16(m, s, b16.as<uint16_t>());
        if (st) return st;
        DITCH_LAUNCH(dev, bf16_to_f32(b16.as<uint16_t>(), dst, (long long)n, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        return DITCH_CUDA_OK;
    }
    }
}

// Whether the segments can stay in a GEMM-decoded quantised format.
int native_format(const std::vector<Seg> &segs) {
    const ditch_cuda_tensor *t0 = segs[0].t;
    for (const Seg &s : segs)
        if (s.t->format != t0->format || s.t->cols != t0->cols) return -1;
    const size_t cols = t0->cols;
    switch (t0->format) {
    case DITCH_FMT_FP8_BLOCK: {
        if (cols % 16 || t0->block_cols % 8 || t0->scales_dtype != DITCH_SCALE_F32) return -1;
        for (size_t i = 0; i < segs.size(); i++) {
            const ditch_cuda_tensor *t = segs[i].t;
            if (t->block_rows != t0->block_rows || t->block_cols != t0->block_cols) return -1;
            if (i + 1 < segs.size() && t->rows % t->block_rows) return -1;
        }
        return kFmtFp8;
    }
    case DITCH_FMT_MXFP4:
        return cols % 32 ? -1 : kFmtMxfp4;
    case DITCH_FMT_Q8_0:  // repacked for the GEMM; single matrices (expert stacks decode to bf16)
        for (const Seg &s : segs)
            if (std::max<size_t>(s.t->slabs, 1) > 1) return -1;
        return cols % 32 ? -1 : kFmtQ8_0;
    case DITCH_FMT_Q4_K:  // likewise, in 256-element super-blocks
        for (const Seg &s : segs)
            if (std::max<size_t>(s.t->slabs, 1) > 1) return -1;
        return cols % 256 ? -1 : kFmtQ4K;
    case DITCH_FMT_INT_PACKED: {
        if (t0->bits != 4 || t0->block_cols % 64 || cols % 32 || !t0->zeros) return -1;
        for (size_t i = 0; i < segs.size(); i++) {
            const ditch_cuda_tensor *t = segs[i].t;
            if (t->bits != 4 || t->block_cols != t0->block_cols || !t->zeros) return -1;
            if (i + 1 < segs.size() && t->rows % 8) return -1;
        }
        return kFmtInt4;
    }
    }
    return -1;
}

// Builds one GEMM operand from row segments concatenated in order.
int build_mat(ditch_cuda_model *m, const std::vector<Seg> &segs, int slabs, Mat &out, const char *what) {
    ditch_cuda_device *dev = m->dev;
    size_t rows = 0;
    const size_t cols = segs[0].t->cols;
    for (const Seg &s : segs) {
        REQUIRE(s.t->cols == cols, "%s: concatenated tensors differ in width", what);
        REQUIRE(s.slab < (int)std::max<size_t>(s.t->slabs, 1), "%s: slab out of range", what);
        rows += s.t->rows;
    }
    REQUIRE(rows % slabs == 0, "%s: rows do not split into slabs", what);
    out.rows = (int)(rows / slabs);
    out.cols = (int)cols;
    out.slabs = slabs;
    // split mode decodes every format once (the split operand is bf16)
    const int fmt = m->split3 ? -1 : native_format(segs);
    if (fmt == kFmtFp8) {
        const ditch_cuda_tensor *t0 = segs[0].t;
        out.fmt = kFmtFp8;
        out.br = t0->block_rows;
        out.bc = t0->block_cols;
        out.scols = (int)((cols + out.bc - 1) / out.bc);
        out.row_bytes = (long long)cols;
        size_t srows = 0;
        for (const Seg &s : segs) srows += (s.t->rows + out.br - 1) / out.br;
        DITCH_CUDA(out.data.reserve(rows * cols));
        DITCH_CUDA(out.scales.reserve(srows * out.scols * 4));
        size_t r = 0, sr = 0;
        for (const Seg &s : segs) {
            const size_t db = slab_bytes(s.t->data_bytes, s.t->slabs), sb = slab_bytes(s.t->scales_bytes, s.t->slabs);
            REQUIRE(db >= s.t->rows * cols, "%s: FP8 data too short", what);
            DITCH_CUDA(copy_in(m, out.data.as<uint8_t>() + r * cols, s.t->data, db * s.slab, s.t->rows * cols, s.t));
            const size_t ns = (s.t->rows + out.br - 1) / out.br * out.scols;
            REQUIRE(sb >= ns * 4, "%s: FP8 scales too short", what);
            DITCH_CUDA(copy_in(m, out.scales.as<float>() + sr * out.scols, s.t->scales, sb * s.slab, ns * 4, s.t));
            r += s.t->rows;
            sr += (s.t->rows + out.br - 1) / out.br;
        }
    } else if (fmt == kFmtQ8_0) {
        out.fmt = kFmtQ8_0;
        out.row_bytes = (long long)cols;
        out.scols = (int)(cols / 32);
        DITCH_CUDA(out.data.reserve(rows * cols));
        DITCH_CUDA(out.scales.reserve(rows * (cols / 32) * 4));
        size_t r = 0;
        for (const Seg &s : segs) {
            const size_t bytes = s.t->rows * (cols / 32) * 34;
            REQUIRE(s.t->data_bytes >= bytes, "%s: Q8_0 data too short", what);
            DevBuf raw;
            DITCH_CUDA(raw.reserve(bytes));
            DITCH_CUDA(copy_in(m, raw.ptr, s.t->data, 0, bytes, s.t));
            DITCH_LAUNCH(dev, repack_q8_0(raw.as<uint8_t>(), (long long)s.t->rows * (cols / 32),
                                          out.data.as<int8_t>() + r * cols, out.scales.as<float>() + r * (cols / 32),
                                          dev->stream));
            DITCH_CUDA(cudaStreamSynchronize(dev->stream));
            r += s.t->rows;
        }
    } else if (fmt == kFmtQ4K) {
        out.fmt = kFmtQ4K;
        out.row_bytes = (long long)cols / 2;
        out.scols = (int)(cols / 32);
        DITCH_CUDA(out.data.reserve(rows * cols / 2));
        DITCH_CUDA(out.scales.reserve(rows * (cols / 32) * 8));  // (d1, m1) pairs
        size_t r = 0;
        for (const Seg &s : segs) {
            const size_t bytes = s.t->rows * (cols / 256) * 144;
            REQUIRE(s.t->data_bytes >= bytes, "%s: Q4_K data too short", what);
            DevBuf raw;
            DITCH_CUDA(raw.reserve(bytes));
            DITCH_CUDA(copy_in(m, raw.ptr, s.t->data, 0, bytes, s.t));
            DITCH_LAUNCH(dev, repack_q4_k(raw.as<uint8_t>(), (long long)s.t->rows * (cols / 256),
                                          out.data.as<uint8_t>() + r * cols / 2, out.scales.as<float>() + r * (cols / 32) * 2,
                                          dev->stream));
            DITCH_CUDA(cudaStreamSynchronize(dev->stream));
            r += s.t->rows;
        }
    } else if (fmt == kFmtMxfp4) {
        out.fmt = kFmtMxfp4;
        out.row_bytes = (long long)cols / 2;
        DITCH_CUDA(out.data.reserve(rows * cols / 2));
        DITCH_CUDA(out.scales.reserve(rows * cols / 32));
        size_t r = 0;
        for (const Seg &s : segs) {
            const size_t db = slab_bytes(s.t->data_bytes, s.t->slabs), sb = slab_bytes(s.t->scales_bytes, s.t->slabs);
            REQUIRE(db >= s.t->rows * cols / 2 && sb >= s.t->rows * cols / 32, "%s: MXFP4 data too short", what);
            DITCH_CUDA(copy_in(m, out.data.as<uint8_t>() + r * cols / 2, s.t->data, db * s.slab, s.t->rows * cols / 2, s.t));
            DITCH_CUDA(copy_in(m, out.scales.as<uint8_t>() + r * cols / 32, s.t->scales, sb * s.slab, s.t->rows * cols / 32,
                               s.t));
            r += s.t->rows;
        }
    } else if (fmt == kFmtInt4) {
        const ditch_cuda_tensor *t0 = segs[0].t;
        out.fmt = kFmtInt4;
        out.group = t0->block_cols;
        out.groups = (int)((cols + out.group - 1) / out.group);
        out.row_bytes = (long long)cols / 2;
        DITCH_CUDA(out.data.reserve(rows * cols / 2));
        DITCH_CUDA(out.scales.reserve(rows * out.groups * 4));
        DITCH_CUDA(out.zeros.reserve(((rows + 7) / 8) * out.groups * 4));
        size_t r = 0;
        for (const Seg &s : segs) {
            const ditch_cuda_tensor *t = s.t;
            const size_t db = slab_bytes(t->data_bytes, t->slabs), sb = slab_bytes(t->scales_bytes, t->slabs);
            const size_t zb = slab_bytes(t->zeros_bytes, t->slabs);
            const size_t nsc = t->rows * out.groups, nz = (t->rows + 7) / 8 * out.groups;
            REQUIRE(db >= t->rows * cols / 2 && zb >= nz * 4, "%s: INT4 data too short", what);
            DITCH_CUDA(copy_in(m, out.data.as<uint8_t>() + r * cols / 2, t->data, db * s.slab, t->rows * cols / 2, t));
            if (t->scales_dtype == DITCH_SCALE_BF16) {
                DevBuf s16;
                DITCH_CUDA(s16.reserve(nsc * 2));
                DITCH_CUDA(copy_in(m, s16.ptr, t->scales, sb * s.slab, nsc * 2, t));
                DITCH_LAUNCH(dev, bf16_to_f32(s16.as<uint16_t>(), out.scales.as<float>() + r * out.groups, (long long)nsc,
                                              dev->stream));
                DITCH_CUDA(cudaStreamSynchronize(dev->stream));
            } else {
                DITCH_CUDA(copy_in(m, out.scales.as<float>() + r * out.groups, t->scales, sb * s.slab, nsc * 4, t));
            }
            DITCH_CUDA(copy_in(m, out.zeros.as<uint32_t>() + (r / 8) * out.groups, t->zeros, zb * s.slab, nz * 4, t));
            r += t->rows;
        }
    } else {
        // bf16 rows, zero-padded to a multiple of 8 columns (TMA row strides
        // are multiples of 16 bytes); the padding multiplies zero activations.
        const size_t kp = (cols + 7) / 8 * 8;
        out.fmt = kFmtBf16;
        out.cols = (int)kp;
        out.row_bytes = (long long)kp * 2;
        DITCH_CUDA(out.data.reserve(rows * kp * 2));
        DevBuf tmp;
        if (kp != cols) {
            DITCH_CUDA(cudaMemsetAsync(out.data.ptr, 0, rows * kp * 2, dev->stream));
            size_t mx = 0;
            for (const Seg &s : segs) mx = std::max(mx, s.t->rows);
            DITCH_CUDA(tmp.reserve(mx * cols * 2));
        }
        size_t r = 0;
        for (const Seg &s : segs) {
            if (kp == cols) {
                int st = decode_seg_bf16(m, s, out.data.as<uint16_t>() + r * cols);
                if (st) return st;
            } else {
                int st = decode_seg_bf16(m, s, tmp.as<uint16_t>());
                if (st) return st;
                DITCH_CUDA(cudaMemcpy2DAsync(out.data.as<uint16_t>() + r * kp, kp * 2, tmp.ptr, cols * 2, cols * 2,
                                             s.t->rows, cudaMemcpyDeviceToDevice, dev->stream));
                DITCH_CUDA(cudaStreamSynchronize(dev->stream));
            }
            r += s.t->rows;
        }
        if (m->split3) {
            // the f32-level operand [hi | lo | hi] from the values as ditch holds them
            out.split_k = (int)kp;
            DITCH_CUDA(out.split.reserve(rows * 3 * kp * 2));
            size_t mx = 0;
            for (const Seg &s : segs) mx = std::max(mx, s.t->rows);
            DevBuf f;
            DITCH_CUDA(f.reserve(mx * cols * 4));
            r = 0;
            for (const Seg &s : segs) {
                int st = decode_seg_f32(m, s, f.as<float>());
                if (st) return st;
                DITCH_LAUNCH(dev, split_weight_rows(f.as<float>(), (int)s.t->rows, (int)cols, (int)kp,
                                                    out.split.as<uint16_t>() + r * 3 * kp, dev->stream));
                DITCH_CUDA(cudaStreamSynchronize(dev->stream));  // f is reused
                r += s.t->rows;
            }
        }
    }
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    return DITCH_CUDA_OK;
}

// A 1-D f32 vector (norm weight or bias) of any float format.
int load_vec(ditch_cuda_model *m, const ditch_cuda_tensor *t, size_t n, DevBuf &out, const char *what) {
    REQUIRE(t->rows * t->cols == n || (t->rows == n && t->cols <= 1) || (t->cols == n && t->rows <= 1),
            "%s: expected %zu values", what, n);
    DITCH_CUDA(out.reserve(n * 4));
    ditch_cuda_device *dev = m->dev;
    if (t->format == DITCH_FMT_F32) {
        DITCH_CUDA(copy_in(m, out.ptr, t->data, 0, n * 4, t));
    } else if (t->format == DITCH_FMT_BF16 || t->format == DITCH_FMT_F16) {
        DevBuf raw;
        DITCH_CUDA(raw.reserve(n * 2));
        DITCH_CUDA(copy_in(m, raw.ptr, t->data, 0, n * 2, t));
        if (t->format == DITCH_FMT_BF16) DITCH_LAUNCH(dev, bf16_to_f32(raw.as<uint16_t>(), out.as<float>(), (long long)n, dev->stream));
        else DITCH_LAUNCH(dev, f16_to_f32(raw.as<uint16_t>(), out.as<float>(), (long long)n, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    } else {
        set_error("%s: vectors must be f32, bf16 or f16", what);
        return DITCH_CUDA_UNSUPPORTED;
    }
    return DITCH_CUDA_OK;
}

// The inverse frequencies with the config's scaling and the f64 angle table
// (src/model.zig:2200-2282): llama3's smoothed divisor, linear, YaRN's ramp
// between interpolated and extrapolated frequencies (Hugging Face's
// correction dims, optionally truncated), or per-frequency divisors; cos /
// sin times the attention factor (YaRN, LongRoPE).
int build_rope(ditch_cuda_model *m) {
    const Config &c = m->cfg;
    const int half = c.head_dim / 2;
    const int len = std::max(c.max_seq, 1);
    std::vector<double> inv(half);
    for (int i = 0; i < half; i++) inv[i] = 1.0 / std::pow(c.rope_theta, (double)(2 * i) / (double)c.head_dim);
    double attn = 1.0;
    if (c.rope_scaling == 1) {
        const double low_wl = c.rope_orig_max / c.rope_low_ff, high_wl = c.rope_orig_max / c.rope_high_ff;
        for (int i = 0; i < half; i++) {
            const double wl = 2.0 * M_PI / inv[i];
            if (wl < high_wl) {
            } else if (wl > low_wl) {
                inv[i] /= c.rope_factor;
            } else {
                const double smooth = (c.rope_orig_max / wl - c.rope_low_ff) / (c.rope_high_ff - c.rope_low_ff);
                inv[i] = (1.0 - smooth) * inv[i] / c.rope_factor + smooth * inv[i];
            }
        }
    } else if (c.rope_scaling == 2) {
        for (int i = 0; i < half; i++) inv[i] /= c.rope_factor;
    } else if (c.rope_scaling == 3) {
        const double dim = (double)c.head_dim, base = c.rope_theta;
        auto corr_dim = [&](double rot) {
            return dim * std::log(c.rope_orig_max / (rot * 2.0 * M_PI)) / (2.0 * std::log(base));
        };
        double low = corr_dim(c.rope_beta_fast), high = corr_dim(c.rope_beta_slow);
        if (c.rope_truncate) {
            low = std::floor(low);
            high = std::ceil(high);
        }
        low = std::max(low, 0.0);
        high = std::min(high, dim - 1);
        if (low == high) high += 0.001;
        for (int i = 0; i < half; i++) {
            const double ramp = std::min(1.0, std::max(0.0, ((double)i - low) / (high - low)));
            const double extrap = 1.0 - ramp;
            inv[i] = inv[i] / c.rope_factor * (1.0 - extrap) + inv[i] * extrap;
        }
        attn = c.rope_attention_factor;
    } else if (c.rope_scaling == 4) {
        for (int i = 0; i < half && i < (int)c.rope_factors.size(); i++) inv[i] /= (double)c.rope_factors[i];
        attn = c.rope_attention_factor;
    }
    std::vector<float> cs((size_t)len * half), sn((size_t)len * half);
    for (int p = 0; p < len; p++)
        for (int i = 0; i < half; i++) {
            const double a = (double)p * inv[i];
            cs[(size_t)p * half + i] = (float)(std::cos(a) * attn);
            sn[(size_t)p * half + i] = (float)(std::sin(a) * attn);
        }
    DITCH_CUDA(m->rope_cos.reserve(cs.size() * 4));
    DITCH_CUDA(m->rope_sin.reserve(sn.size() * 4));
    // on the model's stream (non-blocking: the legacy stream would not order
    // these copies before its kernels), done before the host tables go
    DITCH_CUDA(cudaMemcpyAsync(m->rope_cos.ptr, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, m->dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(m->rope_sin.ptr, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, m->dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(m->dev->stream));
    m->rope_len = len;
    return DITCH_CUDA_OK;
}

}  // namespace

extern "C" {

int ditch_cuda_model_load(ditch_cuda_device *dev, const ditch_cuda_model_config *cfg, const ditch_cuda_tensor *tensors,
                          size_t n_tensors, ditch_cuda_model **out) {
    clear_error();
    REQUIRE(dev && cfg && out && (tensors || n_tensors == 0), "null argument");
    *out = nullptr;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    REQUIRE(cfg->n_layers > 0 && cfg->hidden > 0 && cfg->heads > 0 && cfg->kv_heads > 0 && cfg->head_dim > 0 &&
                cfg->vocab > 0,
            "config dimensions must be positive");
    REQUIRE(cfg->heads % cfg->kv_heads == 0, "heads must be a multiple of kv heads");
    REQUIRE(cfg->head_dim % 2 == 0, "head_dim must be even");
    REQUIRE(cfg->hidden % 8 == 0, "hidden must be a multiple of 8");
    // device-resident inputs may still be in flight on their producers' streams
    for (size_t i = 0; i < n_tensors; i++)
        if (tensors[i].on_device) {
            DITCH_CUDA(cudaDeviceSynchronize());
            break;
        }
    REQUIRE((cfg->heads * cfg->head_dim) % 8 == 0, "heads * head_dim must be a multiple of 8");
    std::unique_ptr<ditch_cuda_model> m(new ditch_cuda_model());
    m->dev = dev;
    Config &c = m->cfg;
    c.n_layers = cfg->n_layers;
    c.hidden = cfg->hidden;
    c.heads = cfg->heads;
    c.kv_heads = cfg->kv_heads;
    c.head_dim = cfg->head_dim;
    c.inter = cfg->inter;
    c.vocab = cfg->vocab;
    c.eps = cfg->eps;
    c.rope_theta = cfg->rope_theta;
    c.rope_scaling = cfg->rope_scaling;
    c.rope_factor = cfg->rope_factor;
    c.rope_low_ff = cfg->rope_low_ff;
    c.rope_high_ff = cfg->rope_high_ff;
    c.rope_orig_max = cfg->rope_orig_max;
    REQUIRE(c.rope_scaling >= 0 && c.rope_scaling <= 4, "rope_scaling %d is not 0 to 4", c.rope_scaling);
    REQUIRE(c.rope_scaling != 4 || cfg->n_rope_factors == 0 || cfg->rope_factors,
            "rope_factors is null with n_rope_factors > 0");
    if (c.rope_scaling == 4 && cfg->n_rope_factors)
        c.rope_factors.assign(cfg->rope_factors, cfg->rope_factors + cfg->n_rope_factors);
    c.rope_attention_factor = cfg->rope_attention_factor != 0 ? cfg->rope_attention_factor : 1.0;
    c.rope_beta_fast = cfg->rope_beta_fast;
    c.rope_beta_slow = cfg->rope_beta_slow;
    c.rope_truncate = cfg->rope_truncate;
    REQUIRE(c.rope_scaling != 3 || (c.rope_factor > 0 && c.rope_orig_max > 0 && c.rope_beta_fast > 0 &&
                                    c.rope_beta_slow > 0 && c.rope_theta > 1),
            "yarn rope scaling needs a positive factor, original length and betas");
    c.qk_norm = cfg->qk_norm;
    c.n_experts = cfg->n_experts;
    c.top_k = cfg->top_k;
    c.moe_inter = cfg->moe_inter;
    c.norm_topk = cfg->norm_topk;
    c.max_seq = cfg->max_seq > 0 ? cfg->max_seq : 4096;
    c.ep_world = cfg->ep_world > 1 ? cfg->ep_world : 1;
    c.ep_rank = c.ep_world > 1 ? cfg->ep_rank : 0;
    REQUIRE(c.ep_rank >= 0 && c.ep_rank < c.ep_world, "ep_rank out of range");
    REQUIRE(c.ep_world == 1 || (c.n_experts > 0 && c.n_experts % c.ep_world == 0),
            "expert parallelism needs the experts to split evenly over ep_world");
    c.e_loc = c.ep_world > 1 ? c.n_experts / c.ep_world : c.n_experts;
    c.e0 = c.ep_rank * c.e_loc;
    c.moe_layers.assign(c.n_layers, 0);
    if (cfg->moe_layers)
        for (int i = 0; i < c.n_layers; i++) c.moe_layers[i] = cfg->moe_layers[i] ? 1 : 0;
    c.tp_world = cfg->tp_world > 1 ? cfg->tp_world : 1;
    c.tp_rank = c.tp_world > 1 ? cfg->tp_rank : 0;
    REQUIRE(c.tp_rank >= 0 && c.tp_rank < c.tp_world, "tp_rank out of range");
    m->split3 = dev->f32_split;
    if (m->split3) {
        bool any_moe = false;
        for (uint8_t f : c.moe_layers) any_moe |= f != 0;
        if (any_moe || c.tp_world > 1 || c.ep_world > 1) {
            set_error("f32 split products are for dense models on one GPU (no routed experts, no tensor or expert "
                      "parallelism)");
            return DITCH_CUDA_UNSUPPORTED;
        }
    }
    if (c.tp_world > 1) {
        bool any_moe = false;
        for (uint8_t f : c.moe_layers) any_moe |= f != 0;
        REQUIRE(!any_moe && c.ep_world == 1, "tensor parallelism is for dense models");
        REQUIRE(c.heads % c.tp_world == 0 && c.kv_heads % c.tp_world == 0 && c.inter % (8 * c.tp_world) == 0,
                "tensor parallelism needs heads, kv heads and inter / 8 divisible by tp_world");
    }
    // full (as stored) dimensions; the config keeps this rank's share
    const int W_tp = c.tp_world, r_tp = c.tp_rank;
    const int qd_full = c.qd(), kvd_full = c.kvd(), inter_full = c.inter;
    c.heads /= W_tp;
    c.kv_heads /= W_tp;
    c.inter /= W_tp;

    std::map<std::string, const ditch_cuda_tensor *> byname;
    for (size_t i = 0; i < n_tensors; i++) {
        REQUIRE(tensors[i].name, "tensor %zu has no name", i);
        byname[tensors[i].name] = &tensors[i];
    }
    auto get = [&](const std::string &name) -> const ditch_cuda_tensor * {
        auto it = byname.find(name);
        return it == byname.end() ? nullptr : it->second;
    };
    const int H = c.hidden, qd = c.qd(), kvd = c.kvd();  // this rank's widths
    int st;
    // Tensor-parallel shards: a tensor given whole is sliced (rows: a view;
    // columns: a device copy of the window), one given at the shard's shape is
    // taken as is. Views and copies live until the load returns.
    std::vector<std::unique_ptr<ditch_cuda_tensor>> views;
    std::vector<DevBuf> windows;
    auto esz = [](const ditch_cuda_tensor *t) -> size_t {
        return t->format == DITCH_FMT_F32 ? 4 : (t->format == DITCH_FMT_BF16 || t->format == DITCH_FMT_F16) ? 2 : 0;
    };
    auto shard_rows = [&](const ditch_cuda_tensor *t, size_t full, size_t part) -> const ditch_cuda_tensor * {
        if (!t || W_tp == 1 || t->rows == part) return t;
        if (t->rows != full || !esz(t) || t->slabs > 1) return nullptr;
        const size_t e = esz(t);
        views.emplace_back(new ditch_cuda_tensor(*t));
        ditch_cuda_tensor *v = views.back().get();
        v->data = static_cast<const uint8_t *>(t->data) + (size_t)r_tp * part * t->cols * e;
        v->rows = part;
        v->data_bytes = part * t->cols * e;
        return v;
    };
    auto shard_cols = [&](const ditch_cuda_tensor *t, size_t full, size_t part) -> const ditch_cuda_tensor * {
        if (!t || W_tp == 1 || t->cols == part) return t;
        if (t->cols != full || !esz(t) || t->slabs > 1) return nullptr;
        const size_t e = esz(t);
        windows.emplace_back();
        DevBuf &w = windows.back();
        if (w.reserve(t->rows * part * e) != cudaSuccess) return nullptr;
        if (cudaMemcpy2DAsync(w.ptr, part * e, static_cast<const uint8_t *>(t->data) + (size_t)r_tp * part * e,
                              full * e, part * e, t->rows, kind_of(t), m->dev->stream) != cudaSuccess)
            return nullptr;
        views.emplace_back(new ditch_cuda_tensor(*t));
        ditch_cuda_tensor *v = views.back().get();
        v->data = w.ptr;
        v->cols = part;
        v->data_bytes = t->rows * part * e;
        v->on_device = 1;
        return v;
    };
    // embedding table: bf16 or f32 as stored
    const ditch_cuda_tensor *emb = get("embed");
    REQUIRE(emb && emb->rows == (size_t)c.vocab && emb->cols == (size_t)H, "embed [vocab][hidden] missing");
    if (emb->format == DITCH_FMT_F32 || emb->format == DITCH_FMT_BF16) {
        m->embed_bf16 = emb->format == DITCH_FMT_BF16;
        const size_t bytes = (size_t)c.vocab * H * (m->embed_bf16 ? 2 : 4);
        DITCH_CUDA(m->embed.reserve(bytes));
        DITCH_CUDA(copy_in(m.get(), m->embed.ptr, emb->data, 0, bytes, emb));
    } else {
        m->embed_bf16 = true;
        DITCH_CUDA(m->embed.reserve((size_t)c.vocab * H * 2));
        st = decode_seg_bf16(m.get(), Seg{emb, 0}, m->embed.as<uint16_t>());
        if (st) return st;
    }
    const ditch_cuda_tensor *fn = get("final_norm");
    REQUIRE(fn, "final_norm missing");
    if ((st = load_vec(m.get(), fn, H, m->final_norm, "final_norm"))) return st;
    const ditch_cuda_tensor *lm = get("lm_head");
    REQUIRE(lm && lm->rows == (size_t)c.vocab && lm->cols == (size_t)H, "lm_head [vocab][hidden] missing");
    if ((st = build_mat(m.get(), {Seg{lm, 0}}, 1, m->lm_head, "lm_head"))) return st;

    m->layers.resize(c.n_layers);
    for (int i = 0; i < c.n_layers; i++) {
        Layer &L = m->layers[i];
        char nm[64];
        auto t = [&](const char *f) {
            snprintf(nm, sizeof nm, "L%d.%s", i, f);
            return get(nm);
        };
        const ditch_cuda_tensor *in = t("input_norm"), *post = t("post_norm");
        REQUIRE(in && post, "layer %d: norms missing", i);
        if ((st = load_vec(m.get(), in, H, L.input_norm, "input_norm"))) return st;
        if ((st = load_vec(m.get(), post, H, L.post_norm, "post_norm"))) return st;
        if (c.qk_norm) {
            const ditch_cuda_tensor *qn = t("q_norm"), *kn = t("k_norm");
            REQUIRE(qn && kn, "layer %d: q/k norms missing", i);
            if ((st = load_vec(m.get(), qn, c.head_dim, L.q_norm, "q_norm"))) return st;
            if ((st = load_vec(m.get(), kn, c.head_dim, L.k_norm, "k_norm"))) return st;
        }
        const ditch_cuda_tensor *q = t("q"), *k = t("k"), *v = t("v"), *o = t("o");
        REQUIRE(q && k && v && o, "layer %d: attention projections missing", i);
        if (W_tp > 1) {
            q = shard_rows(q, qd_full, qd);
            k = shard_rows(k, kvd_full, kvd);
            v = shard_rows(v, kvd_full, kvd);
            o = shard_cols(o, qd_full, qd);
            REQUIRE(q && k && v && o, "layer %d: tensor-parallel shards need f32 / f16 / bf16 q, k, v, o", i);
        }
        REQUIRE(q->rows == (size_t)qd && k->rows == (size_t)kvd && v->rows == (size_t)kvd && q->cols == (size_t)H,
                "layer %d: q/k/v shapes", i);
        REQUIRE(o->rows == (size_t)H && o->cols == (size_t)qd, "layer %d: o shape", i);
        if ((st = build_mat(m.get(), {Seg{q, 0}, Seg{k, 0}, Seg{v, 0}}, 1, L.qkv, "qkv"))) return st;
        if ((st = build_mat(m.get(), {Seg{o, 0}}, 1, L.o, "o"))) return st;
        const ditch_cuda_tensor *qb = shard_rows(t("qb"), qd_full, qd), *kb = shard_rows(t("kb"), kvd_full, kvd),
                                *vb = shard_rows(t("vb"), kvd_full, kvd);
        if (qb || kb || vb) {
            std::vector<float> zeros(c.qkv_width(), 0.0f);
            DITCH_CUDA(L.qkv_bias.reserve(c.qkv_width() * 4));
            // every copy on the model's stream: load_vec's upload of an f32
            // vector is asynchronous there, and the legacy stream does not
            // wait for it
            DITCH_CUDA(cudaMemsetAsync(L.qkv_bias.ptr, 0, c.qkv_width() * 4, dev->stream));
            DevBuf tmp;
            const ditch_cuda_tensor *bs[3] = {qb, kb, vb};
            const int off[3] = {0, qd, qd + kvd}, len[3] = {qd, kvd, kvd};
            for (int j = 0; j < 3; j++) {
                if (!bs[j]) continue;
                if ((st = load_vec(m.get(), bs[j], len[j], tmp, "qkv bias"))) return st;
                DITCH_CUDA(cudaMemcpyAsync(L.qkv_bias.as<float>() + off[j], tmp.ptr, len[j] * 4, cudaMemcpyDeviceToDevice,
                                           dev->stream));
                DITCH_CUDA(cudaStreamSynchronize(dev->stream));  // before tmp is reused or freed
            }
        }
        if (c.moe_layers[i]) {
            L.moe = true;
            const int E = c.n_experts, mi = c.moe_inter;
            REQUIRE(E > 0 && c.top_k > 0 && c.top_k <= E && mi > 0, "layer %d: MoE config", i);
            const ditch_cuda_tensor *r = t("router"), *eg = t("e_gate"), *eu = t("e_up"), *ed = t("e_down");
            REQUIRE(r && eg && eu && ed, "layer %d: router / expert stacks missing", i);
            REQUIRE(r->rows == (size_t)E && r->cols == (size_t)H, "layer %d: router shape", i);
            REQUIRE(eg->slabs == (size_t)E && eg->rows == (size_t)mi && eg->cols == (size_t)H, "layer %d: e_gate shape", i);
            REQUIRE(eu->slabs == (size_t)E && eu->rows == (size_t)mi && eu->cols == (size_t)H, "layer %d: e_up shape", i);
            REQUIRE(ed->slabs == (size_t)E && ed->rows == (size_t)H && ed->cols == (size_t)mi, "layer %d: e_down shape", i);
            if ((st = build_mat(m.get(), {Seg{r, 0}}, 1, L.router, "router"))) return st;
            {
                // f32 router weights for the split-precision router product
                DevBuf rf;
                DITCH_CUDA(rf.reserve((size_t)E * H * 4));
                if (r->format == DITCH_FMT_F32) {
                    DITCH_CUDA(copy_in(m.get(), rf.ptr, r->data, 0, (size_t)E * H * 4, r));
                } else {
                    DITCH_LAUNCH(dev, bf16_to_f32(L.router.data.as<uint16_t>(), rf.as<float>(), (long long)E * H,
                                                  dev->stream));
                }
                if ((st = build_router_split(dev, rf.as<float>(), E, H, L.router3))) return st;
            }
            // this rank's experts only (all of them without expert parallelism)
            const int El = c.e_loc;
            std::vector<Seg> gu, dn;
            for (int e = c.e0; e < c.e0 + El; e++) {
                gu.push_back(Seg{eg, e});
                gu.push_back(Seg{eu, e});
                dn.push_back(Seg{ed, e});
            }
            if ((st = build_mat(m.get(), gu, El, L.e_gate_up, "e_gate_up"))) return st;
            if ((st = build_mat(m.get(), dn, El, L.e_down, "e_down"))) return st;
            L.e_edit.assign(El, 0);
            DITCH_CUDA(L.e_a.reserve((size_t)El * L.e_down.cols * 4 * kMaxDeltaRank));
            DITCH_CUDA(L.e_b.reserve((size_t)El * H * 4 * kMaxDeltaRank));
            DITCH_CUDA(L.e_edit_dev.reserve((size_t)El * 4));
            DITCH_CUDA(cudaMemsetAsync(L.e_edit_dev.ptr, 0, (size_t)El * 4, dev->stream));
        } else {
            const ditch_cuda_tensor *g = t("gate"), *u = t("up"), *d = t("down");
            REQUIRE(g && u && d, "layer %d: MLP projections missing", i);
            if (W_tp > 1) {
                g = shard_rows(g, inter_full, c.inter);
                u = shard_rows(u, inter_full, c.inter);
                d = shard_cols(d, inter_full, c.inter);
                REQUIRE(g && u && d, "layer %d: tensor-parallel shards need f32 / f16 / bf16 gate, up, down", i);
            }
            REQUIRE(g->rows == (size_t)c.inter && u->rows == (size_t)c.inter && g->cols == (size_t)H &&
                        d->rows == (size_t)H && d->cols == (size_t)c.inter,
                    "layer %d: MLP shapes", i);
            if ((st = build_mat(m.get(), {Seg{g, 0}, Seg{u, 0}}, 1, L.gate_up, "gate_up"))) return st;
            if ((st = build_mat(m.get(), {Seg{d, 0}}, 1, L.down, "down"))) return st;
            DITCH_CUDA(L.down_a.reserve((size_t)L.down.cols * 4 * kMaxDeltaRank));
            DITCH_CUDA(L.down_b.reserve((size_t)H * 4 * kMaxDeltaRank));
        }
        DITCH_CUDA(L.o_a.reserve((size_t)qd * 4 * kMaxDeltaRank));
        DITCH_CUDA(L.o_b.reserve((size_t)H * 4 * kMaxDeltaRank));
    }
    if ((st = build_rope(m.get()))) return st;
    DITCH_CUDA(m->dirs.reserve((size_t)(c.n_layers + 1) * H * 4));
    DITCH_CUDA(m->vtmp.reserve((size_t)H * 4));
    uint64_t bytes = m->embed.bytes + m->final_norm.bytes + m->lm_head.bytes() + m->lm_head.split.bytes;
    for (const Layer &L : m->layers)
        bytes += L.qkv.bytes() + L.o.bytes() + L.gate_up.bytes() + L.down.bytes() + L.router.bytes() +
                 L.e_gate_up.bytes() + L.e_down.bytes() + L.qkv.split.bytes + L.o.split.bytes +
                 L.gate_up.split.bytes + L.down.split.bytes;
    m->bytes = bytes;
    DITCH_CUDA(cudaDeviceSynchronize());
    *out = m.release();
    return DITCH_CUDA_OK;
}

void ditch_cuda_model_free(ditch_cuda_model *m) {
    if (!m) return;
    std::lock_guard<std::mutex> lk(m->dev->mu);
    cudaSetDevice(m->dev->ordinal);
    cudaStreamSynchronize(m->dev->stream);
    delete m;
}

uint64_t ditch_cuda_model_bytes(const ditch_cuda_model *m) { return m ? m->bytes : 0; }

}  // extern "C"

namespace ditch {

int build_weight(ditch_cuda_device *dev, const ditch_cuda_tensor *t, Mat &out) {
    ditch_cuda_model tmp;  // the loader helpers only need the device
    tmp.dev = dev;
    std::vector<Seg> segs;
    const int slabs = (int)std::max<size_t>(t->slabs, 1);
    for (int s = 0; s < slabs; s++) segs.push_back(Seg{t, s});
    return build_mat(&tmp, segs, slabs, out, t->name ? t->name : "weight");
}

}  // namespace ditch

struct ditch_cuda_weight {
    ditch_cuda_device *dev;
    ditch::Mat mat;
};

extern "C" {

int ditch_cuda_weight_load(ditch_cuda_device *dev, const ditch_cuda_tensor *t, ditch_cuda_weight **out) {
    clear_error();
    REQUIRE(dev && t && out, "null argument");
    *out = nullptr;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    // device-resident input may still be in flight on the producer's stream
    if (t->on_device) DITCH_CUDA(cudaDeviceSynchronize());
    std::unique_ptr<ditch_cuda_weight> w(new ditch_cuda_weight());
    w->dev = dev;
    int st = build_weight(dev, t, w->mat);
    if (st) return st;
    *out = w.release();
    return DITCH_CUDA_OK;
}

void ditch_cuda_weight_free(ditch_cuda_weight *w) {
    if (!w) return;
    std::lock_guard<std::mutex> lk(w->dev->mu);
    cudaSetDevice(w->dev->ordinal);
    cudaStreamSynchronize(w->dev->stream);
    delete w;
}

int ditch_cuda_weight_format(const ditch_cuda_weight *w) { return w ? w->mat.fmt : -1; }

int ditch_cuda_weight_gemm(ditch_cuda_weight *w, const void *x, size_t m, float *out, int k_splits) {
    clear_error();
    REQUIRE(w && x && out, "null argument");
    if (m == 0) return DITCH_CUDA_OK;
    ditch_cuda_device *dev = w->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const Mat &mat = w->mat;
    REQUIRE(mat.slabs == 1, "stacked weights take the grouped path");
    GemmExtra ex;
    ex.k_splits = std::max(k_splits, 1);
    int flags = 0;
    if (ex.k_splits > 1) {
        DITCH_CUDA(cudaMemsetAsync(out, 0, m * (size_t)mat.rows * 4, dev->stream));
        flags = kEpiAtomic;
    }
    return gemm_mat(dev, mat, 0, mat.rows, static_cast<const uint16_t *>(x), (int)m, out, mat.rows, flags, nullptr,
                    nullptr, nullptr, 0, &ex);
}

int ditch_cuda_weight_decode(ditch_cuda_weight *w, uint16_t *out) {
    clear_error();
    REQUIRE(w && out, "null argument");
    ditch_cuda_device *dev = w->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const Mat &mt = w->mat;
    const int rows = mt.rows * mt.slabs;
    switch (mt.fmt) {
    case kFmtBf16:
        DITCH_CUDA(cudaMemcpyAsync(out, mt.data.ptr, (size_t)rows * mt.cols * 2, cudaMemcpyDeviceToDevice, dev->stream));
        break;
    case kFmtFp8:
        DITCH_LAUNCH(dev, dequant_fp8_bf16(mt.data.as<uint8_t>(), mt.scales.as<float>(), rows, mt.cols, mt.br, mt.bc,
                                           out, dev->stream));
        break;
    case kFmtMxfp4:
        DITCH_LAUNCH(dev, dequant_mxfp4_bf16(mt.data.as<uint8_t>(), mt.scales.as<uint8_t>(), rows, mt.cols, out,
                                             dev->stream));
        break;
    case kFmtInt4:
        DITCH_LAUNCH(dev, dequant_int_bf16(mt.data.as<uint32_t>(), mt.cols / 8, mt.scales.as<float>(),
                                           mt.zeros.as<uint32_t>(), nullptr, mt.groups, rows, mt.cols, 4, mt.group, out,
                                           dev->stream));
        break;
    case kFmtQ8_0:    // the GEMM operand itself: bf16(d * q)
    case kFmtQ4K: {   // bf16(d1 * q - m1)
        StageArgs sa{};
        sa.fmt = mt.fmt;
        sa.data = mt.data.as<uint8_t>();
        sa.row_bytes = mt.row_bytes;
        sa.rows = rows;
        sa.cols = mt.cols;
        sa.scales = mt.scales.as<float>();
        sa.scale_cols = mt.scols;
        sa.out = out;
        DITCH_LAUNCH(dev, launch_stage_decode(sa, dev->sms, dev->stream));
        break;
    }
    default:
        set_error("weight format %d cannot be decoded", mt.fmt);
        return DITCH_CUDA_UNSUPPORTED;
    }
    return DITCH_CUDA_OK;
}

}  // extern "C"
