// C ABI: the element-wise seam entries, standalone decoders, the
// materialised rank-1 weight edit and timing support.
#include <algorithm>

#include "device.cuh"

using namespace ditch;

namespace {

#define REQUIRE(cond, msg)             \
    do {                               \
        if (!(cond)) {                 \
            set_error("%s", msg);      \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)

// Uploads `bytes` from host into a device scratch buffer.
cudaError_t up(ditch_cuda_device *dev, DevBuf &buf, const void *src, size_t bytes) {
    cudaError_t e = buf.reserve(bytes);
    if (e != cudaSuccess || bytes == 0) return e;
    return cudaMemcpyAsync(buf.ptr, src, bytes, cudaMemcpyHostToDevice, dev->stream);
}

int finish(ditch_cuda_device *dev, void *dst, const DevBuf &buf, size_t bytes, const char *what) {
    if (bytes) {
        cudaError_t e = cudaMemcpyAsync(dst, buf.ptr, bytes, cudaMemcpyDeviceToHost, dev->stream);
        if (e != cudaSuccess) return cuda_status(e, what);
    }
    return check_status(dev, what);
}

// Extra scratch for entries with more than the handle's five buffers.
struct Scratch3 {
    DevBuf a, b, c;
};

}  // namespace

extern "C" {

int ditch_cuda_attention_scores(ditch_cuda_device *dev, float *scores, size_t n_keys, const float *q, size_t hd,
                                const float *k, size_t k_len, size_t stride, float scale) {
    clear_error();
    REQUIRE(dev && scores && q && k, "null argument");
    if (n_keys == 0) return DITCH_CUDA_OK;
    REQUIRE(k_len >= (n_keys - 1) * stride + hd, "key slice too short");
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, q, hd * 4));
    DITCH_CUDA(up(dev, dev->bw, k, k_len * 4));
    DITCH_CUDA(dev->bo.reserve(n_keys * 4));
    DITCH_LAUNCH(dev, attention_scores_f32(dev->bo.as<float>(), dev->bx.as<float>(), (int)hd, dev->bw.as<float>(),
                                           (int)n_keys, (long long)stride, scale, dev->stream));
    return finish(dev, scores, dev->bo, n_keys * 4, "attention_scores");
}

int ditch_cuda_attention_values(ditch_cuda_device *dev, float *out, size_t vd, const float *scores, size_t n_keys,
                                const float *v, size_t v_len, size_t stride) {
    clear_error();
    REQUIRE(dev && out && scores && v, "null argument");
    if (vd == 0) return DITCH_CUDA_OK;
    REQUIRE(n_keys == 0 || v_len >= (n_keys - 1) * stride + vd, "value slice too short");
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, scores, n_keys * 4));
    DITCH_CUDA(up(dev, dev->bw, v, v_len * 4));
    DITCH_CUDA(dev->bo.reserve(vd * 4));
    DITCH_LAUNCH(dev, attention_values_f32(dev->bo.as<float>(), dev->bx.as<float>(), (int)n_keys, dev->bw.as<float>(),
                                           (int)vd, (long long)stride, dev->stream));
    return finish(dev, out, dev->bo, vd * 4, "attention_values");
}

int ditch_cuda_gated_activation(ditch_cuda_device *dev, uint32_t act, float *out, const float *gate, const float *up_,
                                size_t n, size_t len, size_t in_stride, size_t out_stride) {
    clear_error();
    REQUIRE(dev && out && gate, "null argument");
    if (act != 0) {
        set_error("activation %u is not implemented on this device", act);
        return DITCH_CUDA_UNSUPPORTED;
    }
    if (n == 0 || len == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const size_t in_elems = (n - 1) * in_stride + len, out_elems = (n - 1) * out_stride + len;
    DITCH_CUDA(up(dev, dev->bx, gate, in_elems * 4));
    if (up_) DITCH_CUDA(up(dev, dev->bw, up_, in_elems * 4));
    // `out` may alias `gate` (src/tensor.zig:1333): read the host output first.
    DITCH_CUDA(up(dev, dev->bo, out, out_elems * 4));
    DITCH_LAUNCH(dev, gated_silu_f32(dev->bx.as<float>(), up_ ? dev->bw.as<float>() : nullptr, (int)n, (int)len,
                                     (long long)in_stride, (long long)out_stride, dev->bo.as<float>(), dev->stream));
    return finish(dev, out, dev->bo, out_elems * 4, "gated_activation");
}

int ditch_cuda_rmsnorm_rows(ditch_cuda_device *dev, float *out, const float *x, const float *weight, size_t w_len,
                            size_t n, size_t len, float eps, int gemma_style) {
    clear_error();
    REQUIRE(dev && out && x, "null argument");
    REQUIRE(w_len == 0 || w_len >= len, "weight shorter than the row");
    if (n == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, x, n * len * 4));
    if (w_len) DITCH_CUDA(up(dev, dev->bw, weight, len * 4));
    DITCH_CUDA(dev->bo.reserve(n * len * 4));
    DITCH_LAUNCH(dev, rmsnorm_rows_f32(dev->bx.as<float>(), w_len ? dev->bw.as<float>() : nullptr, (int)n, (int)len, eps,
                                       gemma_style, dev->bo.as<float>(), dev->stream));
    return finish(dev, out, dev->bo, n * len * 4, "rmsnorm_rows");
}

int ditch_cuda_layernorm_rows(ditch_cuda_device *dev, float *out, const float *x, const float *weight, size_t w_len,
                              const float *bias, size_t n, size_t len, float eps, int one_plus) {
    clear_error();
    REQUIRE(dev && out && x, "null argument");
    REQUIRE(w_len == 0 || w_len >= len, "weight shorter than the row");
    if (n == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, x, n * len * 4));
    if (w_len) DITCH_CUDA(up(dev, dev->bw, weight, len * 4));
    if (bias) DITCH_CUDA(up(dev, dev->by, bias, len * 4));
    DITCH_CUDA(dev->bo.reserve(n * len * 4));
    DITCH_LAUNCH(dev, layernorm_rows_f32(dev->bx.as<float>(), w_len ? dev->bw.as<float>() : nullptr,
                                         bias ? dev->by.as<float>() : nullptr, (int)n, (int)len, eps, one_plus,
                                         dev->bo.as<float>(), dev->stream));
    return finish(dev, out, dev->bo, n * len * 4, "layernorm_rows");
}

int ditch_cuda_softmax_rows(ditch_cuda_device *dev, float *x, size_t n, size_t len) {
    clear_error();
    REQUIRE(dev && x, "null argument");
    if (n == 0 || len == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bo, x, n * len * 4));
    DITCH_LAUNCH(dev, softmax_rows_f32(dev->bo.as<float>(), (int)n, (int)len, dev->stream));
    return finish(dev, x, dev->bo, n * len * 4, "softmax_rows");
}

int ditch_cuda_rope_rows(ditch_cuda_device *dev, float *x, size_t n, size_t dim, const float *cos_t,
                         const float *sin_t, size_t table_len, size_t half, const uint32_t *pos, int style) {
    clear_error();
    REQUIRE(dev && x && cos_t && sin_t && pos, "null argument");
    REQUIRE(style == 0 || style == 1, "style must be 0 (neox) or 1 (gptj)");
    REQUIRE(2 * half <= dim, "rotated half exceeds the head");
    for (size_t i = 0; i < n; i++) REQUIRE(pos[i] < table_len, "position outside the RoPE table");
    if (n == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bo, x, n * dim * 4));
    DITCH_CUDA(up(dev, dev->bx, cos_t, table_len * half * 4));
    DITCH_CUDA(up(dev, dev->bw, sin_t, table_len * half * 4));
    DITCH_CUDA(up(dev, dev->by, pos, n * 4));
    DITCH_LAUNCH(dev, rope_rows_f32(dev->bo.as<float>(), (int)n, (int)dim, dev->bx.as<float>(), dev->bw.as<float>(),
                                    (int)half, dev->by.as<uint32_t>(), style, dev->stream));
    return finish(dev, x, dev->bo, n * dim * 4, "rope_rows");
}

// ---- decoders ----
int ditch_cuda_dequant_fp8(ditch_cuda_device *dev, const uint8_t *codes, const float *scales, size_t rows,
                           size_t cols, size_t br, size_t bc, uint16_t *out) {
    clear_error();
    REQUIRE(dev && codes && scales && out && br > 0 && bc > 0, "bad argument");
    if (rows == 0 || cols == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const size_t sn = ((rows + br - 1) / br) * ((cols + bc - 1) / bc);
    DITCH_CUDA(up(dev, dev->bx, codes, rows * cols));
    DITCH_CUDA(up(dev, dev->bw, scales, sn * 4));
    DITCH_CUDA(dev->bo.reserve(rows * cols * 2));
    DITCH_LAUNCH(dev, dequant_fp8_bf16(dev->bx.as<uint8_t>(), dev->bw.as<float>(), (int)rows, (int)cols, (int)br,
                                       (int)bc, dev->bo.as<uint16_t>(), dev->stream));
    return finish(dev, out, dev->bo, rows * cols * 2, "dequant_fp8");
}

int ditch_cuda_dequant_int(ditch_cuda_device *dev, const uint32_t *packed, size_t wpr, const float *scales,
                           size_t groups, const uint32_t *zeros, const uint32_t *g_idx, size_t rows, size_t cols,
                           int bits, size_t group, uint16_t *out) {
    clear_error();
    REQUIRE(dev && packed && scales && out, "null argument");
    REQUIRE(bits >= 1 && bits <= 8, "bits must be 1..8");
    REQUIRE(wpr * 32 >= cols * (size_t)bits, "packed rows too short");
    if (rows == 0 || cols == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, packed, rows * wpr * 4));
    DITCH_CUDA(up(dev, dev->bw, scales, rows * groups * 4));
    const size_t zrows = (rows * bits + 31) / 32;
    if (zeros) DITCH_CUDA(up(dev, dev->by, zeros, zrows * groups * 4));
    if (g_idx) DITCH_CUDA(up(dev, dev->braw, g_idx, cols * 4));
    DITCH_CUDA(dev->bo.reserve(rows * cols * 2));
    DITCH_LAUNCH(dev, dequant_int_bf16(dev->bx.as<uint32_t>(), (long long)wpr, dev->bw.as<float>(),
                                       zeros ? dev->by.as<uint32_t>() : nullptr, g_idx ? dev->braw.as<uint32_t>() : nullptr,
                                       (int)groups, (int)rows, (int)cols, bits, (int)group, dev->bo.as<uint16_t>(),
                                       dev->stream));
    return finish(dev, out, dev->bo, rows * cols * 2, "dequant_int");
}

int ditch_cuda_dequant_mxfp4(ditch_cuda_device *dev, const uint8_t *blocks, const uint8_t *scales, size_t rows,
                             size_t cols, int transposed, uint16_t *out) {
    clear_error();
    REQUIRE(dev && blocks && scales && out, "null argument");
    if (cols % 32) {
        set_error("MXFP4 needs a multiple of 32 columns");
        return DITCH_CUDA_UNSUPPORTED;
    }
    if (rows == 0 || cols == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, blocks, rows * cols / 2));
    DITCH_CUDA(up(dev, dev->bw, scales, rows * cols / 32));
    DITCH_CUDA(dev->bo.reserve(rows * cols * 2));
    if (transposed)
        DITCH_LAUNCH(dev, dequant_mxfp4t_bf16(dev->bx.as<uint8_t>(), dev->bw.as<uint8_t>(), (int)rows, (int)cols,
                                              dev->bo.as<uint16_t>(), dev->stream));
    else
        DITCH_LAUNCH(dev, dequant_mxfp4_bf16(dev->bx.as<uint8_t>(), dev->bw.as<uint8_t>(), (int)rows, (int)cols,
                                             dev->bo.as<uint16_t>(), dev->stream));
    return finish(dev, out, dev->bo, rows * cols * 2, "dequant_mxfp4");
}

int ditch_cuda_dequant_ggml(ditch_cuda_device *dev, int dtype, const uint8_t *src, size_t src_len, size_t n,
                            float *out) {
    clear_error();
    REQUIRE(dev && src && out, "null argument");
    if (dtype < DITCH_DTYPE_Q8_0 || dtype > DITCH_DTYPE_Q8_K) {
        set_error("dtype %d is not a ggml block format", dtype);
        return DITCH_CUDA_UNSUPPORTED;
    }
    const size_t bs = dtype >= DITCH_DTYPE_Q4_K ? 256 : 32;
    static const size_t bb[] = {34, 18, 20, 22, 24, 144, 210, 292};
    REQUIRE(n % bs == 0, "n is not a whole number of blocks");
    REQUIRE(src_len >= n / bs * bb[dtype - DITCH_DTYPE_Q8_0], "source shorter than n elements");
    if (n == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(up(dev, dev->bx, src, n / bs * bb[dtype - DITCH_DTYPE_Q8_0]));
    DITCH_CUDA(dev->bo.reserve(n * 4));
    DITCH_LAUNCH(dev, dequant_ggml_f32(dtype, dev->bx.as<uint8_t>(), (long long)n, dev->bo.as<float>(), dev->stream));
    return finish(dev, out, dev->bo, n * 4, "dequant_ggml");
}

// W <- W - alpha r (r^T W): a = r^T W (GEMV-T, one read of W), then the
// rank-1 update with b = -alpha r (one read and one write of W).
int ditch_cuda_edit_weight_bf16(ditch_cuda_device *dev, void *w, size_t rows, size_t cols, const float *r,
                                float alpha) {
    clear_error();
    REQUIRE(dev && w && r, "null argument");
    // bf16 elements and f32 entries must sit on their own size; rows that are
    // not 16-byte aligned take the kernels' 2-byte path
    REQUIRE((reinterpret_cast<uintptr_t>(w) & 1) == 0, "w is not 2-byte aligned");
    REQUIRE((reinterpret_cast<uintptr_t>(r) & 3) == 0, "r is not 4-byte aligned");
    REQUIRE(rows <= (size_t)INT32_MAX && cols <= (size_t)INT32_MAX, "rows or cols above 2^31 - 1");
    if (rows == 0 || cols == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(dev->bo.reserve(cols * 4));
    DITCH_CUDA(dev->bx.reserve(rows * 4));
    DITCH_CUDA(cudaMemsetAsync(dev->bo.ptr, 0, cols * 4, dev->stream));
    DITCH_LAUNCH(dev, gemv_t_bf16(static_cast<const uint16_t *>(w), (int)rows, (int)cols, r, dev->bo.as<float>(),
                                  dev->stream));
    DITCH_LAUNCH(dev, scale_vec(r, alpha, (int)rows, dev->bx.as<float>(), dev->stream));
    DITCH_LAUNCH(dev, rank1_update_bf16(static_cast<uint16_t *>(w), (int)rows, (int)cols, dev->bx.as<float>(),
                                        dev->bo.as<float>(), dev->stream));
    return check_status(dev, "edit_weight_bf16");
}

// ---- timing ----
int ditch_cuda_set_decode_staging(ditch_cuda_device *dev, int min_tokens) {
    REQUIRE(dev, "null device");
    REQUIRE(min_tokens >= 0, "min_tokens must be >= 0");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->stage_min_tokens = min_tokens;
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_decode_cache(ditch_cuda_device *dev, int enabled) {
    REQUIRE(dev, "null device");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->decode_cache = enabled != 0;
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_cta_pairs(ditch_cuda_device *dev, int level) {
    REQUIRE(dev, "null device");
    REQUIRE(level >= 0 && level <= 2, "CTA-pair level must be 0, 1 or 2");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->cta_pairs = level;
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_attention_tc(ditch_cuda_device *dev, int level) {
    REQUIRE(dev, "null device");
    REQUIRE(level >= 0 && level <= 2, "attention level must be 0, 1 or 2");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->attn_tc = level;
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_f32_split(ditch_cuda_device *dev, int enabled) {
    REQUIRE(dev, "null device");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->f32_split = enabled != 0;
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_deterministic(ditch_cuda_device *dev, int enabled) {
    REQUIRE(dev, "null device");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->deterministic = enabled != 0;
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_profiling(ditch_cuda_device *dev, int enabled) {
    REQUIRE(dev, "null device");
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->profiling = enabled != 0;
    return DITCH_CUDA_OK;
}

int ditch_cuda_gemm_stats(ditch_cuda_device *dev, double *ms, uint64_t *launches, double *flops) {
    REQUIRE(dev, "null device");
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    for (size_t i = 0; i < dev->n_events; i++) {
        float t = 0;
        DITCH_CUDA(cudaEventElapsedTime(&t, dev->events[i].start, dev->events[i].stop));
        dev->gemm_ms_done += t;
        dev->gemm_flops_done += dev->events[i].flops;
    }
    dev->gemm_launches += dev->n_events;
    dev->n_events = 0;
    if (ms) *ms = dev->gemm_ms_done;
    if (launches) *launches = dev->gemm_launches;
    if (flops) *flops = dev->gemm_flops_done;
    return DITCH_CUDA_OK;
}

int ditch_cuda_reset_stats(ditch_cuda_device *dev) {
    REQUIRE(dev, "null device");
    std::lock_guard<std::mutex> lk(dev->mu);
    cudaStreamSynchronize(dev->stream);
    dev->n_events = 0;
    dev->gemm_ms_done = dev->gemm_flops_done = 0.0;
    dev->gemm_launches = 0;
    dev->launches = 0;
    return DITCH_CUDA_OK;
}

uint64_t ditch_cuda_launches(const ditch_cuda_device *dev) { return dev ? dev->launches.load() : 0; }

int ditch_cuda_timer_start(ditch_cuda_device *dev) {
    REQUIRE(dev, "null device");
    DITCH_CUDA(cudaEventRecord(dev->t0, dev->stream));
    return DITCH_CUDA_OK;
}

int ditch_cuda_timer_stop(ditch_cuda_device *dev, float *ms) {
    REQUIRE(dev && ms, "null argument");
    DITCH_CUDA(cudaEventRecord(dev->t1, dev->stream));
    DITCH_CUDA(cudaEventSynchronize(dev->t1));
    DITCH_CUDA(cudaEventElapsedTime(ms, dev->t0, dev->t1));
    return DITCH_CUDA_OK;
}

int ditch_cuda_synchronize(ditch_cuda_device *dev) {
    REQUIRE(dev, "null device");
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    return check_status(dev, "synchronize");
}

}  // extern "C"
