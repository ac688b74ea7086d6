// Element-wise entries of the compute seam (src/compute.zig:90-117) on f32
// rows: softmax, gated SiLU, RoPE, single-query attention scores / values and
// LayerNorm. The resident forward fuses these into its own kernels; these are
// the per-call device versions a host engine may dispatch one by one.
#include "kernels.cuh"

namespace ditch {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// softmaxInPlace (src/tensor.zig:1181-1200), one warp per row.
__global__ void k_softmax(float *x, int n, int len) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    float *r = x + (long long)row * len;
    float m = -INFINITY;
    for (int i = lane; i < len; i += 32) m = fmaxf(m, r[i]);
    m = warp_max(m);
    float s = 0.0f;
    for (int i = lane; i < len; i += 32) {
        const float e = expf(r[i] - m);
        r[i] = e;
        s += e;
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    for (int i = lane; i < len; i += 32) r[i] *= inv;
}

// gatedActivation with silu (src/tensor.zig:1309-1337).
__global__ void k_gated_silu(const float *gate, const float *up, int n, int len, long long in_stride,
                             long long out_stride, float *out) {
    const long long total = (long long)n * len;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long i = e / len, j = e % len;
        const float g = gate[i * in_stride + j];
        float v = g / (1.0f + expf(-g));
        if (up) v *= up[i * in_stride + j];
        out[i * out_stride + j] = v;
    }
}

// ropeRows (src/compute.zig:519-537): neox rotate-half or gptj interleaved.
__global__ void k_rope(float *x, int n, int dim, const float *cos_t, const float *sin_t, int half,
                       const uint32_t *pos, int style) {
    const long long total = (long long)n * half;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(e / half), k = (int)(e % half);
        float *row = x + (long long)i * dim;
        const float c = cos_t[(long long)pos[i] * half + k], s = sin_t[(long long)pos[i] * half + k];
        const int a = style == 0 ? k : 2 * k, b = style == 0 ? k + half : 2 * k + 1;
        const float x1 = row[a], x2 = row[b];
        row[a] = x1 * c - x2 * s;
        row[b] = x2 * c + x1 * s;
    }
}

// attentionScores: scores[p] = scale * dot(q, k[p * stride ..][0..hd]).
__global__ void k_attn_scores(float *scores, const float *q, int hd, const float *k, int n_keys, long long stride,
                              float scale) {
    const int p = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (p >= n_keys) return;
    float s = 0.0f;
    for (int i = lane; i < hd; i += 32) s = fmaf(q[i], k[(long long)p * stride + i], s);
    s = warp_sum(s);
    if (lane == 0) scores[p] = s * scale;
}

// attentionValues: out[j] = sum_p scores[p] * v[p * stride + j].
__global__ void k_attn_values(float *out, const float *scores, int n_keys, const float *v, int vd, long long stride) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= vd) return;
    float a = 0.0f;
    for (int p = 0; p < n_keys; p++) a = fmaf(scores[p], v[(long long)p * stride + j], a);
    out[j] = a;
}

// layernorm (src/tensor.zig:1341-1356), one warp per row.
__global__ void k_layernorm(const float *x, const float *w, const float *b, int n, int len, float eps, int one_plus,
                            float *out) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const float *r = x + (long long)row * len;
    float s = 0.0f;
    for (int i = lane; i < len; i += 32) s += r[i];
    const float mean = warp_sum(s) / (float)len;
    float v = 0.0f;
    for (int i = lane; i < len; i += 32) v += (r[i] - mean) * (r[i] - mean);
    const float inv = 1.0f / sqrtf(warp_sum(v) / (float)len + eps);
    float *o = out + (long long)row * len;
    for (int i = lane; i < len; i += 32) {
        float y = (r[i] - mean) * inv;
        if (w) y *= one_plus ? 1.0f + w[i] : w[i];
        if (b) y += b[i];
        o[i] = y;
    }
}

inline int grid_for(long long n) {
    long long b = (n + 255) / 256;
    return (int)(b < 1 ? 1 : (b > 65535 ? 65535 : b));
}

}  // namespace

cudaError_t softmax_rows_f32(float *x, int n, int len, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_softmax<<<(n + 7) / 8, 256, 0, st>>>(x, n, len);
    return cudaGetLastError();
}

cudaError_t gated_silu_f32(const float *gate, const float *up, int n, int len, long long in_stride,
                           long long out_stride, float *out, cudaStream_t st) {
    if (n <= 0 || len <= 0) return cudaSuccess;
    k_gated_silu<<<grid_for((long long)n * len), 256, 0, st>>>(gate, up, n, len, in_stride, out_stride, out);
    return cudaGetLastError();
}

cudaError_t rope_rows_f32(float *x, int n, int dim, const float *cos, const float *sin, int half, const uint32_t *pos,
                          int style, cudaStream_t st) {
    if (n <= 0 || half <= 0) return cudaSuccess;
    k_rope<<<grid_for((long long)n * half), 256, 0, st>>>(x, n, dim, cos, sin, half, pos, style);
    return cudaGetLastError();
}

cudaError_t attention_scores_f32(float *scores, const float *q, int hd, const float *k, int n_keys, long long stride,
                                 float scale, cudaStream_t st) {
    if (n_keys <= 0) return cudaSuccess;
    k_attn_scores<<<(n_keys + 7) / 8, 256, 0, st>>>(scores, q, hd, k, n_keys, stride, scale);
    return cudaGetLastError();
}

cudaError_t attention_values_f32(float *out, const float *scores, int n_keys, const float *v, int vd,
                                 long long stride, cudaStream_t st) {
    if (vd <= 0) return cudaSuccess;
    k_attn_values<<<(vd + 255) / 256, 256, 0, st>>>(out, scores, n_keys, v, vd, stride);
    return cudaGetLastError();
}

cudaError_t layernorm_rows_f32(const float *x, const float *w, const float *b, int n, int len, float eps,
                               int one_plus, float *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_layernorm<<<(n + 7) / 8, 256, 0, st>>>(x, w, b, n, len, eps, one_plus, out);
    return cudaGetLastError();
}

}  // namespace ditch
