// Warp helpers shared by the prefill and decode attention kernels: warp
// reductions, and the per-head RMSNorm and neox RoPE of one head vector held
// by a warp (lane l owns elements l, l + 32, ...).
#pragma once

#include "common.cuh"

namespace ditch {
namespace attn {

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

// Rotary embedding, neox pairing (x[i], x[i + hd / 2]) at position `pos`
// (src/tensor.zig:1360-1369 with the table of src/model.zig:2200-2282).
__device__ __forceinline__ void rope_neox_inplace(float *v, int hd, int pos, const float *cos_t, const float *sin_t,
                                                  int lane) {
    const int half = hd / 2;
    const float *c = cos_t + (long long)pos * half;
    const float *s = sin_t + (long long)pos * half;
    for (int i = lane; i < half; i += 32) {
        const float x1 = v[i], x2 = v[i + half];
        v[i] = x1 * c[i] - x2 * s[i];
        v[i + half] = x2 * c[i] + x1 * s[i];
    }
}

// Per-head RMSNorm (q_norm / k_norm of qwen3-style models), in place.
__device__ __forceinline__ void rms_inplace(float *v, int hd, const float *w, float eps, int lane) {
    float ss = 0.0f;
    for (int i = lane; i < hd; i += 32) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
    __syncwarp();
    for (int i = lane; i < hd; i += 32) v[i] = v[i] * inv * w[i];
    __syncwarp();
}

}  // namespace attn
}  // namespace ditch
