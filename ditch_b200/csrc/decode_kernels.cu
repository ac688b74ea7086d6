// Kernels of greedy generation: storing keys and values into the KV cache,
// single-token attention over the cache, and the argmax of the logit rows.
#include "attn_common.cuh"
#include "kernels.cuh"

namespace ditch {

namespace {

using attn::rms_inplace;
using attn::rope_neox_inplace;
using attn::warp_max;
using attn::warp_sum;

constexpr int kStoreWarps = 8;

// One block per row, one warp per head slot: the row's q heads (normed and
// roped in place when prep_q), its k heads (normed and roped when prep_k)
// and v heads, the last two copied to the cache at (slot, position).
__global__ void __launch_bounds__(kStoreWarps * 32) k_kv_store(KvParams p) {
    extern __shared__ float sm[];  // [kStoreWarps][head_dim]
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = p.head_dim, nh = p.heads, nkv = p.kv_heads, qd = nh * hd, kvd = nkv * hd;
    const int b = p.row_b[r], pos = p.row_pos[r];
    if (b < 0 || b >= p.slots || pos < 0 || pos >= p.max_len) {
        if (threadIdx.x == 0 && p.status) atomicExch(p.status, kKernelBadArgument);
        return;
    }
    float *row = p.qkv + (long long)r * (qd + 2 * kvd);
    const long long at = ((long long)b * p.max_len + pos) * kvd;
    float *v = sm + warp * hd;
    const int q_slots = p.prep_q ? nh : 0;
    for (int s = warp; s < q_slots + 2 * nkv; s += kStoreWarps) {
        if (s >= q_slots + nkv) {  // a value head: plain copy
            const int j = s - q_slots - nkv;
            const float *src = row + qd + kvd + j * hd;
            float *dst = p.cache_v + at + j * hd;
            for (int i = lane; i < hd; i += 32) dst[i] = src[i];
            continue;
        }
        const bool is_q = s < q_slots;
        float *src = is_q ? row + s * hd : row + qd + (s - q_slots) * hd;
        for (int i = lane; i < hd; i += 32) v[i] = src[i];
        __syncwarp();
        if (is_q || p.prep_k) {
            const float *nw = is_q ? p.q_norm : p.k_norm;
            if (nw) rms_inplace(v, hd, nw, p.eps, lane);
            rope_neox_inplace(v, hd, pos, p.rope_cos, p.rope_sin, lane);
            __syncwarp();
        }
        float *dst = is_q ? src : p.cache_k + at + (s - q_slots) * hd;
        for (int i = lane; i < hd; i += 32) dst[i] = v[i];
        __syncwarp();
    }
}

// ---- single-token attention over the cache --------------------------------
// Block = (row, kv head). Keys and values 0..pos of the row's slot are staged
// in shared memory kDecChunk at a time and shared by the group's q heads;
// each warp owns heads warp, warp + kDecWarps, ... and keeps an online
// softmax per head (running max, sum and the weighted value sum).
constexpr int kDecChunk = 64;
constexpr int kDecWarps = 4;

__global__ void __launch_bounds__(kDecWarps * 32) k_attention_decode(DecodeAttnParams p) {
    extern __shared__ float sm[];
    const int r = blockIdx.x, kvh = blockIdx.y;
    const int hd = p.head_dim, nh = p.heads, nkv = p.kv_heads;
    const int qd = nh * hd, kvd = nkv * hd, groups = nh / nkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = p.row_b[r], len = p.row_pos[r] + 1;
    const int ks = hd + 1;                     // padded key stride
    float *kbuf = sm;                          // [kDecChunk][hd + 1]
    float *vbuf = kbuf + kDecChunk * ks;       // [kDecChunk][hd]
    float *qbuf = vbuf + kDecChunk * hd;       // [groups][hd]
    float *acc = qbuf + groups * hd;           // [groups][hd]
    float *pbuf = acc + groups * hd;           // [kDecWarps][kDecChunk]
    float *ml = pbuf + kDecWarps * kDecChunk;  // [groups][2]: running max, sum
    float *pw = pbuf + warp * kDecChunk;
    const float *qsrc = p.qkv + (long long)r * (qd + 2 * kvd) + kvh * groups * hd;
    for (int i = threadIdx.x; i < groups * hd; i += blockDim.x) {
        qbuf[i] = qsrc[i];
        acc[i] = 0.0f;
    }
    for (int i = threadIdx.x; i < groups; i += blockDim.x) {
        ml[2 * i] = -INFINITY;
        ml[2 * i + 1] = 0.0f;
    }
    const float *kc = p.cache_k + (long long)b * p.max_len * kvd + kvh * hd;
    const float *vc = p.cache_v + (long long)b * p.max_len * kvd + kvh * hd;
    for (int k0 = 0; k0 < len; k0 += kDecChunk) {
        const int nk = min(kDecChunk, len - k0);
        __syncthreads();
        for (int i = threadIdx.x; i < nk * hd; i += blockDim.x) {
            const int kr = i / hd, d = i - kr * hd;
            kbuf[kr * ks + d] = kc[(long long)(k0 + kr) * kvd + d];
            vbuf[kr * hd + d] = vc[(long long)(k0 + kr) * kvd + d];
        }
        __syncthreads();
        for (int h = warp; h < groups; h += kDecWarps) {
            const float *q = qbuf + h * hd;
            float cmax = -INFINITY;
            for (int kr = lane; kr < kDecChunk; kr += 32) {
                float s = -INFINITY;
                if (kr < nk) {
                    const float *kd = kbuf + kr * ks;
                    float d = 0.0f;
                    for (int i = 0; i < hd; i++) d = fmaf(q[i], kd[i], d);
                    s = d * p.scale;
                }
                pw[kr] = s;
                cmax = fmaxf(cmax, s);
            }
            cmax = warp_max(cmax);
            const float m = ml[2 * h], mnew = fmaxf(m, cmax);
            const float corr = m == -INFINITY ? 0.0f : expf(m - mnew);
            float csum = 0.0f;
            for (int kr = lane; kr < kDecChunk; kr += 32) {
                const float e = kr < nk ? expf(pw[kr] - mnew) : 0.0f;
                pw[kr] = e;
                csum += e;
            }
            csum = warp_sum(csum);
            __syncwarp();
            float *a = acc + h * hd;
            for (int i = lane; i < hd; i += 32) {
                float t = a[i] * corr;
                for (int kr = 0; kr < nk; kr++) t = fmaf(pw[kr], vbuf[kr * hd + i], t);
                a[i] = t;
            }
            __syncwarp();
            if (lane == 0) {
                ml[2 * h] = mnew;
                ml[2 * h + 1] = ml[2 * h + 1] * corr + csum;
            }
            __syncwarp();
        }
    }
    __syncthreads();
    uint16_t *dst = p.out + (long long)r * qd + kvh * groups * hd;
    for (int i = threadIdx.x; i < groups * hd; i += blockDim.x)
        dst[i] = f32_to_bf16_bits(acc[i] * (1.0f / ml[2 * (i / hd) + 1]));
}

// ---- argmax per row --------------------------------------------------------
// Each thread scans its stride in increasing order with a strict `>`, so its
// candidate is its first maximum; candidates merge by value, then by the
// lower index. Only values above -inf ever become candidates, as in the
// reference scan starting from -inf at index 0.
__global__ void __launch_bounds__(512) k_argmax_rows(const float *x, int len, uint32_t *out) {
    __shared__ float sv[16];
    __shared__ int si[16];
    const float *row = x + (long long)blockIdx.x * len;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
        const float v = row[i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < nw; w++)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        out[blockIdx.x] = bi == INT_MAX ? 0u : (uint32_t)bi;
    }
}

}  // namespace

cudaError_t kv_store(const KvParams &p, cudaStream_t st) {
    if (p.n <= 0) return cudaSuccess;
    if (p.head_dim % 2 || p.heads % p.kv_heads) return cudaErrorInvalidValue;
    k_kv_store<<<p.n, kStoreWarps * 32, sizeof(float) * kStoreWarps * p.head_dim, st>>>(p);
    return cudaGetLastError();
}

cudaError_t attention_decode(const DecodeAttnParams &p, cudaStream_t st) {
    if (p.n <= 0) return cudaSuccess;
    if (p.heads % p.kv_heads) return cudaErrorInvalidValue;
    const int hd = p.head_dim, groups = p.heads / p.kv_heads;
    const size_t smem = sizeof(float) * (kDecChunk * (hd + 1) + kDecChunk * hd + 2 * groups * hd +
                                         kDecWarps * kDecChunk + 2 * groups);
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e =
            cudaFuncSetAttribute(k_attention_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    k_attention_decode<<<dim3(p.n, p.kv_heads), kDecWarps * 32, smem, st>>>(p);
    return cudaGetLastError();
}

cudaError_t argmax_rows(const float *x, int n, int len, uint32_t *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_argmax_rows<<<n, 512, 0, st>>>(x, len, out);
    return cudaGetLastError();
}

}  // namespace ditch
