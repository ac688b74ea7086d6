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
    const long long o0 = (long long)r * qd + kvh * groups * hd;
    for (int i = threadIdx.x; i < groups * hd; i += blockDim.x) {
        const float y = acc[i] * (1.0f / ml[2 * (i / hd) + 1]);
        if (p.out_f32) p.out_f32[o0 + i] = y;
        else p.out[o0 + i] = f32_to_bf16_bits(y);
    }
}

// ---- single-token attention, register path (head size 64 / 128) -----------
// Block = (row, kv head), kRegWarps warps; warp w takes key groups w, w + 4,
// ... of KG keys. Lane l holds head dims [l * HD / 32, (l + 1) * HD / 32) of
// the group's GP (padded) query heads and of its running value sums. Per
// key group: the KG key rows (coalesced, 16 or 8 bytes per lane) give each
// lane KG x GP partial dot products; a butterfly reduce-scatter over the
// lanes leaves the full dot of pair (key, head) = index l >> SH in lane l.
// Each lane then keeps the online-softmax state (max, sum) of its own head,
// and the weights reach the value update through shuffles. Padded heads
// have zero queries (finite, discarded). The warps' states merge through
// shared memory at the end.
constexpr int kRegWarps = 4;

template <int HD, int GP>
__global__ void __launch_bounds__(kRegWarps * 32) k_attention_decode_reg(DecodeAttnParams p) {
    constexpr int D = HD / 32;                          // dims per lane
    constexpr int KG = (32 / GP) < 8 ? (32 / GP) : 8;   // keys per group
    constexpr int NV = KG * GP;                         // values reduced per group (a power of two)
    constexpr int LOGN = NV == 32 ? 5 : NV == 16 ? 4 : NV == 8 ? 3 : NV == 4 ? 2 : 1;
    constexpr int SH = 5 - LOGN;                        // lane l holds value index l >> SH
    constexpr int LOGG = GP == 8 ? 3 : GP == 4 ? 2 : GP == 2 ? 1 : 0;
    __shared__ float s_m[kRegWarps][GP], s_l[kRegWarps][GP];
    __shared__ __align__(16) float s_acc[kRegWarps][GP][HD];
    const int r = blockIdx.x, kvh = blockIdx.y;
    const int nh = p.heads, nkv = p.kv_heads, G = nh / nkv;
    const int qd = nh * HD, kvd = nkv * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = p.row_b[r], len = p.row_pos[r] + 1;
    float q[GP][D], acc[GP][D];
    const float *qsrc = p.qkv + (long long)r * (qd + 2 * kvd) + (long long)kvh * G * HD + lane * D;
#pragma unroll
    for (int h = 0; h < GP; h++)
#pragma unroll
        for (int d = 0; d < D; d++) {
            q[h][d] = h < G ? qsrc[h * HD + d] : 0.0f;
            acc[h][d] = 0.0f;
        }
    const int my_index = lane >> SH, my_h = my_index & (GP - 1), my_key = my_index >> LOGG;
    float m_run = -INFINITY, l_run = 0.0f;
    const float *kc = p.cache_k + (long long)b * p.max_len * kvd + kvh * HD + lane * D;
    const float *vc = p.cache_v + (long long)b * p.max_len * kvd + kvh * HD + lane * D;
    for (int k0 = warp * KG; k0 < len; k0 += kRegWarps * KG) {
        float kr[KG][D], vr[KG][D];
#pragma unroll
        for (int j = 0; j < KG; j++) {
            const long long at = (long long)min(k0 + j, len - 1) * kvd;  // past the end: a valid row, weight 0
            if (D == 4) {
                const float4 a = *reinterpret_cast<const float4 *>(kc + at);
                const float4 c = *reinterpret_cast<const float4 *>(vc + at);
                kr[j][0] = a.x; kr[j][1] = a.y; kr[j][2] = a.z; kr[j][3] = a.w;
                vr[j][0] = c.x; vr[j][1] = c.y; vr[j][2] = c.z; vr[j][3] = c.w;
            } else {
                const float2 a = *reinterpret_cast<const float2 *>(kc + at);
                const float2 c = *reinterpret_cast<const float2 *>(vc + at);
                kr[j][0] = a.x; kr[j][1] = a.y;
                vr[j][0] = c.x; vr[j][1] = c.y;
            }
        }
        // partial dots, index = key * GP + head
        float v[NV];
#pragma unroll
        for (int j = 0; j < KG; j++)
#pragma unroll
            for (int h = 0; h < GP; h++) {
                float t = 0.0f;
#pragma unroll
                for (int d = 0; d < D; d++) t = fmaf(q[h][d], kr[j][d], t);
                v[j * GP + h] = t;
            }
        // reduce-scatter: after the step of lane bit s the lanes with that
        // bit set hold the upper half of the remaining indices
#pragma unroll
        for (int n = NV, s = 16; n > 1; n >>= 1, s >>= 1) {
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; i++) {
                const float send = upper ? v[i] : v[i + n / 2];
                const float keep = upper ? v[i + n / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
            }
        }
#pragma unroll
        for (int s = (1 << SH) >> 1; s > 0; s >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], s);
        const float score = k0 + my_key < len ? v[0] * p.scale : -INFINITY;
        // the group's max and sum per head: over the key bits of the lane
        float gmax = score;
#pragma unroll
        for (int s = 1 << (SH + LOGG); s < 32; s <<= 1) gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, s));
        const float m_new = fmaxf(m_run, gmax);
        const float corr = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
        const float pw = score == -INFINITY ? 0.0f : expf(score - m_new);
        float psum = pw;
#pragma unroll
        for (int s = 1 << (SH + LOGG); s < 32; s <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, s);
        l_run = l_run * corr + psum;
        m_run = m_new;
#pragma unroll
        for (int h = 0; h < GP; h++) {
            const float c = __shfl_sync(0xffffffffu, corr, h << SH);
#pragma unroll
            for (int d = 0; d < D; d++) acc[h][d] *= c;
#pragma unroll
            for (int j = 0; j < KG; j++) {
                const float w = __shfl_sync(0xffffffffu, pw, (j * GP + h) << SH);
#pragma unroll
                for (int d = 0; d < D; d++) acc[h][d] = fmaf(w, vr[j][d], acc[h][d]);
            }
        }
    }
    if (my_key == 0 && (lane & ((1 << SH) - 1)) == 0) {
        s_m[warp][my_h] = m_run;
        s_l[warp][my_h] = l_run;
    }
#pragma unroll
    for (int h = 0; h < GP; h++)
#pragma unroll
        for (int d = 0; d < D; d++) s_acc[warp][h][lane * D + d] = acc[h][d];
    __syncthreads();
    const long long o0 = (long long)r * qd + (long long)kvh * G * HD;
    for (int i = threadIdx.x; i < G * HD; i += blockDim.x) {
        const int h = i / HD, d = i - h * HD;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kRegWarps; w++) mx = fmaxf(mx, s_m[w][h]);
        float num = 0.0f, den = 0.0f;
#pragma unroll
        for (int w = 0; w < kRegWarps; w++) {
            const float e = s_m[w][h] == -INFINITY ? 0.0f : expf(s_m[w][h] - mx);
            num = fmaf(s_acc[w][h][d], e, num);
            den = fmaf(s_l[w][h], e, den);
        }
        if (p.out_f32) p.out_f32[o0 + i] = num / den;
        else p.out[o0 + i] = f32_to_bf16_bits(num / den);
    }
}

// ---- argmax per row --------------------------------------------------------
// Each thread scans its stride in increasing order with a strict `>`, so its
// candidate is its first maximum; candidates merge by value, then by the
// lower index. Only values above -inf ever become candidates, as in the
// reference scan starting from -inf at index 0.
__device__ __forceinline__ void argmax_take(float v, int i, float &bv, int &bi) {
    if (v > bv) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(1024) k_argmax_rows(const float *x, int len, uint32_t *out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *row = x + (long long)blockIdx.x * len;
    float bv = -INFINITY;
    int bi = INT_MAX;
    const int bd = blockDim.x;
    if ((len & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        // four 16-byte loads in flight per thread, taken in index order
        const float4 *r4 = reinterpret_cast<const float4 *>(row);
        const int n4 = len >> 2;
        int i = threadIdx.x;
        for (; i + 3 * bd < n4; i += 4 * bd) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = r4[i + u * bd];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int e = 4 * (i + u * bd);
                argmax_take(v[u].x, e, bv, bi);
                argmax_take(v[u].y, e + 1, bv, bi);
                argmax_take(v[u].z, e + 2, bv, bi);
                argmax_take(v[u].w, e + 3, bv, bi);
            }
        }
        for (; i < n4; i += bd) {
            const float4 v = r4[i];
            argmax_take(v.x, 4 * i, bv, bi);
            argmax_take(v.y, 4 * i + 1, bv, bi);
            argmax_take(v.z, 4 * i + 2, bv, bi);
            argmax_take(v.w, 4 * i + 3, bv, bi);
        }
    } else {
        for (int i = threadIdx.x; i < len; i += bd) argmax_take(row[i], i, bv, bi);
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

template <int HD>
cudaError_t launch_decode_reg(const DecodeAttnParams &p, int groups, cudaStream_t st) {
    const dim3 grid(p.n, p.kv_heads);
    switch (groups <= 1 ? 1 : groups <= 2 ? 2 : groups <= 4 ? 4 : 8) {
    case 1: k_attention_decode_reg<HD, 1><<<grid, kRegWarps * 32, 0, st>>>(p); break;
    case 2: k_attention_decode_reg<HD, 2><<<grid, kRegWarps * 32, 0, st>>>(p); break;
    case 4: k_attention_decode_reg<HD, 4><<<grid, kRegWarps * 32, 0, st>>>(p); break;
    default: k_attention_decode_reg<HD, 8><<<grid, kRegWarps * 32, 0, st>>>(p); break;
    }
    return cudaGetLastError();
}

cudaError_t attention_decode(const DecodeAttnParams &p, cudaStream_t st) {
    if (p.n <= 0) return cudaSuccess;
    if (p.heads % p.kv_heads) return cudaErrorInvalidValue;
    const int hd = p.head_dim, groups = p.heads / p.kv_heads;
    const bool aligned = (reinterpret_cast<uintptr_t>(p.cache_k) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(p.cache_v) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(p.qkv) & 15) == 0;
    if (!p.force_generic && aligned && groups <= 8) {
        if (hd == 128) return launch_decode_reg<128>(p, groups, st);
        if (hd == 64) return launch_decode_reg<64>(p, groups, st);
    }
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
    k_argmax_rows<<<n, 1024, 0, st>>>(x, len, out);
    return cudaGetLastError();
}

}  // namespace ditch
