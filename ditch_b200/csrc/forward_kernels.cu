// Forward-pass kernels around the GEMMs: embedding gather, RMSNorm with the
// residual capture fused in, causal GQA attention with RoPE and q/k norms,
// and the x . A row dot of a rank-1 delta.
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

// One warp per row. Token ids past the table set status (the reference's
// embedRowIndex error, src/model.zig:2547) and leave the row zero.
__global__ void k_embed(const void *table, int table_bf16, const uint32_t *tokens, int n, int hidden, float *x,
                        const int *cap_slot, float *res, int *status, int vocab) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const uint32_t t = tokens[row];
    float *xr = x + (long long)row * hidden;
    const int slot = cap_slot ? cap_slot[row] : -1;
    float *cr = slot >= 0 ? res + (long long)slot * hidden : nullptr;
    if (t >= (uint32_t)vocab) {
        if (lane == 0 && status) atomicExch(status, kKernelBadArgument);
        for (int i = lane; i < hidden; i += 32) xr[i] = 0.0f;
        return;
    }
    for (int i = lane; i < hidden; i += 32) {
        const float v = table_bf16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t *>(table)[(long long)t * hidden + i])
                                   : reinterpret_cast<const float *>(table)[(long long)t * hidden + i];
        xr[i] = v;
        if (cr) cr[i] = v;
    }
}

// RMSNorm of one f32 row (src/tensor.zig:1167-1179: inv = 1/sqrt(mean(x^2) + eps),
// out = x * inv * w) to bf16; the captured copy is the un-normalised row.
template <int HIDDEN_MAX>
__global__ void k_rmsnorm_bf16(const float *x, const float *w, int n, int hidden, float eps, uint16_t *h,
                               const int *cap_slot, float *res, const int *row_index) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const int src = row_index ? row_index[row] : row;
    const float *xr = x + (long long)src * hidden;
    float ss = 0.0f;
    if ((hidden & 3) == 0) {
        for (int i = lane * 4; i < hidden; i += 128) {
            float4 v = *reinterpret_cast<const float4 *>(xr + i);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int i = lane; i < hidden; i += 32) ss += xr[i] * xr[i];
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hidden + eps);
    uint16_t *hr = h + (long long)row * hidden;
    const int slot = cap_slot ? cap_slot[src] : -1;
    float *cr = slot >= 0 ? res + (long long)slot * hidden : nullptr;
    if ((hidden & 3) == 0) {  // four elements per lane and access
        for (int i = lane * 4; i < hidden; i += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + i);
            const float4 g = *reinterpret_cast<const float4 *>(w + i);
            uint2 o;
            o.x = pack_bf16x2(v.x * inv * g.x, v.y * inv * g.y);
            o.y = pack_bf16x2(v.z * inv * g.z, v.w * inv * g.w);
            *reinterpret_cast<uint2 *>(hr + i) = o;
            if (cr) *reinterpret_cast<float4 *>(cr + i) = v;
        }
        return;
    }
    for (int i = lane; i < hidden; i += 32) {
        const float v = xr[i];
        hr[i] = f32_to_bf16_bits(v * inv * w[i]);
        if (cr) cr[i] = v;
    }
}

__global__ void k_rmsnorm_f32(const float *x, const float *w, int n, int len, float eps, int gemma, float *out) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const float *xr = x + (long long)row * len;
    float ss = 0.0f;
    for (int i = lane; i < len; i += 32) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)len + eps);
    float *o = out + (long long)row * len;
    for (int i = lane; i < len; i += 32) {
        float v = xr[i] * inv;
        if (w) v *= gemma ? (1.0f + w[i]) : w[i];
        o[i] = v;
    }
}

// ---- attention ----------------------------------------------------------
// Block = (prompt, kv head). Keys and values of the prompt's rows for this kv
// head are roped / normed once into shared memory in chunks of kKeyChunk;
// each warp takes (query row, q head) pairs and runs an online softmax over
// the causal key range.
constexpr int kKeyChunk = 64;
constexpr int kAttnWarps = 8;

__device__ __forceinline__ void rope_neox_inplace(float *v, int hd, int pos, const float *cos_t, const float *sin_t,
                                                  int lane) {
    const int half = hd / 2;
    const float *c = cos_t + (long long)pos * half;
    const float *s = sin_t + (long long)pos * half;
    // lanes split the half; x1 = v[i], x2 = v[i + half]
    for (int i = lane; i < half; i += 32) {
        const float x1 = v[i], x2 = v[i + half];
        v[i] = x1 * c[i] - x2 * s[i];
        v[i + half] = x2 * c[i] + x1 * s[i];
    }
}

__device__ __forceinline__ void rms_inplace(float *v, int hd, const float *w, float eps, int lane) {
    float ss = 0.0f;
    for (int i = lane; i < hd; i += 32) ss += v[i] * v[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
    __syncwarp();
    for (int i = lane; i < hd; i += 32) v[i] = v[i] * inv * w[i];
    __syncwarp();
}

__global__ void __launch_bounds__(kAttnWarps * 32) k_attention(AttnParams p) {
    extern __shared__ float sm[];
    const int b = blockIdx.x, kvh = blockIdx.y;
    const int hd = p.head_dim, nh = p.heads, nkv = p.kv_heads;
    const int qd = nh * hd, kvd = nkv * hd, width = qd + 2 * kvd;
    const int groups = nh / nkv;
    const int start = p.seq_start[b], len = p.seq_len[b];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int ks = hd + 1;  // padded key stride (bank-conflict-free row reads)
    float *kbuf = sm;                                  // [kKeyChunk][hd + 1]
    float *vbuf = kbuf + kKeyChunk * ks;               // [kKeyChunk][hd]
    float *qbuf = vbuf + kKeyChunk * hd;               // [kAttnWarps][hd]
    float *pbuf = qbuf + kAttnWarps * hd;              // [kAttnWarps][kKeyChunk]
    float *obuf = pbuf + kAttnWarps * kKeyChunk;       // [kAttnWarps][hd] accumulators
    float *q = qbuf + warp * hd;
    float *pw = pbuf + warp * kKeyChunk;
    float *acc = obuf + warp * hd;

    // Each warp owns query tasks t = warp, warp + kAttnWarps, ... over (row, head in group).
    const int tasks = len * groups;
    for (int t0 = 0; t0 < tasks; t0 += kAttnWarps) {
        const int t = t0 + warp;
        const bool active = t < tasks;
        const int qi = active ? t / groups : 0;
        const int h = kvh * groups + (active ? t % groups : 0);
        float m = -INFINITY, l = 0.0f;
        if (active) {
            const float *src = p.qkv + (long long)(start + qi) * width + h * hd;
            for (int i = lane; i < hd; i += 32) {
                q[i] = src[i];
                acc[i] = 0.0f;
            }
            __syncwarp();
            if (p.q_norm) rms_inplace(q, hd, p.q_norm, p.eps, lane);
            rope_neox_inplace(q, hd, qi, p.rope_cos, p.rope_sin, lane);
            __syncwarp();
        }
        // The causal range of this batch of tasks spans keys [0, max qi].
        const int last_q = min(len - 1, (min(t0 + kAttnWarps, tasks) - 1) / groups);
        for (int k0 = 0; k0 <= last_q; k0 += kKeyChunk) {
            const int nk = min(kKeyChunk, last_q + 1 - k0);
            __syncthreads();
            // Stage roped / normed keys and values for this chunk (all warps).
            for (int kr = warp; kr < nk; kr += kAttnWarps) {
                const float *row = p.qkv + (long long)(start + k0 + kr) * width;
                float *kd = kbuf + kr * ks;
                for (int i = lane; i < hd; i += 32) {
                    kd[i] = row[qd + kvh * hd + i];
                    vbuf[kr * hd + i] = row[qd + kvd + kvh * hd + i];
                }
                __syncwarp();
                if (p.k_norm) rms_inplace(kd, hd, p.k_norm, p.eps, lane);
                rope_neox_inplace(kd, hd, k0 + kr, p.rope_cos, p.rope_sin, lane);
                __syncwarp();
            }
            __syncthreads();
            if (active && k0 <= qi) {
                const int nvalid = min(nk, qi - k0 + 1);
                // scores: lanes over keys
                float cmax = -INFINITY;
                for (int kr = lane; kr < kKeyChunk; kr += 32) {
                    float s = -INFINITY;
                    if (kr < nvalid) {
                        const float *kd = kbuf + kr * ks;
                        float d = 0.0f;
                        for (int i = 0; i < hd; i++) d = fmaf(q[i], kd[i], d);
                        s = d * p.scale;
                    }
                    pw[kr] = s;
                    cmax = fmaxf(cmax, s);
                }
                cmax = warp_max(cmax);
                const float mnew = fmaxf(m, cmax);
                const float corr = (m == -INFINITY) ? 0.0f : expf(m - mnew);
                float csum = 0.0f;
                for (int kr = lane; kr < kKeyChunk; kr += 32) {
                    const float e = kr < nvalid ? expf(pw[kr] - mnew) : 0.0f;
                    pw[kr] = e;
                    csum += e;
                }
                csum = warp_sum(csum);
                l = l * corr + csum;
                m = mnew;
                __syncwarp();
                for (int i = lane; i < hd; i += 32) {
                    float a = acc[i] * corr;
                    for (int kr = 0; kr < nvalid; kr++) a = fmaf(pw[kr], vbuf[kr * hd + i], a);
                    acc[i] = a;
                }
                __syncwarp();
            }
        }
        if (active) {
            const float inv = 1.0f / l;
            uint16_t *dst = p.out + (long long)(start + qi) * qd + h * hd;
            for (int i = lane; i < hd; i += 32) dst[i] = f32_to_bf16_bits(acc[i] * inv);
        }
        __syncwarp();
    }
}

// ---- q/k norm and RoPE, once per (token, head) ---------------------------
// Warp per (token, head slot) with the head's values in registers: lane l
// holds elements l, l + 32, ... (the order rms_inplace and rope_neox_inplace
// use), so the arithmetic is theirs. Applied in place to the q and k columns
// of the QKV rows before the tiled attention reads them.
template <int HD>
__global__ void __launch_bounds__(256) k_qk_prep(float *qkv, AttnParams p) {
    constexpr int V = HD / 32, H2 = V / 2;  // values per lane; pair (k, k + H2) = (i, i + HD / 2)
    const int b = blockIdx.x;
    const int start = p.seq_start[b], len = p.seq_len[b];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = blockIdx.y * 8 + warp;
    if (pos >= len) return;
    const int nh = p.heads, nkv = p.kv_heads;
    const int width = (nh + 2 * nkv) * HD;
    float *row = qkv + (long long)(start + pos) * width;
    const float *c = p.rope_cos + (long long)pos * (HD / 2);
    const float *sn = p.rope_sin + (long long)pos * (HD / 2);
    float cs[H2], ss[H2];
#pragma unroll
    for (int k = 0; k < H2; k++) {
        cs[k] = __ldg(c + lane + 32 * k);
        ss[k] = __ldg(sn + lane + 32 * k);
    }
    for (int slot = 0; slot < nh + nkv; slot++) {  // q heads, then k heads
        float *v = row + slot * HD;
        const float *nw = slot < nh ? p.q_norm : p.k_norm;
        float x[V];
#pragma unroll
        for (int k = 0; k < V; k++) x[k] = v[lane + 32 * k];
        if (nw) {
            float sq = 0.0f;
#pragma unroll
            for (int k = 0; k < V; k++) sq += x[k] * x[k];
            sq = warp_sum(sq);
            const float inv = 1.0f / sqrtf(sq / (float)HD + p.eps);
#pragma unroll
            for (int k = 0; k < V; k++) x[k] = x[k] * inv * __ldg(nw + lane + 32 * k);
        }
#pragma unroll
        for (int k = 0; k < H2; k++) {
            const float x1 = x[k], x2 = x[k + H2];
            x[k] = x1 * cs[k] - x2 * ss[k];
            x[k + H2] = x2 * cs[k] + x1 * ss[k];
        }
#pragma unroll
        for (int k = 0; k < V; k++) v[lane + 32 * k] = x[k];
    }
}

// ---- register-tiled attention for head_dim 64 / 128 ----------------------
// Block = (prompt, kv head and part of its group, chunk of 64 query
// positions); 256 threads; up to kMaxHeads query heads of the group one after
// another, so a prompt whose keys fit one 64-key chunk stages K and V once
// for them. Q (64 rows) and each
// 64-key chunk of K are staged transposed in f32 shared memory (rows across
// lanes: conflict-free), V natural, from rows already normed and roped.
// Scores: thread (ty, tx) owns queries 4ty..4ty+3 x keys 4tx..4tx+3 (two
// LDS.128 per 16 FMAs); the output: the same 4 queries x HD/16 dimensions
// (float4 groups tx, tx + 16, ..., so a quarter-warp's value loads are
// conflict-free). Online softmax across key chunks, f32.
constexpr int kQB = 64, kKB = 64;
constexpr int kMaxHeads = 4;  // query heads per block

template <int HD>
__global__ void __launch_bounds__(256) k_attention_tiled(AttnParams p) {
    extern __shared__ float sm[];
    float *qt = sm;                    // [HD][kQB]
    float *kt = qt + HD * kQB;         // [HD][kKB]
    float *vs = kt + HD * kKB;         // [kKB][HD]
    float *pt = vs + kKB * HD;         // [kKB][kQB]
    const int nh = p.heads, nkv = p.kv_heads, groups = nh / nkv;
    // blockIdx.y = (kv head, part): a group wider than kMaxHeads query heads
    // is split over several blocks (each stages its own K / V)
    const int parts = (groups + kMaxHeads - 1) / kMaxHeads;
    const int kvh = blockIdx.y / parts, part = blockIdx.y % parts;
    const int g0 = part * kMaxHeads, g1 = min(groups, g0 + kMaxHeads);
    const int b = blockIdx.x, i0 = blockIdx.z * kQB;
    const int start = p.seq_start[b], len = p.seq_len[b];
    if (i0 >= len) return;
    const int qd = nh * HD, kvd = nkv * HD, width = qd + 2 * kvd;
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    constexpr int DPT = HD / 16;  // output dimensions per thread
    constexpr int C4 = HD / 4;    // float4 per row
    const int last_q = min(len, i0 + kQB) - 1;  // causal: keys 0 .. last_q
    const bool one_chunk = last_q < kKB;

    for (int g = g0; g < g1; g++) {
        const int h = kvh * groups + g;
        __syncthreads();  // the previous head's reads of the buffers are done
        for (int idx = tid; idx < kQB * C4; idx += 256) {
            const int r = idx % kQB, c4 = idx / kQB, i = i0 + r;
            float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < len) q = *reinterpret_cast<const float4 *>(p.qkv + (long long)(start + i) * width + h * HD + 4 * c4);
            qt[(4 * c4 + 0) * kQB + r] = q.x;
            qt[(4 * c4 + 1) * kQB + r] = q.y;
            qt[(4 * c4 + 2) * kQB + r] = q.z;
            qt[(4 * c4 + 3) * kQB + r] = q.w;
        }
        float m[4], l[4], o[4][DPT];
#pragma unroll
        for (int a = 0; a < 4; a++) {
            m[a] = -INFINITY;
            l[a] = 0.0f;
#pragma unroll
            for (int c = 0; c < DPT; c++) o[a][c] = 0.0f;
        }
        for (int k0 = 0; k0 <= last_q; k0 += kKB) {
            if (!one_chunk || g == g0) {
                if (k0 > 0) __syncthreads();  // the previous chunk's reads of kt / vs / pt are done
                for (int idx = tid; idx < kKB * C4; idx += 256) {
                    const int r = idx % kKB, c4 = idx / kKB, j = k0 + r;
                    float4 k = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (j < len) k = *reinterpret_cast<const float4 *>(p.qkv + (long long)(start + j) * width + qd +
                                                                       kvh * HD + 4 * c4);
                    kt[(4 * c4 + 0) * kKB + r] = k.x;
                    kt[(4 * c4 + 1) * kKB + r] = k.y;
                    kt[(4 * c4 + 2) * kKB + r] = k.z;
                    kt[(4 * c4 + 3) * kKB + r] = k.w;
                }
                for (int idx = tid; idx < kKB * C4; idx += 256) {
                    const int r = idx / C4, c4 = idx % C4, j = k0 + r;
                    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (j < len) v = *reinterpret_cast<const float4 *>(p.qkv + (long long)(start + j) * width + qd +
                                                                       kvd + kvh * HD + 4 * c4);
                    *reinterpret_cast<float4 *>(vs + r * HD + 4 * c4) = v;
                }
            }
            __syncthreads();
            // scores of queries 4ty.. x keys 4tx..
            float s[4][4];
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int c = 0; c < 4; c++) s[a][c] = 0.0f;
#pragma unroll 8
            for (int d = 0; d < HD; d++) {
                const float4 qv = *reinterpret_cast<const float4 *>(qt + d * kQB + 4 * ty);
                const float4 kv = *reinterpret_cast<const float4 *>(kt + d * kKB + 4 * tx);
                const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int c = 0; c < 4; c++) s[a][c] = fmaf(qa[a], ka[c], s[a][c]);
            }
            float corr[4];
#pragma unroll
            for (int a = 0; a < 4; a++) {
                const int qi = i0 + 4 * ty + a;
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int kj = k0 + 4 * tx + c;
                    s[a][c] = (kj <= qi && kj < len) ? s[a][c] * p.scale : -INFINITY;
                    mx = fmaxf(mx, s[a][c]);
                }
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float mnew = fmaxf(m[a], mx);
                corr[a] = (m[a] == -INFINITY) ? 0.0f : expf(m[a] - mnew);
                float sum = 0.0f;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const float e = (s[a][c] == -INFINITY) ? 0.0f : expf(s[a][c] - mnew);
                    s[a][c] = e;
                    sum += e;
                }
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
                l[a] = l[a] * corr[a] + sum;
                m[a] = (mnew == -INFINITY) ? m[a] : mnew;
            }
            // P^T [key][query] for the value product
#pragma unroll
            for (int c = 0; c < 4; c++)
                *reinterpret_cast<float4 *>(pt + (4 * tx + c) * kQB + 4 * ty) =
                    make_float4(s[0][c], s[1][c], s[2][c], s[3][c]);
            __syncthreads();
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int c = 0; c < DPT; c++) o[a][c] *= corr[a];
            const int nk = min(kKB, last_q + 1 - k0);
            for (int k = 0; k < nk; k++) {
                const float4 pv = *reinterpret_cast<const float4 *>(pt + k * kQB + 4 * ty);
                const float pa[4] = {pv.x, pv.y, pv.z, pv.w};
                float vv[DPT];
#pragma unroll
                for (int c = 0; c < DPT; c += 4) {  // dimensions 4 (tx + 16 c/4) ..: a quarter-warp reads 128 B
                    const float4 t = *reinterpret_cast<const float4 *>(vs + k * HD + 4 * tx + 16 * c);
                    vv[c] = t.x;
                    vv[c + 1] = t.y;
                    vv[c + 2] = t.z;
                    vv[c + 3] = t.w;
                }
#pragma unroll
                for (int a = 0; a < 4; a++)
#pragma unroll
                    for (int c = 0; c < DPT; c++) o[a][c] = fmaf(pa[a], vv[c], o[a][c]);
            }
        }
#pragma unroll
        for (int a = 0; a < 4; a++) {
            const int qi = i0 + 4 * ty + a;
            if (qi >= len) continue;
            const float inv = 1.0f / l[a];
            uint16_t *dst = p.out + (long long)(start + qi) * qd + h * HD + 4 * tx;
#pragma unroll
            for (int c = 0; c < DPT; c += 4) {
                uint2 w;
                w.x = pack_bf16x2(o[a][c] * inv, o[a][c + 1] * inv);
                w.y = pack_bf16x2(o[a][c + 2] * inv, o[a][c + 3] * inv);
                *reinterpret_cast<uint2 *>(dst + 16 * c) = w;
            }
        }
    }
}

template <int HD>
cudaError_t launch_attention_tiled(const AttnParams &p, cudaStream_t st) {
    const size_t smem = sizeof(float) * (2 * HD * kQB + kKB * HD + kKB * kQB);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_tiled<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    int max_len = p.max_len > 0 ? p.max_len : kQB;
    // q / k norm and RoPE in place on the workspace rows (the buffer is the
    // forward's own QKV output, read only by this attention)
    k_qk_prep<HD><<<dim3(p.n_prompts, (max_len + 7) / 8), 256, 0, st>>>(const_cast<float *>(p.qkv), p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int groups = p.heads / p.kv_heads, parts = (groups + kMaxHeads - 1) / kMaxHeads;
    dim3 grid(p.n_prompts, p.kv_heads * parts, (max_len + kQB - 1) / kQB);
    k_attention_tiled<HD><<<grid, 256, smem, st>>>(p);
    return cudaGetLastError();
}

// xa[m] = sum_k act[m][k] * a[k], one warp per row.
__global__ void k_rowdot_bf16(const uint16_t *act, const float *a, int m, int k, float *xa) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= m) return;
    const uint16_t *r = act + (long long)row * k;
    float s = 0.0f;
    if ((k & 7) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(act) & 15) == 0) {
        // four 16-byte loads in flight per lane, four independent sums
        float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int i = lane * 8;
        for (; i + 3 * 256 < k; i += 4 * 256) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = __ldg(reinterpret_cast<const uint4 *>(r + i + u * 256));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                const float4 a0 = __ldg(reinterpret_cast<const float4 *>(a + i + u * 256));
                const float4 a1 = __ldg(reinterpret_cast<const float4 *>(a + i + u * 256 + 4));
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    t[u] = fmaf(__uint_as_float(w[j] << 16), av[2 * j], t[u]);
                    t[u] = fmaf(__uint_as_float(w[j] & 0xffff0000u), av[2 * j + 1], t[u]);
                }
            }
        }
        for (; i < k; i += 256) {
            uint4 v = __ldg(reinterpret_cast<const uint4 *>(r + i));
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                t[0] = fmaf(__uint_as_float(w[j] << 16), a[i + 2 * j], t[0]);
                t[0] = fmaf(__uint_as_float(w[j] & 0xffff0000u), a[i + 2 * j + 1], t[0]);
            }
        }
        s = (t[0] + t[1]) + (t[2] + t[3]);
    } else {
        for (int i = lane; i < k; i += 32) s = fmaf(bf16_bits_to_f32(r[i]), a[i], s);
    }
    s = warp_sum(s);
    if (lane == 0) xa[row] = s;
}

}  // namespace

cudaError_t embed_rows(const void *table, int table_bf16, const uint32_t *tokens, int n, int hidden, float *x,
                       const int *cap_slot, float *res, int *status, int vocab, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_embed<<<(n + 7) / 8, 256, 0, st>>>(table, table_bf16, tokens, n, hidden, x, cap_slot, res, status, vocab);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows_bf16(const float *x, const float *w, int n, int hidden, float eps, uint16_t *h,
                              const int *cap_slot, float *res, const int *row_index, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_rmsnorm_bf16<0><<<(n + 7) / 8, 256, 0, st>>>(x, w, n, hidden, eps, h, cap_slot, res, row_index);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows_f32(const float *x, const float *w, int n, int len, float eps, int gemma, float *out,
                             cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_rmsnorm_f32<<<(n + 7) / 8, 256, 0, st>>>(x, w, n, len, eps, gemma, out);
    return cudaGetLastError();
}

cudaError_t gather_rmsnorm_bf16(const float *x, const int *rows, int n, int hidden, float eps, const float *w,
                                uint16_t *h, cudaStream_t st) {
    return rmsnorm_rows_bf16(x, w, n, hidden, eps, h, nullptr, nullptr, rows, st);
}

cudaError_t attention_prefill(const AttnParams &p, cudaStream_t st) {
    if (p.n_prompts <= 0) return cudaSuccess;
    if (p.heads % p.kv_heads) return cudaErrorInvalidValue;
    const int hd = p.head_dim;
    if (hd == 128 && !p.force_generic) return launch_attention_tiled<128>(p, st);
    if (hd == 64 && !p.force_generic) return launch_attention_tiled<64>(p, st);
    // other head sizes: one warp per (query, head) with an online softmax
    const size_t smem = sizeof(float) * (kKeyChunk * (hd + 1) + kKeyChunk * hd + kAttnWarps * hd +
                                         kAttnWarps * kKeyChunk + kAttnWarps * hd);
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    dim3 grid(p.n_prompts, p.kv_heads);
    k_attention<<<grid, kAttnWarps * 32, smem, st>>>(p);
    return cudaGetLastError();
}

cudaError_t rowdot_bf16(const uint16_t *act, const float *a, int m, int k, float *xa, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    k_rowdot_bf16<<<(m + 7) / 8, 256, 0, st>>>(act, a, m, k, xa);
    return cudaGetLastError();
}

}  // namespace ditch
