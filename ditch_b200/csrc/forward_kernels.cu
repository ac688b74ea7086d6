// Forward-pass kernels around the GEMMs: embedding gather, RMSNorm with the
// residual capture fused in, causal GQA attention with RoPE and q/k norms,
// and the x . A row dot of a rank-1 delta.
#include "attn_common.cuh"
#include "kernels.cuh"

namespace ditch {

namespace {

using attn::warp_max;
using attn::warp_sum;
using attn::rope_neox_inplace;
using attn::rms_inplace;

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
    if (table_bf16 && (hidden & 3) == 0 &&
        ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(res)) & 15) ==
            0) {
        // four elements per lane and access: 8-byte reads of the bf16 row, 16-byte writes
        const uint2 *tr = reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(table) + (long long)t * hidden);
        for (int i = lane; i < hidden / 4; i += 32) {
            const uint2 q = __ldg(tr + i);
            const float4 v = make_float4(__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xffff0000u),
                                         __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xffff0000u));
            reinterpret_cast<float4 *>(xr)[i] = v;
            if (cr) reinterpret_cast<float4 *>(cr)[i] = v;
        }
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
                               const int *cap_slot, float *res, const int *row_index, int split_k) {
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
    const int slot = cap_slot ? cap_slot[src] : -1;
    float *cr = slot >= 0 ? res + (long long)slot * hidden : nullptr;
    if (split_k > 0) {  // f32-level operand: [hi | hi | lo] segments of split_k columns (padding zero)
        uint16_t *hr = h + (long long)row * 3 * split_k;
        for (int i = lane; i < split_k; i += 32) {
            const float v = i < hidden ? xr[i] : 0.0f;
            const float y = i < hidden ? v * inv * w[i] : 0.0f;
            const uint16_t hi = f32_to_bf16_bits(y);
            hr[i] = hi;
            hr[split_k + i] = hi;
            hr[2 * split_k + i] = f32_to_bf16_bits(y - bf16_bits_to_f32(hi));
            if (cr && i < hidden) cr[i] = v;
        }
        return;
    }
    uint16_t *hr = h + (long long)row * hidden;
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

// The same RMSNorm with a block per row and the row held in registers (up
// to 8 float4 per thread, element i = 4 (v blockDim + tid) + e): x is read
// once, where the warp-per-row form above reads it twice (once for the sum
// of squares, once for the output, the second mostly missing L1 at 16 KB
// per row). hidden a multiple of 4, at most 32 x blockDim.
__global__ void __launch_bounds__(1024) k_rmsnorm_row(const float *x, const float *w, int hidden, float eps,
                                                      uint16_t *h, const int *cap_slot, float *res,
                                                      const int *row_index) {
    __shared__ float sh[32];
    const int row = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
    const int src = row_index ? row_index[row] : row;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (long long)src * hidden);
    const int n4 = hidden / 4;
    float4 v[8];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = k * nt + tid;
        v[k] = i < n4 ? xr[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int k = 0; k < 8; k++) ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
    ss = warp_sum(ss);
    if ((tid & 31) == 0) sh[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < (nt + 31) / 32; k++) tot += sh[k];
    const float inv = 1.0f / sqrtf(tot / (float)hidden + eps);
    const int slot = cap_slot ? cap_slot[src] : -1;
    float4 *cr = slot >= 0 ? reinterpret_cast<float4 *>(res + (long long)slot * hidden) : nullptr;
    uint2 *hr = reinterpret_cast<uint2 *>(h + (long long)row * hidden);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = k * nt + tid;
        if (i >= n4) break;
        const float4 g = __ldg(w4 + i);
        uint2 o;
        o.x = pack_bf16x2(v[k].x * inv * g.x, v[k].y * inv * g.y);
        o.y = pack_bf16x2(v[k].z * inv * g.z, v[k].w * inv * g.w);
        hr[i] = o;
        if (cr) cr[i] = v[k];
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
            if (p.out_f32) {
                float *dst = p.out_f32 + (long long)(start + qi) * qd + h * hd;
                for (int i = lane; i < hd; i += 32) dst[i] = acc[i] * inv;
            } else {
                uint16_t *dst = p.out + (long long)(start + qi) * qd + h * hd;
                for (int i = lane; i < hd; i += 32) dst[i] = f32_to_bf16_bits(acc[i] * inv);
            }
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
    // q heads, then k heads; the next head's values load while this one is
    // normed and rotated
    const int slots = nh + nkv;
    float xn[V];
#pragma unroll
    for (int k = 0; k < V; k++) xn[k] = row[lane + 32 * k];
    for (int slot = 0; slot < slots; slot++) {
        float *v = row + slot * HD;
        const float *nw = slot < nh ? p.q_norm : p.k_norm;
        float x[V];
#pragma unroll
        for (int k = 0; k < V; k++) x[k] = xn[k];
        if (slot + 1 < slots)
#pragma unroll
            for (int k = 0; k < V; k++) xn[k] = v[HD + lane + 32 * k];
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

// ---- tensor-core attention for head_dim 64 / 128 -------------------------
// Block = (prompt, kv head and part of its group, chunk of 64 query
// positions); 4 warps, warp w owns query rows 16w .. 16w + 15 of the chunk.
// Up to kMaxHeads query heads of the group run one after another, so a prompt
// whose keys fit one 64-key chunk stages K and V once for them. Q, K and V
// (already normed and roped by k_qk_prep) are staged in shared memory as
// bf16 pairs x = hi + lo (hi = bf16(x), lo = bf16(x - hi)); every product is
// hi*hi + hi*lo + lo*hi on mma.sync m16n8k16 with f32 accumulation, which
// keeps the scores and the P.V sums to about 2^-16 relative (f32-like). The
// scores never leave registers: the S accumulator fragments are the A
// operand of the P.V product. Online softmax in f32 across key chunks; the
// causal limit skips the 8-key tiles and 16-key steps above each warp's rows.
constexpr int kQB = 64, kKB = 64;
constexpr int kMaxHeads = 4;  // query heads per block
constexpr int kBatch = 4;     // staging loads in flight per thread

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (a, b) -> bf16x2 hi and the bf16x2 of the remainders (low half = a).
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
    hi = pack_bf16x2(a, b);
    const float ah = __uint_as_float(hi << 16), bh = __uint_as_float(hi & 0xffff0000u);
    lo = pack_bf16x2(a - ah, b - bh);
}

template <int HD>
__global__ void __launch_bounds__(128) k_attention_mma(AttnParams p) {
    constexpr int QS = HD + 8;   // row stride (bf16) of the Q and K tiles: conflict-free fragment loads
    constexpr int VS = kKB + 8;  // row stride of the transposed V tile
    constexpr int C4 = HD / 4;
    extern __shared__ __align__(16) uint16_t smb[];
    uint16_t *qh = smb, *ql = qh + kQB * QS;
    uint16_t *kh = ql + kQB * QS, *kl = kh + kKB * QS;
    uint16_t *vh = kl + kKB * QS, *vl = vh + HD * VS;  // [dim][key]
    const int nh = p.heads, nkv = p.kv_heads, groups = nh / nkv;
    const int parts = (groups + kMaxHeads - 1) / kMaxHeads;
    const int kvh = blockIdx.y / parts, part = blockIdx.y % parts;
    const int gh0 = part * kMaxHeads, gh1 = min(groups, gh0 + kMaxHeads);
    const int b = blockIdx.x, i0 = blockIdx.z * kQB;
    const int start = p.seq_start[b], len = p.seq_len[b];
    if (i0 >= len) return;
    const int qd = nh * HD, kvd = nkv * HD, width = qd + 2 * kvd;
    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int r0 = 16 * w;                      // this warp's first row in the chunk
    const int last_q = min(len, i0 + kQB) - 1;  // causal: keys 0 .. last_q
    const bool one_chunk = last_q < kKB;
    const int row_a = i0 + r0 + g, row_b = row_a + 8;            // this thread's two query positions
    const int warp_last = min(i0 + r0 + 15, len - 1);            // last query position of the warp

    auto ld32 = [](const uint16_t *p_) { return *reinterpret_cast<const uint32_t *>(p_); };

    for (int gh = gh0; gh < gh1; gh++) {
        const int h = kvh * groups + gh;
        __syncthreads();  // the previous head's reads of the buffers are done
        // staging: kBatch loads in flight per thread before their conversions
        // (a load per conversion waits one memory round trip each)
#pragma unroll
        for (int b0 = 0; b0 < kQB * C4 / 128; b0 += kBatch) {
            float4 q[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; u++) {
                const int idx = tid + 128 * (b0 + u), r = idx / C4, c4 = idx % C4, i = i0 + r;
                q[u] = i < len ? *reinterpret_cast<const float4 *>(p.qkv + (long long)(start + i) * width + h * HD + 4 * c4)
                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < kBatch; u++) {
                const int idx = tid + 128 * (b0 + u), r = idx / C4, c4 = idx % C4;
                uint2 hi, lo;
                split_bf16x2(q[u].x, q[u].y, hi.x, lo.x);
                split_bf16x2(q[u].z, q[u].w, hi.y, lo.y);
                *reinterpret_cast<uint2 *>(qh + r * QS + 4 * c4) = hi;
                *reinterpret_cast<uint2 *>(ql + r * QS + 4 * c4) = lo;
            }
        }
        float o[HD / 8][4];
#pragma unroll
        for (int d = 0; d < HD / 8; d++) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;
        float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;

        for (int k0 = 0; k0 <= last_q; k0 += kKB) {
            if (!one_chunk || gh == gh0) {
                if (k0 > 0) __syncthreads();  // the previous chunk's reads of the K / V tiles are done
#pragma unroll
                for (int b0 = 0; b0 < kKB * C4 / 128; b0 += kBatch) {
                    float4 k[kBatch];
#pragma unroll
                    for (int u = 0; u < kBatch; u++) {
                        const int idx = tid + 128 * (b0 + u), r = idx / C4, c4 = idx % C4, j = k0 + r;
                        k[u] = j < len ? *reinterpret_cast<const float4 *>(p.qkv + (long long)(start + j) * width + qd +
                                                                           kvh * HD + 4 * c4)
                                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    }
#pragma unroll
                    for (int u = 0; u < kBatch; u++) {
                        const int idx = tid + 128 * (b0 + u), r = idx / C4, c4 = idx % C4;
                        uint2 hi, lo;
                        split_bf16x2(k[u].x, k[u].y, hi.x, lo.x);
                        split_bf16x2(k[u].z, k[u].w, hi.y, lo.y);
                        *reinterpret_cast<uint2 *>(kh + r * QS + 4 * c4) = hi;
                        *reinterpret_cast<uint2 *>(kl + r * QS + 4 * c4) = lo;
                    }
                }
#pragma unroll
                for (int b0 = 0; b0 < kKB * C4 / 128; b0 += kBatch) {  // keys across lanes: conflict-free transposed stores
                    float4 v[kBatch];
#pragma unroll
                    for (int u = 0; u < kBatch; u++) {
                        const int idx = tid + 128 * (b0 + u), r = idx % kKB, c4 = idx / kKB, j = k0 + r;
                        v[u] = j < len ? *reinterpret_cast<const float4 *>(p.qkv + (long long)(start + j) * width + qd +
                                                                           kvd + kvh * HD + 4 * c4)
                                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    }
#pragma unroll
                    for (int u = 0; u < kBatch; u++) {
                        const int idx = tid + 128 * (b0 + u), r = idx % kKB, c4 = idx / kKB;
                        const float vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const uint16_t hb = f32_to_bf16_bits(vv[e]);
                            vh[(4 * c4 + e) * VS + r] = hb;
                            vl[(4 * c4 + e) * VS + r] = f32_to_bf16_bits(vv[e] - bf16_bits_to_f32(hb));
                        }
                    }
                }
            }
            __syncthreads();
            // 8-key tiles this warp needs (causal limit) and the 16-key steps of P . V
            const int nt = max(0, min(8, (warp_last - k0) / 8 + 1));
            float s[8][4];
#pragma unroll
            for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < HD / 16; kk++) {
                const int c = 16 * kk + 2 * t;
                const uint32_t ah0 = ld32(qh + (r0 + g) * QS + c), ah1 = ld32(qh + (r0 + g + 8) * QS + c);
                const uint32_t ah2 = ld32(qh + (r0 + g) * QS + c + 8), ah3 = ld32(qh + (r0 + g + 8) * QS + c + 8);
                const uint32_t al0 = ld32(ql + (r0 + g) * QS + c), al1 = ld32(ql + (r0 + g + 8) * QS + c);
                const uint32_t al2 = ld32(ql + (r0 + g) * QS + c + 8), al3 = ld32(ql + (r0 + g + 8) * QS + c + 8);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (j < nt) {
                        const uint32_t bh0 = ld32(kh + (8 * j + g) * QS + c), bh1 = ld32(kh + (8 * j + g) * QS + c + 8);
                        const uint32_t bl0 = ld32(kl + (8 * j + g) * QS + c), bl1 = ld32(kl + (8 * j + g) * QS + c + 8);
                        mma_bf16_16816(s[j], ah0, ah1, ah2, ah3, bh0, bh1);
                        mma_bf16_16816(s[j], ah0, ah1, ah2, ah3, bl0, bl1);
                        mma_bf16_16816(s[j], al0, al1, al2, al3, bh0, bh1);
                    }
                }
            }
            // scale, causal mask, online softmax (rows row_a: s[j][0..1], row_b: s[j][2..3])
            float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; j++) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int key = k0 + 8 * j + 2 * t + (e & 1);
                    const int row = (e < 2) ? row_a : row_b;
                    const bool ok = j < nt && key <= row && key < len;
                    s[j][e] = ok ? s[j][e] * p.scale : -INFINITY;
                }
                mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
                mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
            }
#pragma unroll
            for (int off = 1; off < 4; off <<= 1) {
                mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
                mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
            }
            const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
            const float corr_a = (m_a == -INFINITY) ? 0.0f : expf(m_a - mn_a);
            const float corr_b = (m_b == -INFINITY) ? 0.0f : expf(m_b - mn_b);
            float sum_a = 0.0f, sum_b = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float mref = e < 2 ? mn_a : mn_b;
                    const float pe = (s[j][e] == -INFINITY) ? 0.0f : expf(s[j][e] - mref);
                    s[j][e] = pe;
                    if (e < 2) sum_a += pe;
                    else sum_b += pe;
                }
            }
#pragma unroll
            for (int off = 1; off < 4; off <<= 1) {
                sum_a += __shfl_xor_sync(0xffffffffu, sum_a, off);
                sum_b += __shfl_xor_sync(0xffffffffu, sum_b, off);
            }
            l_a = l_a * corr_a + sum_a;
            l_b = l_b * corr_b + sum_b;
            m_a = (mn_a == -INFINITY) ? m_a : mn_a;
            m_b = (mn_b == -INFINITY) ? m_b : mn_b;
#pragma unroll
            for (int d = 0; d < HD / 8; d++) {
                o[d][0] *= corr_a;
                o[d][1] *= corr_a;
                o[d][2] *= corr_b;
                o[d][3] *= corr_b;
            }
            // O += P . V over the 16-key steps this warp needs
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                if (2 * kk >= nt) break;
                uint32_t ph0, ph1, ph2, ph3, pl0, pl1, pl2, pl3;
                split_bf16x2(s[2 * kk][0], s[2 * kk][1], ph0, pl0);
                split_bf16x2(s[2 * kk][2], s[2 * kk][3], ph1, pl1);
                split_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1], ph2, pl2);
                split_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3], ph3, pl3);
                const int c = 16 * kk + 2 * t;
#pragma unroll
                for (int d = 0; d < HD / 8; d++) {
                    const uint16_t *vrh = vh + (8 * d + g) * VS, *vrl = vl + (8 * d + g) * VS;
                    const uint32_t bh0 = ld32(vrh + c), bh1 = ld32(vrh + c + 8);
                    const uint32_t bl0 = ld32(vrl + c), bl1 = ld32(vrl + c + 8);
                    mma_bf16_16816(o[d], ph0, ph1, ph2, ph3, bh0, bh1);
                    mma_bf16_16816(o[d], ph0, ph1, ph2, ph3, bl0, bl1);
                    mma_bf16_16816(o[d], pl0, pl1, pl2, pl3, bh0, bh1);
                }
            }
        }
        const float inv_a = 1.0f / l_a, inv_b = 1.0f / l_b;
#pragma unroll
        for (int d = 0; d < HD / 8; d++) {
            const int dim = h * HD + 8 * d + 2 * t;
            if (p.out_f32) {
                if (row_a < len)
                    *reinterpret_cast<float2 *>(p.out_f32 + (long long)(start + row_a) * qd + dim) =
                        make_float2(o[d][0] * inv_a, o[d][1] * inv_a);
                if (row_b < len)
                    *reinterpret_cast<float2 *>(p.out_f32 + (long long)(start + row_b) * qd + dim) =
                        make_float2(o[d][2] * inv_b, o[d][3] * inv_b);
                continue;
            }
            if (row_a < len)
                *reinterpret_cast<uint32_t *>(p.out + (long long)(start + row_a) * qd + dim) =
                    pack_bf16x2(o[d][0] * inv_a, o[d][1] * inv_a);
            if (row_b < len)
                *reinterpret_cast<uint32_t *>(p.out + (long long)(start + row_b) * qd + dim) =
                    pack_bf16x2(o[d][2] * inv_b, o[d][3] * inv_b);
        }
    }
}

template <int HD>
cudaError_t launch_attention_tiled(const AttnParams &p, cudaStream_t st) {
    const size_t smem = sizeof(uint16_t) * (2 * kQB * (HD + 8) + 2 * kKB * (HD + 8) + 2 * HD * (kKB + 8));
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_mma<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
    if (attention_tc_eligible(p)) return attention_tc(p, st);
    const int groups = p.heads / p.kv_heads, parts = (groups + kMaxHeads - 1) / kMaxHeads;
    dim3 grid(p.n_prompts, p.kv_heads * parts, (max_len + kQB - 1) / kQB);
    k_attention_mma<HD><<<grid, 128, smem, st>>>(p);
    return cudaGetLastError();
}

// xa[m] = sum_k act[m][k] * a[k], one warp per row.
__global__ void k_rowdot_bf16(const uint16_t *act, const float *a, int m, int k, float *xa, int stride) {
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
    if (lane == 0) xa[(long long)row * stride] = s;
}

// The same dot products, four rows per warp: each lane's eight values of `a`
// are loaded once and used against the four rows, so the vector costs half a
// byte of L1 traffic per activation byte instead of two. Needs k % 8 == 0 and
// 16-byte aligned act and a. Rows past m repeat the last row and are not
// stored.
constexpr int kDotRows = 4;
__global__ void __launch_bounds__(128) k_rowdot_bf16_rows(const uint16_t *act, const float *a, int m, int k,
                                                          float *xa, int stride) {
    const int row0 = (blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * kDotRows;
    const int lane = threadIdx.x & 31;
    if (row0 >= m) return;
    const uint16_t *r[kDotRows];
#pragma unroll
    for (int q = 0; q < kDotRows; q++) r[q] = act + (long long)min(row0 + q, m - 1) * k;
    float t[kDotRows][2] = {};
    int i = lane * 8;
    for (; i + 256 < k; i += 2 * 256) {
        uint4 v[2][kDotRows];
#pragma unroll
        for (int u = 0; u < 2; u++)
#pragma unroll
            for (int q = 0; q < kDotRows; q++) v[u][q] = __ldg(reinterpret_cast<const uint4 *>(r[q] + i + u * 256));
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const float4 a0 = __ldg(reinterpret_cast<const float4 *>(a + i + u * 256));
            const float4 a1 = __ldg(reinterpret_cast<const float4 *>(a + i + u * 256 + 4));
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int q = 0; q < kDotRows; q++) {
                const uint32_t w[4] = {v[u][q].x, v[u][q].y, v[u][q].z, v[u][q].w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    t[q][u] = fmaf(__uint_as_float(w[j] << 16), av[2 * j], t[q][u]);
                    t[q][u] = fmaf(__uint_as_float(w[j] & 0xffff0000u), av[2 * j + 1], t[q][u]);
                }
            }
        }
    }
    if (i < k) {
        const float4 a0 = __ldg(reinterpret_cast<const float4 *>(a + i));
        const float4 a1 = __ldg(reinterpret_cast<const float4 *>(a + i + 4));
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int q = 0; q < kDotRows; q++) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(r[q] + i));
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                t[q][0] = fmaf(__uint_as_float(w[j] << 16), av[2 * j], t[q][0]);
                t[q][0] = fmaf(__uint_as_float(w[j] & 0xffff0000u), av[2 * j + 1], t[q][0]);
            }
        }
    }
#pragma unroll
    for (int q = 0; q < kDotRows; q++) {
        const float s = warp_sum(t[q][0] + t[q][1]);
        if (lane == 0 && row0 + q < m) xa[(long long)(row0 + q) * stride] = s;
    }
}

cudaError_t launch_rowdot_bf16(const uint16_t *act, const float *a, int m, int k, float *xa, int stride,
                               cudaStream_t st) {
    if ((k & 7) == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(act)) & 15) == 0) {
        const int warps = (m + kDotRows - 1) / kDotRows;
        k_rowdot_bf16_rows<<<(warps + 3) / 4, 128, 0, st>>>(act, a, m, k, xa, stride);
    } else {
        k_rowdot_bf16<<<(m + 7) / 8, 256, 0, st>>>(act, a, m, k, xa, stride);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t embed_rows(const void *table, int table_bf16, const uint32_t *tokens, int n, int hidden, float *x,
                       const int *cap_slot, float *res, int *status, int vocab, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_embed<<<(n + 7) / 8, 256, 0, st>>>(table, table_bf16, tokens, n, hidden, x, cap_slot, res, status, vocab);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows_bf16(const float *x, const float *w, int n, int hidden, float eps, uint16_t *h,
                              const int *cap_slot, float *res, const int *row_index, cudaStream_t st, int split_k) {
    if (n <= 0) return cudaSuccess;
    const int nt = ((hidden + 31) / 32 + 31) / 32 * 32;  // threads: 32 elements each, whole warps
    if (split_k == 0 && (hidden & 3) == 0 && nt <= 1024 &&
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(h) |
          reinterpret_cast<uintptr_t>(res)) & 15) == 0) {
        k_rmsnorm_row<<<n, nt, 0, st>>>(x, w, hidden, eps, h, cap_slot, res, row_index);
        return cudaGetLastError();
    }
    k_rmsnorm_bf16<0><<<(n + 7) / 8, 256, 0, st>>>(x, w, n, hidden, eps, h, cap_slot, res, row_index, split_k);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows_f32(const float *x, const float *w, int n, int len, float eps, int gemma, float *out,
                             cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_rmsnorm_f32<<<(n + 7) / 8, 256, 0, st>>>(x, w, n, len, eps, gemma, out);
    return cudaGetLastError();
}

cudaError_t gather_rmsnorm_bf16(const float *x, const int *rows, int n, int hidden, float eps, const float *w,
                                uint16_t *h, cudaStream_t st, int split_k) {
    return rmsnorm_rows_bf16(x, w, n, hidden, eps, h, nullptr, nullptr, rows, st, split_k);
}

bool attention_prefill_preps_in_place(int head_dim, int force_generic) {
    return !force_generic && (head_dim == 128 || head_dim == 64);
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
    return launch_rowdot_bf16(act, a, m, k, xa, 1, st);
}

cudaError_t rowdot_bf16_strided(const uint16_t *act, const float *a, int m, int k, float *xa, int stride,
                                cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    return launch_rowdot_bf16(act, a, m, k, xa, stride, st);
}

// ---- split operands -------------------------------------------------------
namespace {

__device__ __forceinline__ void split_store(uint16_t *row, int kp, int c, float v, bool weight) {
    const uint16_t hi = f32_to_bf16_bits(v);
    const uint16_t lo = f32_to_bf16_bits(v - bf16_bits_to_f32(hi));
    row[c] = hi;
    row[kp + c] = weight ? lo : hi;
    row[2 * kp + c] = weight ? hi : lo;
}

// One thread per (row, column < kp); columns past k are zero.
__global__ void k_split_rows(const float *x, long long rows, int k, int kp, uint16_t *out, bool weight) {
    const long long total = rows * kp;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / kp;
        const int c = (int)(e - r * kp);
        split_store(out + r * 3 * kp, kp, c, c < k ? x[r * k + c] : 0.0f, weight);
    }
}

// silu(g) * u with the scalar exp (src/tensor.zig:1212-1214, 1334-1337).
__global__ void k_swiglu_split(const float *gu, long long n, int inter, int kp, float *act32, uint16_t *act) {
    const long long total = n * kp;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / kp;
        const int c = (int)(e - r * kp);
        float y = 0.0f;
        if (c < inter) {
            const float g = gu[r * 2 * inter + c], u = gu[r * 2 * inter + inter + c];
            y = g / (1.0f + expf(-g)) * u;
        }
        act32[r * kp + c] = y;
        split_store(act + r * 3 * kp, kp, c, y, false);
    }
}

// Warp per row.
__global__ void k_rowdot_f32(const float *x, const float *a, int m, int k, float *xa, int stride) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= m) return;
    const float *xr = x + (long long)row * k;
    float s = 0.0f;
    for (int i = lane; i < k; i += 32) s = fmaf(xr[i], a[i], s);
    s = warp_sum(s);
    if (lane == 0) xa[(long long)row * stride] = s;
}

__global__ void k_add_split_halves(const float *s, int kp, float *out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < kp) out[c] = s[c] + s[kp + c];
}

__global__ void k_merge_split(const uint16_t *split, long long rows, int kp, float *out) {
    const long long total = rows * kp;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / kp;
        const int c = (int)(e - r * kp);
        const uint16_t *row = split + r * 3 * kp;
        out[e] = bf16_bits_to_f32(row[c]) + bf16_bits_to_f32(row[kp + c]);
    }
}

int grid_for(long long total) { return (int)std::min<long long>((total + 255) / 256, 148LL * 16); }

}  // namespace

cudaError_t split_weight_rows(const float *w, int rows, int k, int kp, uint16_t *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_split_rows<<<grid_for((long long)rows * kp), 256, 0, st>>>(w, rows, k, kp, out, true);
    return cudaGetLastError();
}

cudaError_t split_act_rows(const float *x, int n, int k, int kp, uint16_t *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_split_rows<<<grid_for((long long)n * kp), 256, 0, st>>>(x, n, k, kp, out, false);
    return cudaGetLastError();
}

cudaError_t swiglu_split(const float *gu, int n, int inter, int kp, float *act32, uint16_t *act, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_swiglu_split<<<grid_for((long long)n * kp), 256, 0, st>>>(gu, n, inter, kp, act32, act);
    return cudaGetLastError();
}

cudaError_t rowdot_f32_strided(const float *x, const float *a, int m, int k, float *xa, int stride, cudaStream_t st) {
    if (m <= 0) return cudaSuccess;
    k_rowdot_f32<<<(m + 7) / 8, 256, 0, st>>>(x, a, m, k, xa, stride);
    return cudaGetLastError();
}

cudaError_t merge_split_rows(const uint16_t *split, int rows, int kp, float *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_merge_split<<<grid_for((long long)rows * kp), 256, 0, st>>>(split, rows, kp, out);
    return cudaGetLastError();
}

cudaError_t add_split_halves(const float *s, int kp, float *out, cudaStream_t st) {
    if (kp <= 0) return cudaSuccess;
    k_add_split_halves<<<(kp + 255) / 256, 256, 0, st>>>(s, kp, out);
    return cudaGetLastError();
}

}  // namespace ditch
