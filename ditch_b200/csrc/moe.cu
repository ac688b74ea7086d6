// Routed-expert MLP (src/moe.zig:998-1228, softmax top-k path) on the device:
//   1. router logits as a split-bf16 tcgen05 GEMM (about 2^-16 relative, so
//      the top-k picks agree with ditch's f32 router but for exact ties);
//   2. per token: softmax, top-k (the first maximum wins ties,
//      src/moe.zig:971-985), renormalisation (norm_topk_prob);
//   3. a stable counting sort of the (token, slot) pairs by expert: experts in
//      index order, tokens in order within an expert (the reference's
//      gather order, src/moe.zig:1144-1152);
//   4. the expert MLPs as two grouped GEMMs over the sorted rows (SwiGLU
//      gate/up with the decode of MXFP4 / FP8 / INT4 experts fused into the
//      operand load, then down with the per-expert rank-1 delta);
//   5. the weighted combine, each token's experts summed in index order
//      (acc += w * out, src/moe.zig:1197-1199), added to the residual.
#include <algorithm>

#include "model.cuh"

namespace ditch {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// RMSNorm (src/tensor.zig:1167-1179) written as [hi | hi | lo] bf16 segments
// of width cp: the activation side of the split-precision router product.
__global__ void k_rmsnorm_split3(const float *x, const float *w, int n, int hidden, int cp, float eps, uint16_t *h3) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const float *xr = x + (long long)row * hidden;
    float ss = 0.0f;
    for (int i = lane; i < hidden; i += 32) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)hidden + eps);
    uint16_t *o = h3 + (long long)row * 3 * cp;
    for (int i = lane; i < cp; i += 32) {
        uint16_t hi = 0, lo = 0;
        if (i < hidden) {
            const float v = xr[i] * inv * w[i];
            hi = f32_to_bf16_bits(v);
            lo = f32_to_bf16_bits(v - bf16_bits_to_f32(hi));
        }
        o[i] = hi;
        o[cp + i] = hi;
        o[2 * cp + i] = lo;
    }
}

// Softmax over the E router logits, top-k, renormalisation; one warp per token.
constexpr int kMaxExpertsPerLane = 32;  // E <= 1024

__global__ void k_route(const float *logits, int n, int E, int k, int norm_topk, int *sel, float *wts) {
    const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (t >= n) return;
    const float *row = logits + (long long)t * E;
    float p[kMaxExpertsPerLane];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; j++) {
        const int e = j * 32 + lane;
        p[j] = e < E ? row[e] : -INFINITY;
        m = fmaxf(m, p[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; j++) {
        const int e = j * 32 + lane;
        p[j] = e < E ? expf(p[j] - m) : 0.0f;
        s += p[j];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; j++) p[j] *= inv;
    // top-k: the largest probability, ties to the lowest expert index
    bool taken[kMaxExpertsPerLane];
#pragma unroll
    for (int j = 0; j < kMaxExpertsPerLane; j++) taken[j] = (j * 32 + lane) >= E;
    float selw[16];
    int sele[16];
    for (int q = 0; q < k; q++) {
        float bv = -INFINITY;
        int be = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < kMaxExpertsPerLane; j++) {
            const int e = j * 32 + lane;
            if (!taken[j] && (p[j] > bv || (p[j] == bv && e < be))) {
                bv = p[j];
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        sele[q] = be;
        selw[q] = bv;
        if ((be & 31) == lane) {
#pragma unroll
            for (int j = 0; j < kMaxExpertsPerLane; j++)
                if (j == (be >> 5)) taken[j] = true;
        }
    }
    if (lane == 0) {
        float sum = 0.0f;
        for (int q = 0; q < k; q++) sum += selw[q];
        for (int q = 0; q < k; q++) {
            sel[(long long)t * k + q] = sele[q];
            wts[(long long)t * k + q] = (norm_topk && sum > 0.0f) ? selw[q] / sum : selw[q];
        }
    }
}

// Selections are bucketed by expert in chunks of kChunk (token-major order):
// per-chunk histograms, then per expert an exclusive prefix over chunks, so
// the scatter places every selection with one pass and the order within an
// expert stays the selection order (tokens ascending, as src/moe.zig gathers).
constexpr int kChunk = 256;

__global__ void k_chunk_counts(const int *sel, int nk, int E, int *cc) {
    extern __shared__ int hist[];  // [E]
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int i = blockIdx.x * kChunk + threadIdx.x;
    if (i < nk) atomicAdd(&hist[sel[i]], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) cc[(long long)blockIdx.x * E + e] = hist[e];
}

// In place: cc[c][e] <- sum of cc[c'][e] for c' < c; counts[e] = the total.
// One block per expert: each thread sums a run of consecutive chunks, a block
// scan turns the run sums into run bases, and the runs are rewritten.
__global__ void __launch_bounds__(256) k_chunk_prefix(int *cc, int chunks, int E, int *counts) {
    __shared__ int warp_tot[8];
    const int e = blockIdx.x;
    const int per = (chunks + 255) / 256;
    const int c0 = threadIdx.x * per, c1 = min(chunks, c0 + per);
    int run = 0;
    for (int c = c0; c < c1; c++) run += cc[(long long)c * E + e];
    // exclusive scan of the run sums across the block
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    int base = 0, total = 0;
    for (int j = 0; j < 8; j++) {
        if (j < w) base += warp_tot[j];
        total += warp_tot[j];
    }
    int acc = base + incl - run;
    for (int c = c0; c < c1; c++) {
        const int t = cc[(long long)c * E + e];
        cc[(long long)c * E + e] = acc;
        acc += t;
    }
    if (threadIdx.x == 0) counts[e] = total;
}

// One block: expert offsets and the two grouped-GEMM tile schedules
// (expert-major, then token chunk, then weight tile).
__global__ void k_schedule(const int *counts, int E, int bn_gu, int wt_gu, int bn_d, int wt_d, int *offsets,
                           int4 *sched_gu, int *n_gu, int4 *sched_d, int *n_d) {
    __shared__ int s_cnt[1024], s_off[1024], s_tgu[1024], s_td[1024];
    const int e = threadIdx.x;
    const int c = e < E ? counts[e] : 0;
    s_cnt[e] = c;
    s_tgu[e] = e < E ? (c + bn_gu - 1) / bn_gu * wt_gu : 0;
    s_td[e] = e < E ? (c + bn_d - 1) / bn_d * wt_d : 0;
    __syncthreads();
    if (e == 0) {  // E <= 1024: a serial scan is cheap next to the GEMMs
        int a = 0, b = 0, d = 0;
        for (int i = 0; i < E; i++) {
            s_off[i] = a;
            a += s_cnt[i];
            const int tg = s_tgu[i], td = s_td[i];
            s_tgu[i] = b;
            b += tg;
            s_td[i] = d;
            d += td;
        }
        offsets[E] = a;
        *n_gu = b;
        *n_d = d;
    }
    __syncthreads();
    if (e >= E) return;
    offsets[e] = s_off[e];
    int tile = s_tgu[e];
    for (int ch = 0; ch * bn_gu < c; ch++)
        for (int w = 0; w < wt_gu; w++) sched_gu[tile++] = make_int4(e, s_off[e] + ch * bn_gu, min(bn_gu, c - ch * bn_gu), w);
    tile = s_td[e];
    for (int ch = 0; ch * bn_d < c; ch++)
        for (int w = 0; w < wt_d; w++) sched_d[tile++] = make_int4(e, s_off[e] + ch * bn_d, min(bn_d, c - ch * bn_d), w);
}

// Stable scatter: block e walks all (token, slot) pairs in order and places
// those routed to expert e at offsets[e] + rank.
// One block of kChunk threads per chunk: thread i's rank among the equal
// experts of its warp (match_any), plus the counts of the earlier warps of the
// chunk, plus the chunk's base in the expert's segment.
__global__ void __launch_bounds__(kChunk) k_scatter(const int *sel, const float *wts, int nk, int k, int E,
                                                    const int *cc, const int *offsets, int *perm, float *pw,
                                                    int *pexp, int *slot) {
    extern __shared__ int cnt[];  // [kChunk / 32][E]
    constexpr int kW = kChunk / 32;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int j = threadIdx.x; j < kW * E; j += kChunk) cnt[j] = 0;
    __syncthreads();
    const int i = blockIdx.x * kChunk + threadIdx.x;
    const bool valid = i < nk;
    const int e = valid ? sel[i] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & ((1u << lane) - 1));
    if (valid && rank == 0) cnt[w * E + e] = __popc(same);
    __syncthreads();
    for (int x = threadIdx.x; x < E; x += kChunk) {  // exclusive prefix over the warps
        int run = 0;
        for (int ww = 0; ww < kW; ww++) {
            const int t = cnt[ww * E + x];
            cnt[ww * E + x] = run;
            run += t;
        }
    }
    __syncthreads();
    if (valid) {
        const int pos = offsets[e] + cc[(long long)blockIdx.x * E + e] + cnt[w * E + e] + rank;
        perm[pos] = i / k;
        pw[pos] = wts[i];
        pexp[pos] = e;
        slot[i] = pos;
    }
}

// dst[pos][0..H) = src[perm[pos]][0..H) (bf16 rows, source row stride `ss`).
__global__ void k_gather_rows(const uint16_t *src, long long ss, const int *perm, int rows, int hidden, uint16_t *dst) {
    const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const uint16_t *s = src + (long long)perm[r] * ss;
    uint16_t *d = dst + (long long)r * hidden;
    if ((hidden & 7) == 0 && (ss & 7) == 0) {
        for (int i = lane * 8; i < hidden; i += 256)
            *reinterpret_cast<uint4 *>(d + i) = *reinterpret_cast<const uint4 *>(s + i);
    } else {
        for (int i = lane; i < hidden; i += 32) d[i] = s[i];
    }
}

// xa[pos][t] = act[pos] . a_t[e(pos)] for experts with an edit (the x . A
// terms of the per-expert rank-`rank` delta, a [E][rank][mi]), 0 otherwise.
__global__ void k_rowdot_grouped(const uint16_t *act, const float *e_a, const int *pexp, const int *e_flags, int rows,
                                 int mi, int rank, float *xa) {
    const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int e = pexp[r];
    if (!e_flags[e]) {
        if (lane < rank) xa[(long long)r * rank + lane] = 0.0f;
        return;
    }
    const uint16_t *ar = act + (long long)r * mi;
    for (int t = 0; t < rank; t++) {
        const float *a = e_a + ((long long)e * rank + t) * mi;
        float s = 0.0f;
        for (int i = lane; i < mi; i += 32) s = fmaf(bf16_bits_to_f32(ar[i]), a[i], s);
        s = warp_sum(s);
        if (lane == 0) xa[(long long)r * rank + t] = s;
    }
}

// x[t] += sum over t's experts in index order of w * eo[slot], accumulated
// from zero as src/moe.zig:1197-1199 (acc += w * out), then added to x.
__global__ void k_combine(const float *eo, const int *sel, const float *wts, const int *slot, int n, int k, int hidden,
                          float *x) {
    const int t = blockIdx.x;
    __shared__ int s_slot[16];
    __shared__ float s_w[16];
    if (threadIdx.x == 0) {
        int order[16], e[16];
        for (int q = 0; q < k; q++) {
            order[q] = q;
            e[q] = sel[(long long)t * k + q];
        }
        for (int a = 1; a < k; a++) {  // insertion sort by expert index
            const int oq = order[a], ev = e[a];
            int b = a;
            while (b > 0 && e[b - 1] > ev) {
                e[b] = e[b - 1];
                order[b] = order[b - 1];
                b--;
            }
            e[b] = ev;
            order[b] = oq;
        }
        for (int q = 0; q < k; q++) {
            s_slot[q] = slot[(long long)t * k + order[q]];
            s_w[q] = wts[(long long)t * k + order[q]];
        }
    }
    __syncthreads();
    float *xr = x + (long long)t * hidden;
    if ((hidden & 3) == 0) {
        for (int i = threadIdx.x * 4; i < hidden; i += blockDim.x * 4) {
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int q = 0; q < k; q++) {
                const float wq = s_w[q];
                const float4 v = __ldg(reinterpret_cast<const float4 *>(eo + (long long)s_slot[q] * hidden + i));
                acc.x = acc.x + wq * v.x;
                acc.y = acc.y + wq * v.y;
                acc.z = acc.z + wq * v.z;
                acc.w = acc.w + wq * v.w;
            }
            float4 xv = *reinterpret_cast<const float4 *>(xr + i);
            xv.x = xv.x + acc.x;
            xv.y = xv.y + acc.y;
            xv.z = xv.z + acc.z;
            xv.w = xv.w + acc.w;
            *reinterpret_cast<float4 *>(xr + i) = xv;
        }
        return;
    }
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float acc = 0.0f;
        for (int q = 0; q < k; q++) acc = acc + s_w[q] * eo[(long long)s_slot[q] * hidden + i];
        xr[i] = xr[i] + acc;
    }
}

// ---- expert parallelism over a peer group ---------------------------------
// Layout of the group region's data part (offsets from peer_data), per rank.
struct EpLayout {
    size_t cnt, scores, eo, xg, meta, end;
    size_t cap;  // receive rows: every rank's pairs could land on one rank
};

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

EpLayout ep_layout(const Config &c, size_t max_tokens) {
    EpLayout l{};
    const size_t W = c.ep_world, E = c.n_experts, H = c.hidden, nk = max_tokens * c.top_k;
    l.cap = W * nk;
    l.cnt = 0;
    l.scores = align256(l.cnt + W * E * 4);
    l.eo = align256(l.scores + 2 * E * 4);
    l.xg = align256(l.eo + nk * H * 4);
    l.meta = align256(l.xg + l.cap * H * 2);
    l.end = align256(l.meta + l.cap * 8);
    return l;
}

template <class T>
__device__ __forceinline__ T *region(const PeerPtrs &pp, int r, size_t off) {
    return reinterpret_cast<T *>(pp.p[r] + kPeerFlagBytes + off);
}

// This rank's per-expert pair counts into every rank's [world][E] table.
__global__ void k_ep_put_counts(const int *counts, int E, PeerPtrs pp, size_t off, int rank) {
    int *dst = region<int>(pp, blockIdx.x, off) + (size_t)rank * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) dst[e] = counts[e];
    __threadfence_system();
}

// From the gathered counts: where this rank's pairs of expert e land in the
// owner's receive rows (dst_base[e] + local sorted position), and how many
// rows each of this rank's own experts receives. Receive rows are ordered by
// local expert, then source rank, then the source's order.
__global__ void k_ep_plan(const int *cnt_all, const int *offsets_local, int E, int El, int world, int rank,
                          int *dst_base, int *rcnt) {
    __shared__ int tot[1024];
    const int e = threadIdx.x;
    int before = 0;
    if (e < E) {
        int t = 0;
        for (int s = 0; s < world; s++) {
            const int c = cnt_all[(size_t)s * E + e];
            if (s < rank) before += c;
            t += c;
        }
        tot[e] = t;
    }
    __syncthreads();
    if (e >= E) return;
    const int d = e / El;
    int base = 0;
    for (int x = d * El; x < e; x++) base += tot[x];
    dst_base[e] = base + before - offsets_local[e];
    if (d == rank) rcnt[e - d * El] = tot[e];
}

// One warp per local (token, expert) pair in expert-sorted order: the pair's
// normalised row (bf16, the hi part of the split rows) and (source rank,
// position) into the owner's receive region.
__global__ void k_ep_dispatch(const uint16_t *h3, long long ss, const int *perm, const int *pexp, int nk,
                              const int *dst_base, int El, PeerPtrs pp, size_t xg_off, size_t meta_off, int H,
                              int rank) {
    const int pos = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (pos < nk) {
        const int e = pexp[pos], d = e / El;
        const long long row = (long long)dst_base[e] + pos;
        const uint16_t *src = h3 + (long long)perm[pos] * ss;
        uint16_t *dst = region<uint16_t>(pp, d, xg_off) + row * H;
        for (int i = lane * 8; i < H; i += 256)
            *reinterpret_cast<uint4 *>(dst + i) = *reinterpret_cast<const uint4 *>(src + i);
        if (lane == 0) region<int2>(pp, d, meta_off)[row] = make_int2(rank, pos);
    }
    __threadfence_system();
}

// Local expert of every receive row (rows past the total get -1).
__global__ void k_ep_fill_pexp(const int *offsets, int El, int cap, int *pexp) {
    const int total = offsets[El];
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < cap; r += gridDim.x * blockDim.x) {
        if (r >= total) {
            pexp[r] = -1;
            continue;
        }
        int lo = 0, hi = El - 1;  // last expert whose offset <= r
        while (lo < hi) {
            const int mid = (lo + hi + 1) / 2;
            if (offsets[mid] <= r) lo = mid;
            else hi = mid - 1;
        }
        pexp[r] = lo;
    }
}

// xa of receive rows of edited local experts (rows with pexp < 0 skipped),
// `rank` terms per row as k_rowdot_grouped.
__global__ void k_ep_rowdot(const uint16_t *act, const float *e_a, const int *pexp, const int *e_flags, int cap,
                            int mi, int rank, float *xa) {
    const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= cap) return;
    const int e = pexp[r];
    if (e < 0) return;
    if (!e_flags[e]) {
        if (lane < rank) xa[(long long)r * rank + lane] = 0.0f;
        return;
    }
    const uint16_t *ar = act + (long long)r * mi;
    for (int t = 0; t < rank; t++) {
        const float *a = e_a + ((long long)e * rank + t) * mi;
        float s = 0.0f;
        for (int i = lane; i < mi; i += 32) s = fmaf(bf16_bits_to_f32(ar[i]), a[i], s);
        s = warp_sum(s);
        if (lane == 0) xa[(long long)r * rank + t] = s;
    }
}

// One warp per receive row: its expert output back to the source rank's eo
// rows at the pair's position there.
__global__ void k_ep_return(const float *eo, const int2 *meta, const int *offsets, int El, PeerPtrs pp,
                            size_t eo_off, int H) {
    const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r < offsets[El]) {
        const int2 sp = meta[r];
        const float *src = eo + (long long)r * H;
        float *dst = region<float>(pp, sp.x, eo_off) + (long long)sp.y * H;
        for (int i = lane * 4; i < H; i += 128)
            *reinterpret_cast<float4 *>(dst + i) = *reinterpret_cast<const float4 *>(src + i);
    }
    __threadfence_system();
}

// This rank's expert scores into every rank's score buffer (double-buffered).
__global__ void k_ep_put_scores(const float *local, int El, int rank, PeerPtrs pp, size_t off) {
    float *dst = region<float>(pp, blockIdx.x, off) + (size_t)rank * El;
    for (int e = threadIdx.x; e < El; e += blockDim.x) dst[e] = local[e];
    __threadfence_system();
}

// Token tile of a grouped GEMM from the mean rows per expert.
int tile_for(int avg, bool dual, bool quant) {
    if (avg <= 32) return 32;
    if (avg <= 64) return 64;
    if ((dual && !quant) || avg <= 160) return 128;
    return 256;
}

}  // namespace

int build_router_split(ditch_cuda_device *dev, const float *router_f32, int E, int hidden, Mat &out) {
    const int cp = (hidden + 63) / 64 * 64;
    out.fmt = kFmtBf16;
    out.rows = E;
    out.cols = 3 * cp;
    out.slabs = 1;
    out.row_bytes = (long long)out.cols * 2;
    DITCH_CUDA(out.data.reserve((size_t)E * out.cols * 2));
    // weights [Wh | Wl | Wh] against activations [xh | xh | xl]
    DITCH_LAUNCH(dev, split_bf16(router_f32, E, hidden, cp, 3, 2, out.data.as<uint16_t>(), dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    return DITCH_CUDA_OK;
}

int moe_mlp_ep(ditch_cuda_model *m, Layer &L, int n);

int moe_mlp(ditch_cuda_model *m, Layer &L, int li, int n) {
    (void)li;
    if (m->group) return moe_mlp_ep(m, L, n);
    ditch_cuda_device *dev = m->dev;
    cudaStream_t st = dev->stream;
    const Config &c = m->cfg;
    const int H = c.hidden, E = c.n_experts, k = c.top_k, mi = c.moe_inter;
    if (E > 1024 || k > 16) {
        set_error("MoE with %d experts / top-%d is not supported (<= 1024 / 16)", E, k);
        return DITCH_CUDA_UNSUPPORTED;
    }
    const int nk = n * k;
    const int mip = L.e_down.cols;  // stored (8-aligned) expert width: the act row stride
    const int cp = (H + 63) / 64 * 64;
    const int avg = (nk + E - 1) / E;
    // quantised expert stacks with a kept bf16 copy run the bf16 grouped GEMM
    const bool gu_q = L.e_gate_up.fmt != kFmtBf16 && !expert_stack_cached(dev, L.e_gate_up);
    const bool d_q = L.e_down.fmt != kFmtBf16 && !expert_stack_cached(dev, L.e_down);
    const int bn_gu = tile_for(avg, true, gu_q);
    const int bn_d = tile_for(avg, false, d_q);
    const int wt_gu = (mi + 127) / 128, wt_d = (H + 127) / 128;
    const int max_gu = (nk / bn_gu + E) * wt_gu, max_d = (nk / bn_d + E) * wt_d;
    DITCH_CUDA(m->moe_h3.reserve((size_t)n * 3 * cp * 2));
    DITCH_CUDA(m->moe_logits.reserve((size_t)n * E * 4));
    DITCH_CUDA(m->moe_sel.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_w.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_counts.reserve((size_t)E * 4));
    DITCH_CUDA(m->moe_cc.reserve((size_t)((nk + kChunk - 1) / kChunk) * E * 4));
    DITCH_CUDA(m->moe_offsets.reserve((size_t)(E + 1) * 4 + 8));
    DITCH_CUDA(m->moe_perm.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_pw.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_pexp.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_slot.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_xg.reserve((size_t)nk * H * 2));
    DITCH_CUDA(m->moe_act.reserve((size_t)nk * mip * 2));
    DITCH_CUDA(m->moe_eo.reserve((size_t)nk * H * 4));
    DITCH_CUDA(m->moe_xa.reserve((size_t)nk * 4 * kMaxDeltaRank));
    DITCH_CUDA(m->moe_sched_gu.reserve((size_t)max_gu * 16));
    DITCH_CUDA(m->moe_sched_d.reserve((size_t)max_d * 16));
    DITCH_CUDA(m->moe_nsched.reserve(16));
    int *n_gu = m->moe_nsched.as<int>(), *n_d = n_gu + 1;

    k_rmsnorm_split3<<<(n + 7) / 8, 256, 0, st>>>(m->x.as<float>(), L.post_norm.as<float>(), n, H, cp, c.eps,
                                                   m->moe_h3.as<uint16_t>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    int s;
    if ((s = gemm_mat(dev, L.router3, 0, E, m->moe_h3.as<uint16_t>(), n, m->moe_logits.ptr, E, 0, nullptr, nullptr,
                      nullptr, 0, nullptr)))
        return s;
    k_route<<<(n + 7) / 8, 256, 0, st>>>(m->moe_logits.as<float>(), n, E, k, c.norm_topk, m->moe_sel.as<int>(),
                                         m->moe_w.as<float>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    const int chunks = (nk + kChunk - 1) / kChunk;
    k_chunk_counts<<<chunks, kChunk, (size_t)E * 4, st>>>(m->moe_sel.as<int>(), nk, E, m->moe_cc.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    k_chunk_prefix<<<E, 256, 0, st>>>(m->moe_cc.as<int>(), chunks, E, m->moe_counts.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    k_schedule<<<1, 1024, 0, st>>>(m->moe_counts.as<int>(), E, bn_gu, wt_gu, bn_d, wt_d, m->moe_offsets.as<int>(),
                                   m->moe_sched_gu.as<int4>(), n_gu, m->moe_sched_d.as<int4>(), n_d);
    DITCH_LAUNCH(dev, cudaGetLastError());
    k_scatter<<<chunks, kChunk, (size_t)(kChunk / 32) * E * 4, st>>>(
        m->moe_sel.as<int>(), m->moe_w.as<float>(), nk, k, E, m->moe_cc.as<int>(), m->moe_offsets.as<int>(),
        m->moe_perm.as<int>(), m->moe_pw.as<float>(), m->moe_pexp.as<int>(), m->moe_slot.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    k_gather_rows<<<(nk + 7) / 8, 256, 0, st>>>(m->moe_h3.as<uint16_t>(), 3LL * cp, m->moe_perm.as<int>(), nk, H,
                                                m->moe_xg.as<uint16_t>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    GemmExtra gu;
    gu.sched = m->moe_sched_gu.as<int4>();
    gu.n_sched = n_gu;
    gu.slab_rows = 2 * mi;
    gu.bn = bn_gu;
    if (mip != mi) DITCH_CUDA(cudaMemsetAsync(m->moe_act.ptr, 0, (size_t)nk * mip * 2, st));
    if ((s = gemm_mat(dev, L.e_gate_up, 0, mi, m->moe_xg.as<uint16_t>(), nk, m->moe_act.ptr, mip, kEpiSwiglu, nullptr,
                      nullptr, nullptr, mi, &gu)))
        return s;
    bool any_edit = false;
    for (uint8_t f : L.e_edit) any_edit |= f != 0;
    if (any_edit) {
        k_rowdot_grouped<<<(nk + 7) / 8, 256, 0, st>>>(m->moe_act.as<uint16_t>(), L.e_a.as<float>(),
                                                       m->moe_pexp.as<int>(), L.e_edit_dev.as<int>(), nk, mip,
                                                       L.e_rank, m->moe_xa.as<float>());
        DITCH_LAUNCH(dev, cudaGetLastError());
    }
    GemmExtra dn;
    dn.sched = m->moe_sched_d.as<int4>();
    dn.n_sched = n_d;
    dn.slab_rows = H;
    dn.bn = bn_d;
    dn.e_flags = L.e_edit_dev.as<int>();
    dn.db_stride = H * L.e_rank;
    if ((s = gemm_mat(dev, L.e_down, 0, H, m->moe_act.as<uint16_t>(), nk, m->moe_eo.ptr, H, 0, nullptr,
                      any_edit ? m->moe_xa.as<float>() : nullptr, any_edit ? L.e_b.as<float>() : nullptr, 0, &dn,
                      L.e_rank)))
        return s;
    k_combine<<<n, 256, 0, st>>>(m->moe_eo.as<float>(), m->moe_sel.as<int>(), m->moe_w.as<float>(),
                                 m->moe_slot.as<int>(), n, k, H, m->x.as<float>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    return DITCH_CUDA_OK;
}

namespace {

#define EP_REQUIRE(cond, ...)          \
    do {                               \
        if (!(cond)) {                 \
            set_error(__VA_ARGS__);    \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)

// One exchange of the model's peer group: signal this rank's epoch to every
// peer, then wait (bounded) until every peer has signalled it.
int ep_exchange(ditch_cuda_model *m) { return group_exchange(m->dev, m->group, m->group->wait_s); }

}  // namespace

// Expert-parallel MoE MLP: routing on this rank's tokens, the pairs sent to
// their experts' owners, the owners' grouped GEMMs over every rank's rows,
// the outputs returned to the pairs' positions, then the same ordered combine
// as one GPU (so the result equals the single-GPU forward bit for bit).
// Exchange order per layer: counts, rows, outputs.
int moe_mlp_ep(ditch_cuda_model *m, Layer &L, int n) {
    ditch_cuda_device *dev = m->dev;
    cudaStream_t st = dev->stream;
    const Config &c = m->cfg;
    ditch_cuda_group *g = m->group;
    const int H = c.hidden, E = c.n_experts, El = c.e_loc, k = c.top_k, mi = c.moe_inter;
    const int W = g->world, rank = g->rank;
    EP_REQUIRE(E <= 1024 && k <= 16, "MoE with %d experts / top-%d is not supported (<= 1024 / 16)", E, k);
    EP_REQUIRE((size_t)n <= m->group_tokens, "%d tokens exceed the %zu the peer group was sized for", n,
               m->group_tokens);
    const EpLayout lay = ep_layout(c, m->group_tokens);
    const int nk = n * k;
    const int cap = (int)lay.cap;
    const int mip = L.e_down.cols;
    const int cp = (H + 63) / 64 * 64;
    const int avg = (int)(((long long)W * nk + E - 1) / E);  // rows per expert with balanced routing
    // quantised expert stacks with a kept bf16 copy run the bf16 grouped GEMM
    const bool gu_q = L.e_gate_up.fmt != kFmtBf16 && !expert_stack_cached(dev, L.e_gate_up);
    const bool d_q = L.e_down.fmt != kFmtBf16 && !expert_stack_cached(dev, L.e_down);
    const int bn_gu = tile_for(avg, true, gu_q);
    const int bn_d = tile_for(avg, false, d_q);
    const int wt_gu = (mi + 127) / 128, wt_d = (H + 127) / 128;
    const int src_gu = (nk / bn_gu + E) * wt_gu, src_d = (nk / bn_d + E) * wt_d;
    const int max_gu = (cap / bn_gu + El) * wt_gu, max_d = (cap / bn_d + El) * wt_d;
    DITCH_CUDA(m->moe_h3.reserve((size_t)n * 3 * cp * 2));
    DITCH_CUDA(m->moe_logits.reserve((size_t)n * E * 4));
    DITCH_CUDA(m->moe_sel.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_w.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_counts.reserve((size_t)E * 4));
    DITCH_CUDA(m->moe_cc.reserve((size_t)((nk + kChunk - 1) / kChunk) * E * 4));
    DITCH_CUDA(m->moe_offsets.reserve((size_t)(E + 1) * 4 + 8));
    DITCH_CUDA(m->moe_perm.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_pw.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_pexp.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_slot.reserve((size_t)nk * 4));
    DITCH_CUDA(m->moe_sched_gu.reserve((size_t)src_gu * 16));
    DITCH_CUDA(m->moe_sched_d.reserve((size_t)src_d * 16));
    DITCH_CUDA(m->moe_nsched.reserve(16));
    DITCH_CUDA(m->ep_dst.reserve((size_t)E * 4));
    DITCH_CUDA(m->ep_rcnt.reserve((size_t)El * 4));
    DITCH_CUDA(m->ep_roff.reserve((size_t)(El + 1) * 4 + 8));
    DITCH_CUDA(m->ep_pexp.reserve((size_t)cap * 4));
    DITCH_CUDA(m->ep_act.reserve((size_t)cap * mip * 2));
    DITCH_CUDA(m->ep_eo.reserve((size_t)cap * H * 4));
    DITCH_CUDA(m->ep_xa.reserve((size_t)cap * 4 * kMaxDeltaRank));
    DITCH_CUDA(m->ep_sched_gu.reserve((size_t)max_gu * 16));
    DITCH_CUDA(m->ep_sched_d.reserve((size_t)max_d * 16));
    DITCH_CUDA(m->ep_nsched.reserve(16));
    uint8_t *own = peer_data(g->base);

    // routing of this rank's tokens, pairs sorted by expert (as one GPU)
    k_rmsnorm_split3<<<(n + 7) / 8, 256, 0, st>>>(m->x.as<float>(), L.post_norm.as<float>(), n, H, cp, c.eps,
                                                   m->moe_h3.as<uint16_t>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    int s;
    if ((s = gemm_mat(dev, L.router3, 0, E, m->moe_h3.as<uint16_t>(), n, m->moe_logits.ptr, E, 0, nullptr, nullptr,
                      nullptr, 0, nullptr)))
        return s;
    k_route<<<(n + 7) / 8, 256, 0, st>>>(m->moe_logits.as<float>(), n, E, k, c.norm_topk, m->moe_sel.as<int>(),
                                         m->moe_w.as<float>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    const int chunks = (nk + kChunk - 1) / kChunk;
    k_chunk_counts<<<chunks, kChunk, (size_t)E * 4, st>>>(m->moe_sel.as<int>(), nk, E, m->moe_cc.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    k_chunk_prefix<<<E, 256, 0, st>>>(m->moe_cc.as<int>(), chunks, E, m->moe_counts.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    int *src_n = m->moe_nsched.as<int>();
    k_schedule<<<1, 1024, 0, st>>>(m->moe_counts.as<int>(), E, bn_gu, wt_gu, bn_d, wt_d, m->moe_offsets.as<int>(),
                                   m->moe_sched_gu.as<int4>(), src_n, m->moe_sched_d.as<int4>(), src_n + 1);
    DITCH_LAUNCH(dev, cudaGetLastError());
    k_scatter<<<chunks, kChunk, (size_t)(kChunk / 32) * E * 4, st>>>(
        m->moe_sel.as<int>(), m->moe_w.as<float>(), nk, k, E, m->moe_cc.as<int>(), m->moe_offsets.as<int>(),
        m->moe_perm.as<int>(), m->moe_pw.as<float>(), m->moe_pexp.as<int>(), m->moe_slot.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());

    // exchange 1: every rank's per-expert pair counts
    k_ep_put_counts<<<W, 256, 0, st>>>(m->moe_counts.as<int>(), E, g->peers, lay.cnt, rank);
    DITCH_LAUNCH(dev, cudaGetLastError());
    if ((s = ep_exchange(m))) return s;
    k_ep_plan<<<1, 1024, 0, st>>>(reinterpret_cast<const int *>(own + lay.cnt), m->moe_offsets.as<int>(), E, El, W,
                                  rank, m->ep_dst.as<int>(), m->ep_rcnt.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    int *n_gu = m->ep_nsched.as<int>(), *n_d = n_gu + 1;
    k_schedule<<<1, 1024, 0, st>>>(m->ep_rcnt.as<int>(), El, bn_gu, wt_gu, bn_d, wt_d, m->ep_roff.as<int>(),
                                   m->ep_sched_gu.as<int4>(), n_gu, m->ep_sched_d.as<int4>(), n_d);
    DITCH_LAUNCH(dev, cudaGetLastError());

    // exchange 2: the rows to their experts' owners
    k_ep_dispatch<<<(nk + 7) / 8, 256, 0, st>>>(m->moe_h3.as<uint16_t>(), 3LL * cp, m->moe_perm.as<int>(),
                                                m->moe_pexp.as<int>(), nk, m->ep_dst.as<int>(), El, g->peers, lay.xg,
                                                lay.meta, H, rank);
    DITCH_LAUNCH(dev, cudaGetLastError());
    if ((s = ep_exchange(m))) return s;

    // this rank's experts over every rank's rows
    k_ep_fill_pexp<<<std::min((cap + 255) / 256, 4096), 256, 0, st>>>(m->ep_roff.as<int>(), El, cap,
                                                                      m->ep_pexp.as<int>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    const uint16_t *xg = reinterpret_cast<const uint16_t *>(own + lay.xg);
    GemmExtra gu;
    gu.sched = m->ep_sched_gu.as<int4>();
    gu.n_sched = n_gu;
    gu.slab_rows = 2 * mi;
    gu.bn = bn_gu;
    if (mip != mi) DITCH_CUDA(cudaMemsetAsync(m->ep_act.ptr, 0, (size_t)cap * mip * 2, st));
    if ((s = gemm_mat(dev, L.e_gate_up, 0, mi, xg, cap, m->ep_act.ptr, mip, kEpiSwiglu, nullptr, nullptr, nullptr, mi,
                      &gu)))
        return s;
    bool any_edit = false;
    for (uint8_t f : L.e_edit) any_edit |= f != 0;
    if (any_edit) {
        k_ep_rowdot<<<(cap + 7) / 8, 256, 0, st>>>(m->ep_act.as<uint16_t>(), L.e_a.as<float>(), m->ep_pexp.as<int>(),
                                                   L.e_edit_dev.as<int>(), cap, mip, L.e_rank, m->ep_xa.as<float>());
        DITCH_LAUNCH(dev, cudaGetLastError());
    }
    GemmExtra dn;
    dn.sched = m->ep_sched_d.as<int4>();
    dn.n_sched = n_d;
    dn.slab_rows = H;
    dn.bn = bn_d;
    dn.e_flags = L.e_edit_dev.as<int>();
    dn.db_stride = H * L.e_rank;
    if ((s = gemm_mat(dev, L.e_down, 0, H, m->ep_act.as<uint16_t>(), cap, m->ep_eo.ptr, H, 0, nullptr,
                      any_edit ? m->ep_xa.as<float>() : nullptr, any_edit ? L.e_b.as<float>() : nullptr, 0, &dn,
                      L.e_rank)))
        return s;

    // exchange 3: the outputs back to the pairs' positions on their source ranks
    k_ep_return<<<(cap + 7) / 8, 256, 0, st>>>(m->ep_eo.as<float>(), reinterpret_cast<const int2 *>(own + lay.meta),
                                               m->ep_roff.as<int>(), El, g->peers, lay.eo, H);
    DITCH_LAUNCH(dev, cudaGetLastError());
    if ((s = ep_exchange(m))) return s;
    k_combine<<<n, 256, 0, st>>>(reinterpret_cast<const float *>(own + lay.eo), m->moe_sel.as<int>(),
                                 m->moe_w.as<float>(), m->moe_slot.as<int>(), n, k, H, m->x.as<float>());
    DITCH_LAUNCH(dev, cudaGetLastError());
    return DITCH_CUDA_OK;
}

// Every rank's `per_rank` values (this rank's `local`) gathered in rank order
// through the layout's score area (two halves used in turn: a rank is at most
// one exchange ahead of another, so it never overwrites the half a peer is
// still reading).
static int ep_allgather_f32(ditch_cuda_model *m, const float *local, int per_rank, std::vector<float> &all) {
    ditch_cuda_device *dev = m->dev;
    cudaStream_t st = dev->stream;
    const Config &c = m->cfg;
    ditch_cuda_group *g = m->group;
    const int E = c.n_experts, W = g->world;
    EP_REQUIRE(per_rank >= 0 && (size_t)per_rank * W <= (size_t)E, "%d values per rank exceed the score area",
               per_rank);
    const EpLayout lay = ep_layout(c, m->group_tokens);
    const size_t off = lay.scores + (size_t)m->ep_score_parity * E * 4;
    m->ep_score_parity ^= 1;
    DITCH_CUDA(m->ep_scores.reserve((size_t)std::max(per_rank, 1) * 4));
    DITCH_CUDA(cudaMemcpyAsync(m->ep_scores.ptr, local, (size_t)per_rank * 4, cudaMemcpyHostToDevice, st));
    k_ep_put_scores<<<W, 256, 0, st>>>(m->ep_scores.as<float>(), per_rank, g->rank, g->peers, off);
    DITCH_LAUNCH(dev, cudaGetLastError());
    int s;
    if ((s = ep_exchange(m))) return s;
    all.assign((size_t)per_rank * W, 0.0f);
    DITCH_CUDA(cudaMemcpyAsync(all.data(), peer_data(g->base) + off, all.size() * 4, cudaMemcpyDeviceToHost, st));
    DITCH_CUDA(cudaStreamSynchronize(st));
    return DITCH_CUDA_OK;
}

int ep_allgather_scores(ditch_cuda_model *m, const std::vector<float> &local, std::vector<float> &all) {
    EP_REQUIRE((int)local.size() == m->cfg.e_loc, "local scores size");
    int s;
    if ((s = ep_allgather_f32(m, local.data(), m->cfg.e_loc, all))) return s;
    return check_status(m->dev, "expert score exchange");
}

int ep_any_active(ditch_cuda_model *m, size_t local_active, bool *any) {
    const float v = local_active ? 1.0f : 0.0f;
    std::vector<float> all;
    int s;
    if ((s = ep_allgather_f32(m, &v, 1, all))) return s;
    if ((s = check_status(m->dev, "generation step agreement"))) return s;
    *any = false;
    for (float x : all) *any |= x != 0.0f;
    return DITCH_CUDA_OK;
}

}  // namespace ditch

extern "C" {

size_t ditch_cuda_model_group_bytes(const ditch_cuda_model *m, size_t max_tokens) {
    if (!m) return 0;
    if (m->cfg.ep_world > 1) return ditch::ep_layout(m->cfg, max_tokens).end;
    if (m->cfg.tp_world > 1) return ditch::tp_group_bytes(m->cfg, max_tokens);
    return 0;
}

int ditch_cuda_model_set_group(ditch_cuda_model *m, ditch_cuda_group *g, size_t max_tokens) {
    using namespace ditch;
    clear_error();
    EP_REQUIRE(m && g, "null argument");
    const Config &c = m->cfg;
    const bool ep = c.ep_world > 1, tp = c.tp_world > 1;
    EP_REQUIRE(ep || tp, "the model was loaded without expert or tensor parallelism");
    EP_REQUIRE(g->opened, "the group is not opened");
    EP_REQUIRE(g->dev == m->dev, "the group lives on another device");
    EP_REQUIRE(g->world == (ep ? c.ep_world : c.tp_world) && g->rank == (ep ? c.ep_rank : c.tp_rank),
               "group rank %d / world %d differ from the model's", g->rank, g->world);
    EP_REQUIRE(max_tokens > 0, "max_tokens must be positive");
    const size_t need = ep ? ep_layout(c, max_tokens).end : tp_group_bytes(c, max_tokens);
    EP_REQUIRE(need <= g->bytes, "the group region holds %zu bytes; %zu needed", g->bytes, need);
    std::lock_guard<std::mutex> lk(m->dev->mu);
    m->group = g;
    m->group_tokens = max_tokens;
    // tensor parallel ranks recompute the replicated parts (norms, the LM
    // head) and must agree bit for bit: products summed in a fixed order
    if (tp) m->dev->deterministic = true;
    return DITCH_CUDA_OK;
}

}  // extern "C"
