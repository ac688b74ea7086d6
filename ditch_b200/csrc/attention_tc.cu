// Causal GQA prefill attention on the fifth-generation tensor cores, for
// batches whose prompts are at most 128 tokens long (the trial workload's
// prompts). Same arithmetic as the mma.sync kernel in forward_kernels.cu
// (src/model.zig:4226-4374): Q, K, V and the softmax weights P are split
// into bf16 pairs x = hi + lo, every product is hi*hi + hi*lo + lo*hi with
// f32 accumulation, the softmax is f32 with CUDA's expf, and the output is
// the P.V sum times 1 / (sum of P).
//
// Work item = (prompt, kv head). Its keys (NK = 64 or 128 rows, zero past the
// prompt) and values (transposed: one row per dimension) are held in shared
// memory as bf16 hi / lo, K-major with the 128-byte swizzle. The group's
// query heads are stacked into tiles of 128 query rows (two heads of 64 rows
// when NK is 64), and per tile:
//   S = Q . K^T     tcgen05.mma M 128 x N NK, f32 accumulator in TMEM
//   P = softmax(S)  each thread owns one row (its TMEM lane) and half of its
//                   columns; P is written over the Q tile, bf16 hi / lo
//   O = P . V       tcgen05.mma M 128 x N head_dim into TMEM
//   out = O / l     read back with tcgen05.ld, bf16 rows to global memory
// The next Q rows are loaded into registers while the current products run.
//
// Prompts of at most 64 tokens (k_attention_tc2, the default): two CTAs per
// SM, so that one CTA's loads and barrier waits overlap the other's work;
// the Q tile is staged one 64-dim half at a time and the output rows leave
// through shared memory as whole-row stores. Prompts of 65 to 128 tokens
// (k_attention_tc): one CTA per SM with the whole Q tile staged.
//
// Every wait on the MMA barrier is bounded; on a timeout the status word is
// set and the CTA frees its TMEM and returns.
#include "common.cuh"
#include "kernels.cuh"

namespace ditch {
namespace {

constexpr int kTcThreads = 256;
constexpr int kTcRows = 128;  // query rows per tile (the MMA's M)

template <int HD, int NK>
struct AttnTc {
    static constexpr int kHpt = kTcRows / NK;                       // heads per tile
    static constexpr int kQRegion = kTcRows * 128;                  // one 64-dim region of the Q tile
    static constexpr int kPRegion = kTcRows * 128;                  // one 64-key region of the P tile
    static constexpr int kQBytes = kQRegion * (HD / 64);
    static constexpr int kPBytes = kPRegion * (NK / 64);
    static constexpr int kQPBytes = kQBytes > kPBytes ? kQBytes : kPBytes;
    static constexpr int kKRegion = NK * 128;                       // one 64-dim region of K
    static constexpr int kKBytes = kKRegion * (HD / 64);
    static constexpr int kVRegion = HD * 128;                       // one 64-key region of V^T
    static constexpr int kVBytes = kVRegion * (NK / 64);
    static constexpr int kOperandBytes = 2 * (kQPBytes + kKBytes + kVBytes);
    static constexpr int kRedBytes = 4 * kTcRows * sizeof(float);  // per-row max and sum of two column halves
    static constexpr int kSmemBytes = 1024 + kOperandBytes + kRedBytes + 64;
    static constexpr uint32_t kTmemCols = (NK + HD) <= 128 ? 128 : 256;
    static constexpr int kQLoads = kTcRows * HD / 4 / kTcThreads;   // float4 loads per thread for a Q tile
    static constexpr int kKLoads = NK * HD / 4 / kTcThreads;
    static constexpr int kVTotal = (NK / 8) * (HD / 4);              // 8-key x 4-dim blocks of V
    static constexpr int kVUnits = (kVTotal + kTcThreads - 1) / kTcThreads;
    static_assert(kQLoads > 0 && kKLoads > 0 && kVUnits > 0, "tile shape");
};

// Shared memory of one CTA: the operand tiles, the softmax row statistics,
// the barriers and the TMEM base (from a 1024-byte aligned base).
struct TcSmem {
    uint8_t *qh, *ql, *kh, *kl, *vh, *vl;  // Q tile (P over it), K, V^T: bf16 hi / lo
    float *red;                              // [2][128] row max, then [2][128] row sum
    uint64_t *bar;                           // MMA completion
    uint32_t *tmem_slot;
    volatile int *abort;
};

template <int HD, int NK>
__device__ __forceinline__ TcSmem carve_tc(uint8_t *smem_raw) {
    using C = AttnTc<HD, NK>;
    TcSmem s;
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    s.qh = base;
    s.ql = s.qh + C::kQPBytes;
    s.kh = s.ql + C::kQPBytes;
    s.kl = s.kh + C::kKBytes;
    s.vh = s.kl + C::kKBytes;
    s.vl = s.vh + C::kVBytes;
    s.red = reinterpret_cast<float *>(s.vl + C::kVBytes);
    s.bar = reinterpret_cast<uint64_t *>(s.red + 4 * kTcRows);
    s.tmem_slot = reinterpret_cast<uint32_t *>(s.bar + 1);
    s.abort = reinterpret_cast<volatile int *>(s.tmem_slot + 1);
    return s;
}

// Byte offset of chunk j (8 bf16) of row r in a K-major 128-byte-swizzled region.
__device__ __forceinline__ int sw_off(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

// bf16 hi of (a, b) and the bf16 of the remainders (low half = a).
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    hi = pack_bf16x2(a, b);
    lo = pack_bf16x2(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
}

// Stores a float4 of dims d .. d + 3 of row r into a K-major hi / lo pair of
// regions (64 dims each).
__device__ __forceinline__ void put_rowvec(uint8_t *hi, uint8_t *lo, int region_bytes, int r, int d, float4 v) {
    const int off = (d >> 6) * region_bytes + sw_off(r, (d & 63) >> 3) + ((d & 4) ? 8 : 0);
    uint2 h, l;
    split2(v.x, v.y, h.x, l.x);
    split2(v.z, v.w, h.y, l.y);
    *reinterpret_cast<uint2 *>(hi + off) = h;
    *reinterpret_cast<uint2 *>(lo + off) = l;
}

// Eight consecutive keys of one dimension of V as one 16-byte chunk of row
// `d` of the transposed hi / lo tiles.
template <int HD, int NK>
__device__ __forceinline__ void put_vchunk(const TcSmem &s, int d, int kg, const float (&x)[8]) {
    using C = AttnTc<HD, NK>;
    uint4 h, l;
    split2(x[0], x[1], h.x, l.x);
    split2(x[2], x[3], h.y, l.y);
    split2(x[4], x[5], h.z, l.z);
    split2(x[6], x[7], h.w, l.w);
    const int off = (kg >> 3) * C::kVRegion + sw_off(d, kg & 7);
    *reinterpret_cast<uint4 *>(s.vh + off) = h;
    *reinterpret_cast<uint4 *>(s.vl + off) = l;
}

template <int HD, int NK>
__device__ __forceinline__ void load_q_tile(const AttnParams &p, int start, int len, int kvh, int groups, int tile,
                                            float4 (&q)[AttnTc<HD, NK>::kQLoads]) {
    using C = AttnTc<HD, NK>;
    const int width = (p.heads + 2 * p.kv_heads) * HD;
#pragma unroll
    for (int u = 0; u < C::kQLoads; u++) {
        const int f = threadIdx.x + kTcThreads * u, r = f / (HD / 4), d = 4 * (f % (HD / 4));
        const int slot = tile * C::kHpt + r / NK, pos = r % NK;
        q[u] = (slot < groups && pos < len)
                   ? __ldg(reinterpret_cast<const float4 *>(p.qkv + (long long)(start + pos) * width +
                                                            (kvh * groups + slot) * HD + d))
                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
}

template <int HD, int NK>
__device__ __forceinline__ void store_q_tile(const TcSmem &s, const float4 (&q)[AttnTc<HD, NK>::kQLoads]) {
    using C = AttnTc<HD, NK>;
#pragma unroll
    for (int u = 0; u < C::kQLoads; u++) {
        const int f = threadIdx.x + kTcThreads * u, r = f / (HD / 4), d = 4 * (f % (HD / 4));
        put_rowvec(s.qh, s.ql, C::kQRegion, r, d, q[u]);
    }
}

// S (+)= A . B^T for the three hi / lo products of one 16-wide K step.
__device__ __forceinline__ void mma3(uint32_t d, uint64_t ah, uint64_t al, uint64_t bh, uint64_t bl, uint32_t idesc,
                                     uint32_t acc) {
    tc_mma_bf16(d, ah, bh, idesc, acc);
    tc_mma_bf16(d, ah, bl, idesc, 1u);
    tc_mma_bf16(d, al, bh, idesc, 1u);
}

// The softmax of one row of S (this thread's half of its NK columns, the
// row max and sum exchanged with the other half's thread through s.red),
// written as P hi / lo over the Q tile. Row sums stay in s.red[256 + ...]
// for the output's 1 / l. Warp-collective (tcgen05.ld) and CTA-wide
// (__syncthreads): every thread calls it.
template <int HD, int NK>
__device__ __forceinline__ void softmax_to_p(const AttnParams &p, const TcSmem &s, uint32_t s_row, int half, int row,
                                             bool valid, int pos) {
    using C = AttnTc<HD, NK>;
    constexpr int kHalf = NK / 2;
    float sc[kHalf];
#pragma unroll
    for (int c = 0; c < kHalf; c += 32) {
        float t[32];
        tmem_ld32(s_row + half * kHalf + c, t);
#pragma unroll
        for (int i = 0; i < 32; i++) sc[c + i] = t[i];
    }
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kHalf; i++) {
        const int key = half * kHalf + i;
        sc[i] = (valid && key <= pos) ? sc[i] * p.scale : -INFINITY;
        mx = fmaxf(mx, sc[i]);
    }
    s.red[half * kTcRows + row] = mx;
    __syncthreads();
    mx = fmaxf(s.red[row], s.red[kTcRows + row]);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < kHalf; i++) {
        sc[i] = sc[i] == -INFINITY ? 0.0f : expf(sc[i] - mx);
        sum += sc[i];
    }
    s.red[2 * kTcRows + half * kTcRows + row] = sum;
#pragma unroll
    for (int j = 0; j < kHalf / 8; j++) {
        const int kc = half * (kHalf / 8) + j;  // 8-key chunk of the row
        uint4 h, l;
        split2(sc[8 * j + 0], sc[8 * j + 1], h.x, l.x);
        split2(sc[8 * j + 2], sc[8 * j + 3], h.y, l.y);
        split2(sc[8 * j + 4], sc[8 * j + 5], h.z, l.z);
        split2(sc[8 * j + 6], sc[8 * j + 7], h.w, l.w);
        const int off = (kc >> 3) * C::kPRegion + sw_off(row, kc & 7);
        *reinterpret_cast<uint4 *>(s.qh + off) = h;
        *reinterpret_cast<uint4 *>(s.ql + off) = l;
    }
}

// One query tile of an item: S = Q . K^T, the softmax into P (over the Q
// tile), O = P . V and the bf16 output rows. `prefetch` runs while S is
// computed (the caller's next Q rows into registers). Returns false when a
// wait ran out (the abort flag and the status word are set).
template <int HD, int NK, class F>
__device__ __forceinline__ bool attend_tile(const AttnParams &p, const TcSmem &s, uint32_t tmem, int start, int len,
                                            int kvh, int groups, int tile, uint32_t &phase, F &&prefetch) {
    using C = AttnTc<HD, NK>;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int row = 32 * quarter + lane;  // this thread's query row of the tile
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
    const uint32_t s_cols = tmem, o_cols = tmem + NK;
    const int qd = p.heads * HD;

    // ---- S = Q . K^T ----
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(kTcRows, NK);
#pragma unroll
        for (int dr = 0; dr < HD / 64; dr++) {
            const uint64_t ah = sw128_kmajor_desc(smem_u32(s.qh + dr * C::kQRegion));
            const uint64_t al = sw128_kmajor_desc(smem_u32(s.ql + dr * C::kQRegion));
            const uint64_t bh = sw128_kmajor_desc(smem_u32(s.kh + dr * C::kKRegion));
            const uint64_t bl = sw128_kmajor_desc(smem_u32(s.kl + dr * C::kKRegion));
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                mma3(s_cols, ah + 2 * kk, al + 2 * kk, bh + 2 * kk, bl + 2 * kk, idesc, (dr | kk) ? 1u : 0u);
        }
        tc_commit(s.bar);
    }
    prefetch();
    if (!mbar_wait(s.bar, phase, s.abort, p.status)) return false;
    phase ^= 1;
    tc_fence_after();

    // ---- softmax over this thread's half of the row, P over the Q tile ----
    const int slot = tile * C::kHpt + row / NK, pos = row % NK;
    const bool valid = slot < groups && pos < len;
    softmax_to_p<HD, NK>(p, s, s_cols + lane_addr, half, row, valid, pos);

    // ---- O = P . V ----
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16_f32(kTcRows, HD);
        const int key_steps = max(1, (min(len, NK) + 15) / 16);  // P and V are zero past the prompt
        for (int ks = 0; ks < key_steps; ks++) {
            const int kr = ks >> 2, kk = ks & 3;
            const uint64_t ah = sw128_kmajor_desc(smem_u32(s.qh + kr * C::kPRegion)) + 2 * kk;
            const uint64_t al = sw128_kmajor_desc(smem_u32(s.ql + kr * C::kPRegion)) + 2 * kk;
            const uint64_t bh = sw128_kmajor_desc(smem_u32(s.vh + kr * C::kVRegion)) + 2 * kk;
            const uint64_t bl = sw128_kmajor_desc(smem_u32(s.vl + kr * C::kVRegion)) + 2 * kk;
            mma3(o_cols, ah, al, bh, bl, idesc, ks ? 1u : 0u);
        }
        tc_commit(s.bar);
    }
    if (!mbar_wait(s.bar, phase, s.abort, p.status)) return false;
    phase ^= 1;
    tc_fence_after();

    // ---- out = O / l, this thread's half of the dims ----
    // (tcgen05.ld is warp-collective: every lane loads, valid rows store)
    const float inv = valid ? 1.0f / (s.red[2 * kTcRows + row] + s.red[3 * kTcRows + row]) : 0.0f;
    uint16_t *dst =
        valid ? p.out + (long long)(start + pos) * qd + (kvh * groups + slot) * HD + half * (HD / 2) : nullptr;
#pragma unroll
    for (int c = 0; c < HD / 2; c += 32) {
        float t[32];
        tmem_ld32(o_cols + lane_addr + half * (HD / 2) + c, t);
        if (!valid) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint4 w;
            w.x = pack_bf16x2(t[8 * j + 0] * inv, t[8 * j + 1] * inv);
            w.y = pack_bf16x2(t[8 * j + 2] * inv, t[8 * j + 3] * inv);
            w.z = pack_bf16x2(t[8 * j + 4] * inv, t[8 * j + 5] * inv);
            w.w = pack_bf16x2(t[8 * j + 6] * inv, t[8 * j + 7] * inv);
            *reinterpret_cast<uint4 *>(dst + c + 8 * j) = w;
        }
    }
    return true;
}

// One CTA per item, loads through registers.
template <int HD, int NK>
__global__ void __launch_bounds__(kTcThreads, 1) k_attention_tc(AttnParams p) {
    using C = AttnTc<HD, NK>;
    const int b = blockIdx.x, kvh = blockIdx.y;
    const int start = p.seq_start[b], len = min(p.seq_len[b], NK);
    if (len <= 0) return;
    extern __shared__ uint8_t smem_raw[];
    const TcSmem s = carve_tc<HD, NK>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int groups = p.heads / p.kv_heads, tiles = (groups + C::kHpt - 1) / C::kHpt;
    const int width = (p.heads + 2 * p.kv_heads) * HD, qd = p.heads * HD, kvd = p.kv_heads * HD;

    if (tid == 0) {
        mbar_init(s.bar, 1);
        *s.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(s.tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }

    // first Q tile, keys and values: all loads of a batch in flight before
    // their conversions
    float4 q[C::kQLoads];
    load_q_tile<HD, NK>(p, start, len, kvh, groups, 0, q);
    {
        float4 k[C::kKLoads];
#pragma unroll
        for (int u = 0; u < C::kKLoads; u++) {
            const int f = tid + kTcThreads * u, r = f / (HD / 4), d = 4 * (f % (HD / 4));
            k[u] = r < len ? __ldg(reinterpret_cast<const float4 *>(p.qkv + (long long)(start + r) * width + qd +
                                                                     kvh * HD + d))
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < C::kKLoads; u++) {
            const int f = tid + kTcThreads * u, r = f / (HD / 4), d = 4 * (f % (HD / 4));
            put_rowvec(s.kh, s.kl, C::kKRegion, r, d, k[u]);
        }
    }
#pragma unroll
    for (int u = 0; u < C::kVUnits; u++) {
        // unit: 8 keys x 4 dims; the 8 lanes of a dim group take the 8 key
        // groups, so each store instruction covers whole 128-byte rows
        const int un = tid + kTcThreads * u;
        if (un >= C::kVTotal) break;
        const int rest = un >> 3, dg = rest % (HD / 4), kg = (rest / (HD / 4)) * 8 + (un & 7);
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int key = 8 * kg + i;
            v[i] = key < len ? __ldg(reinterpret_cast<const float4 *>(p.qkv + (long long)(start + key) * width + qd +
                                                                       kvd + kvh * HD + 4 * dg))
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = e == 0 ? v[i].x : e == 1 ? v[i].y : e == 2 ? v[i].z : v[i].w;
            put_vchunk<HD, NK>(s, 4 * dg + e, kg, x);
        }
    }
    store_q_tile<HD, NK>(s, q);

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s.tmem_slot;
    uint32_t phase = 0;
    for (int tile = 0; tile < tiles; tile++) {
        const bool more = tile + 1 < tiles;
        if (!attend_tile<HD, NK>(p, s, tmem, start, len, kvh, groups, tile, phase, [&] {
                if (more) load_q_tile<HD, NK>(p, start, len, kvh, groups, tile + 1, q);
            }))
            break;
        if (more) store_q_tile<HD, NK>(s, q);  // P is consumed: the next queries go over it
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// Prompts of at most 64 tokens with two CTAs per SM, so that one CTA's
// loads and waits overlap the other's work. The Q tile is staged one 64-dim
// half at a time (S accumulates over the halves); P and then the tile's bf16
// output rows reuse those 32 KB. Operands take 96 KB per CTA (head_dim 128),
// registers at most 128 per thread. The output rows leave through shared
// memory as whole-row stores.
template <int HD>
struct AttnTc2 {
    static constexpr int NK = 64;
    static constexpr int kHalfBytes = kTcRows * 128;  // one 64-dim half of the Q tile, hi or lo
    static constexpr int kKRegion = NK * 128;
    static constexpr int kKBytes = kKRegion * (HD / 64);
    static constexpr int kVBytes = HD * 128;  // V^T: HD rows of 64 keys
    static constexpr int kOperandBytes = 2 * (kHalfBytes + kKBytes + kVBytes);
    static constexpr int kSmemBytes = 1024 + kOperandBytes + 4 * kTcRows * sizeof(float) + 64;
    static constexpr uint32_t kTmemCols = (NK + HD) <= 128 ? 128 : 256;
    static constexpr int kQLoads = kTcRows * 64 / 4 / kTcThreads;  // float4 per thread for a Q half
    static constexpr int kKLoads = NK * HD / 4 / kTcThreads;
    static constexpr int kVTotal = (NK / 8) * (HD / 4);
    static constexpr int kVUnits = (kVTotal + kTcThreads - 1) / kTcThreads;
    static constexpr int kCpr = HD / 8;  // 16-byte chunks per output row
    static_assert(kTcRows * HD * 2 <= 2 * kHalfBytes, "output rows fit over the Q halves");
};

template <int HD>
__device__ __forceinline__ void load_q_half(const AttnParams &p, int start, int len, int kvh, int groups, int tile,
                                            int dr, float4 (&q)[AttnTc2<HD>::kQLoads]) {
    using C = AttnTc2<HD>;
    const int width = (p.heads + 2 * p.kv_heads) * HD;
#pragma unroll
    for (int u = 0; u < C::kQLoads; u++) {
        const int f = threadIdx.x + kTcThreads * u, r = f / 16, d = 64 * dr + 4 * (f % 16);
        const int slot = tile * 2 + r / C::NK, pos = r % C::NK;
        q[u] = (slot < groups && pos < len)
                   ? __ldg(reinterpret_cast<const float4 *>(p.qkv + (long long)(start + pos) * width +
                                                            (kvh * groups + slot) * HD + d))
                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
}

template <int HD>
__device__ __forceinline__ void store_q_half(const TcSmem &s, const float4 (&q)[AttnTc2<HD>::kQLoads]) {
#pragma unroll
    for (int u = 0; u < AttnTc2<HD>::kQLoads; u++) {
        const int f = threadIdx.x + kTcThreads * u;
        put_rowvec(s.qh, s.ql, 0, f / 16, 4 * (f % 16), q[u]);
    }
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, 2) k_attention_tc2(AttnParams p) {
    using C = AttnTc2<HD>;
    constexpr int NK = C::NK;
    const int b = blockIdx.x, kvh = blockIdx.y;
    const int start = p.seq_start[b], len = min(p.seq_len[b], NK);
    if (len <= 0) return;
    extern __shared__ uint8_t smem_raw[];
    TcSmem s;
    {
        uint8_t *base =
            reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
        s.qh = base;
        s.ql = s.qh + C::kHalfBytes;
        s.kh = s.ql + C::kHalfBytes;
        s.kl = s.kh + C::kKBytes;
        s.vh = s.kl + C::kKBytes;
        s.vl = s.vh + C::kVBytes;
        s.red = reinterpret_cast<float *>(s.vl + C::kVBytes);
        s.bar = reinterpret_cast<uint64_t *>(s.red + 4 * kTcRows);
        s.tmem_slot = reinterpret_cast<uint32_t *>(s.bar + 1);
        s.abort = reinterpret_cast<volatile int *>(s.tmem_slot + 1);
    }
    uint8_t *stage = s.qh;  // the tile's bf16 output rows, [128][HD] with swizzled 16-byte chunks
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int groups = p.heads / p.kv_heads, tiles = (groups + 1) / 2;
    const int width = (p.heads + 2 * p.kv_heads) * HD, qd = p.heads * HD, kvd = p.kv_heads * HD;

    if (tid == 0) {
        mbar_init(s.bar, 1);
        *s.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(s.tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }

    float4 q[C::kQLoads];
    load_q_half<HD>(p, start, len, kvh, groups, 0, 0, q);
    {
        float4 k[C::kKLoads];
#pragma unroll
        for (int u = 0; u < C::kKLoads; u++) {
            const int f = tid + kTcThreads * u, r = f / (HD / 4), d = 4 * (f % (HD / 4));
            k[u] = r < len ? __ldg(reinterpret_cast<const float4 *>(p.qkv + (long long)(start + r) * width + qd +
                                                                     kvh * HD + d))
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < C::kKLoads; u++) {
            const int f = tid + kTcThreads * u, r = f / (HD / 4), d = 4 * (f % (HD / 4));
            put_rowvec(s.kh, s.kl, C::kKRegion, r, d, k[u]);
        }
    }
#pragma unroll
    for (int u = 0; u < C::kVUnits; u++) {
        const int un = tid + kTcThreads * u;
        if (un >= C::kVTotal) break;
        const int rest = un >> 3, dg = rest % (HD / 4), kg = un & 7;
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int key = 8 * kg + i;
            v[i] = key < len ? __ldg(reinterpret_cast<const float4 *>(p.qkv + (long long)(start + key) * width + qd +
                                                                       kvd + kvh * HD + 4 * dg))
                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = e == 0 ? v[i].x : e == 1 ? v[i].y : e == 2 ? v[i].z : v[i].w;
            put_vchunk<HD, NK>(s, 4 * dg + e, kg, x);
        }
    }
    store_q_half<HD>(s, q);

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s.tmem_slot;
    const uint32_t s_cols = tmem, o_cols = tmem + NK;
    const int quarter = warp & 3, half = warp >> 2;
    const int row = 32 * quarter + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
    uint32_t phase = 0;
    bool ok = true;

    for (int tile = 0; tile < tiles && ok; tile++) {
        // ---- S = Q . K^T, one 64-dim half of Q at a time ----
        for (int dr = 0; dr < HD / 64; dr++) {
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                constexpr uint32_t idesc = idesc_bf16_f32(kTcRows, NK);
                const uint64_t ah = sw128_kmajor_desc(smem_u32(s.qh)), al = sw128_kmajor_desc(smem_u32(s.ql));
                const uint64_t bh = sw128_kmajor_desc(smem_u32(s.kh + dr * C::kKRegion));
                const uint64_t bl = sw128_kmajor_desc(smem_u32(s.kl + dr * C::kKRegion));
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    mma3(s_cols, ah + 2 * kk, al + 2 * kk, bh + 2 * kk, bl + 2 * kk, idesc, (dr | kk) ? 1u : 0u);
                tc_commit(s.bar);
            }
            const bool next_half = dr + 1 < HD / 64;
            if (next_half) load_q_half<HD>(p, start, len, kvh, groups, tile, dr + 1, q);
            if (!mbar_wait(s.bar, phase, s.abort, p.status)) {
                ok = false;
                break;
            }
            phase ^= 1;
            tc_fence_after();
            if (next_half) store_q_half<HD>(s, q);  // this half's products are done
        }
        if (!ok) break;

        // ---- softmax into P over the Q region ----
        const int slot = tile * 2 + row / NK, pos = row % NK;
        const bool valid = slot < groups && pos < len;
        softmax_to_p<HD, NK>(p, s, s_cols + lane_addr, half, row, valid, pos);

        // ---- O = P . V ----
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            constexpr uint32_t idesc = idesc_bf16_f32(kTcRows, HD);
            const int key_steps = (len + 15) / 16;  // P and V are zero past the prompt
            const uint64_t ah = sw128_kmajor_desc(smem_u32(s.qh)), al = sw128_kmajor_desc(smem_u32(s.ql));
            const uint64_t bh = sw128_kmajor_desc(smem_u32(s.vh)), bl = sw128_kmajor_desc(smem_u32(s.vl));
            for (int kk = 0; kk < key_steps; kk++)
                mma3(o_cols, ah + 2 * kk, al + 2 * kk, bh + 2 * kk, bl + 2 * kk, idesc, kk ? 1u : 0u);
            tc_commit(s.bar);
        }
        const bool more = tile + 1 < tiles;
        if (more) load_q_half<HD>(p, start, len, kvh, groups, tile + 1, 0, q);
        if (!mbar_wait(s.bar, phase, s.abort, p.status)) {
            ok = false;
            break;
        }
        phase ^= 1;
        tc_fence_after();

        // ---- out = O / l: bf16 rows into the staging area, then whole-row stores ----
        const float inv = valid ? 1.0f / (s.red[2 * kTcRows + row] + s.red[3 * kTcRows + row]) : 0.0f;
#pragma unroll
        for (int c = 0; c < HD / 2; c += 32) {
            float t[32];
            tmem_ld32(o_cols + lane_addr + half * (HD / 2) + c, t);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint4 w;
                w.x = pack_bf16x2(t[8 * j + 0] * inv, t[8 * j + 1] * inv);
                w.y = pack_bf16x2(t[8 * j + 2] * inv, t[8 * j + 3] * inv);
                w.z = pack_bf16x2(t[8 * j + 4] * inv, t[8 * j + 5] * inv);
                w.w = pack_bf16x2(t[8 * j + 6] * inv, t[8 * j + 7] * inv);
                const int jj = (half * (HD / 2) + c) / 8 + j;
                *reinterpret_cast<uint4 *>(stage + row * (HD * 2) + ((jj ^ (row & (C::kCpr - 1))) << 4)) = w;
            }
        }
        tc_fence_before();
        __syncthreads();
#pragma unroll
        for (int idx = tid; idx < kTcRows * C::kCpr; idx += kTcThreads) {
            const int r = idx / C::kCpr, j = idx % C::kCpr;
            const int rs = tile * 2 + r / NK, rp = r % NK;
            if (rs < groups && rp < len) {
                const uint4 w =
                    *reinterpret_cast<const uint4 *>(stage + r * (HD * 2) + ((j ^ (r & (C::kCpr - 1))) << 4));
                *reinterpret_cast<uint4 *>(p.out + (long long)(start + rp) * qd + (kvh * groups + rs) * HD + 8 * j) =
                    w;
            }
        }
        if (more) {
            __syncthreads();  // the staging area is read out
            store_q_half<HD>(s, q);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}
template <int HD, int NK>
cudaError_t launch_tc(const AttnParams &p, cudaStream_t st) {
    using C = AttnTc<HD, NK>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_tc<HD, NK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    k_attention_tc<HD, NK><<<dim3(p.n_prompts, p.kv_heads), kTcThreads, C::kSmemBytes, st>>>(p);
    return cudaGetLastError();
}

template <int HD>
cudaError_t launch_tc2(const AttnParams &p, cudaStream_t st) {
    using C = AttnTc2<HD>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_tc2<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    k_attention_tc2<HD><<<dim3(p.n_prompts, p.kv_heads), kTcThreads, C::kSmemBytes, st>>>(p);
    return cudaGetLastError();
}
}  // namespace

bool attention_tc_eligible(const AttnParams &p) {
    return p.tc > 0 && !p.force_generic && !p.out_f32 && (p.head_dim == 64 || p.head_dim == 128) &&
           p.max_len >= 1 && p.max_len <= 128 && p.kv_heads <= 65535;
}

cudaError_t attention_tc(const AttnParams &p, cudaStream_t st) {
    if (p.n_prompts <= 0) return cudaSuccess;
    if (!attention_tc_eligible(p)) return cudaErrorInvalidValue;
    if (p.max_len > 64) return p.head_dim == 128 ? launch_tc<128, 128>(p, st) : launch_tc<64, 128>(p, st);
    if (p.tc >= 2) return p.head_dim == 128 ? launch_tc2<128>(p, st) : launch_tc2<64>(p, st);
    return p.head_dim == 128 ? launch_tc<128, 64>(p, st) : launch_tc<64, 64>(p, st);
}

}  // namespace ditch
