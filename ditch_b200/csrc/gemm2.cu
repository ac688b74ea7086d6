// CTA-pair tcgen05 GEMM (cta_group::2) for bf16 weights and wide token tiles:
// the products of a prefill-sized forward (C2: 8192 tokens per GEMM).
//
// Two CTAs of a cluster share one 256-row output tile. CTA r of the pair
// loads weight rows [128 r, 128 r + 128) of the tile and token rows
// [BN/2 r, BN/2 r + BN/2) of the token tile; the even CTA issues one
// tcgen05.mma.cta_group::2 (M = 256) per 16-wide k-step, which reads both
// CTAs' shared memory and writes each CTA's 128 accumulator rows (all BN
// token columns) into that CTA's TMEM. Per SM and k-stage this moves 32 KB
// through shared memory for 128 x BN x 64 products instead of the one-CTA
// kernel's 16 + BN/8 KB for 128 x BN x 64: a third less operand traffic at
// BN = 256, which is what limits the one-CTA kernel's tensor-pipe occupancy.
//
// Roles per CTA (192 threads, 320 for SwiGLU): warp 0 TMA producer (both CTAs: their own
// halves, completing on the even CTA's stage barrier); warp 1 TMEM
// allocator (both, a pair allocation) and MMA issuer (even CTA only); warps
// 2-5 (2-9 for SwiGLU) epilogue (both: their own 128 rows). The even CTA's MMA commits free a
// stage and hand over an accumulator in both CTAs at once (multicast commit).
// No TMA multicast: each CTA loads only its own tiles from this GPU's memory.
//
// Every mbarrier wait is bounded; a timeout sets the status word and the
// roles unwind. The pair meets at a cluster barrier before TMEM is freed,
// so neither CTA leaves while the other may still touch its shared memory.
#include <algorithm>

#include "gemm.cuh"

namespace ditch {

namespace {

constexpr int PBM = 128;  // weight rows per CTA (256 per pair)
constexpr int PBK = 64;
// epilogue warps: 4 (one per TMEM lane quarter), 8 for SwiGLU (two per lane
// quarter, each taking half the token columns: the two accumulators fill
// TMEM, so the next tile's MMAs wait until the SwiGLU values are in
// registers; the stores follow the hand-back)
template <bool DUAL>
constexpr int pair_epi_warps() { return DUAL ? 8 : 4; }
constexpr int kPSmemBudget = 224 * 1024;

template <int BN, bool DUAL>
struct PairCfg {
    static constexpr int kNA = DUAL ? 2 : 1;
    static constexpr int kABytes = PBM * PBK * 2;
    static constexpr int kBBytes = (BN / 2) * PBK * 2;  // this CTA's half of the token tile
    static constexpr int kStageBytes = kNA * kABytes + kBBytes;
    static constexpr int kStagesFit = kPSmemBudget / kStageBytes;
    static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
    static constexpr int kAccCols = kNA * BN;
    static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
    static constexpr int kTmemColsRaw = kAccBufs * kAccCols;
    static constexpr int kTmemCols = kTmemColsRaw < 32 ? 32 : kTmemColsRaw;
    static constexpr int kEpi = pair_epi_warps<DUAL>();
    static constexpr int kWarps = 2 + kEpi;
    static constexpr int kThreads = kWarps * 32;
    // full, empty, 2 tfull, 2 tempty; then the TMEM base and the abort word
    static constexpr int kBarBytes = (8 * (2 * kStages + 4) + 16 + 63) / 64 * 64;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + kBarBytes;
    static_assert(kSmemBytes <= 232448, "over the 227 KB of shared memory per block");
    static_assert(kStages >= 3, "shared memory too small");
    static_assert(kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM columns");
    static_assert(BN % 16 == 0 && BN / 2 >= 16 && BN <= 256, "N of a cta_group::2 MMA");
};

template <class C>
struct PairSmem {
    uint8_t *base;
    uint64_t *full, *empty, *tfull, *tempty;
    uint32_t *tmem_base;
    int *abort;
    __device__ __forceinline__ uint8_t *a(int s, int i) const { return base + s * C::kStageBytes + i * C::kABytes; }
    __device__ __forceinline__ uint8_t *b(int s) const { return base + s * C::kStageBytes + C::kNA * C::kABytes; }
};

template <class C>
__device__ __forceinline__ PairSmem<C> pair_carve(uint8_t *smem_raw) {
    PairSmem<C> L;
    uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    L.base = reinterpret_cast<uint8_t *>(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(L.base + C::kStages * C::kStageBytes);
    L.full = bars;
    L.empty = bars + C::kStages;
    L.tfull = bars + 2 * C::kStages;
    L.tempty = L.tfull + 2;
    L.tmem_base = reinterpret_cast<uint32_t *>(L.tempty + 2);
    L.abort = reinterpret_cast<int *>(L.tmem_base + 1);
    return L;
}

// ---- PTX of the CTA pair ----------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of the variable at shared::cta address `addr`
// in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2D tiled load into this CTA's shared memory, completing on the mbarrier at
// shared::cluster address `bar` (the even CTA's stage barrier).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap *map, uint32_t bar, void *dst, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on the mbarrier at `bar` (shared::cta offset) in both CTAs of the
// pair once every earlier tcgen05.mma of this thread has completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// A bounded wait with cluster-scope acquire (the barrier receives arrivals
// or transaction bytes from the other CTA of the pair).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort, int *status) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    long long start = clock64();
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - start > kWaitBudgetCycles) {
            *abort = 1;
            if (status) atomicExch(status, kKernelWaitTimeout);
            return false;
        }
    }
}

// silu with the approximate exponential and division of the SFU (a few ulp
// of f32, far below the bf16 rounding of the product that follows)
__device__ __forceinline__ float silu_p(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// 32 lanes x 16 columns of TMEM into registers, without waiting: the values
// are defined only after tmem_wait_pass on the same array.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

#define DITCH_R8(a, i) "+r"(a[i]), "+r"(a[i + 1]), "+r"(a[i + 2]), "+r"(a[i + 3]), \
    "+r"(a[i + 4]), "+r"(a[i + 5]), "+r"(a[i + 6]), "+r"(a[i + 7])

// Waits for every TMEM load this thread issued. Both arrays pass through the
// asm statement, so no use of their values can be scheduled above the wait.
__device__ __forceinline__ void tmem_wait_pass(uint32_t (&a)[16], uint32_t (&b)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : DITCH_R8(a, 0), DITCH_R8(a, 8), DITCH_R8(b, 0), DITCH_R8(b, 8)
                 :
                 : "memory");
}
#undef DITCH_R8

// silu(g + bias) * u over 16 columns, rounded to bf16 (to nearest even, as
// f32_to_bf16_bits for every non-NaN value) and packed two per word.
__device__ __forceinline__ void swiglu16_bf16(const uint32_t (&g)[16], const uint32_t (&u)[16], float bias,
                                              uint32_t (&pk)[8]) {
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float lo = silu_p(__uint_as_float(g[2 * j]) + bias) * __uint_as_float(u[2 * j]);
        const float hi = silu_p(__uint_as_float(g[2 * j + 1]) + bias) * __uint_as_float(u[2 * j + 1]);
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pk[j]) : "f"(hi), "f"(lo));
    }
}

// Pair tile `tile`: weight tile (256 rows) and token tile (BN), in bands of
// 16 token tiles run weight tile by weight tile (the tiles the 74 pairs hold
// at once share a few operand tiles, which stay in L2). Measured on the C2
// trial over two boxes: bands of 16 took 1.3-1.7 % less time per trial than
// bands of 8; 4, 24 and 32 were slower than 8 or level with it; 12 came
// within run-to-run noise of 16.
__device__ __forceinline__ void pair_tile(const GemmParams &p, int tile, int bn, int &wt, int &tok0) {
    constexpr int kBand = 16;
    const int band = tile / (kBand * p.w_tiles);
    const int idx = tile - band * kBand * p.w_tiles;
    const int g = min(kBand, p.t_tiles - band * kBand);
    wt = idx / g;
    tok0 = (band * kBand + idx % g) * bn;
}

template <int BN, bool DUAL>
__global__ void __launch_bounds__(PairCfg<BN, DUAL>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                     const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using C = PairCfg<BN, DUAL>;
    extern __shared__ uint8_t smem_raw[];
    PairSmem<C> L = pair_carve<C>(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0: the even CTA (MMA issuer)
    volatile int *abort = L.abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&L.full[s], 1);   // the even CTA's producer arrives; both CTAs' bytes complete it
            mbar_init(&L.empty[s], 1);  // the MMA commit
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&L.tfull[b], 1);
            mbar_init(&L.tempty[b], 2 * C::kEpi);  // both CTAs' epilogue warps (used in the even CTA)
        }
        *L.abort = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (DUAL) tma_prefetch_desc(&tmA2);
    }
    if (warp == 1) {
        tmem_alloc_pair(L.tmem_base, C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *L.tmem_base;

    const int pairs = gridDim.x / 2, pair = blockIdx.x / 2;
    const int tiles = p.w_tiles * p.t_tiles;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int it = 0;
            const uint32_t full0 = mapa_shared(smem_u32(&L.full[0]), 0);
            for (int tile = pair; tile < tiles && !*abort; tile += pairs) {
                int wt, tok0;
                pair_tile(p, tile, BN, wt, tok0);
                const int arow = p.a_row0 + wt * 2 * PBM + (int)rank * PBM;
                const int brow = tok0 + (int)rank * (BN / 2);
                for (int kt = 0; kt < p.k_tiles; kt++, it++) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait_cluster(&L.empty[s], ph ^ 1, abort, p.status)) break;
                    const uint32_t fb = full0 + s * 8;  // the even CTA's full[s]
                    if (rank == 0) mbar_arrive_expect_tx(&L.full[s], 2 * C::kStageBytes);
                    tma_load_2d_pair(&tmA, fb, L.a(s, 0), kt * PBK, arow);
                    if (DUAL) tma_load_2d_pair(&tmA2, fb, L.a(s, 1), kt * PBK, arow + p.a2_row_offset);
                    tma_load_2d_pair(&tmB, fb, L.b(s), kt * PBK, brow);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (the even CTA) ----------------
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(2 * PBM, BN);
            int it = 0, local = 0;
            for (int tile = pair; tile < tiles && !*abort; tile += pairs, local++) {
                const int buf = local % C::kAccBufs;
                const uint32_t use_ph = (local / C::kAccBufs) & 1;
                if (!mbar_wait_cluster(&L.tempty[buf], use_ph ^ 1, abort, p.status)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * C::kAccCols;
                bool ok = true;
                for (int kt = 0; kt < p.k_tiles; kt++, it++) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait_cluster(&L.full[s], ph, abort, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_kmajor_desc(smem_u32(L.a(s, 0)));
                    const uint64_t bdesc = sw128_kmajor_desc(smem_u32(L.b(s)));
                    const uint64_t a2desc = DUAL ? sw128_kmajor_desc(smem_u32(L.a(s, 1))) : 0;
#pragma unroll
                    for (int kk = 0; kk < PBK / 16; kk++) {
                        const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
                        tc_mma_bf16_pair(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, acc);
                        if (DUAL) tc_mma_bf16_pair(d + BN, a2desc + 2 * kk, bdesc + 2 * kk, idesc, acc);
                    }
                    tc_commit_pair(&L.empty[s]);
                }
                if (!ok) break;
                tc_commit_pair(&L.tfull[buf]);
            }
        }
    } else {
        // ---------------- epilogue (both CTAs: their own 128 rows) ----------------
        const int q = warp & 3;                   // TMEM lane quarter of this warp
        const int part = (warp - 2) / 4;          // column half (8 epilogue warps) or 0
        const int c_beg = part * (BN * 4 / C::kEpi), c_end = c_beg + BN * 4 / C::kEpi;
        const int trow = q * 32 + lane;
        const uint32_t tempty0 = mapa_shared(smem_u32(&L.tempty[0]), 0);
        int local = 0;
        for (int tile = pair; tile < tiles && !*abort; tile += pairs, local++) {
            int wt, tok0;
            pair_tile(p, tile, BN, wt, tok0);
            const int buf = local % C::kAccBufs;
            const uint32_t use_ph = (local / C::kAccBufs) & 1;
            if (!mbar_wait_cluster(&L.tfull[buf], use_ph, abort, p.status)) break;
            tc_fence_after();
            const int n = wt * 2 * PBM + (int)rank * PBM + trow;  // weight row = output feature
            const bool n_ok = n < p.m_w;
            const float bias = (p.bias && n_ok) ? p.bias[n] : 0.0f;
            const int drank = p.delta_rank > 1 ? p.delta_rank : 1;
            float dbn[kMaxDeltaRank];
            bool any_delta = false;
#pragma unroll
            for (int t = 0; t < kMaxDeltaRank; t++) {
                dbn[t] = (p.db && n_ok && t < drank) ? p.db[(long long)n * drank + t] : 0.0f;
                any_delta |= dbn[t] != 0.0f;
            }
            const uint32_t tbase = tmem + buf * C::kAccCols + (static_cast<uint32_t>(q * 32) << 16);
            const int m_end = min(p.n_tok, tok0 + BN);
            if constexpr (DUAL) {
                // One accumulator buffer: the next tile's MMAs wait for it.
                // So the warp reads its gate and up columns (both loads of a
                // chunk in flight together), forms silu(gate) * up as bf16 in
                // registers, hands the accumulator back, and only then stores.
                constexpr int kCh = BN * 4 / C::kEpi / 16;  // 16-column chunks per warp
                static_assert(kCh % 2 == 0, "chunks go in pairs");
                uint32_t pk[kCh][8];                         // bf16 pairs (even token low)
                const uint32_t tw = tbase + c_beg;
                // chunk ci holds tokens from tok0 + c_beg + 16 ci; once one is past
                // the last token, so are the later ones (warp-uniform)
                auto live = [&](int ci) { return tok0 + c_beg + ci * 16 < m_end; };
                // the next chunk's two loads are in flight while this chunk is formed
                uint32_t ga[16], ua[16], gb[16], ub[16];
                if (live(0)) {
                    tmem_ld16_issue(tw, ga);
                    tmem_ld16_issue(tw + BN, ua);
                }
#pragma unroll
                for (int ci = 0; ci < kCh; ci += 2) {
                    if (live(ci)) {
                        tmem_wait_pass(ga, ua);
                        if (live(ci + 1)) {
                            tmem_ld16_issue(tw + (ci + 1) * 16, gb);
                            tmem_ld16_issue(tw + BN + (ci + 1) * 16, ub);
                        }
                        swiglu16_bf16(ga, ua, bias, pk[ci]);
                    }
                    if (live(ci + 1)) {
                        tmem_wait_pass(gb, ub);
                        if (ci + 2 < kCh && live(ci + 2)) {
                            tmem_ld16_issue(tw + (ci + 2) * 16, ga);
                            tmem_ld16_issue(tw + BN + (ci + 2) * 16, ua);
                        }
                        swiglu16_bf16(gb, ub, bias, pk[ci + 1]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tempty0 + buf * 8);  // the even CTA's tempty[buf]
                if (n_ok) {
                    uint16_t *ob = reinterpret_cast<uint16_t *>(p.out) + n;
#pragma unroll
                    for (int ci = 0; ci < kCh; ci++) {
                        const int m0 = tok0 + c_beg + ci * 16;
                        if (m0 < m_end) {
                            const int mv = min(16, m_end - m0);
#pragma unroll
                            for (int j = 0; j < 16; j++)
                                if (j < mv)
                                    ob[(long long)(m0 + j) * p.ldo] =
                                        static_cast<uint16_t>((j & 1) ? (pk[ci][j >> 1] >> 16) : pk[ci][j >> 1]);
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c0 = c_beg; c0 < c_end; c0 += 32) {
                    if (tok0 + c0 >= m_end) break;  // warp-uniform
                    float v[32], u[32];
                    tmem_ld32(tbase + c0, v);
                    if (DUAL) tmem_ld32(tbase + BN + c0, u);
                    const int m0 = tok0 + c0;
                    const int mv = min(32, m_end - m0);
                    // every load of a chunk before its first store (see the one-CTA kernel)
                    float r[32];
#pragma unroll
                    for (int j = 0; j < 32; j++) r[j] = v[j];
                    if (p.xa && any_delta) {
#pragma unroll 1
                        for (int t = 0; t < drank; t++) {
                            float xa[32];
#pragma unroll
                            for (int j = 0; j < 32; j++) xa[j] = j < mv ? __ldg(p.xa + (long long)(m0 + j) * drank + t) : 0.0f;
#pragma unroll
                            for (int j = 0; j < 32; j++) r[j] += xa[j] * dbn[t];
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; j++) r[j] += bias;
                    const long long o0 = (long long)m0 * p.ldo + n;
                    if (!n_ok) {
                    } else if (DUAL) {
                        uint16_t *ob = reinterpret_cast<uint16_t *>(p.out) + o0;
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (j < mv) ob[(long long)j * p.ldo] = f32_to_bf16_bits(silu_p(r[j]) * u[j]);
                    } else if (p.flags & kEpiResidual) {
                        float *of = reinterpret_cast<float *>(p.out) + o0;
                        float old[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) old[j] = j < mv ? of[(long long)j * p.ldo] : 0.0f;
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (j < mv) of[(long long)j * p.ldo] = old[j] + r[j];
                    } else if (p.flags & kEpiOutBf16) {
                        uint16_t *ob = reinterpret_cast<uint16_t *>(p.out) + o0;
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (j < mv) ob[(long long)j * p.ldo] = f32_to_bf16_bits(r[j]);
                    } else {
                        float *of = reinterpret_cast<float *>(p.out) + o0;
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (j < mv) of[(long long)j * p.ldo] = r[j];
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tempty0 + buf * 8);  // the even CTA's tempty[buf]
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the pair's MMAs, loads and arrivals are done before TMEM goes
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, C::kTmemCols);
}

template <int BN, bool DUAL>
cudaError_t launch_pair_t(const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p,
                          int num_sms, cudaStream_t stream) {
    using C = PairCfg<BN, DUAL>;
    CUtensorMap ma, ma2, mb;
    bool ok = gemm_map_bf16(&ma, a.ptr, a.cols, a.rows, a.row_bytes, PBM);
    if (ok && DUAL) ok = gemm_map_bf16(&ma2, a2->ptr, a2->cols, a2->rows, a2->row_bytes, PBM);
    if (!DUAL) ma2 = ma;
    if (ok) ok = gemm_map_bf16(&mb, b.ptr, b.cols, b.rows, b.row_bytes, BN / 2);
    if (!ok) return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<BN, DUAL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    p.k_tiles = (p.k + PBK - 1) / PBK;
    p.kt_unit = 1;
    p.k_splits = 1;
    p.w_tiles = (p.m_w + 2 * PBM - 1) / (2 * PBM);
    p.t_tiles = (p.n_tok + BN - 1) / BN;
    const int tiles = p.w_tiles * p.t_tiles;
    const int pairs = std::min(tiles, num_sms / 2);
    if (pairs <= 0) return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<BN, DUAL>, ma, ma2, mb, p);
}

}  // namespace

bool gemm_pair_fits(const GemmParams &p, int fmt, int k, int num_sms) {
    // dense bf16 products over at least one full pair tile of weights and
    // enough token tiles to fill the pairs; no K splits, stream-K or atomics;
    // SwiGLU pairs only at level 2
    const bool dual = (p.flags & kEpiSwiglu) != 0;
    // (a SwiGLU product with a delta term, which no caller makes, takes the one-CTA kernel)
    return p.cta_pairs >= (dual ? 2 : 1) && !(dual && p.xa) && fmt == kFmtBf16 && !p.sched && p.k_splits <= 1 &&
           !p.stream_k &&
           !(p.flags & kEpiAtomic) && p.m_w >= 2 * PBM && p.n_tok >= 512 && k >= 4 * PBK && num_sms >= 2;
}

cudaError_t launch_gemm_pair(const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p,
                             int num_sms, cudaStream_t stream) {
    const bool dual = (p.flags & kEpiSwiglu) != 0;
    if (dual) {
        // gate and up accumulators of 256 tokens fill TMEM (one buffer): the
        // epilogue does not overlap the next tile (eight epilogue warps keep
        // it short), but each SM moves 48 KB per 2 x 128 x 256 x 64 products
        if (!a2) return cudaErrorInvalidValue;
        return launch_pair_t<256, true>(a, a2, b, p, num_sms, stream);
    }
    return launch_pair_t<256, false>(a, a2, b, p, num_sms, stream);
}

}  // namespace ditch
