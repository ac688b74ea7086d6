// Persistent, warp-specialised tcgen05 GEMM with TMEM accumulators and
// fused weight decode. See gemm.cuh for the contract.
//
// Roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: weight tile (or its raw quantised codes) and
//               token tile into a ring of shared-memory stages;
//   warp 1      TMEM allocator and MMA issuer (one elected lane): 4 x
//               tcgen05.mma (K = 16 each) per 64-wide k-stage, commits to
//               free the stage and, after the last k-stage, to hand the
//               accumulator to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (double-buffered in
//               TMEM so the next tile's MMAs overlap this tile's stores),
//               fused bias / rank-1 delta / residual add / SwiGLU, stores;
//   warps 6-9   (quantised weights only) transform: expand the raw tile into
//               bf16 in the 128B-swizzled K-major operand layout.
#include "gemm.cuh"

#include <algorithm>
#include <mutex>

namespace ditch {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 4;
constexpr int kXformWarps = 4;

template <int BN, bool DUAL, int FMT>
struct Cfg {
    static constexpr bool kQuant = FMT != kFmtBf16;
    static constexpr int kNA = DUAL ? 2 : 1;
    static constexpr int kABytes = BM * BK * 2;
    static constexpr int kBBytes = BN * BK * 2;
    static constexpr int kRawBytes = FMT == kFmtFp8 ? BM * BK : (FMT == kFmtMxfp4 || FMT == kFmtInt4) ? BM * BK / 2 : 0;
    static constexpr int kStageBytes = kNA * (kABytes + kRawBytes) + kBBytes;
    static constexpr int kStagesRaw = (220 * 1024) / kStageBytes;
    static constexpr int kStages = kStagesRaw > 6 ? 6 : kStagesRaw;
    static constexpr int kAccCols = kNA * BN;
    static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;
    static constexpr int kWarps = 2 + kEpiWarps + (kQuant ? kXformWarps : 0);
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
    static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
    static_assert((kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation must be a power of two");
};

// Stage s holds [A_0 | A_1 (dual) | B | raw_0 | raw_1 (dual)]; every operand
// buffer is 1024-byte aligned (the 128B swizzle atom).
template <class C>
struct SmemLayout {
    uint8_t *base;
    uint64_t *full, *empty, *rawfull, *tfull, *tempty;
    uint32_t *tmem_base;
    int *abort;
    __device__ __forceinline__ uint8_t *a(int s, int i) const { return base + s * C::kStageBytes + i * C::kABytes; }
    __device__ __forceinline__ uint8_t *b(int s) const { return base + s * C::kStageBytes + C::kNA * C::kABytes; }
    __device__ __forceinline__ uint8_t *raw(int s, int i) const {
        return base + s * C::kStageBytes + C::kNA * C::kABytes + C::kBBytes + i * C::kRawBytes;
    }
};

template <class C>
__device__ __forceinline__ SmemLayout<C> carve(uint8_t *smem_raw) {
    SmemLayout<C> L;
    uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    L.base = reinterpret_cast<uint8_t *>(base);
    uint64_t *bars = reinterpret_cast<uint64_t *>(L.base + C::kStages * C::kStageBytes);
    L.full = bars;
    L.empty = bars + C::kStages;
    L.rawfull = bars + 2 * C::kStages;
    L.tfull = bars + 3 * C::kStages;
    L.tempty = bars + 3 * C::kStages + 2;
    L.tmem_base = reinterpret_cast<uint32_t *>(bars + 3 * C::kStages + 4);
    L.abort = reinterpret_cast<int *>(L.tmem_base + 1);
    return L;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Where a tile's operands and outputs live, in dense or grouped mode.
struct TileInfo {
    int wt;        // weight tile within the matrix (slab)
    int tok0;      // first token row (of the B operand and of the output)
    int tok_cnt;   // valid token rows
    int a_row0;    // first weight row of the matrix (slab) in the A map
    int e;         // expert (grouped mode), else -1
    int kt0, kt1;  // k-tiles of this tile's split
    bool first_split;
};

template <int BN>
__device__ __forceinline__ TileInfo tile_info(const GemmParams &p, int tile, int kt_per_split) {
    TileInfo t;
    if (p.sched) {
        const int4 s = p.sched[tile];
        t.e = s.x;
        t.tok0 = s.y;
        t.tok_cnt = s.z;
        t.wt = s.w;
        t.a_row0 = p.a_row0 + s.x * p.slab_rows;
        t.kt0 = 0;
        t.kt1 = p.k_tiles;
        t.first_split = true;
        return t;
    }
    const int split = tile % p.k_splits;
    const int rest = tile / p.k_splits;
    t.e = -1;
    t.wt = rest / p.t_tiles;
    t.tok0 = (rest % p.t_tiles) * BN;
    t.tok_cnt = min(BN, p.n_tok - t.tok0);
    t.a_row0 = p.a_row0;
    t.kt0 = split * kt_per_split;
    t.kt1 = min(p.k_tiles, t.kt0 + kt_per_split);
    t.first_split = split == 0;
    return t;
}

// ---- weight decode into the swizzled operand layout ------------------------
// Thread `r` (0..127) of the transform warps writes row r of the 128 x 64 bf16
// tile: eight 16-byte chunks, chunk j at (j ^ (r & 7)) within its 128-byte row.

__device__ __forceinline__ void e4m3x4_to_f32(uint32_t w, float *f) {
    uint32_t h01, h23;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
        : "=r"(h01), "=r"(h23)
        : "r"(w));
    float2 a = __half22float2(*reinterpret_cast<__half2 *>(&h01));
    float2 b = __half22float2(*reinterpret_cast<__half2 *>(&h23));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

// FP8 E4M3 with f32 block scales: bf16(code * scale[row / br][col / bc]).
__device__ __forceinline__ void xform_fp8(const uint8_t *raw, uint8_t *arow_tile, int r, int grow, int k0,
                                          const GemmParams &p) {
    uint8_t *arow = arow_tile + r * 128;
    const int rs = (r >> 1) & 3;  // 64B swizzle of the raw tile
    const float *srow = p.scales + (long long)(grow / p.blk_rows) * p.scale_cols;
    // Block columns that are a multiple of the 64-wide k-tile share one scale
    // per tile (the 128 x 128 blocks of the BASELINE checkpoints).
    const bool one_scale = (p.blk_cols & 63) == 0;
    const float s_tile = one_scale ? __ldg(srow + k0 / p.blk_cols) : 0.0f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 64 + ((c ^ rs) << 4));
        uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = 2 * c + h;
            int col = k0 + 8 * j;
            float s = one_scale ? s_tile : ((col < p.k) ? __ldg(srow + col / p.blk_cols) : 0.0f);
            float f[8];
            e4m3x4_to_f32(words[2 * h], f);
            e4m3x4_to_f32(words[2 * h + 1], f + 4);
            uint4 o;
            o.x = pack_bf16x2(f[0] * s, f[1] * s);
            o.y = pack_bf16x2(f[2] * s, f[3] * s);
            o.z = pack_bf16x2(f[4] * s, f[5] * s);
            o.w = pack_bf16x2(f[6] * s, f[7] * s);
            *reinterpret_cast<uint4 *>(arow + ((j ^ (r & 7)) << 4)) = o;
        }
    }
}

__device__ __constant__ float kE2M1[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                           -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

__device__ __forceinline__ float e8m0_scale(uint32_t b) {
    return __uint_as_float(b == 0 ? 0x00400000u : (b << 23));
}

// MXFP4 (natural layout): bf16(e2m1[nibble] * 2^(e - 127)), low nibble first.
__device__ __forceinline__ void xform_mxfp4(const uint8_t *raw, uint8_t *arow_tile, int r, int grow, int k0,
                                            const GemmParams &p) {
    uint8_t *arow = arow_tile + r * 128;
    const uint8_t *srow = p.scales_u8 + (long long)grow * (p.k / 32);
#pragma unroll
    for (int c = 0; c < 2; c++) {  // 2 x 16 raw bytes = 64 elements
        uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 32 + c * 16);
        uint32_t words[4] = {q.x, q.y, q.z, q.w};
        const int blk = (k0 >> 5) + c;
        float s = (blk * 32 < p.k) ? e8m0_scale(__ldg(srow + blk)) : 0.0f;
#pragma unroll
        for (int h = 0; h < 4; h++) {  // one word = 8 elements = one output chunk
            const int j = 4 * c + h;
            uint32_t w = words[h];
            uint4 o;
            uint32_t *op = &o.x;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                uint32_t byte = (w >> (8 * e)) & 0xff;
                op[e] = pack_bf16x2(kE2M1[byte & 0xf] * s, kE2M1[byte >> 4] * s);
            }
            *reinterpret_cast<uint4 *>(arow + ((j ^ (r & 7)) << 4)) = o;
        }
    }
}

// INT4 pack-quantized, contiguous groups: bf16(f32(q - zp) * scale[row][g]).
__device__ __forceinline__ void xform_int4(const uint8_t *raw, uint8_t *arow_tile, int r, int grow, int k0,
                                           const GemmParams &p) {
    uint8_t *arow = arow_tile + r * 128;
    const int groups = p.scale_cols;
    const int g = k0 / p.blk_cols;  // a 64-wide k-tile lies in one group (group % 64 == 0)
    float s = (k0 < p.k) ? __ldg(p.scales + (long long)grow * groups + g) : 0.0f;
    int zq = 8;
    if (p.zeros) {
        uint32_t zw = __ldg(p.zeros + (long long)(grow >> 3) * groups + g);
        zq = (zw >> ((grow & 7) * 4)) & 0xf;
    }
#pragma unroll
    for (int c = 0; c < 2; c++) {
        uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 32 + c * 16);
        uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int h = 0; h < 4; h++) {
            const int j = 4 * c + h;
            uint32_t w = words[h];
            uint4 o;
            uint32_t *op = &o.x;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                int lo = (int)((w >> (8 * e)) & 0xf) - zq;
                int hi = (int)((w >> (8 * e + 4)) & 0xf) - zq;
                op[e] = pack_bf16x2((float)lo * s, (float)hi * s);
            }
            *reinterpret_cast<uint4 *>(arow + ((j ^ (r & 7)) << 4)) = o;
        }
    }
}

template <int BN, bool DUAL, int FMT>
__global__ void __launch_bounds__(Cfg<BN, DUAL, FMT>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
                const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using C = Cfg<BN, DUAL, FMT>;
    extern __shared__ uint8_t smem_raw[];
    SmemLayout<C> L = carve<C>(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    volatile int *abort = L.abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(&L.full[s], 1 + (C::kQuant ? kXformWarps : 0));
            mbar_init(&L.empty[s], 1);
            mbar_init(&L.rawfull[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&L.tfull[b], 1);
            mbar_init(&L.tempty[b], kEpiWarps);
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
        tmem_alloc(L.tmem_base, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *L.tmem_base;

    const int tiles = p.sched ? *p.n_sched : p.w_tiles * p.t_tiles * p.k_splits;
    const int kt_per_split = (p.k_tiles + p.k_splits - 1) / p.k_splits;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int it = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
                const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
                const int arow = ti.a_row0 + ti.wt * BM;
                for (int kt = ti.kt0; kt < ti.kt1; kt++, it++) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&L.empty[s], ph ^ 1, abort, p.status)) break;
                    if (C::kQuant) {
                        mbar_arrive_expect_tx(&L.rawfull[s], C::kNA * C::kRawBytes);
                        const int xb = kt * (FMT == kFmtFp8 ? BK : BK / 2);  // raw bytes along K
                        tma_load_2d(&tmA, &L.rawfull[s], L.raw(s, 0), xb, arow);
                        if (DUAL) tma_load_2d(&tmA2, &L.rawfull[s], L.raw(s, 1), xb, arow + p.a2_row_offset);
                        mbar_arrive_expect_tx(&L.full[s], C::kBBytes);
                    } else {
                        mbar_arrive_expect_tx(&L.full[s], C::kNA * C::kABytes + C::kBBytes);
                        tma_load_2d(&tmA, &L.full[s], L.a(s, 0), kt * BK, arow);
                        if (DUAL) tma_load_2d(&tmA2, &L.full[s], L.a(s, 1), kt * BK, arow + p.a2_row_offset);
                    }
                    tma_load_2d(&tmB, &L.full[s], L.b(s), kt * BK, ti.tok0);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
            int it = 0, local = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x, local++) {
                const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
                const int kt0 = ti.kt0, kt1 = ti.kt1;
                const int buf = local & 1;
                const uint32_t use_ph = (local >> 1) & 1;
                if (!mbar_wait(&L.tempty[buf], use_ph ^ 1, abort, p.status)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * C::kAccCols;
                bool ok = true;
                for (int kt = kt0; kt < kt1; kt++, it++) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&L.full[s], ph, abort, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_kmajor_desc(smem_u32(L.a(s, 0)));
                    const uint64_t bdesc = sw128_kmajor_desc(smem_u32(L.b(s)));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint32_t acc = (kt > kt0 || kk > 0) ? 1u : 0u;
                        tc_mma_bf16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, acc);
                        if (DUAL) {
                            const uint64_t a2desc = sw128_kmajor_desc(smem_u32(L.a(s, 1)));
                            tc_mma_bf16(d + BN, a2desc + 2 * kk, bdesc + 2 * kk, idesc, acc);
                        }
                    }
                    tc_commit(&L.empty[s]);
                }
                if (!ok) break;
                tc_commit(&L.tfull[buf]);
            }
        }
    } else if (warp < 2 + kEpiWarps) {
        // ---------------- epilogue ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int local = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x, local++) {
            const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
            const bool first_split = ti.first_split;  // bias and delta once per output
            const int buf = local & 1;
            const uint32_t use_ph = (local >> 1) & 1;
            if (!mbar_wait(&L.tfull[buf], use_ph, abort, p.status)) break;
            tc_fence_after();
            const int n = ti.wt * BM + q * 32 + lane;  // weight row = output feature
            const bool n_ok = n < p.m_w;
            const float bias = (p.bias && n_ok && first_split) ? p.bias[n] : 0.0f;
            bool delta = p.db && n_ok && first_split;
            const float *dbp = p.db;
            if (delta && ti.e >= 0) {
                delta = p.e_flags == nullptr || p.e_flags[ti.e] != 0;
                dbp = p.db + ti.e * p.db_stride;
            }
            const float dbn = delta ? dbp[n] : 0.0f;
            const uint32_t tbase = tmem + buf * C::kAccCols + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(tbase + c0, v);
                float u[32];
                if (DUAL) tmem_ld32(tbase + BN + c0, u);
                const int m0 = ti.tok0 + c0;
                const int m_end = ti.tok0 + ti.tok_cnt;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int m = m0 + j;
                    if (!n_ok || m >= m_end) continue;
                    float r = v[j];
                    if (p.xa && dbn != 0.0f) r += p.xa[m] * dbn;
                    r += bias;
                    const long long o = (long long)m * p.ldo + n;
                    if (DUAL) {
                        float g = r;
                        float up = u[j];
                        reinterpret_cast<uint16_t *>(p.out)[o] = f32_to_bf16_bits(silu_f(g) * up);
                    } else if (p.flags & kEpiAtomic) {
                        atomicAdd(reinterpret_cast<float *>(p.out) + o, r);
                    } else if (p.flags & kEpiResidual) {
                        float *po = reinterpret_cast<float *>(p.out) + o;
                        *po = *po + r;
                    } else if (p.flags & kEpiOutBf16) {
                        reinterpret_cast<uint16_t *>(p.out)[o] = f32_to_bf16_bits(r);
                    } else {
                        reinterpret_cast<float *>(p.out)[o] = r;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&L.tempty[buf]);
        }
    } else if (C::kQuant) {
        // ---------------- weight transform ----------------
        const int r = threadIdx.x - (2 + kEpiWarps) * 32;  // 0..127: tile row
        const int xw = warp - (2 + kEpiWarps);
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles && !*abort; tile += gridDim.x) {
            const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
            const int wt = ti.wt;
            bool ok = true;
            for (int kt = ti.kt0; kt < ti.kt1; kt++, it++) {
                const int s = it % C::kStages;
                const uint32_t ph = (it / C::kStages) & 1;
                if (!mbar_wait(&L.rawfull[s], ph, abort, p.status)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int i = 0; i < C::kNA; i++) {
                    int grow = ti.a_row0 + wt * BM + r + (i ? p.a2_row_offset : 0);
                    int vrow = min(grow, ti.a_row0 + (i ? p.a2_row_offset : 0) + p.m_w - 1);  // clamp side-data reads
                    if (FMT == kFmtFp8) xform_fp8(L.raw(s, i), L.a(s, i), r, vrow, kt * BK, p);
                    if (FMT == kFmtMxfp4) xform_mxfp4(L.raw(s, i), L.a(s, i), r, vrow, kt * BK, p);
                    if (FMT == kFmtInt4) xform_int4(L.raw(s, i), L.a(s, i), r, vrow, kt * BK, p);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&L.full[s]);
            }
            if (!ok) break;
            (void)xw;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// ---- host side ----------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// A 2D map over a row-major [rows][inner] tensor of `elem_bytes` elements.
bool make_map(CUtensorMap *map, const void *ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
              uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    CUresult r = fn(map, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, bool DUAL, int FMT>
cudaError_t launch_t(const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p, int num_sms,
                     cudaStream_t stream) {
    using C = Cfg<BN, DUAL, FMT>;
    CUtensorMap ma, ma2, mb;
    bool ok;
    if (FMT == kFmtBf16) {
        ok = make_map(&ma, a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.cols, a.rows, a.row_bytes, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
        if (ok && DUAL)
            ok = make_map(&ma2, a2->ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a2->cols, a2->rows, a2->row_bytes, BK,
                          BM, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
        const uint32_t raw_inner = FMT == kFmtFp8 ? BK : BK / 2;  // bytes per row per k-tile
        const CUtensorMapSwizzle sw = FMT == kFmtFp8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
        ok = make_map(&ma, a.ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.row_bytes, a.rows, a.row_bytes, raw_inner, BM,
                      sw);
        if (ok && DUAL)
            ok = make_map(&ma2, a2->ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a2->row_bytes, a2->rows, a2->row_bytes,
                          raw_inner, BM, sw);
    }
    if (!DUAL) ma2 = ma;
    if (ok)
        ok = make_map(&mb, b.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b.cols, b.rows, b.row_bytes, BK, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN, DUAL, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             C::kSmemBytes);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    p.k_tiles = (p.k + BK - 1) / BK;
    p.w_tiles = (p.m_w + BM - 1) / BM;
    p.t_tiles = (p.n_tok + BN - 1) / BN;
    if (p.k_splits < 1) p.k_splits = 1;
    if (p.k_splits > p.k_tiles) p.k_splits = p.k_tiles;
    if (p.sched) p.k_splits = 1;  // grouped tiles are whole-K
    const int tiles = p.w_tiles * p.t_tiles * p.k_splits;
    // grouped mode: the tile count is on the device; the grid is persistent
    const int grid = p.sched ? num_sms : std::min(tiles, num_sms);
    if (grid <= 0) return cudaSuccess;
    gemm_kernel<BN, DUAL, FMT><<<grid, C::kThreads, C::kSmemBytes, stream>>>(ma, ma2, mb, p);
    return cudaGetLastError();
}

template <int BN, bool DUAL>
cudaError_t dispatch_fmt(int fmt, const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p,
                         int sms, cudaStream_t st) {
    switch (fmt) {
    case kFmtBf16: return launch_t<BN, DUAL, kFmtBf16>(a, a2, b, p, sms, st);
    case kFmtFp8: return launch_t<BN, DUAL, kFmtFp8>(a, a2, b, p, sms, st);
    case kFmtMxfp4: return launch_t<BN, DUAL, kFmtMxfp4>(a, a2, b, p, sms, st);
    case kFmtInt4: return launch_t<BN, DUAL, kFmtInt4>(a, a2, b, p, sms, st);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace

cudaError_t launch_gemm(int fmt, const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p,
                        int num_sms, cudaStream_t stream) {
    const bool dual = (p.flags & kEpiSwiglu) != 0;
    if (dual && !a2) return cudaErrorInvalidValue;
    const int bn = p.bn ? p.bn : gemm_token_tile(p.n_tok, dual);
    if (dual) {
        if (bn == 32) return dispatch_fmt<32, true>(fmt, a, a2, b, p, num_sms, stream);
        if (bn == 64) return dispatch_fmt<64, true>(fmt, a, a2, b, p, num_sms, stream);
        if (bn == 128) return dispatch_fmt<128, true>(fmt, a, a2, b, p, num_sms, stream);
        return cudaErrorInvalidValue;
    }
    if (bn == 32) return dispatch_fmt<32, false>(fmt, a, a2, b, p, num_sms, stream);
    if (bn == 64) return dispatch_fmt<64, false>(fmt, a, a2, b, p, num_sms, stream);
    if (bn == 128) return dispatch_fmt<128, false>(fmt, a, a2, b, p, num_sms, stream);
    if (bn == 256) return dispatch_fmt<256, false>(fmt, a, a2, b, p, num_sms, stream);
    return cudaErrorInvalidValue;
}

// Narrow token tiles for small batches (decode-like calls stay weight-
// bandwidth bound and need no padding to 256 tokens).
int gemm_token_tile(int n_tok, bool dual) {
    if (n_tok <= 32) return 32;
    if (n_tok <= 64) return 64;
    if (dual || n_tok <= 128) return 128;
    return 256;
}

}  // namespace ditch
