// Persistent, warp-specialised tcgen05 GEMM with TMEM accumulators and
// fused weight decode. See gemm.cuh for the contract.
//
// Roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: the token tile and the weight tile (bf16) or its
//               raw quantised codes into rings of shared-memory stages;
//   warp 1      TMEM allocator and MMA issuer (one elected lane): 4 x
//               tcgen05.mma (K = 16 each) per 64-wide k-stage (two per kk in
//               SwiGLU mode: gate and up), commits to free the stage and,
//               after the last k-stage, to hand the accumulator over;
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (double-buffered in
//               TMEM when it fits, so the next tile's MMAs overlap these
//               stores), fused bias / rank-1 delta / residual add / SwiGLU;
//   warps 6-13  (quantised weights only) transform: expand the raw tile into
//               bf16 in the 128B-swizzled K-major operand layout, two threads
//               per weight row.
//
// Shared memory: S stages of [A_0 | A_1 (SwiGLU) | B] and R stages of the raw
// quantised tiles [raw_0 | raw_1]; every buffer 1024-byte aligned.
#include "gemm.cuh"

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace ditch {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 4;
constexpr int kXformWarps = 8;
// Each decode thread owns one row part of a k-tile: 64 / kParts elements of
// one of the 128 rows. (Measured on B200: 16 decode warps, a quarter row
// each, were 4-9 % faster for FP8 at 128-512 tokens but 10-18 % slower for
// MXFP4 and INT4, and the MoE trial lost 3 %.)
constexpr int kParts = kXformWarps / 4;
constexpr int kSmemBudget = 224 * 1024;

template <int BN, bool DUAL, int FMT>
struct Cfg {
    static constexpr bool kQuant = FMT != kFmtBf16;
    static constexpr int kNA = DUAL ? 2 : 1;
    static constexpr int kABytes = BM * BK * 2;
    static constexpr int kBBytes = BN * BK * 2;
    // raw weight tile of one k-tile: 128 rows x 64 bytes (8-bit codes, TMA
    // 64-byte swizzle) or x 32 bytes (4-bit codes, no swizzle)
    static constexpr int kRawBytes = (FMT == kFmtFp8 || FMT == kFmtQ8_0)  ? BM * BK
                                     : (FMT == kFmtMxfp4 || FMT == kFmtInt4 || FMT == kFmtQ4K) ? BM * BK / 2
                                                                             : 0;
    static constexpr int kStageBytes = kNA * kABytes + kBBytes;
    static constexpr int kRawStageBytes = kNA * kRawBytes;
    // raw-tile stages in flight: narrow token tiles (decode-like products,
    // bound by streaming the weight) keep more of the weight in flight. A raw
    // tile is loaded together with its stage's token tile, so at most
    // min(kStages, kRawStages) raw tiles are in flight. (Measured on B200: a
    // separate raw-tile producer running up to 16 tiles ahead, with fewer
    // operand stages, and 128-byte raw rows were both slower at 128 tokens.)
    static constexpr int kRawStages = !kQuant ? 0 : BN <= 64 ? (DUAL ? 4 : 8) : 3;
    static constexpr int kRawRing = kRawStages > 0 ? kRawStages : 1;  // modulus (unused without raw tiles)
    static constexpr int kStagesFit = (kSmemBudget - kRawStages * kRawStageBytes) / kStageBytes;
    static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
    static constexpr int kAccCols = kNA * BN;
    static constexpr int kAccBufs = 2 * kAccCols <= 512 ? 2 : 1;
    static constexpr int kTmemColsRaw = kAccBufs * kAccCols;
    static constexpr int kTmemCols = kTmemColsRaw < 32 ? 32 : kTmemColsRaw;
    // producer, MMA, epilogue, then (quantised) the decode warps
    static constexpr int kWarps = 2 + kEpiWarps + (kQuant ? kXformWarps : 0);
    static constexpr int kThreads = kWarps * 32;
    // mbarriers (full, empty, raw full, raw empty, 2 + 2 accumulator, 2 stream-K), then the
    // TMEM base, the abort word and the stream-K flag
    static constexpr int kBarBytes = (8 * (2 * kStages + 2 * kRawStages + 6) + 16 + 63) / 64 * 64;
    static constexpr int kSmemBytes = kStages * kStageBytes + kRawStages * kRawStageBytes + 1024 + kBarBytes;
    static_assert(kSmemBytes <= 232448, "over the 227 KB of shared memory per block");
    static_assert(kStages >= 2, "shared memory too small for two stages");
    static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
    static_assert((kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation must be a power of two");
};

template <class C>
struct SmemLayout {
    uint8_t *base;
    uint64_t *full, *empty, *rawfull, *rawempty, *tfull, *tempty;
    uint64_t *skbar;  // stream-K: [0] parts stored (one arrival per epilogue warp), [1] flag set
    uint32_t *tmem_base;
    int *abort;
    int *sk_flag;  // stream-K: this CTA finishes the current split tile
    __device__ __forceinline__ uint8_t *a(int s, int i) const { return base + s * C::kStageBytes + i * C::kABytes; }
    __device__ __forceinline__ uint8_t *b(int s) const { return base + s * C::kStageBytes + C::kNA * C::kABytes; }
    __device__ __forceinline__ uint8_t *raw(int s, int i) const {
        return base + C::kStages * C::kStageBytes + s * C::kRawStageBytes + i * C::kRawBytes;
    }
};

template <class C>
__device__ __forceinline__ SmemLayout<C> carve(uint8_t *smem_raw) {
    SmemLayout<C> L;
    uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    L.base = reinterpret_cast<uint8_t *>(base);
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(L.base + C::kStages * C::kStageBytes + C::kRawStages * C::kRawStageBytes);
    L.full = bars;
    L.empty = bars + C::kStages;
    L.rawfull = bars + 2 * C::kStages;
    L.rawempty = L.rawfull + C::kRawStages;
    L.tfull = L.rawempty + C::kRawStages;
    L.tempty = L.tfull + 2;
    L.skbar = L.tempty + 2;
    L.tmem_base = reinterpret_cast<uint32_t *>(L.skbar + 2);
    L.abort = reinterpret_cast<int *>(L.tmem_base + 1);
    L.sk_flag = L.abort + 1;
    return L;
}

// silu with the approximate exponential and division of the SFU (a few ulp
// of f32, far below the bf16 rounding of the product that follows; the
// CTA-pair kernel forms it the same way)
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Where a tile's operands and outputs live, in dense or grouped mode.
struct TileInfo {
    int wt;        // weight tile within the matrix (slab)
    int tok0;      // first token row (of the B operand and of the output)
    int tok_cnt;   // valid token rows
    int a_row0;    // first weight row of the matrix (slab) in the A map
    int e;         // expert (grouped mode), else -1
    int kt0, kt1;  // k-tiles of this tile's split
    bool first_split;
    bool sk_partial;  // stream-K: the tile is split between CTAs
    int sk_tile;      // stream-K: the tile's index
};

// k-units: runs of p.kt_unit k-tiles (the k-tiles one raw weight tile holds),
// the grain of K splits and stream-K ranges.
__device__ __forceinline__ int k_units(const GemmParams &p) { return (p.k_tiles + p.kt_unit - 1) / p.kt_unit; }

// Stream-K range of CTA `cta` of `grid`: units [u0, u1) of tiles x k-units.
__device__ __forceinline__ void sk_range(const GemmParams &p, int cta, int grid, long long &u0, long long &u1) {
    const long long U = (long long)p.w_tiles * p.t_tiles * k_units(p);
    u0 = U * cta / grid;
    u1 = U * (cta + 1) / grid;
}

// The CTA whose stream-K range holds unit u: the largest c with u0(c) <= u.
__device__ __forceinline__ int sk_owner(const GemmParams &p, long long u, int grid) {
    const long long U = (long long)p.w_tiles * p.t_tiles * k_units(p);
    return (int)(((u + 1) * grid - 1) / U);
}

// This CTA's work: tiles first, first + step, ... below end (whole tiles or
// k-splits), or under stream-K its segments 0, 1, ... (one per tile its
// range touches).
__device__ __forceinline__ void work_range(const GemmParams &p, int tiles, int &first, int &end, int &step) {
    if (!p.stream_k) {
        first = blockIdx.x;
        end = tiles;
        step = gridDim.x;
        return;
    }
    long long u0, u1;
    sk_range(p, blockIdx.x, gridDim.x, u0, u1);
    first = 0;
    step = 1;
    const int ku = k_units(p);
    end = u1 > u0 ? (int)((u1 - 1) / ku - u0 / ku + 1) : 0;
}

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
        t.sk_partial = false;
        t.sk_tile = -1;
        return t;
    }
    // Output tiles run in bands of kBand token tiles, weight tile by weight
    // tile within a band: the tiles the persistent CTAs hold at one time share
    // a few weight tiles and a few token tiles, which then stay in L2.
    constexpr int kBand = 8;
    int split, rest;
    if (p.stream_k) {  // `tile` is the segment index within this CTA's range
        long long u0, u1;
        sk_range(p, blockIdx.x, gridDim.x, u0, u1);
        const int ku = k_units(p);
        rest = (int)(u0 / ku) + tile;
        const long long k0 = (long long)rest * ku;
        t.kt0 = (int)max(u0 - k0, 0LL) * p.kt_unit;
        t.kt1 = (int)min((long long)p.k_tiles, min(u1 - k0, (long long)ku) * p.kt_unit);
        t.first_split = true;  // the epilogue runs once, on the whole sum
        t.sk_partial = !(t.kt0 == 0 && t.kt1 == p.k_tiles);
        t.sk_tile = rest;
        split = 0;
    } else {
        split = tile % p.k_splits;
        rest = tile / p.k_splits;
        t.kt0 = split * kt_per_split;
        t.kt1 = min(p.k_tiles, t.kt0 + kt_per_split);
        t.first_split = split == 0;
        t.sk_partial = false;
        t.sk_tile = -1;
    }
    const int band = rest / (kBand * p.w_tiles);
    const int idx = rest - band * kBand * p.w_tiles;
    const int g = min(kBand, p.t_tiles - band * kBand);
    t.e = -1;
    t.wt = idx / g;
    t.tok0 = (band * kBand + idx % g) * BN;
    t.tok_cnt = min(BN, p.n_tok - t.tok0);
    t.a_row0 = p.a_row0;
    (void)split;
    return t;
}

// ---- weight decode into the swizzled operand layout ------------------------
// Transform thread t (0..255) owns row r = t & 127 of the 128 x 64 bf16 tile and
// half h = t >> 7 of it: output chunks 4h .. 4h + 3 (16 bytes = 8 elements
// each); chunk j lands at (j ^ (r & 7)) within the row's 128 bytes.

// Four E4M3 codes (one word, low byte first) times one block scale s, as two
// bf16x2 words (codes 0, 1 and 2, 3). (Measured on B200: building the f32
// values with integer shifts and one multiply by s * 2^120, exact but with
// twice the instructions, made the decode-bound GEMMs slower.)
__device__ __forceinline__ void e4m3x4_scaled(uint32_t w, float s, uint32_t &lo, uint32_t &hi) {
    lo = scale_pack(e4m3x2_f32(w & 0xffff), s);
    hi = scale_pack(e4m3x2_f32(w >> 16), s);
}

// The decoded operand tile is bf16 K-major with the 128-byte swizzle: output
// chunk j (eight elements) of row r at j ^ (r & 7). Half h of a row's k-tile
// is elements [32 h, 32 h + 32), output chunks 4 h .. 4 h + 3.
__device__ __forceinline__ void put_chunk(uint8_t *atile, int r, int j, uint4 o) {
    *reinterpret_cast<uint4 *>(atile + r * 128 + ((j ^ (r & 7)) << 4)) = o;
}

// FP8 E4M3 with f32 block scales: bf16(code * scale[row / br][col / bc]).
// Raw tile: 128 rows x 64 bytes, TMA 64B swizzle (chunk c at c ^ ((r >> 1) & 3)).
// srow: the scale row of this weight row; s_tile: the k-tile's scale when the
// block columns are a multiple of 64 (one_scale), loaded by the caller ahead
// of the barrier wait.
__device__ __forceinline__ void xform_fp8(const uint8_t *raw, uint8_t *atile, int r, int h, const float *srow,
                                          bool one_scale, float s_tile, int k0, const GemmParams &p) {
    const int rs = (r >> 1) & 3;
#pragma unroll
    for (int cc = 0; cc < 4 / kParts; cc++) {
        const int c = (4 / kParts) * h + cc;  // raw 16-byte chunk: output chunks 2c, 2c + 1
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 64 + ((c ^ rs) << 4));
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int j = 2 * c + half;
            const int col = k0 + 8 * j;
            const float s = one_scale ? s_tile : ((col < p.k) ? __ldg(srow + col / p.blk_cols) : 0.0f);
            uint4 o;
            e4m3x4_scaled(words[2 * half], s, o.x, o.y);
            e4m3x4_scaled(words[2 * half + 1], s, o.z, o.w);
            put_chunk(atile, r, j, o);
        }
    }
}

// MXFP4 (natural layout): bf16(e2m1[nibble] * 2^(e - 127)), low nibble first.
// Raw tile: 128 rows x 32 bytes (no swizzle); half h reads 16 bytes = one
// 32-element block with scale s (loaded by the caller ahead of the wait).
__device__ __forceinline__ void xform_mxfp4(const uint8_t *raw, uint8_t *atile, int r, int h, float s) {
    // part h: 32 / kParts bytes = 64 / kParts elements, output chunks (8 / kParts) h ...
    uint32_t words[8 / kParts];
    if constexpr (kParts == 2) {
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 32 + h * 16);
        words[0] = q.x, words[1] = q.y, words[2] = q.z, words[3] = q.w;
    } else {
        const uint2 q = *reinterpret_cast<const uint2 *>(raw + r * 32 + h * 8);
        words[0] = q.x, words[1] = q.y;
    }
#pragma unroll
    for (int jj = 0; jj < 8 / kParts; jj++) {  // one word = 8 elements = one output chunk
        const uint32_t w = words[jj];
        uint4 o;
        o.x = scale_pack(e2m1x2_f32(w & 0xff), s);
        o.y = scale_pack(e2m1x2_f32((w >> 8) & 0xff), s);
        o.z = scale_pack(e2m1x2_f32((w >> 16) & 0xff), s);
        o.w = scale_pack(e2m1x2_f32(w >> 24), s);
        put_chunk(atile, r, (8 / kParts) * h + jj, o);
    }
}

// INT4 pack-quantized, contiguous groups (a multiple of 64):
// bf16(f32(q - zp) * scale[row][g]); s and the zero point zq of the k-tile's
// group are loaded by the caller. Raw tile as MXFP4.
__device__ __forceinline__ void xform_int4(const uint8_t *raw, uint8_t *atile, int r, int h, float s, int zq) {
    uint32_t words[8 / kParts];
    if constexpr (kParts == 2) {
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 32 + h * 16);
        words[0] = q.x, words[1] = q.y, words[2] = q.z, words[3] = q.w;
    } else {
        const uint2 q = *reinterpret_cast<const uint2 *>(raw + r * 32 + h * 8);
        words[0] = q.x, words[1] = q.y;
    }
#pragma unroll
    for (int jj = 0; jj < 8 / kParts; jj++) {
        const uint32_t w = words[jj];
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int lo = (int)((w >> (8 * e)) & 0xf) - zq;
            const int hi = (int)((w >> (8 * e + 4)) & 0xf) - zq;
            o[e] = scale_pack(make_float2((float)lo, (float)hi), s);
        }
        put_chunk(atile, r, (8 / kParts) * h + jj, make_uint4(o[0], o[1], o[2], o[3]));
    }
}

// Eight int8 codes (two words) to four bf16x2 of bf16(f32(code) * d): the
// ggml Q8_0 value d * q in f32 (src/quant.zig:81-85), rounded to bf16.
__device__ __forceinline__ uint4 q8x8_bf16(uint32_t w0, uint32_t w1, float d) {
    uint32_t o[4];
    const uint32_t w[2] = {w0, w1};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const uint32_t word = w[k >> 1];
        const int sh = 16 * (k & 1);
        const float lo = (float)(int8_t)((word >> sh) & 0xff), hi = (float)(int8_t)((word >> (sh + 8)) & 0xff);
        o[k] = scale_pack(make_float2(lo, hi), d);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// GGUF Q8_0 repacked at load: int8 codes [rows][cols] and the block scales d
// as f32 [rows][cols / 32]. Raw tile as FP8; half h is one 32-code block
// with scale d (loaded by the caller).
__device__ __forceinline__ void xform_q8_0(const uint8_t *raw, uint8_t *atile, int r, int h, float d) {
    const int rs = (r >> 1) & 3;
#pragma unroll
    for (int cc = 0; cc < 4 / kParts; cc++) {
        const int c = (4 / kParts) * h + cc;  // raw 16-byte chunk: output chunks 2c, 2c + 1
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 64 + ((c ^ rs) << 4));
        put_chunk(atile, r, 2 * c, q8x8_bf16(q.x, q.y, d));
        put_chunk(atile, r, 2 * c + 1, q8x8_bf16(q.z, q.w, d));
    }
}

// A pair of Q4_K codes to bf16x2 of bf16(d1 * q - m1): the ggml value in f32
// (src/quant.zig:148-173; d1 = d * scale and m1 = dmin * min were formed at
// repack, every product here is exact), rounded to bf16.
__device__ __forceinline__ uint32_t q4k_pair(uint32_t lo, uint32_t hi, float d1, float m1) {
    return pack_bf16x2(__fsub_rn(__fmul_rn(d1, (float)lo), m1), __fsub_rn(__fmul_rn(d1, (float)hi), m1));
}

// GGUF Q4_K repacked at load: 4-bit codes [rows][cols / 2] in element order
// (low nibble first) and (d1, m1) f32 pairs per 32-element sub-block
// [rows][cols / 32]. Raw tile as MXFP4; half h is one sub-block.
__device__ __forceinline__ void xform_q4k(const uint8_t *raw, uint8_t *atile, int r, int h, float d1, float m1) {
    uint32_t words[8 / kParts];
    if constexpr (kParts == 2) {
        const uint4 q = *reinterpret_cast<const uint4 *>(raw + r * 32 + h * 16);
        words[0] = q.x, words[1] = q.y, words[2] = q.z, words[3] = q.w;
    } else {
        const uint2 q = *reinterpret_cast<const uint2 *>(raw + r * 32 + h * 8);
        words[0] = q.x, words[1] = q.y;
    }
#pragma unroll
    for (int jj = 0; jj < 8 / kParts; jj++) {
        const uint32_t w = words[jj];
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) o[e] = q4k_pair((w >> (8 * e)) & 0xf, (w >> (8 * e + 4)) & 0xf, d1, m1);
        put_chunk(atile, r, (8 / kParts) * h + jj, make_uint4(o[0], o[1], o[2], o[3]));
    }
}

// The side data of half h of one row's k-tile at k0, loaded ahead of the
// barrier waits: the scale (FP8 one_scale, MXFP4, Q8_0, INT4) and the INT4
// zero point.
template <int FMT>
__device__ __forceinline__ void load_side(const GemmParams &p, int vrow, const float *srow, bool one_scale, int k0,
                                          int h, float &s, int &zq, float &mn) {
    s = 0.0f;
    zq = 8;
    mn = 0.0f;
    if (FMT == kFmtFp8) {
        if (one_scale) s = __ldg(srow + k0 / p.blk_cols);
    } else if (FMT == kFmtMxfp4) {
        const int blk = (k0 >> 5) + h * 2 / kParts;  // the 32-element block of part h
        if (blk * 32 < p.k) s = e8m0_scale(__ldg(p.scales_u8 + (long long)vrow * (p.k / 32) + blk));
    } else if (FMT == kFmtQ8_0) {
        const int blk = (k0 >> 5) + h * 2 / kParts;  // the 32-element block of part h
        if (blk * 32 < p.k) s = __ldg(p.scales + (long long)vrow * p.scale_cols + blk);
    } else if (FMT == kFmtInt4) {
        const int groups = p.scale_cols, g = k0 / p.blk_cols;
        if (k0 < p.k) s = __ldg(p.scales + (long long)vrow * groups + g);
        if (p.zeros) zq = (__ldg(p.zeros + (long long)(vrow >> 3) * groups + g) >> ((vrow & 7) * 4)) & 0xf;
    } else if (FMT == kFmtQ4K) {
        const int blk = (k0 >> 5) + h * 2 / kParts;  // the 32-element sub-block of part h
        if (blk * 32 < p.k) {
            const float2 dm = __ldg(reinterpret_cast<const float2 *>(p.scales) + (long long)vrow * p.scale_cols + blk);
            s = dm.x, mn = dm.y;
        }
    }
}

// ---- staged decode ----------------------------------------------------------
// Rows [row0, row0 + rows) of a quantised weight decoded once to bf16
// [rows][cols] with the transforms' own arithmetic, so that the bf16 GEMM over
// the staged copy equals the fused GEMM bit for bit. One thread decodes one
// 16-byte chunk of codes: 16 FP8 elements, or 32 MXFP4 / INT4 elements.
__global__ void __launch_bounds__(256) k_stage_decode(const StageArgs a) {
    const int epc = (a.fmt == kFmtFp8 || a.fmt == kFmtQ8_0) ? 16 : 32;  // elements per chunk
    const int chunks = a.cols / epc;
    const long long total = (long long)a.rows * chunks;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / chunks), ch = (int)(i % chunks);
        const int grow = a.row0 + r, c0 = ch * epc;
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(a.data + (long long)grow * a.row_bytes + ch * 16));
        const uint32_t words[4] = {q.x, q.y, q.z, q.w};
        uint4 *dst = reinterpret_cast<uint4 *>(a.out + (long long)r * a.cols + c0);
        if (a.fmt == kFmtFp8) {
            const float *srow = a.scales + (long long)(grow / a.blk_rows) * a.scale_cols;
            const bool one = (a.blk_cols & 15) == 0;
            const float s0 = __ldg(srow + c0 / a.blk_cols);
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t o[4];
                if (one) {
                    e4m3x4_scaled(words[2 * half], s0, o[0], o[1]);
                    e4m3x4_scaled(words[2 * half + 1], s0, o[2], o[3]);
                } else {  // block columns not a multiple of 16: a scale per element
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int c = c0 + 8 * half + 2 * e;
                        const uint32_t two = words[2 * half + (e >> 1)] >> (16 * (e & 1));
                        const float2 v = e4m3x2_f32(two & 0xffff);
                        const float sl = __ldg(srow + c / a.blk_cols), sh = __ldg(srow + (c + 1) / a.blk_cols);
                        o[e] = pack_bf16x2(v.x * sl, v.y * sh);
                    }
                }
                dst[half] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        } else if (a.fmt == kFmtQ8_0) {
            const float d = __ldg(a.scales + (long long)grow * a.scale_cols + c0 / 32);
            dst[0] = q8x8_bf16(words[0], words[1], d);
            dst[1] = q8x8_bf16(words[2], words[3], d);
        } else if (a.fmt == kFmtMxfp4) {
            const float s = e8m0_scale(__ldg(a.scales_u8 + (long long)grow * (a.cols / 32) + ch));
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint32_t w = words[jj];
                dst[jj] = make_uint4(scale_pack(e2m1x2_f32(w & 0xff), s), scale_pack(e2m1x2_f32((w >> 8) & 0xff), s),
                                     scale_pack(e2m1x2_f32((w >> 16) & 0xff), s), scale_pack(e2m1x2_f32(w >> 24), s));
            }
        } else if (a.fmt == kFmtQ4K) {
            const float2 dm = __ldg(reinterpret_cast<const float2 *>(a.scales) + (long long)grow * a.scale_cols + c0 / 32);
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint32_t w = words[jj];
                dst[jj] = make_uint4(q4k_pair(w & 0xf, (w >> 4) & 0xf, dm.x, dm.y),
                                     q4k_pair((w >> 8) & 0xf, (w >> 12) & 0xf, dm.x, dm.y),
                                     q4k_pair((w >> 16) & 0xf, (w >> 20) & 0xf, dm.x, dm.y),
                                     q4k_pair((w >> 24) & 0xf, w >> 28, dm.x, dm.y));
            }
        } else {  // kFmtInt4
            const int g = c0 / a.blk_cols;
            const float s = __ldg(a.scales + (long long)grow * a.scale_cols + g);
            int zq = 8;
            if (a.zeros) zq = (__ldg(a.zeros + (long long)(grow >> 3) * a.scale_cols + g) >> ((grow & 7) * 4)) & 0xf;
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint32_t w = words[jj];
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int lo = (int)((w >> (8 * e)) & 0xf) - zq;
                    const int hi = (int)((w >> (8 * e + 4)) & 0xf) - zq;
                    o[e] = scale_pack(make_float2((float)lo, (float)hi), s);
                }
                dst[jj] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// ---- weight-streaming product for at most 16 tokens ----------------------
// out[m][n] = x[m] . W[n] for m < M <= 16, the weight read once in its
// stored format. Block = 8 warps over 16 weight rows (two n8 tiles); the
// warps share the block's K range chunk by chunk and their partial sums are
// added in shared memory (then across grid.y K splits: atomically, or in
// split order in deterministic mode). Lane
// (g, t) streams 16 bytes of row g (and g + 8) per chunk with plain loads,
// decodes them to bf16 pairs with the in-GEMM arithmetic, and feeds
// mma.sync m16n8k16 with the tokens as A (rows g, g + 8) and the weight as B.
// K is permuted consistently for A and B: the lane's EPL consecutive weight
// elements fill k-positions {2t, 2t + 1, 2t + 8, 2t + 9} of EPL / 4 steps,
// and its A fragments read the same x elements (one 8-byte load per row and
// step). A dot product does not depend on the order of its K terms.
template <int FMT>
struct Skinny {
    static constexpr int kEPL = FMT == kFmtBf16 ? 8 : (FMT == kFmtFp8 || FMT == kFmtQ8_0) ? 16 : 32;
    static constexpr int kChunk = 4 * kEPL;  // K per chunk (four lanes per row)
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The EPL / 2 bf16 pairs of one lane's 16 raw bytes of weight row `row` at
// element k0 (a multiple of EPL).
template <int FMT>
__device__ __forceinline__ void skinny_decode(const uint4 q, int row, int k0, const GemmParams &p, uint32_t *pr) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    if (FMT == kFmtBf16) {
#pragma unroll
        for (int i = 0; i < 4; i++) pr[i] = w[i];
    } else if (FMT == kFmtFp8) {
        const float s = __ldg(p.scales + (long long)(row / p.blk_rows) * p.scale_cols + k0 / p.blk_cols);
#pragma unroll
        for (int i = 0; i < 4; i++) e4m3x4_scaled(w[i], s, pr[2 * i], pr[2 * i + 1]);
    } else if (FMT == kFmtQ8_0) {
        const float d = __ldg(p.scales + (long long)row * p.scale_cols + k0 / 32);
        const uint4 a = q8x8_bf16(w[0], w[1], d), b = q8x8_bf16(w[2], w[3], d);
        pr[0] = a.x; pr[1] = a.y; pr[2] = a.z; pr[3] = a.w;
        pr[4] = b.x; pr[5] = b.y; pr[6] = b.z; pr[7] = b.w;
    } else if (FMT == kFmtMxfp4) {
        const float s = e8m0_scale(__ldg(p.scales_u8 + (long long)row * (p.k / 32) + k0 / 32));
#pragma unroll
        for (int i = 0; i < 16; i++) pr[i] = scale_pack(e2m1x2_f32((w[i >> 2] >> (8 * (i & 3))) & 0xff), s);
    } else if (FMT == kFmtQ4K) {
        const float2 dm = __ldg(reinterpret_cast<const float2 *>(p.scales) + (long long)row * p.scale_cols + k0 / 32);
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xff;
            pr[i] = q4k_pair(byte & 0xf, byte >> 4, dm.x, dm.y);
        }
    } else {  // kFmtInt4
        const int g = k0 / p.blk_cols;
        const float s = __ldg(p.scales + (long long)row * p.scale_cols + g);
        int zq = 8;
        if (p.zeros) zq = (__ldg(p.zeros + (long long)(row >> 3) * p.scale_cols + g) >> ((row & 7) * 4)) & 0xf;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const uint32_t byte = (w[i >> 2] >> (8 * (i & 3))) & 0xff;
            pr[i] = scale_pack(make_float2((float)((int)(byte & 0xf) - zq), (float)((int)(byte >> 4) - zq)), s);
        }
    }
}

template <int FMT>
__global__ void __launch_bounds__(256) k_skinny(const uint8_t *wdata, long long row_bytes, const uint16_t *x,
                                                long long ldx, const GemmParams p, int chunks_per_split) {
    using S = Skinny<FMT>;
    constexpr int EPL = S::kEPL, STEPS = EPL / 4;
    constexpr int kNum = EPL == 8 ? 2 : 1, kDen = EPL == 32 ? 2 : 1;  // bytes per element = kNum / kDen
    __shared__ float red[8][16][17];  // [warp][row of 16][token]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int n0 = blockIdx.x * 16;
    const int c_lo = blockIdx.y * chunks_per_split;
    const int c_hi = min((p.k + S::kChunk - 1) / S::kChunk, c_lo + chunks_per_split);
    const int M = p.n_tok;
    float acc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
    const int rows[2] = {min(n0 + g, p.m_w - 1), min(n0 + 8 + g, p.m_w - 1)};  // clamped: stores are masked
    const uint16_t *xa = x + (long long)min(g, M - 1) * ldx, *xb = x + (long long)min(g + 8, M - 1) * ldx;
    const bool va = g < M, vb = g + 8 < M;
    // kU chunks per round: all their weight loads are issued before any is
    // decoded, so each lane keeps 2 kU 16-byte loads in flight
    constexpr int kU = 4;
    const uint8_t *wrow[2] = {wdata + (long long)(p.a_row0 + rows[0]) * row_bytes,
                              wdata + (long long)(p.a_row0 + rows[1]) * row_bytes};
    for (int c0 = c_lo + warp; c0 < c_hi; c0 += 8 * kU) {
        uint4 q[kU][2];
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int c = c0 + 8 * u;
            const long long off = (long long)(c * S::kChunk + t * EPL) * kNum / kDen;
#pragma unroll
            for (int j = 0; j < 2; j++)
                q[u][j] = c < c_hi ? __ldg(reinterpret_cast<const uint4 *>(wrow[j] + off)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kU; u++) {
            const int c = c0 + 8 * u;
            if (c >= c_hi) break;
            const int k0 = c * S::kChunk + t * EPL;  // this lane's first element
            uint2 ax[STEPS], bx[STEPS];
#pragma unroll
            for (int s2 = 0; s2 < STEPS; s2++) {
                ax[s2] = va ? *reinterpret_cast<const uint2 *>(xa + k0 + 4 * s2) : make_uint2(0, 0);
                bx[s2] = vb ? *reinterpret_cast<const uint2 *>(xb + k0 + 4 * s2) : make_uint2(0, 0);
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                uint32_t pr[EPL / 2];
                skinny_decode<FMT>(q[u][j], p.a_row0 + rows[j], k0, p, pr);
#pragma unroll
                for (int s2 = 0; s2 < STEPS; s2++)
                    mma_16816(acc[j], ax[s2].x, bx[s2].x, ax[s2].y, bx[s2].y, pr[2 * s2], pr[2 * s2 + 1]);
            }
        }
    }
    // acc[j]: tokens (g, g + 8) x weight rows 8 j + 2 t, + 1 -> red[warp][row][token]
#pragma unroll
    for (int j = 0; j < 2; j++) {
        red[warp][8 * j + 2 * t][g] = acc[j][0];
        red[warp][8 * j + 2 * t + 1][g] = acc[j][1];
        red[warp][8 * j + 2 * t][g + 8] = acc[j][2];
        red[warp][8 * j + 2 * t + 1][g + 8] = acc[j][3];
    }
    __syncthreads();
    // thread (row, token): warps added in order
    const int row = threadIdx.x >> 4, m = threadIdx.x & 15, n = n0 + row;
    float r = 0.0f;
#pragma unroll
    for (int w2 = 0; w2 < 8; w2++) r += red[w2][row][m];
    if (gridDim.y > 1 && p.sk_ws) {
        // K split over the grid, deterministic mode: each block leaves its
        // partial sums in sk_ws; the block that arrives last adds them in
        // split order (the result does not depend on timing) and runs the
        // epilogue. Otherwise every split adds its sum atomically.
        __shared__ int s_last;
        float *ws = p.sk_ws + (size_t)blockIdx.x * 256;
        const size_t split_stride = (size_t)gridDim.x * 256;
        __stcg(ws + blockIdx.y * split_stride + threadIdx.x, r);
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const int old = atomicAdd(p.sk_cnt + blockIdx.x, 1);
            s_last = old == (int)gridDim.y - 1;
            if (s_last) p.sk_cnt[blockIdx.x] = 0;  // every split has arrived: ready for the next launch
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        r = 0.0f;
        for (int y = 0; y < (int)gridDim.y; y++) r += __ldcg(ws + y * split_stride + threadIdx.x);
    }
    if (m >= M || n >= p.m_w) return;
    if (blockIdx.y == 0 || p.sk_ws) {  // bias and delta once per output
        if (p.xa && p.db) {
            const int drank = p.delta_rank > 1 ? p.delta_rank : 1;
            for (int t = 0; t < drank; t++) r += p.xa[m * drank + t] * p.db[(long long)n * drank + t];
        }
        if (p.bias) r += p.bias[n];
    }
    float *o = reinterpret_cast<float *>(p.out) + (long long)m * p.ldo + n;
    if (p.flags & kEpiAtomic) atomicAdd(o, r);
    else if (p.flags & kEpiResidual) *o = *o + r;
    else *o = r;
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
        }
        for (int s = 0; s < C::kRawStages; s++) {
            mbar_init(&L.rawfull[s], 1);
            mbar_init(&L.rawempty[s], kXformWarps);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&L.tfull[b], 1);
            mbar_init(&L.tempty[b], kEpiWarps);
        }
        mbar_init(&L.skbar[0], kEpiWarps);
        mbar_init(&L.skbar[1], 1);
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
    const int kt_per_split = (k_units(p) + p.k_splits - 1) / p.k_splits * p.kt_unit;
    int w_first, w_end, w_step;
    work_range(p, tiles, w_first, w_end, w_step);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            // one or two token tiles (decode-sized products): every weight tile
            // is read once and every token tile by all CTAs, so the weight
            // stream goes first out of L2 and the token tiles stay
            const bool hint = !p.sched && p.t_tiles <= 2;
            const uint64_t pol_w = l2_policy_evict_first(), pol_t = l2_policy_evict_last();
            int it = 0;
            for (int tile = w_first; tile < w_end && !*abort; tile += w_step) {
                const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
                const int arow = ti.a_row0 + ti.wt * BM;
                for (int kt = ti.kt0; kt < ti.kt1; kt++, it++) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&L.empty[s], ph ^ 1, abort, p.status)) break;
                    if (C::kQuant) {
                        const int rs = it % C::kRawRing;
                        const uint32_t rph = (it / C::kRawRing) & 1;
                        if (!mbar_wait(&L.rawempty[rs], rph ^ 1, abort, p.status)) break;
                        mbar_arrive_expect_tx(&L.rawfull[rs], C::kRawStageBytes);
                        const int xb = kt * ((FMT == kFmtFp8 || FMT == kFmtQ8_0) ? BK : BK / 2);  // raw bytes along K
                        if (hint) {
                            tma_load_2d_hint(&tmA, &L.rawfull[rs], L.raw(rs, 0), xb, arow, pol_w);
                            if (DUAL)
                                tma_load_2d_hint(&tmA2, &L.rawfull[rs], L.raw(rs, 1), xb, arow + p.a2_row_offset, pol_w);
                        } else {
                            tma_load_2d(&tmA, &L.rawfull[rs], L.raw(rs, 0), xb, arow);
                            if (DUAL) tma_load_2d(&tmA2, &L.rawfull[rs], L.raw(rs, 1), xb, arow + p.a2_row_offset);
                        }
                        mbar_arrive_expect_tx(&L.full[s], C::kBBytes);
                    } else {
                        mbar_arrive_expect_tx(&L.full[s], C::kNA * C::kABytes + C::kBBytes);
                        if (hint) {
                            tma_load_2d_hint(&tmA, &L.full[s], L.a(s, 0), kt * BK, arow, pol_w);
                            if (DUAL)
                                tma_load_2d_hint(&tmA2, &L.full[s], L.a(s, 1), kt * BK, arow + p.a2_row_offset, pol_w);
                        } else {
                            tma_load_2d(&tmA, &L.full[s], L.a(s, 0), kt * BK, arow);
                            if (DUAL) tma_load_2d(&tmA2, &L.full[s], L.a(s, 1), kt * BK, arow + p.a2_row_offset);
                        }
                    }
                    if (hint) tma_load_2d_hint(&tmB, &L.full[s], L.b(s), kt * BK, ti.tok0, pol_t);
                    else tma_load_2d(&tmB, &L.full[s], L.b(s), kt * BK, ti.tok0);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
            int it = 0, local = 0;
            for (int tile = w_first; tile < w_end && !*abort; tile += w_step, local++) {
                const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
                const int buf = local % C::kAccBufs;
                const uint32_t use_ph = (local / C::kAccBufs) & 1;
                if (!mbar_wait(&L.tempty[buf], use_ph ^ 1, abort, p.status)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * C::kAccCols;
                bool ok = true;
                for (int kt = ti.kt0; kt < ti.kt1; kt++, it++) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&L.full[s], ph, abort, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_kmajor_desc(smem_u32(L.a(s, 0)));
                    const uint64_t bdesc = sw128_kmajor_desc(smem_u32(L.b(s)));
                    const uint64_t a2desc = DUAL ? sw128_kmajor_desc(smem_u32(L.a(s, 1))) : 0;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint32_t acc = (kt > ti.kt0 || kk > 0) ? 1u : 0u;
                        tc_mma_bf16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, acc);
                        if (DUAL) tc_mma_bf16(d + BN, a2desc + 2 * kk, bdesc + 2 * kk, idesc, acc);
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
        const int trow = q * 32 + lane;  // row of the tile (weight row) this thread owns
        int local = 0, sk_uses = 0;
        for (int tile = w_first; tile < w_end && !*abort; tile += w_step, local++) {
            const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
            const bool first_split = ti.first_split;  // bias and delta once per output
            const int buf = local % C::kAccBufs;
            const uint32_t use_ph = (local / C::kAccBufs) & 1;
            if (!mbar_wait(&L.tfull[buf], use_ph, abort, p.status)) break;
            tc_fence_after();
            const int n = ti.wt * BM + trow;  // weight row = output feature
            const bool n_ok = n < p.m_w;
            const float bias = (p.bias && n_ok && first_split) ? p.bias[n] : 0.0f;
            bool delta = p.db && n_ok && first_split;
            const float *dbp = p.db;
            if (delta && ti.e >= 0) {
                delta = p.e_flags == nullptr || p.e_flags[ti.e] != 0;
                dbp = p.db + ti.e * p.db_stride;
            }
            const int drank = p.delta_rank > 1 ? p.delta_rank : 1;
            float dbn[kMaxDeltaRank];
            bool any_delta = false;
#pragma unroll
            for (int t = 0; t < kMaxDeltaRank; t++) {
                dbn[t] = (delta && t < drank) ? dbp[(long long)n * drank + t] : 0.0f;
                any_delta |= dbn[t] != 0.0f;
            }
            const uint32_t tbase = tmem + buf * C::kAccCols + (static_cast<uint32_t>(q * 32) << 16);
            const int m_end = ti.tok0 + ti.tok_cnt;
            // stream-K: a part of a split tile goes to this CTA's slot; the CTA
            // that brings the last part sums them all in k order and finishes
            // accumulator columns (tokens) per step: 16 where the decode warps
            // leave each thread fewer registers
            constexpr int EC = (C::kQuant && kXformWarps > 8) ? 16 : 32;
            bool finish = true;
            int c_lo = 0, c_hi = -1;
            long long t_u0 = 0;
            if (ti.sk_partial) {
                t_u0 = (long long)ti.sk_tile * k_units(p);
                c_lo = sk_owner(p, t_u0, gridDim.x);
                c_hi = sk_owner(p, t_u0 + k_units(p) - 1, gridDim.x);
                float *mine = p.sk_ws + ((size_t)(blockIdx.x * 2 + (tile == 0 ? 0 : 1)) * C::kNA * BM + trow) * BN;
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += EC) {
                    if (ti.tok0 + c0 >= m_end) break;
#pragma unroll
                    for (int i = 0; i < C::kNA; i++)
#pragma unroll
                        for (int hc = 0; hc < EC; hc += 16) {
                            float v[16];
                            tmem_ld16(tbase + i * BN + c0 + hc, v);
                            float4 *dst = reinterpret_cast<float4 *>(mine + (size_t)i * BM * BN + c0 + hc);
#pragma unroll
                            for (int j = 0; j < 4; j++)
                                __stcg(dst + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
                        }
                }
                // all epilogue warps' stores, then one thread counts this part in
                const uint32_t sk_ph = sk_uses++ & 1;
                __syncwarp();
                if (lane == 0) mbar_arrive(&L.skbar[0]);
                bool ok = true;
                if (threadIdx.x == 64) {  // first epilogue thread
                    ok = mbar_wait(&L.skbar[0], sk_ph, abort, p.status);
                    if (ok) {
                        __threadfence();
                        const int old = atomicAdd(p.sk_cnt + ti.sk_tile, 1);
                        const int last = old == c_hi - c_lo;
                        if (last) p.sk_cnt[ti.sk_tile] = 0;  // every part has arrived: ready for the next launch
                        *reinterpret_cast<volatile int *>(L.sk_flag) = last;
                        mbar_arrive(&L.skbar[1]);
                    }
                }
                if (ok) ok = mbar_wait(&L.skbar[1], sk_ph, abort, p.status);
                finish = ok && *reinterpret_cast<volatile int *>(L.sk_flag) != 0;
                if (finish) {
                    // the whole sum, parts in k order (this CTA's from TMEM),
                    // back into TMEM, where the epilogue below reads it
                    __threadfence();
#pragma unroll 1
                    for (int c0 = 0; c0 < BN; c0 += 16) {
                        if (ti.tok0 + c0 >= m_end) break;
#pragma unroll
                        for (int i = 0; i < C::kNA; i++) {
                            float acc[16];
#pragma unroll
                            for (int j = 0; j < 16; j++) acc[j] = 0.0f;
                            for (int c = c_lo; c <= c_hi; c++) {
                                float part[16];
                                if (c == (int)blockIdx.x) {
                                    tmem_ld16(tbase + i * BN + c0, part);
                                } else {
                                    long long cu0, cu1;
                                    sk_range(p, c, gridDim.x, cu0, cu1);
                                    const float4 *src = reinterpret_cast<const float4 *>(
                                        p.sk_ws + ((size_t)((c * 2 + (cu0 >= t_u0 ? 0 : 1)) * C::kNA + i) * BM + trow) * BN +
                                        c0);
#pragma unroll
                                    for (int j = 0; j < 4; j++) {
                                        const float4 a4 = __ldcg(src + j);
                                        part[4 * j] = a4.x;
                                        part[4 * j + 1] = a4.y;
                                        part[4 * j + 2] = a4.z;
                                        part[4 * j + 3] = a4.w;
                                    }
                                }
#pragma unroll
                                for (int j = 0; j < 16; j++) acc[j] += part[j];
                            }
                            tmem_st16(tbase + i * BN + c0, acc);
                        }
                    }
                }
            }
#pragma unroll 1
            for (int c0 = 0; c0 < BN && finish; c0 += EC) {
                if (ti.tok0 + c0 >= m_end) break;  // warp-uniform: no valid token left
                float v[EC], u[EC];
                if constexpr (EC == 32) {
                    tmem_ld32(tbase + c0, v);
                    if (DUAL) tmem_ld32(tbase + BN + c0, u);
                } else {
                    tmem_ld16(tbase + c0, v);
                    if (DUAL) tmem_ld16(tbase + BN + c0, u);
                }
                const int m0 = ti.tok0 + c0;
                const int mv = min(EC, m_end - m0);  // valid tokens of this chunk (>= 1)
                // Every load of a chunk is issued before its first store: as far
                // as the compiler knows the stores may alias the loads, and
                // interleaving them serialises one memory round trip per token.
                float r[EC];
#pragma unroll
                for (int j = 0; j < EC; j++) r[j] = v[j];
                if (p.xa && any_delta) {
#pragma unroll 1
                    for (int t = 0; t < drank; t++) {  // r += (x . a_t) b_t, term by term
                        float xa[EC];
#pragma unroll
                        for (int j = 0; j < EC; j++) xa[j] = j < mv ? __ldg(p.xa + (long long)(m0 + j) * drank + t) : 0.0f;
#pragma unroll
                        for (int j = 0; j < EC; j++) r[j] += xa[j] * dbn[t];
                    }
                }
#pragma unroll
                for (int j = 0; j < EC; j++) r[j] += bias;
                const long long o0 = (long long)m0 * p.ldo + n;
                if (!n_ok) {
                    // weight row past the matrix: nothing to store
                } else if (DUAL) {
                    uint16_t *ob = reinterpret_cast<uint16_t *>(p.out) + o0;
#pragma unroll
                    for (int j = 0; j < EC; j++)
                        if (j < mv) ob[(long long)j * p.ldo] = f32_to_bf16_bits(silu_f(r[j]) * u[j]);
                } else if (p.flags & kEpiAtomic) {
                    float *of = reinterpret_cast<float *>(p.out) + o0;
#pragma unroll
                    for (int j = 0; j < EC; j++)
                        if (j < mv) atomicAdd(of + (long long)j * p.ldo, r[j]);
                } else if (p.flags & kEpiResidual) {
                    float *of = reinterpret_cast<float *>(p.out) + o0;
                    float old[EC];
#pragma unroll
                    for (int j = 0; j < EC; j++) old[j] = j < mv ? of[(long long)j * p.ldo] : 0.0f;
#pragma unroll
                    for (int j = 0; j < EC; j++)
                        if (j < mv) of[(long long)j * p.ldo] = old[j] + r[j];
                } else if (p.flags & kEpiOutBf16) {
                    uint16_t *ob = reinterpret_cast<uint16_t *>(p.out) + o0;
#pragma unroll
                    for (int j = 0; j < EC; j++)
                        if (j < mv) ob[(long long)j * p.ldo] = f32_to_bf16_bits(r[j]);
                } else {
                    float *of = reinterpret_cast<float *>(p.out) + o0;
#pragma unroll
                    for (int j = 0; j < EC; j++)
                        if (j < mv) of[(long long)j * p.ldo] = r[j];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&L.tempty[buf]);
        }
    } else if (C::kQuant) {
        // ---------------- weight transform ----------------
        const int t = threadIdx.x - (2 + kEpiWarps) * 32;  // 0 .. 32 kXformWarps - 1
        const int r = t & 127, h = t >> 7;                  // row, part of the row
        const bool one_scale = FMT == kFmtFp8 && (p.blk_cols & 63) == 0;
        int it = 0;
        for (int tile = w_first; tile < w_end && !*abort; tile += w_step) {
            const TileInfo ti = tile_info<BN>(p, tile, kt_per_split);
            int vrow[C::kNA];
            const float *srow[C::kNA];
#pragma unroll
            for (int i = 0; i < C::kNA; i++) {
                const int off = i ? p.a2_row_offset : 0;
                const int grow = ti.a_row0 + ti.wt * BM + r + off;
                vrow[i] = min(grow, ti.a_row0 + off + p.m_w - 1);  // clamp side-data reads
                srow[i] = FMT == kFmtFp8 ? p.scales + (long long)(vrow[i] / p.blk_rows) * p.scale_cols : nullptr;
            }
            bool ok = true;
            for (int kt = ti.kt0; kt < ti.kt1; kt++, it++) {
                const int s = it % C::kStages;
                const int rs = it % C::kRawRing;
                const uint32_t rph = (it / C::kRawRing) & 1;
                float sd[C::kNA], md[C::kNA];
                int zd[C::kNA];
#pragma unroll
                for (int i = 0; i < C::kNA; i++)  // issued before the wait: their latency hides behind it
                    load_side<FMT>(p, vrow[i], srow[i], one_scale, kt * BK, h, sd[i], zd[i], md[i]);
                // the raw tile has landed (the producer loaded it after operand stage s was free)
                if (!mbar_wait(&L.rawfull[rs], rph, abort, p.status)) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (int i = 0; i < C::kNA; i++) {
                    if (FMT == kFmtFp8) xform_fp8(L.raw(rs, i), L.a(s, i), r, h, srow[i], one_scale, sd[i], kt * BK, p);
                    if (FMT == kFmtMxfp4) xform_mxfp4(L.raw(rs, i), L.a(s, i), r, h, sd[i]);
                    if (FMT == kFmtInt4) xform_int4(L.raw(rs, i), L.a(s, i), r, h, sd[i], zd[i]);
                    if (FMT == kFmtQ8_0) xform_q8_0(L.raw(rs, i), L.a(s, i), r, h, sd[i]);
                    if (FMT == kFmtQ4K) xform_q4k(L.raw(rs, i), L.a(s, i), r, h, sd[i], md[i]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&L.rawempty[rs]);
                    mbar_arrive(&L.full[s]);
                }
            }
            if (!ok) break;
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

// A 2D map over a row-major [rows][inner] tensor. Encodings are cached by
// their full parameter tuple (a map depends on nothing else), which takes the
// driver call off the host path of repeated launches.
struct MapKey {
    const void *ptr;
    uint64_t inner, rows, row_bytes;
    uint32_t box_inner, box_rows;
    int dt, sw;
    bool operator==(const MapKey &o) const {
        return ptr == o.ptr && inner == o.inner && rows == o.rows && row_bytes == o.row_bytes &&
               box_inner == o.box_inner && box_rows == o.box_rows && dt == o.dt && sw == o.sw;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        size_t h = std::hash<const void *>()(k.ptr);
        for (uint64_t v : {k.inner, k.rows, k.row_bytes, (uint64_t)k.box_inner << 32 | k.box_rows,
                           (uint64_t)k.dt << 8 | (uint64_t)k.sw})
            h = h * 1000003u ^ std::hash<uint64_t>()(v);
        return h;
    }
};

bool encode_map(CUtensorMap *map, const void *ptr, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw);

bool make_map(CUtensorMap *map, const void *ptr, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    static std::mutex mu;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{ptr, inner, rows, row_bytes, box_inner, box_rows, (int)dt, (int)sw};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *map = it->second;
            return true;
        }
    }
    if (!encode_map(map, ptr, dt, inner, rows, row_bytes, box_inner, box_rows, sw)) return false;
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, *map);
    return true;
}

bool encode_map(CUtensorMap *map, const void *ptr, CUtensorMapDataType dt, uint64_t inner, uint64_t rows,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
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
        ok = make_map(&ma, a.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.cols, a.rows, a.row_bytes, BK, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
        if (ok && DUAL)
            ok = make_map(&ma2, a2->ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a2->cols, a2->rows, a2->row_bytes, BK, BM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
        const bool bytes8 = FMT == kFmtFp8 || FMT == kFmtQ8_0;  // one byte per element
        const uint32_t raw_inner = bytes8 ? BK : BK / 2;        // bytes per row per k-tile
        const CUtensorMapSwizzle sw = bytes8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
        ok = make_map(&ma, a.ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.row_bytes, a.rows, a.row_bytes, raw_inner, BM, sw);
        if (ok && DUAL)
            ok = make_map(&ma2, a2->ptr, CU_TENSOR_MAP_DATA_TYPE_UINT8, a2->row_bytes, a2->rows, a2->row_bytes,
                          raw_inner, BM, sw);
    }
    if (!DUAL) ma2 = ma;
    if (ok)
        ok = make_map(&mb, b.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, b.cols, b.rows, b.row_bytes, BK, BN,
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
    p.kt_unit = 1;
    p.w_tiles = (p.m_w + BM - 1) / BM;
    p.t_tiles = (p.n_tok + BN - 1) / BN;
    const int ku = (p.k_tiles + p.kt_unit - 1) / p.kt_unit;
    if (p.k_splits < 1) p.k_splits = 1;
    if (p.sched) p.k_splits = 1;  // grouped tiles are whole-K
    if (p.k_splits > 1) {  // splits of whole k-units, none empty
        const int per = (ku + p.k_splits - 1) / p.k_splits;
        p.k_splits = (ku + per - 1) / per;
    }
    const int tiles = p.w_tiles * p.t_tiles * p.k_splits;
    // grouped mode: the tile count is on the device; the grid is persistent
    // stream-K: every CTA gets at least 4 k-units (so none is empty)
    const long long units = (long long)tiles * ku;
    const int grid = p.sched ? num_sms
                     : p.stream_k ? (int)std::max(1LL, std::min<long long>(num_sms, units / 4))
                                  : std::min(tiles, num_sms);
    if (p.stream_k && (p.sched || p.k_splits != 1 || !p.sk_ws || !p.sk_cnt)) return cudaErrorInvalidValue;
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
    case kFmtQ8_0: return launch_t<BN, DUAL, kFmtQ8_0>(a, a2, b, p, sms, st);
    case kFmtQ4K: return launch_t<BN, DUAL, kFmtQ4K>(a, a2, b, p, sms, st);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace

bool gemm_map_bf16(CUtensorMap *map, const void *ptr, uint64_t cols, uint64_t rows, uint64_t row_bytes,
                   uint32_t box_rows) {
    return make_map(map, ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cols, rows, row_bytes, BK, box_rows,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

size_t skinny_split_bytes(int rows, int splits) { return (size_t)((rows + 15) / 16) * splits * 256 * sizeof(float); }

size_t gemm_stream_k_bytes(int grid, int bn, bool dual) {
    return (size_t)grid * 2 * (dual ? 2 : 1) * BM * bn * sizeof(float);
}

bool gemm_wants_stream_k(long long tiles, int k_tiles, int sms) {
    // Only where whole tiles would leave over half the SMs idle: measured on
    // B200, the split tiles' extra partial-sum traffic and fix-up cost more
    // than a ragged last wave of wider occupancy.
    return tiles > 0 && sms > 0 && k_tiles >= 8 && 2 * tiles <= sms;
}

// Token tile width: narrow tiles for small batches (decode-like calls stay
// weight-bandwidth bound and need no padding to 256 tokens); quantised weights
// take 256-token tiles in SwiGLU mode too, halving the decode work per MMA.
int gemm_token_tile(int n_tok, bool dual, bool quant) {
    if (n_tok <= 32) return 32;
    if (n_tok <= 64) return 64;
    if (n_tok <= 128) return 128;
    return (dual && !quant) ? 128 : 256;
}

cudaError_t launch_stage_decode(const StageArgs &a, int num_sms, cudaStream_t stream) {
    const int epc = (a.fmt == kFmtFp8 || a.fmt == kFmtQ8_0) ? 16 : 32;
    if (a.rows <= 0) return cudaSuccess;
    if ((a.fmt != kFmtFp8 && a.fmt != kFmtMxfp4 && a.fmt != kFmtInt4 && a.fmt != kFmtQ8_0 && a.fmt != kFmtQ4K) ||
        a.cols % epc != 0)
        return cudaErrorInvalidValue;
    if (a.fmt == kFmtInt4 && a.blk_cols % 32 != 0) return cudaErrorInvalidValue;
    const long long chunks = (long long)a.rows * (a.cols / epc);
    const long long want = (chunks + 255) / 256;
    const int grid = (int)std::min<long long>(want, (long long)num_sms * 8);
    k_stage_decode<<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

int skinny_chunk(int fmt) {
    switch (fmt) {
    case kFmtBf16: return Skinny<kFmtBf16>::kChunk;
    case kFmtFp8: return Skinny<kFmtFp8>::kChunk;
    case kFmtQ8_0: return Skinny<kFmtQ8_0>::kChunk;
    case kFmtMxfp4: return Skinny<kFmtMxfp4>::kChunk;
    case kFmtInt4: return Skinny<kFmtInt4>::kChunk;
    case kFmtQ4K: return Skinny<kFmtQ4K>::kChunk;
    default: return 0;
    }
}

cudaError_t launch_skinny(int fmt, const GemmOperand &a, const GemmOperand &b, const GemmParams &p, int k_splits,
                          cudaStream_t stream) {
    const int chunk = skinny_chunk(fmt);
    if (!chunk || p.n_tok < 1 || p.n_tok > 16 || p.k % chunk) return cudaErrorInvalidValue;
    if (fmt == kFmtFp8 && p.blk_cols % 16) return cudaErrorInvalidValue;
    if (fmt == kFmtInt4 && p.blk_cols % 32) return cudaErrorInvalidValue;
    const int chunks = p.k / chunk;
    k_splits = std::max(1, std::min(k_splits, chunks));
    const int per = (chunks + k_splits - 1) / k_splits;
    dim3 grid((p.m_w + 15) / 16, (chunks + per - 1) / per);
    if (grid.y > 1 && (p.sk_ws ? !p.sk_cnt : !(p.flags & kEpiAtomic))) return cudaErrorInvalidValue;
    const uint8_t *w = static_cast<const uint8_t *>(a.ptr);
    const uint16_t *x = static_cast<const uint16_t *>(b.ptr);
    const long long ldx = b.row_bytes / 2;
    switch (fmt) {
    case kFmtBf16: k_skinny<kFmtBf16><<<grid, 256, 0, stream>>>(w, a.row_bytes, x, ldx, p, per); break;
    case kFmtFp8: k_skinny<kFmtFp8><<<grid, 256, 0, stream>>>(w, a.row_bytes, x, ldx, p, per); break;
    case kFmtQ8_0: k_skinny<kFmtQ8_0><<<grid, 256, 0, stream>>>(w, a.row_bytes, x, ldx, p, per); break;
    case kFmtMxfp4: k_skinny<kFmtMxfp4><<<grid, 256, 0, stream>>>(w, a.row_bytes, x, ldx, p, per); break;
    case kFmtInt4: k_skinny<kFmtInt4><<<grid, 256, 0, stream>>>(w, a.row_bytes, x, ldx, p, per); break;
    case kFmtQ4K: k_skinny<kFmtQ4K><<<grid, 256, 0, stream>>>(w, a.row_bytes, x, ldx, p, per); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_gemm(int fmt, const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p,
                        int num_sms, cudaStream_t stream) {
    const bool dual = (p.flags & kEpiSwiglu) != 0;
    if (dual && !a2) return cudaErrorInvalidValue;
    if (!p.bn && gemm_pair_fits(p, fmt, p.k, num_sms)) return launch_gemm_pair(a, a2, b, p, num_sms, stream);
    const int bn = p.bn ? p.bn : gemm_token_tile(p.n_tok, dual, fmt != kFmtBf16);
    if (dual) {
        if (bn == 32) return dispatch_fmt<32, true>(fmt, a, a2, b, p, num_sms, stream);
        if (bn == 64) return dispatch_fmt<64, true>(fmt, a, a2, b, p, num_sms, stream);
        if (bn == 128) return dispatch_fmt<128, true>(fmt, a, a2, b, p, num_sms, stream);
        if (bn == 256 && fmt != kFmtBf16) return dispatch_fmt<256, true>(fmt, a, a2, b, p, num_sms, stream);
        return cudaErrorInvalidValue;
    }
    if (bn == 32) return dispatch_fmt<32, false>(fmt, a, a2, b, p, num_sms, stream);
    if (bn == 64) return dispatch_fmt<64, false>(fmt, a, a2, b, p, num_sms, stream);
    if (bn == 128) return dispatch_fmt<128, false>(fmt, a, a2, b, p, num_sms, stream);
    if (bn == 256) return dispatch_fmt<256, false>(fmt, a, a2, b, p, num_sms, stream);
    return cudaErrorInvalidValue;
}

}  // namespace ditch
