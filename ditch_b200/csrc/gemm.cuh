// tcgen05/TMEM GEMM for ditch's weight products (`tensor.matmulT`,
// src/tensor.zig:1023-1045): out[m][n] = x[m][:] . W[n][:] over K.
//
// Orientation: the WEIGHT is the MMA's M operand (128 weight rows per tile,
// TMEM lane = weight row) and the TOKENS are the N operand (BN tokens per
// tile). That makes the epilogue store coalesced (a warp writes 32
// consecutive output features of one token) and lets small token counts
// use a narrow N instead of padding a 128-row M tile.
//
// Weight formats:
//   kFmtBf16  - bf16 weight tiles loaded by TMA straight into the swizzled
//               operand layout;
//   kFmtFp8   - E4M3 codes with f32 block scales (src/dequant.zig:477-514):
//               TMA stages the raw code tile, four transform warps expand it
//               to bf16(code * scale) in the swizzled operand layout;
//   kFmtMxfp4 - E2M1 nibbles with E8M0 scales per 32 (src/dequant.zig:643-673);
//   kFmtInt4  - compressed-tensors pack-quantized INT4 with f32 group scales
//               and packed zero points (src/dequant.zig:518-597);
//   kFmtQ8_0, kFmtQ4K - ggml blocks (src/quant.zig:81-85, 148-173), decoded
//               to f32 and rounded to bf16 for the MMA.
#pragma once

#include "common.cuh"

namespace ditch {

enum WeightFormat : int {
    kFmtBf16 = 0,
    kFmtFp8 = 1,
    kFmtMxfp4 = 2,
    kFmtInt4 = 3,
    kFmtQ8_0 = 4,
    kFmtQ4K = 5,
};

// Epilogue flags.
enum EpilogueFlags : int {
    kEpiOutBf16 = 1,     // store bf16 instead of f32
    kEpiResidual = 2,    // out (f32) += result, in place (the residual add)
    kEpiSwiglu = 4,      // dual accumulators: out = silu(gate) * up (bf16)
    kEpiAtomic = 8,      // split-K: atomically add f32 partial sums
};

struct GemmParams {
    int m_w;       // valid weight rows (output features)
    int n_tok;     // valid tokens
    int k;         // reduction length
    int w_tiles, t_tiles, k_tiles, k_splits;
    int kt_unit;        // k-tiles per raw weight tile: the grain of K splits (set by the launcher)
    int a2_row_offset;  // dual mode: row offset of the up weight in the A2 map
    int a_row0;         // first weight row (a slab of a stacked tensor)
    void *out;
    long long ldo;      // row stride of out, in elements
    int flags;
    const float *bias;  // [m_w] or null
    const float *xa;    // [n_tok][delta_rank]: x . a_t of the delta's rank terms, or null
    const float *db;    // [m_w][delta_rank]: B of the delta (-lambda v for rank 1)
    int delta_rank;     // terms of the delta (0 or 1: rank 1; at most kMaxDeltaRank)
    // quantised weights: per-format side data
    const float *scales;     // fp8 block scales [rows/br][scols]; int4 [rows][groups]
    const uint8_t *scales_u8;  // mxfp4 E8M0 scales [rows][k/32]
    const uint32_t *zeros;   // int4 packed zero points [ceil(rows*4/32)][groups]
    const uint8_t *raw;      // ggml blocks: raw rows (read with plain loads)
    long long raw_row_bytes;
    int blk_rows, blk_cols, scale_cols;  // fp8 block shape; int4 group in blk_cols
    int *status;
    // Grouped mode (token-sorted routed experts): one entry per output tile,
    // (expert, first token row, token rows, weight tile); the weight rows of
    // expert e start at a_row0 + e * slab_rows. Null sched = dense mode.
    const int4 *sched;
    const int *n_sched;
    int slab_rows;
    const int *e_flags;   // per expert: apply the rank-1 delta (xa, db) only when set
    long long db_stride;  // db of expert e at db + e * db_stride
    int bn;               // token tile (32, 64, 128, 256); 0 = chosen from n_tok
    // Stream-K (dense mode, k_splits 1): the grid's CTAs take equal contiguous
    // ranges of the (tile, k-tile) units. A tile split between CTAs is summed
    // in k order by the CTA that finishes the last of its parts (the others
    // leave their partial sums in sk_ws and count themselves in sk_cnt), which
    // then runs the epilogue once: results do not depend on timing.
    int stream_k;
    float *sk_ws;  // [grid][2][accumulators][128][bn] f32 partial sums
    int *sk_cnt;   // [tiles] arrival counters, zero between launches
    // Dense bf16 products over many tokens may run on CTA pairs
    // (cta_group::2, gemm2.cu): 256-row output tiles, each CTA of the pair
    // loading half the weight rows and half the token rows. 0 never, 1
    // single-accumulator products, 2 SwiGLU products too.
    int cta_pairs;
};

// Device bytes of the weight-streaming product's split partial sums (in
// sk_ws; the per-row-block counters are the first (rows + 15) / 16 of sk_cnt).
size_t skinny_split_bytes(int rows, int splits);
// Device bytes of the stream-K partial sums for a grid of `grid` CTAs.
size_t gemm_stream_k_bytes(int grid, int bn, bool dual);
// Whether a dense GEMM of `tiles` whole output tiles runs stream-K on `sms`
// SMs (when the whole tiles would leave over half of them idle).
bool gemm_wants_stream_k(long long tiles, int k_tiles, int sms);

constexpr int kMaxDeltaRank = 4;

// Token tile width the GEMM uses for n_tok tokens (dual = SwiGLU mode,
// quant = a weight format decoded inside the GEMM).
int gemm_token_tile(int n_tok, bool dual, bool quant);

// Host side: launches one GEMM on `stream`. Returns a CUDA error code.
struct GemmOperand {
    const void *ptr;    // device pointer of the operand (or raw codes)
    int rows;           // rows of the whole tensor (for the TMA map)
    int cols;           // K (elements)
    long long row_bytes;
};

// The CTA-pair GEMM (gemm2.cu): whether it takes this product, and its launch.
bool gemm_pair_fits(const GemmParams &p, int fmt, int k, int num_sms);
cudaError_t launch_gemm_pair(const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b, GemmParams p,
                             int num_sms, cudaStream_t stream);
// The 128B-swizzled K-major bf16 tensor map of the GEMMs (64 x box_rows boxes).
bool gemm_map_bf16(CUtensorMap *map, const void *ptr, uint64_t cols, uint64_t rows, uint64_t row_bytes,
                   uint32_t box_rows);

cudaError_t launch_gemm(int fmt, const GemmOperand &a, const GemmOperand *a2, const GemmOperand &b,
                        GemmParams p, int num_sms, cudaStream_t stream);

// Staged decode of rows [row0, row0 + rows) of a quantised weight (FP8 block,
// MXFP4 or INT4 in the GEMM's storage) to bf16 [rows][cols], bit-identical to
// the operand the fused GEMM builds in shared memory. cols must be a multiple
// of 16 (FP8) or 32 (MXFP4, INT4); INT4 groups a multiple of 32.
struct StageArgs {
    int fmt;
    const uint8_t *data;
    long long row_bytes;
    int row0, rows, cols;
    const float *scales;       // FP8 [rows / blk_rows][scale_cols]; INT4 [rows][scale_cols]
    const uint8_t *scales_u8;  // MXFP4 E8M0 [rows][cols / 32]
    const uint32_t *zeros;     // INT4 packed zero points or null
    int blk_rows, blk_cols, scale_cols;
    uint16_t *out;
};

cudaError_t launch_stage_decode(const StageArgs &a, int num_sms, cudaStream_t stream);

// Weight-streaming product for 1..16 tokens (decode-like calls): the weight
// read once in its stored format (bf16, FP8, Q8_0, MXFP4, INT4), tensor-core
// mma.sync with the tokens as the 16-row operand. Plain f32 output, residual
// add or atomic add (p.flags), bias and rank-1 delta (split 0). K must be a
// multiple of skinny_chunk(fmt); 0 = format not supported.
int skinny_chunk(int fmt);
cudaError_t launch_skinny(int fmt, const GemmOperand &a, const GemmOperand &b, const GemmParams &p, int k_splits,
                          cudaStream_t stream);

}  // namespace ditch
