// Bandwidth-bound and small kernels of the trial path (everything that is not
// a weight GEMM). Each launcher runs on the given stream and returns the
// launch's CUDA error code.
#pragma once

#include "common.cuh"

namespace ditch {

// ---- standalone decoders (bit-exact restatements of the reference) --------
// bf16(e4m3[code] * scale[r / br][c / bc])             src/dequant.zig:477-514
cudaError_t dequant_fp8_bf16(const uint8_t *codes, const float *scales, int rows, int cols, int br, int bc,
                             uint16_t *out, cudaStream_t st);
// pack-quantized INT (any bits <= 8), optional zeros and g_idx   dequant.zig:518-597
cudaError_t dequant_int_bf16(const uint32_t *packed, long long wpr, const float *scales, const uint32_t *zeros,
                             const uint32_t *g_idx, int groups, int rows, int cols, int bits, int group,
                             uint16_t *out, cudaStream_t st);
// natural-layout MXFP4                                   dequant.zig:643-673
cudaError_t dequant_mxfp4_bf16(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, uint16_t *out,
                               cudaStream_t st);
// gpt-oss transposed MXFP4                               dequant.zig:603-637
cudaError_t dequant_mxfp4t_bf16(const uint8_t *blocks, const uint8_t *scales, int src_rows, int src_cols,
                                uint16_t *out, cudaStream_t st);
// ggml blocks to f32 (dtype codes of src/tensor.zig:11-32)  quant.zig:57-209
cudaError_t dequant_ggml_f32(int dtype, const uint8_t *src, long long n, float *out, cudaStream_t st);
// Q8_0 blocks to the GEMM's layout (int8 codes [n] and f32 scales [n / 32]),
// and that layout back to the f32 values d * q.
cudaError_t repack_q8_0(const uint8_t *src, long long blocks, int8_t *codes, float *scales, cudaStream_t st);
cudaError_t q8_0_f32(const int8_t *codes, const float *scales, long long n, float *out, cudaStream_t st);
// Q4_K super-blocks to the GEMM's layout (4-bit codes [n / 2] in element
// order and (d * scale, dmin * min) f32 pairs [n / 32]), and that layout back
// to the f32 values d1 * q - m1.
cudaError_t repack_q4_k(const uint8_t *src, long long super_blocks, uint8_t *codes, float *dm, cudaStream_t st);
cudaError_t q4_k_f32(const uint8_t *codes, const float *dm, long long n, float *out, cudaStream_t st);
// ggml blocks to bf16 (the GEMM operand of a GGUF weight)
cudaError_t dequant_ggml_bf16(int dtype, const uint8_t *src, long long n, uint16_t *out, cudaStream_t st);

// Split f32 rows into bf16 segments of width cp (zero padded): segment s is
// the high part bf16(v) (pattern bit s = 0) or the residual bf16(v - hi) (1).
// A product over concatenated segments [xh | xh | xl] . [Wh | Wl | Wh]^T is
// then accurate to about 2^-16 relative on bf16 tensor cores.
cudaError_t split_bf16(const float *src, int rows, int cols, int cp, int nseg, int pattern, uint16_t *dst,
                       cudaStream_t st);
cudaError_t f32_to_bf16(const float *src, uint16_t *dst, long long n, cudaStream_t st);
cudaError_t bf16_to_f32(const uint16_t *src, float *dst, long long n, cudaStream_t st);
cudaError_t f16_to_f32(const uint16_t *src, float *dst, long long n, cudaStream_t st);

// ---- forward pieces -------------------------------------------------------
// x[i] = embed[tokens[i]] (bf16 or f32 table); entry-0 capture of rows with
// cap_slot[i] >= 0 into res[cap_slot][H].
cudaError_t embed_rows(const void *table, int table_bf16, const uint32_t *tokens, int n, int hidden, float *x,
                       const int *cap_slot, float *res, int *status, int vocab, cudaStream_t st);

// h = bf16(rmsnorm(x) * w) per row; rows with cap_slot[i] >= 0 are also
// copied (pre-norm, f32) to res[cap_slot][H] (the residual capture of the
// previous layer's output, src/model.zig:4856-4862). split_k > 0: each row of
// h is [hi | hi | lo] of split_k columns each (the f32-level operand, zero
// padded), where hi = bf16(y) and lo = bf16(y - hi).
cudaError_t rmsnorm_rows_bf16(const float *x, const float *w, int n, int hidden, float eps, uint16_t *h,
                              const int *cap_slot, float *res, const int *row_index, cudaStream_t st,
                              int split_k = 0);
// f32 in/out RMSNorm of n rows (the VTable rmsnormRows, src/tensor.zig:1167-1179).
cudaError_t rmsnorm_rows_f32(const float *x, const float *w, int n, int len, float eps, int gemma, float *out,
                             cudaStream_t st);
// Gather rows then RMSNorm to bf16 (final norm of the logit rows).
cudaError_t gather_rmsnorm_bf16(const float *x, const int *rows, int n, int hidden, float eps, const float *w,
                                uint16_t *h, cudaStream_t st, int split_k = 0);

// ---- f32-level products from bf16 tensor cores (split operands) ----------
// A weight W [rows][k] (f32) becomes [hi | lo | hi] and an activation row
// [hi | hi | lo], segments of kp >= k columns (zero padded), with hi =
// bf16(v) and lo = bf16(v - hi); one GEMM over 3 kp then adds hi.hi + hi.lo
// + lo.hi with f32 accumulation, about 2^-16 relative per product (the
// missing lo.lo term is below that).
// W rows (f32, ld = k) -> out rows of 3 kp.
cudaError_t split_weight_rows(const float *w, int rows, int k, int kp, uint16_t *out, cudaStream_t st);
// Activations x [n][k] (f32) -> out [n][3 kp].
cudaError_t split_act_rows(const float *x, int n, int k, int kp, uint16_t *out, cudaStream_t st);
// SwiGLU of a plain gate | up product gu [n][2 inter] (f32): act32 [n][kp] =
// silu(gate) * up (f32, zero padded) and act [n][3 kp] its split operand.
cudaError_t swiglu_split(const float *gu, int n, int inter, int kp, float *act32, uint16_t *act, cudaStream_t st);
// xa[row * stride] = sum_k x[row][k] a[k] (f32 x, ld = k).
cudaError_t rowdot_f32_strided(const float *x, const float *a, int m, int k, float *xa, int stride, cudaStream_t st);
// out[c] = s[c] + s[kp + c] for c < kp: the v^T W of a split operand's hi and
// lo segments (from a GEMV-T over all 3 kp columns).
cudaError_t add_split_halves(const float *s, int kp, float *out, cudaStream_t st);
// out [rows][kp] f32 = hi + lo of a split weight operand [rows][3 kp].
cudaError_t merge_split_rows(const uint16_t *split, int rows, int kp, float *out, cudaStream_t st);

struct AttnParams {
    const float *qkv;       // [n][qd + 2 kvd] (q | k | v), biases already added
    uint16_t *out;          // [n][qd] bf16
    float *out_f32;         // when set: [n][qd] f32 instead of out
    const int *seq_start;   // per prompt: first row
    const int *seq_len;     // per prompt: rows
    int n_prompts;
    int heads, kv_heads, head_dim;
    const float *rope_cos, *rope_sin;  // [max_pos][head_dim / 2]
    const float *q_norm, *k_norm;      // per-head RMSNorm weights or null
    float eps, scale;
    int *status;
    int max_len;        // longest prompt of the batch
    int force_generic;  // use the one-warp-per-query kernel for any head size
    int tc;             // prompts of at most 128 tokens on tcgen05 (attention_tc.cu): 0 off, 1 a CTA per
                        // (prompt, kv head), 2 two CTAs per SM for prompts of at most 64 tokens
};
// Causal attention within each prompt with GQA, RoPE (neox) and optional q/k
// norms (src/model.zig:4226-4374, attentionWorker 2935-2986).
cudaError_t attention_prefill(const AttnParams &p, cudaStream_t st);
// True when attention_prefill leaves the q and k columns of the QKV rows
// normed and roped in place (the tensor-core path, head sizes 64 and 128).
bool attention_prefill_preps_in_place(int head_dim, int force_generic);
// The tcgen05 kernel for batches whose prompts are all at most 128 tokens
// (head sizes 64 and 128, bf16 output); q and k already normed and roped.
bool attention_tc_eligible(const AttnParams &p);
cudaError_t attention_tc(const AttnParams &p, cudaStream_t st);

// ---- greedy decode with a KV cache (src/model.zig:5378-5444) ---------------
// One layer's cache: keys (normed and roped) and values, f32
// [slots][max_len][kvd] each, the reference's KvCache layout
// (src/model.zig:2586-2724) with a slot per prompt.
struct KvParams {
    float *qkv;                  // [n][qd + 2 kvd]
    const int *row_b, *row_pos;  // per row: cache slot and position
    int n, slots, max_len;
    int heads, kv_heads, head_dim;
    const float *rope_cos, *rope_sin;
    const float *q_norm, *k_norm;
    float eps;
    float *cache_k, *cache_v;
    int prep_k;  // 1: norm and rope the keys while storing them (0: the attention already did, in place)
    int prep_q;  // 1: norm and rope the queries in place (decode rows)
    int *status;
};
// Stores every row's keys and values at (slot, position) of the cache.
cudaError_t kv_store(const KvParams &p, cudaStream_t st);

struct DecodeAttnParams {
    const float *qkv;            // [n][qd + 2 kvd], queries normed and roped
    uint16_t *out;               // [n][qd] bf16
    float *out_f32;              // when set: [n][qd] f32 instead of out
    const int *row_b, *row_pos;  // per row: cache slot and position
    int n, max_len;
    int heads, kv_heads, head_dim;
    const float *cache_k, *cache_v;
    float scale;
    int force_generic;  // the shared-memory kernel for any head size (tests)
};
// Row r attends to keys 0..row_pos[r] of its slot (its own key included:
// kv_store runs first).
cudaError_t attention_decode(const DecodeAttnParams &p, cudaStream_t st);

// out[r] = argmax of row r of x [n][len]: the first maximum wins and NaN
// never does; a row with nothing above -inf gives 0 (src/model.zig:5194-5204).
cudaError_t argmax_rows(const float *x, int n, int len, uint32_t *out, cudaStream_t st);

// xa[m] = sum_k act[m][k] * a[k] (act bf16, a f32): the x . A term of a rank-1
// delta (src/tensor.zig:1036-1042).
cudaError_t rowdot_bf16(const uint16_t *act, const float *a, int m, int k, float *xa, cudaStream_t st);
// The same into xa[row * stride] (one term of a rank-r delta).
cudaError_t rowdot_bf16_strided(const uint16_t *act, const float *a, int m, int k, float *xa, int stride,
                                cudaStream_t st);

// ---- edit (src/abliterate.zig:264-280) and ranking (src/moe.zig:1239-1306) --
// out[c] = sum_r v[r] W[r][c] over a weight in its stored format (bf16 or
// FP8 blocks); out must be zeroed (split-K partial sums are atomically added).
cudaError_t gemv_t_bf16(const uint16_t *w, int rows, int cols, const float *v, float *out, cudaStream_t st);
cudaError_t gemv_t_fp8(const uint8_t *codes, const float *scales, int rows, int cols, int br, int bc,
                       const float *v, float *out, cudaStream_t st);
cudaError_t gemv_t_f32(const float *w, int rows, int cols, const float *v, float *out, cudaStream_t st);
// MXFP4: deterministic (fixed row chunks, partial sums added in order), out
// overwritten; `scratch` holds gemv_t_mxfp4_scratch(slabs, rows, cols) floats.
size_t gemv_t_mxfp4_scratch(int slabs, int rows, int cols);
cudaError_t gemv_t_mxfp4(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, const float *v,
                         float *out, float *scratch, cudaStream_t st);
// The same for each matrix of a stack of `slabs` [rows][cols] MXFP4 matrices
// (one direction v [rows] for all): out[e][c] for e < slabs.
cudaError_t gemv_t_mxfp4_stack(const uint8_t *blocks, const uint8_t *scales, int slabs, int rows, int cols,
                               const float *v, float *out, float *scratch, cudaStream_t st);
// out[r] = ||W_r||_2
cudaError_t row_norms_bf16(const uint16_t *w, int rows, int cols, float *out, cudaStream_t st);
cudaError_t row_norms_f32(const float *w, int rows, int cols, float *out, cudaStream_t st);
cudaError_t row_norms_mxfp4(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, float *out,
                            cudaStream_t st);
// W[r][c] = bf16(W[r][c] + b[r] * a[c]) in place (the materialised edit
// W <- W - alpha r (r^T W) with b = -alpha r, a = r^T W).
cudaError_t rank1_update_bf16(uint16_t *w, int rows, int cols, const float *b, const float *a, cudaStream_t st);
// b[i] = -lambda * v[i]
// Pre-normalised edit (src/abliterate.zig:305-323): vn = v / n (0 where the
// row norm n is 0) and b = -lambda v n.
cudaError_t prenorm_vec(const float *v, const float *n, float lambda, int len, float *vn, float *b, cudaStream_t st);
cudaError_t scale_vec(const float *v, float lambda, int n, float *b, cudaStream_t st);

// ---- scoring ----------------------------------------------------------------
// Per row: logSoftmax with an f64 sum (src/tensor.zig:1203-1210). Rows are
// split into pieces over the SMs; `scratch` holds kl_scratch_bytes(rows,
// vocab) bytes.
cudaError_t log_softmax_rows(const float *x, int rows, int vocab, float *out, void *scratch, cudaStream_t st);
// Per row: sum_j exp(lb_j) (lb_j - logsoftmax(x)_j) in f64 (src/scorers.zig:378-402).
cudaError_t kl_rows(const float *baseline, const float *logits, int rows, int vocab, double *kl, void *scratch,
                    cudaStream_t st);
size_t kl_scratch_bytes(int rows, int vocab);

// ---- capture and directions -------------------------------------------------
// sums[l][h] += mean over take[b] captures of prompt b (f64), per prompt and
// entry (src/engine.zig:414-431); `scratch` holds residual_scratch_bytes(
// entries, hidden, prompts) bytes (the prompt runs' partial sums).
cudaError_t residual_sums(const float *res, int entries, int nc, int hidden, const int *first, const int *take,
                          int prompts, double *sums, double *scratch, cudaStream_t st);
size_t residual_scratch_bytes(int entries, int hidden, int prompts);
// dirs[e] = normalize(bad - good) (orthogonalised against normalize(good)),
// from f64 sums and counts (src/abliterate.zig:88-109, engine.zig:334-336).
cudaError_t directions_from_sums(const double *good_sums, double good_count, const double *bad_sums,
                                 double bad_count, int entries, int hidden, int orthogonalize, float *dirs,
                                 float *good_mean, float *bad_mean, cudaStream_t st);

// ---- element-wise entries of the compute seam (src/compute.zig:90-117) -------
cudaError_t softmax_rows_f32(float *x, int n, int len, cudaStream_t st);
cudaError_t gated_silu_f32(const float *gate, const float *up, int n, int len, long long in_stride,
                           long long out_stride, float *out, cudaStream_t st);
cudaError_t rope_rows_f32(float *x, int n, int dim, const float *cos, const float *sin, int half, const uint32_t *pos,
                          int style, cudaStream_t st);
cudaError_t attention_scores_f32(float *scores, const float *q, int hd, const float *k, int n_keys, long long stride,
                                 float scale, cudaStream_t st);
cudaError_t attention_values_f32(float *out, const float *scores, int n_keys, const float *v, int vd,
                                 long long stride, cudaStream_t st);
cudaError_t layernorm_rows_f32(const float *x, const float *w, const float *b, int n, int len, float eps,
                               int one_plus, float *out, cudaStream_t st);

}  // namespace ditch
