/* CPU restatement of ditch's engine for the trial-evaluation hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * product (`libditch_cuda.so`) and the timed CPU baseline of `bench.py`.  Only
 * `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg load
 * it; the product never calls into it.
 *
 * Every function cites the reference (plyght/ditch v0.8.0) file:line it
 * restates.  Arithmetic follows the reference's f32 kernels with the AVX-512
 * kernel shape (VL = 16 lanes, fused multiply-add), see src/tensor.zig:623-687.
 * Parity is pinned against the reference's own fixtures
 * (tests/fixtures/<family>/reference.json, 2e-3 max abs, src/model_test.zig:58-84)
 * and known-answer tests (src/quant.zig:367-482, src/dequant.zig:1290-1310,
 * src/abliterate.zig:554-742).
 */
#ifndef DITCH_ORACLE_H
#define DITCH_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- conversions (src/tensor.zig:419-440) ---- */
uint16_t or_f32_to_bf16(float v);
float or_bf16_to_f32(uint16_t v);
float or_f16_to_f32(uint16_t v);
uint16_t or_f32_to_f16(float v);
void or_bf16_to_f32_n(const uint16_t *src, float *dst, size_t n);
void or_f32_to_bf16_n(const float *src, uint16_t *dst, size_t n);

/* ---- dot products and matrix products (src/tensor.zig:550-1122) ---- */
float or_dot(const float *a, const float *b, size_t n);
/* out[n][rows] = x[n][cols] . W^T (+ x . (B A)^T), W f32 [rows][cols];
 * delta A [rank][cols], B [rows][rank] (NULL / rank 0 = none). */
void or_matmul_t(float *out, const float *x, size_t n, const float *w, size_t rows,
                 size_t cols, const float *da, const float *db, size_t rank);
/* The same product over bf16 weights (src/tensor.zig:827-883, 449-486): each
 * task converts its weight rows to f32, then the f32 tiles; for at most four
 * inputs ditch's fused path (src/tensor.zig:919-1020) gives the same dot
 * products (every row a VL-lane FMA dot). */
void or_matmul_t_bf16(float *out, const float *x, size_t n, const uint16_t *w, size_t rows,
                      size_t cols, const float *da, const float *db, size_t rank);
/* out[q][cols] = y[q][rows] . W (src/tensor.zig:1079-1094). */
void or_matvec_t_multi(float *out, const float *w, size_t rows, size_t cols,
                       const float *y, size_t q);
/* out[rows] = ||W_i||_2 (src/tensor.zig:1114-1122). */
void or_row_norms(float *out, const float *w, size_t rows, size_t cols);

/* ---- element-wise (src/tensor.zig:1167-1369) ---- */
void or_rmsnorm(float *out, const float *x, const float *w, size_t len, float eps);
void or_softmax_inplace(float *x, size_t n);
void or_log_softmax(float *out, const float *x, size_t n);
float or_silu(float x);
void or_exp_vec16(const float *x, float *out); /* expVec on 16 lanes */
/* out[i][j] = silu(gate[i][j]) * up[i][j] with the reference's VL split
 * (src/tensor.zig:1309-1337). */
void or_gated_silu(float *out, const float *gate, const float *up, size_t n, size_t len,
                   size_t in_stride, size_t out_stride);
void or_apply_rope(float *x, const float *cos_row, const float *sin_row, size_t dim);
/* RoPE frequency scaling (src/arch.zig:132-142): 0 none, 1 llama3 (factor,
 * low/high frequency factors, original context length), 2 linear (factor),
 * 3 yarn (factor, orig_max, beta_fast, beta_slow, truncate,
 * attention_factor), 4 per-frequency divisors (factors, attention_factor). */
typedef struct {
    int scaling;
    double factor, low_ff, high_ff, orig_max;
    const float *factors;
    size_t n_factors;
    double attention_factor, beta_fast, beta_slow;
    int truncate;
} or_rope;
/* [len][dim/2] RoPE table, f64 angles cast to f32 (src/model.zig:2200-2282). */
void or_rope_table_ex(float *cos_t, float *sin_t, size_t len, size_t dim, double theta, const or_rope *r);
/* the same for scaling 0 / 1 / 2 from plain arguments */
void or_rope_table(float *cos_t, float *sin_t, size_t len, size_t dim, double theta,
                   int scaling, double factor, double low_ff, double high_ff, double orig_max);

/* ---- ggml block decode to f32 (src/quant.zig:57-209) ----
 * dtype codes follow src/tensor.zig:11-32: 5 q8_0, 6 q4_0, 7 q4_1, 8 q5_0,
 * 9 q5_1, 10 q4_k, 11 q6_k, 12 q8_k. */
size_t or_ggml_block_size(int dtype);
size_t or_ggml_block_bytes(int dtype);
int or_dequant_ggml(int dtype, const uint8_t *src, float *out, size_t n);
void or_quant_q8_0(const float *x, uint8_t *out, size_t n); /* src/quant.zig:245-255 */
/* A valid Q4_K encoder for synthetic data (the reference has none). */
void or_quant_q4_k(const float *x, uint8_t *out, size_t n);

/* ---- safetensors dequant to bf16 (src/dequant.zig:259-673) ---- */
float or_e4m3_value(uint8_t code);
void or_f32_to_bf16_array(const float *x, size_t n, uint16_t *out);
float or_e8m0_scale(uint8_t b);
/* bf16(e4m3[code] * scale[r / br][c / bc]) (src/dequant.zig:477-514). */
void or_dequant_fp8(const uint8_t *codes, const float *scales, size_t rows, size_t cols,
                    size_t br, size_t bc, uint16_t *out);
/* compressed-tensors pack-quantized INT (src/dequant.zig:518-597).
 * packed: [rows][words_per_row] u32; scales f32 [rows][groups];
 * zeros: NULL or [ceil(rows*bits/32)][groups] u32; g_idx: NULL or [cols]. */
void or_dequant_int_packed(const uint32_t *packed, size_t words_per_row, const float *scales,
                           const uint32_t *zeros, const uint32_t *g_idx, size_t rows,
                           size_t cols, int bits, size_t group, uint16_t *out);
/* Natural-layout MXFP4 (src/dequant.zig:643-673): blocks [rows][cols/2],
 * scales [rows][cols/32]. */
void or_dequant_mxfp4_packed(const uint8_t *blocks, const uint8_t *scales, size_t rows,
                             size_t cols, uint16_t *out);
/* gpt-oss MXFP4, stored transposed (src/dequant.zig:603-637): source
 * [src_rows][src_cols/32][16] + [src_rows][src_cols/32]; out [src_cols][src_rows]. */
void or_dequant_mxfp4_transposed(const uint8_t *blocks, const uint8_t *scales,
                                 size_t src_rows, size_t src_cols, uint16_t *out);
uint32_t or_unpack_field(const uint32_t *words, size_t i, int bits);

/* Synthetic-data quantisers restating tools/make_fixture.py. */
void or_quant_fp8_block(const float *w, size_t rows, size_t cols, size_t br, size_t bc,
                        uint8_t *codes, float *scales); /* make_fixture.py:109-127 */
void or_quant_mxfp4_packed(const float *w, size_t rows, size_t cols, uint8_t *blocks,
                           uint8_t *scales);          /* make_fixture.py:210-224 */
void or_quant_int_packed(const float *w, size_t rows, size_t cols, int bits, size_t group,
                         uint32_t *packed, float *scales, uint32_t *zeros); /* :156-194 */

/* ---- the forward (src/model.zig:4619-4959, src/moe.zig:998-1228) ---- */
typedef struct {
    int n_layers, hidden, heads, kv_heads, head_dim, inter, vocab;
    float eps;
    double rope_theta;
    int qk_norm;           /* 1: per-head RMSNorm of q and k before RoPE (Qwen3) */
    int rope_scaling;      /* or_rope's scaling codes */
    double rope_factor, rope_low_ff, rope_high_ff, rope_orig_max;
    int n_experts, top_k, moe_inter, norm_topk;
    const float *rope_factors;
    size_t n_rope_factors;
    double rope_attention_factor, rope_beta_fast, rope_beta_slow;
    int rope_truncate;
} or_config;

typedef struct {
    const float *input_norm, *post_norm;
    const float *q, *k, *v, *o;       /* [qd][H], [kvd][H], [kvd][H], [H][qd] */
    const float *qb, *kb, *vb;        /* NULL when the family has none */
    const float *q_norm, *k_norm;     /* [head_dim] */
    const float *gate, *up, *down;    /* dense MLP: [I][H], [I][H], [H][I] */
    const float *router;              /* MoE layer: [E][H]; NULL for a dense layer */
    const float *e_gate, *e_up, *e_down; /* [E][mi][H], [E][mi][H], [E][H][mi] */
    const float *o_da, *o_db; size_t o_rank;       /* o_proj delta */
    const float *down_da, *down_db; size_t down_rank;
    const float *const *e_down_da; const float *const *e_down_db; /* per expert, may be NULL */
    const size_t *e_down_rank;        /* per expert terms of its delta (NULL: 1) */
} or_layer;

typedef struct {
    or_config c;
    const float *embed;      /* [V][H] */
    const float *final_norm; /* [H] */
    const float *lm_head;    /* [V][H] */
    const or_layer *layers;
    /* 1: the linear weights (q, k, v, o, gate, up, down, router, expert stacks
     * and lm_head) are bf16 bit arrays (uint16), multiplied through ditch's
     * half-precision path (or_matmul_t_bf16), as a checkpoint held in bf16
     * is in mapped mode */
    int w_bf16;
} or_model;

/* One batched forward (src/model.zig:4619 `forward` + ForwardOptions 3136-3144).
 * rows (b, pos) per token; residuals [L+1][nc][H]; logits [nl][V]. */
int or_forward(const or_model *m, const uint32_t *tokens, const uint32_t *row_b,
               const uint32_t *row_pos, size_t n, const size_t *capture_rows, size_t nc,
               float *residuals, const size_t *logit_rows, size_t nl, float *logits);

/* ---- abliteration (src/abliterate.zig) ---- */
typedef struct { float max_weight, max_weight_position, min_weight, min_weight_distance; } or_params;
/* returns 0 when the layer is untouched (null in the reference) */
int or_kernel_weight(or_params p, size_t layer, float *out);
void or_compute_directions(const float *good, const float *bad, size_t entries, size_t hidden,
                           int orthogonalize, float *dirs);
/* none-mode delta: A = v^T W [cols], B = -lambda v [rows] (abliterate.zig:270-280). */
void or_compute_delta_none(const float *w, size_t rows, size_t cols, const float *v,
                           float lambda, float *a, float *b);
/* W' = W + B A, f32 (abliterate.zig:544-552). */
void or_materialize(const float *w, size_t rows, size_t cols, const float *a, const float *b,
                    size_t rank, float *out);
/* Expert ranking score ||V^T W||/||W||_F (moe.zig:1239-1250). */
float or_score_down(const float *w, size_t rows, size_t cols, const float *v);
void or_rank_scores(const float *scores, size_t n, uint32_t *order); /* moe.zig:1296-1306 */

/* ---- engine capture and scorers ---- */
/* Window means of captured residuals accumulated in f64 (src/engine.zig:369-438).
 * residuals [L+1][nc][H], capture rows grouped per prompt (first_capture[b],
 * take[b]); sums [entries][H] f64 are added to. */
void or_residual_sums(const float *residuals, size_t entries, size_t nc, size_t hidden,
                      const size_t *first_capture, const size_t *take, size_t prompts,
                      double *sums);
/* KL of one trial against baseline log-probs (src/scorers.zig:378-402),
 * kl_tokens = 1: mean over prompts of sum_j exp(lb_j)(lb_j - lt_j). */
double or_kl_first_token(const float *baseline_logp, const float *logits, size_t prompts,
                         size_t vocab, double *per_prompt);

/* threads used by the parallel kernels (0 = all cores) */
void or_set_threads(int n);
int or_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
