/* ditch_cuda: a B200 (sm_100a) backend for ditch's trial-evaluation hot path.
 *
 * A plain C ABI (no C++ or torch types) for a `--device cuda` backend behind
 * ditch's compute seam (src/compute.zig). Two layers:
 *
 *   1. The per-op entries of `compute.VTable` (src/compute.zig:90-117): host
 *      slices in, host slices out, "upload, compute, drop" per weight tile
 *      (the contract of src/vulkan/backend.zig:223-244), with an optional
 *      device-side residency cache of weight tiles (compute.Residency,
 *      src/compute.zig:580-693).
 *   2. Coarse entries for a model kept resident in HBM: the batched forward
 *      with residual capture and logit rows (model.forward,
 *      src/model.zig:4619-4853), the residual-mean pass
 *      (engine.getResidualMeanObserved, src/engine.zig:314-438), directions
 *      (abliterate.computeDirections, src/abliterate.zig:88-109), the
 *      none-mode edit (abliterate.apply, src/abliterate.zig:148-280), expert
 *      ranking (moe.rankScores, src/moe.zig:1239-1306) and the first-token KL
 *      (KlDivergence.init / score, src/scorers.zig:311-402).
 *
 * Errors mirror compute.Error (src/compute.zig:54-60): every entry returns a
 * status; DITCH_CUDA_UNSUPPORTED means "the caller runs the CPU kernel" (the
 * seam's fallback, which lives in ditch, never in this library).
 * ditch_cuda_last_error() describes the last failure on this thread.
 *
 * Threading: a device handle serialises its calls with a mutex (ditch may
 * call from any pool thread, src/compute.zig:161-163).
 */
#ifndef DITCH_CUDA_H
#define DITCH_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: compute.Error (src/compute.zig:54-60) ---- */
#define DITCH_CUDA_OK 0
#define DITCH_CUDA_UNSUPPORTED 1   /* error.Unsupported: shape or dtype not taken */
#define DITCH_CUDA_DEVICE_FAILED 2 /* error.DeviceFailed */
#define DITCH_CUDA_OUT_OF_MEMORY 3 /* error.OutOfMemory */
#define DITCH_CUDA_INVALID 4       /* invalid argument */

/* Weight dtypes: tensor.DType order (src/tensor.zig:11-32). */
#define DITCH_DTYPE_F32 0
#define DITCH_DTYPE_F16 1
#define DITCH_DTYPE_BF16 2
#define DITCH_DTYPE_Q8_0 5
#define DITCH_DTYPE_Q4_0 6
#define DITCH_DTYPE_Q4_1 7
#define DITCH_DTYPE_Q5_0 8
#define DITCH_DTYPE_Q5_1 9
#define DITCH_DTYPE_Q4_K 10
#define DITCH_DTYPE_Q6_K 11
#define DITCH_DTYPE_Q8_K 12

typedef struct ditch_cuda_device ditch_cuda_device;
typedef struct ditch_cuda_model ditch_cuda_model;

/* Text of the last failure on the calling thread (empty when none). */
const char *ditch_cuda_last_error(void);
/* Number of usable CUDA devices (0 when no driver or GPU is present). */
int ditch_cuda_device_count(void);
/* Library version string. */
const char *ditch_cuda_version(void);

/* ---- device: compute.select(.cuda) / Device.deinit (src/compute.zig:224-279) ----
 * memory_budget: bytes the residency cache may keep (0 = upload every tile,
 * compute and drop it), like `--gpu-memory`. */
int ditch_cuda_open(int ordinal, uint64_t memory_budget, ditch_cuda_device **out);
void ditch_cuda_close(ditch_cuda_device *dev);
/* VTable.forgetWeights: drops every resident weight tile. */
void ditch_cuda_forget_weights(ditch_cuda_device *dev);
/* compute.served: weight-tile operations this device served. */
uint64_t ditch_cuda_served(const ditch_cuda_device *dev);
/* Host-stable weight addresses (compute.weights_stable, src/compute.zig:165-172):
 * residency is keyed by host address only while this is set. */
void ditch_cuda_set_weights_stable(ditch_cuda_device *dev, int stable);

/* ---- per-op VTable entries (src/compute.zig:90-117), host buffers ----
 * Weight = {data, dtype, rows, cols} (src/tensor.zig:517-521), w_len bytes.
 * f32 / f16 weights and f32 inputs run as a split-bf16 (hi + lo) product on
 * the tensor cores, accurate to about 2^-16 relative; bf16 weights exactly. */
int ditch_cuda_matmul_t(ditch_cuda_device *dev, float *out, const float *x, size_t n, const uint8_t *w,
                        size_t w_len, int dtype, size_t rows, size_t cols);
int ditch_cuda_matvec_t_multi(ditch_cuda_device *dev, float *out, const uint8_t *w, size_t w_len, int dtype,
                              size_t rows, size_t cols, const float *y, size_t q);
int ditch_cuda_row_norms(ditch_cuda_device *dev, float *out, const uint8_t *w, size_t w_len, int dtype, size_t rows,
                         size_t cols);
int ditch_cuda_attention_scores(ditch_cuda_device *dev, float *scores, size_t n_keys, const float *q, size_t hd,
                                const float *k, size_t k_len, size_t stride, float scale);
int ditch_cuda_attention_values(ditch_cuda_device *dev, float *out, size_t vd, const float *scores, size_t n_keys,
                                const float *v, size_t v_len, size_t stride);
/* act: tensor.Activation code; 0 = silu is implemented, others UNSUPPORTED. */
int ditch_cuda_gated_activation(ditch_cuda_device *dev, uint32_t act, float *out, const float *gate, const float *up,
                                size_t n, size_t len, size_t in_stride, size_t out_stride);
int ditch_cuda_rmsnorm_rows(ditch_cuda_device *dev, float *out, const float *x, const float *weight, size_t w_len,
                            size_t n, size_t len, float eps, int gemma_style);
int ditch_cuda_layernorm_rows(ditch_cuda_device *dev, float *out, const float *x, const float *weight, size_t w_len,
                              const float *bias, size_t n, size_t len, float eps, int one_plus);
int ditch_cuda_softmax_rows(ditch_cuda_device *dev, float *x, size_t n, size_t len);
/* style 0 = neox (rotate half), 1 = gptj (interleaved); tables [table_len][half]. */
int ditch_cuda_rope_rows(ditch_cuda_device *dev, float *x, size_t n, size_t dim, const float *cos_t,
                         const float *sin_t, size_t table_len, size_t half, const uint32_t *pos, int style);

/* ---- standalone decoders, bit-exact against src/dequant.zig / src/quant.zig ----
 * Host buffers in, host buffers out. */
/* bf16(e4m3[code] * scale[r / br][c / bc]), scales f32 (src/dequant.zig:477-514). */
int ditch_cuda_dequant_fp8(ditch_cuda_device *dev, const uint8_t *codes, const float *scales, size_t rows,
                           size_t cols, size_t br, size_t bc, uint16_t *out_bf16);
/* compressed-tensors pack-quantized INT (src/dequant.zig:518-597): packed
 * [rows][words_per_row] u32, scales f32 [rows][groups], zeros NULL or
 * [ceil(rows*bits/32)][groups] u32, g_idx NULL or [cols]. */
int ditch_cuda_dequant_int(ditch_cuda_device *dev, const uint32_t *packed, size_t words_per_row, const float *scales,
                           size_t groups, const uint32_t *zeros, const uint32_t *g_idx, size_t rows, size_t cols,
                           int bits, size_t group, uint16_t *out_bf16);
/* MXFP4, natural layout (src/dequant.zig:643-673) or the transposed gpt-oss
 * layout (transposed = 1, src/dequant.zig:603-637; rows/cols are the source's). */
int ditch_cuda_dequant_mxfp4(ditch_cuda_device *dev, const uint8_t *blocks, const uint8_t *scales, size_t rows,
                             size_t cols, int transposed, uint16_t *out_bf16);
/* ggml blocks to f32 (quant.dequantize, src/quant.zig:57-79). */
int ditch_cuda_dequant_ggml(ditch_cuda_device *dev, int dtype, const uint8_t *src, size_t src_len, size_t n,
                            float *out_f32);

/* ---- resident model ---- */
typedef struct {
    int n_layers, hidden, heads, kv_heads, head_dim, inter, vocab;
    float eps;
    double rope_theta;
    /* RoPE frequency scaling (src/model.zig:2200-2282): 0 none; 1 llama3
     * (rope_factor, rope_low_ff, rope_high_ff, rope_orig_max); 2 linear
     * (inv_freq / rope_factor); 3 yarn (rope_factor, rope_orig_max,
     * rope_beta_fast, rope_beta_slow, rope_truncate, rope_attention_factor);
     * 4 per-frequency divisors inv_freq[i] / rope_factors[i] for i <
     * n_rope_factors (a GGUF rope_freqs.weight, ditch's "ditch_factors", or
     * LongRoPE's short factors with its rope_attention_factor). */
    int rope_scaling;
    double rope_factor, rope_low_ff, rope_high_ff, rope_orig_max;
    int qk_norm; /* per-head q/k RMSNorm before RoPE (Qwen3) */
    int n_experts, top_k, moe_inter, norm_topk;
    const uint8_t *moe_layers; /* [n_layers]: 1 = routed-expert MLP; NULL = dense model */
    int max_seq;               /* longest prompt (RoPE table rows) */
    /* Expert parallelism over ep_world ranks (0 or 1: this model holds every
     * expert): this rank keeps routed experts [ep_rank E / ep_world,
     * (ep_rank + 1) E / ep_world) of the stacks it is given and runs MoE
     * layers through a peer group (ditch_cuda_model_set_group). */
    int ep_rank, ep_world;
    /* Tensor parallelism over tp_world ranks (0 or 1: none; dense models,
     * f32 / f16 / bf16 weights): this rank keeps query heads [tp_rank H_q /
     * tp_world, ...), the matching kv heads and MLP columns; q / k / v / gate /
     * up are split by rows and o / down by columns. Tensors may be given whole
     * (the loader takes this rank's slice) or already sharded. o / down
     * partial sums are all-reduced over the peer group after each layer. */
    int tp_rank, tp_world;
    /* RoPE scaling, continued (read for rope_scaling 3 and 4): cos / sin are
     * multiplied by rope_attention_factor (0 is read as 1); rope_factors is
     * read during the load only. */
    const float *rope_factors;
    size_t n_rope_factors;
    double rope_attention_factor, rope_beta_fast, rope_beta_slow;
    int rope_truncate;
} ditch_cuda_model_config;

/* Storage formats of a resident tensor. */
#define DITCH_FMT_F32 0
#define DITCH_FMT_BF16 1
#define DITCH_FMT_F16 2
#define DITCH_FMT_FP8_BLOCK 3 /* E4M3 codes + f32 scales [ceil(rows/br)][ceil(cols/bc)] */
#define DITCH_FMT_INT_PACKED 4 /* u32 words + scales (f32 or bf16) + optional packed zeros */
#define DITCH_FMT_MXFP4 5      /* natural layout nibbles [rows][cols/2] + E8M0 [rows][cols/32] */
#define DITCH_FMT_Q8_0 6
#define DITCH_FMT_Q4_K 7

#define DITCH_SCALE_F32 0
#define DITCH_SCALE_BF16 1

/* One tensor of the model. Canonical names: "embed", "final_norm", "lm_head",
 * and per layer i "L<i>.input_norm", "L<i>.post_norm", "L<i>.q|k|v|o",
 * "L<i>.qb|kb|vb", "L<i>.q_norm|k_norm", "L<i>.gate|up|down" (dense MLP),
 * "L<i>.router" and the expert stacks "L<i>.e_gate|e_up|e_down" ([slabs =
 * experts][rows][cols]). Host memory (or device memory when on_device is
 * set), read during the call only. With device memory the loader first waits
 * for all work queued on the GPU, so data still being produced on another
 * stream is complete before it is read. */
typedef struct {
    const char *name;
    int format;
    size_t slabs, rows, cols;
    const void *data;
    size_t data_bytes;
    const void *scales;
    size_t scales_bytes;
    int scales_dtype;
    const void *zeros;
    size_t zeros_bytes;
    int block_rows, block_cols; /* FP8 block; INT: block_cols = group size */
    int bits;                   /* INT: bits per field */
    int on_device;              /* 1: data / scales / zeros are device pointers of this GPU */
} ditch_cuda_tensor;

int ditch_cuda_model_load(ditch_cuda_device *dev, const ditch_cuda_model_config *cfg, const ditch_cuda_tensor *tensors,
                          size_t n_tensors, ditch_cuda_model **out);
void ditch_cuda_model_free(ditch_cuda_model *m);

/* A checkpoint from disk (src/safetensors.zig, src/gguf_model.zig,
 * src/dequant.zig:783-1187): a Hugging Face directory (config.json and
 * *.safetensors; model_type llama, mistral, qwen2, qwen3, qwen3_moe or
 * mixtral; bf16 / f16 / f32, FP8 block-scaled with weight_block_size, or
 * compressed-tensors pack-quantized INT without g_idx; routed experts one
 * tensor per expert, mixtral's w1 / w3 / w2, or fused gate_up_proj /
 * down_proj in either orientation) or a GGUF file (general.architecture
 * llama, with experts mixtral, qwen2, qwen3 or qwen3moe; F32, F16, BF16, Q8_0,
 * Q4_K; llama's permuted q / k rows and biases restored; stacked ffn_*_exps
 * experts; an embedded ditch.hf.config_json; rope_freqs.weight as Llama 3's
 * scaling when it matches the standard settings, else as per-frequency
 * divisors). rope_scaling types llama3, linear, yarn, longrope,
 * ditch_factors; dynamic, mrope and default read as plain RoPE. Quantised groups reach the device raw. The files
 * are memory-mapped during the call. A directory holding an export's
 * .incomplete marker is refused.
 * max_seq: the RoPE table rows (0 = 4096). Anything else returns
 * DITCH_CUDA_UNSUPPORTED with the reason in ditch_cuda_last_error(). */
int ditch_cuda_model_load_checkpoint(ditch_cuda_device *dev, const char *path, int max_seq, ditch_cuda_model **out);
/* The config and tensor count the loader would use, without a device
 * (moe_layers, when given, receives up to moe_layers_len flags; rope_factors
 * up to rope_factors_len per-frequency RoPE divisors, their count in
 * cfg->n_rope_factors; cfg's own moe_layers and rope_factors pointers are
 * left NULL). */
int ditch_cuda_checkpoint_inspect(const char *path, ditch_cuda_model_config *cfg, size_t *n_tensors,
                                  uint8_t *moe_layers, size_t moe_layers_len, float *rope_factors,
                                  size_t rope_factors_len);
/* Device bytes the resident model holds. */
uint64_t ditch_cuda_model_bytes(const ditch_cuda_model *m);

/* Export (src/export.zig saveModel): the Hugging Face directory src_dir the
 * model was loaded from, written to out_dir with the model's deltas merged on
 * the device (W' = W + B A, rank terms added in order; fused expert tensors
 * per expert slice, src/moe.zig:368-390). FP8 and pack-quantized groups are
 * written decoded (bf16, config.json without quantization_config); float
 * tensors keep their dtype. export_dtype: DITCH_DTYPE_F32 / F16 / BF16 for
 * every float tensor (config.json's dtype / torch_dtype then name it), or -1.
 * Shards of at most max_shard_bytes (0 = 5 GiB) with
 * model.safetensors.index.json when there are several; tokenizer and side
 * files copied; a .incomplete marker exists until everything is written.
 * Tensor- or expert-parallel models and GGUF sources return
 * DITCH_CUDA_UNSUPPORTED. */
int ditch_cuda_export_checkpoint(ditch_cuda_model *m, const char *src_dir, const char *out_dir, int export_dtype,
                                 uint64_t max_shard_bytes);
/* The config.json text an export writes (no device): quantization_config and
 * expert_dtype removed when strip_quantization_config (dequant.zig:1195-1219),
 * float dtype names replaced by export_dtype's when it is not -1
 * (export.zig:239-283). out receives min(cap, *out_len) bytes. */
int ditch_cuda_export_config(const char *json, size_t len, int export_dtype, int strip_quantization_config, char *out,
                             size_t cap, size_t *out_len);
/* The delta the last edit left on a weight: component 0 = attention output,
 * 1 = MLP down, 2 = routed expert `expert`'s down projection. *rank = 0 when
 * the weight is not edited; else a [rank][cols] and b [rows][rank] (f32) are
 * filled (max_rank at least *rank). */
int ditch_cuda_model_delta(ditch_cuda_model *m, size_t layer, int component, size_t expert, float *a, float *b,
                           size_t max_rank, size_t *rank);
/* The export's rounding of f32 values (host buffers) to bf16
 * (src/tensor.zig:423-430) or IEEE f16 (round to nearest even). */
int ditch_cuda_round_f32(ditch_cuda_device *dev, const float *src, size_t n, int dtype, uint16_t *dst);

/* model.forward (src/model.zig:4619) with ForwardOptions (3136-3144): rows
 * {b, pos} per token (every prompt's rows contiguous, positions 0..len-1);
 * residuals [L+1][nc][H] for capture_rows (entry 0 = embedding, entry l =
 * output of layer l-1); logits [nl][V] for logit_rows. NULL outputs skip. */
int ditch_cuda_forward(ditch_cuda_model *m, const uint32_t *tokens, const uint32_t *row_b, const uint32_t *row_pos,
                       size_t n, const size_t *capture_rows, size_t nc, float *residuals, const size_t *logit_rows,
                       size_t nl, float *logits);

/* Greedy generation, model.generate (src/model.zig:5359-5444) with the cache
 * Engine.generateBatch sizes (src/engine.zig:254-260): one prefill of the
 * prompts (concatenated tokens, prompt_offsets[n_prompts + 1]) filling a
 * device KV cache, the first token from its logits, then one-row decode
 * steps over the prompts still active. A prompt stops after a token in
 * eos_ids (which is kept) or after max_new_tokens tokens; at least one token
 * is produced. Tokens go to out_tokens [n_prompts][max(max_new_tokens, 1)]
 * (row-major), their number per prompt to out_counts [n_prompts]. The
 * argmax keeps the first maximum (src/model.zig:5194-5204). The longest
 * prompt plus max_new_tokens must fit the positions the model was loaded
 * for. Under expert parallelism every rank of the group calls it at the same
 * time with its own prompts (at least one) and the same max_new_tokens: the
 * ranks agree before each decode step whether any rank still decodes, and a
 * rank whose prompts have finished runs that step on one placeholder row so
 * the MoE exchanges stay matched; the prefill's tokens must fit the group's
 * max_tokens. This is the device half of KeywordRate (src/scorers.zig:95-155);
 * detokenising and the keyword match stay on the host. */
int ditch_cuda_generate(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets, size_t n_prompts,
                        size_t max_new_tokens, const uint32_t *eos_ids, size_t n_eos, uint32_t *out_tokens,
                        size_t *out_counts);

/* engine.getResidualMeanObserved (src/engine.zig:314-438) without winsorising:
 * prompts given as concatenated tokens with prompt_offsets[n_prompts + 1];
 * the last `window` tokens of every prompt are averaged and summed in f64
 * into sums [L+1][H] (added to); *count += prompts seen. batch_size bounds
 * the prompts per forward (0 = all). */
int ditch_cuda_residual_sums(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets,
                             size_t n_prompts, size_t window, size_t batch_size, double *sums, uint64_t *count);

/* abliterate.computeDirections (src/abliterate.zig:88-109) from the f64 sums
 * of the good and bad passes; dirs [L+1][H] is returned and kept resident
 * for the edits. */
int ditch_cuda_directions(ditch_cuda_model *m, const double *good_sums, uint64_t good_count, const double *bad_sums,
                          uint64_t bad_count, int orthogonalize, float *dirs);
/* Uploads directions [entries][H] computed elsewhere. */
int ditch_cuda_set_directions(ditch_cuda_model *m, const float *dirs, size_t entries);

/* abliterate.Params (src/abliterate.zig:40-45). */
typedef struct {
    float max_weight, max_weight_position, min_weight, min_weight_distance;
} ditch_cuda_params;

/* abliterate.apply, row_normalization none (src/abliterate.zig:148-280): per
 * layer, lambda = kernelWeight(p, layer); v = dirs[layer + 1] or the
 * interpolated direction (direction_index >= 0, interpolateBasis :119-131);
 * A = v^T W, B = -lambda v on o_proj (attn_o) and down_proj (mlp_down; every
 * expert's down projection on an MoE layer, the broad edit). NULL params =
 * component untouched. The deltas act inside the GEMM epilogues; weights are
 * not modified. */
int ditch_cuda_apply_edit(ditch_cuda_model *m, const ditch_cuda_params *attn_o, const ditch_cuda_params *mlp_down,
                          float direction_index, int use_direction_index);
/* Options.row_normalization for the edits that follow (src/abliterate.zig:
 * 283-350): 0 none (the default); 1 pre, where a = (v / n)^T W and
 * b = -lambda v n with n the row norms ||W_i|| of the decoded weight (the
 * delta stays rank 1); 2 full, W' = diag(n) rownorm(Wn + B A^T), applied as a
 * rank-lora_rank delta (1..4, Options.lora_rank, default 3 in ditch) from a
 * randomised SVD of W' - W with 2 r + 4 sketch vectors and 6 power
 * iterations; the sketch of the k-th edited matrix is seeded with seed + k
 * (Options.seed) from this library's own generator, not ditch's, so the two
 * agree to the SVD's accuracy. Routed experts get one such delta per edited
 * expert, the k of its seed counted as on one device, so expert-parallel
 * ranks agree with a single GPU. On tensor-parallel ranks pre takes the row
 * norms over all ranks' column shards (a collective of the group: every rank
 * edits alike), and full runs the randomised SVD over the shards: the
 * products over columns summed over the group, the column vectors gathered
 * whole, the same sketch as one GPU (collectives of the group in every edit:
 * every rank applies the same edits in the same order). */
int ditch_cuda_set_row_normalization(ditch_cuda_model *m, int mode, size_t lora_rank, uint64_t seed);
/* moe.applyExpertSelective, ranked selection (src/moe.zig:1373-1477): the
 * o_proj edit as above, then per MoE layer the top n_experts experts by
 * ||v^T W_down|| / ||W_down||_F get lambda * strength. */
int ditch_cuda_apply_expert_edit(ditch_cuda_model *m, const ditch_cuda_params *attn_o, const ditch_cuda_params *mlp_down,
                                 float direction_index, int use_direction_index, size_t n_experts, float strength);
/* model.resetDeltas (src/model.zig:2348-2369). */
int ditch_cuda_reset_edits(ditch_cuda_model *m);
/* moe.scoreDown per routed expert of `layer` and rankScores (descending,
 * ties by index): order [E], scores [E] (either may be NULL). */
int ditch_cuda_rank_experts(ditch_cuda_model *m, size_t layer, const float *v, uint32_t *order, float *scores);

/* KlDivergence.init with kl_tokens = 1 (src/scorers.zig:311-369): the prompts
 * stay resident with the unedited model's first-token log-probabilities. */
int ditch_cuda_kl_init(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets, size_t n_prompts);
/* KlDivergence.score (src/scorers.zig:378-402) under the current edits on the
 * resident prompts: mean over prompts of sum_j exp(lb_j)(lb_j - lt_j), f64. */
int ditch_cuda_kl_score(ditch_cuda_model *m, double *kl);
/* Same, uploading the prompts from host memory in the call (they must be the
 * prompts given to ditch_cuda_kl_init). */
int ditch_cuda_kl_score_prompts(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets,
                                size_t n_prompts, double *kl);

/* The materialised rank-1 weight edit W <- W - alpha r (r^T W) on a bf16
 * matrix in device memory (GEMV-T then rank-1 update; the edited matrix of
 * src/abliterate.zig:544-552 rounded to bf16). r is a device f32 [rows].
 * w must be 2-byte and r 4-byte aligned (else DITCH_CUDA_INVALID); a w whose
 * rows are not all 16-byte aligned (a view at an odd storage offset, or cols
 * not a multiple of 8) is edited with 2-byte accesses, more slowly. */
int ditch_cuda_edit_weight_bf16(ditch_cuda_device *dev, void *w, size_t rows, size_t cols, const float *r,
                                float alpha);

/* The same edit for callers that cannot allocate device memory: a host
 * whose own pool owns HBM, code that must not synchronise the device (as
 * cudaMalloc / cudaFree can), or a caller without a ditch_cuda_device handle.
 * No counterpart in the reference: ditch's CPU engine has no device memory.
 *
 * The scratch (a = r^T W and b = -alpha r) is a fixed 512 KiB array inside
 * the library, held by every GPU that loads it until the process exits; the
 * call itself allocates nothing. Limit: rows <= 65536 and cols <= 65536
 * (larger sizes return DITCH_CUDA_INVALID). w and r are device pointers of
 * the current device, aligned as for ditch_cuda_edit_weight_bf16; the work is queued on `stream` (a cudaStream_t, NULL
 * for the default stream) and the call returns without waiting. The first
 * call on a device looks the array's device address up (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture.
 * All calls share the array and it keeps the last call's contents (the call
 * clears what must start at zero), so calls that overlap on the GPU race. */
int ditch_cuda_edit_weight_bf16_noalloc(void *w, size_t rows, size_t cols, const float *r, float alpha,
                                        void *stream);

/* ---- one resident weight and its dequant-fused GEMM ----
 * The product behind `matmulT` (src/tensor.zig:1023-1045) for one weight
 * kept in HBM in its stored format: FP8 blocks, MXFP4 and INT4 groups of 64k
 * are decoded inside the GEMM's operand load (src/dequant.zig:477-673
 * element rules); other formats are decoded to bf16 once at load. */
typedef struct ditch_cuda_weight ditch_cuda_weight;
int ditch_cuda_weight_load(ditch_cuda_device *dev, const ditch_cuda_tensor *t, ditch_cuda_weight **out);
void ditch_cuda_weight_free(ditch_cuda_weight *w);
/* 0 bf16, 1 FP8 block, 2 MXFP4, 3 INT4, 4 Q8_0 (how the GEMM reads the weight). */
int ditch_cuda_weight_format(const ditch_cuda_weight *w);
/* out[m][rows] f32 = x[m][cols] . W^T with x bf16; x and out are device
 * pointers, used in order on the device's own stream (asynchronous; that
 * stream does not wait for other streams, so x must be complete when the call
 * is made). k_splits > 1 splits K (partial sums added atomically; out is
 * zeroed first). */
int ditch_cuda_weight_gemm(ditch_cuda_weight *w, const void *x_bf16, size_t m, float *out, int k_splits);
/* The decoded weight [rows][cols] bf16 into device memory (asynchronous). */
int ditch_cuda_weight_decode(ditch_cuda_weight *w, uint16_t *out_bf16);
/* GEMM plan for FP8 / MXFP4 / INT4 weights (dense products; the routed-expert
 * grouped GEMM always decodes in the GEMM). A product over at least
 * `min_tokens` tokens decodes the weight once into device scratch as bf16 and
 * runs the bf16 GEMM; smaller ones decode tile by tile inside the GEMM. Both
 * plans build the same bf16 operand, so results are identical. 0 = always in
 * the GEMM. Default 1024. No counterpart in the reference (a tuning knob of
 * this backend). */
int ditch_cuda_set_decode_staging(ditch_cuda_device *dev, int min_tokens);
/* A staged GEMM keeps the bf16 copy of the weight it decoded and reuses it on
 * later calls (the resident weights never change; edits are separate deltas):
 * a trial loop then decodes each FP8 / MXFP4 / INT4 / Q8_0 weight once, like
 * ditch's own bf16 copies in mapped mode, at 2 bytes per element of device
 * memory (copies are made only while more than 4 GiB stays free). 0 decodes
 * into scratch on every call. Default on. Results are the same either way. */
int ditch_cuda_set_decode_cache(ditch_cuda_device *dev, int enabled);
/* Deterministic products. GEMMs with few output tiles split K over the SMs;
 * by default the splits add their partial sums with atomics, whose order
 * (and so the last bits of the result) varies from run to run. With
 * deterministic mode on, they run stream-K instead (each CTA takes an equal
 * share of the tile x k-tile work and a tile split between CTAs is summed in
 * k order by the CTA that brings its last part), and the 1..16-token product
 * adds its splits in order: the same inputs give the same bits on every run
 * and every GPU, at some cost in speed. A model joined to a tensor-parallel
 * group turns it on for its device (the ranks' replicated results must
 * agree bit for bit). Default off. No counterpart in the reference. */
int ditch_cuda_set_deterministic(ditch_cuda_device *dev, int enabled);
/* Dense bf16 GEMMs of at least 512 tokens and 256 weight rows (the products
 * of a prefill-sized forward, staged FP8 / MXFP4 / INT4 weights included) run
 * on CTA pairs: two SMs share each 256 x 256 output tile (tcgen05 with
 * cta_group::2), each loading half the weight rows and half the tokens, which
 * cuts the operand traffic per SM by a third. Level 0: never; 1: products
 * with one accumulator (qkv, o_proj, down_proj, LM head); 2: the SwiGLU
 * gate / up products too (256-token tiles, their two accumulators filling
 * TMEM; their epilogue runs on eight warps). The same products either way
 * (f32 accumulation of the same bf16 operands). Default 2 (measured on B200,
 * C2 trial at about 1.52 GHz: 108.5 ms at either level; the SwiGLU pair
 * tile moves a third less operand traffic per FLOP, 1.48 ms per launch
 * under ncu against 1.49 for one CTA per tile).
 * No counterpart in the reference (a tuning knob of this backend). */
int ditch_cuda_set_cta_pairs(ditch_cuda_device *dev, int level);
/* Prefill attention of batches whose prompts are all at most 128 tokens on
 * the tcgen05 tensor cores (Q.K^T and P.V with TMEM accumulators, head sizes
 * 64 and 128). Level 0: never (the mma.sync kernel); 1: one CTA per (prompt,
 * kv head) with the whole 128-row Q tile staged; 2: as 1, and prompts of at
 * most 64 tokens on a kernel that stages Q by 64-dim halves so that two CTAs
 * share each SM (one's loads overlap the other's products). Longer prompts, other head sizes and the f32-level
 * split mode use the mma.sync kernel. Every kernel splits the operands into
 * bf16 hi + lo and sums hi*hi + hi*lo + lo*hi in f32, so they agree to f32
 * rounding. Default 2. No counterpart in the reference (a tuning knob of
 * this backend). */
int ditch_cuda_set_attention_tc(ditch_cuda_device *dev, int level);
/* f32-level products for f32 and f16 weights. By default a resident model
 * rounds f32 / f16 weights to bf16 at load and rounds every GEMM input to
 * bf16 (tensor-core products with f32 accumulation), about 2^-9 relative per
 * operand. With this on, models loaded afterwards keep each dense weight W
 * as [hi | lo | hi] bf16 segments (hi = bf16(W), lo = bf16(W - hi)) and
 * every GEMM input x as [hi | hi | lo], so one bf16 GEMM over three times
 * the K adds hi.hi + hi.lo + lo.hi in f32: about 2^-16 relative per product,
 * the f32 engine's results to about 1e-5 (src/tensor.zig:1023-1045), at three
 * times the tensor-core work and 6 more bytes per weight. The edit deltas
 * read the same operand (A = v^T (hi + lo)) and the f32 activations; the
 * full-mode sketch products read the hi part. Dense models with f32 / f16 /
 * bf16 weights only (quantised weights, routed experts and tensor
 * parallelism are refused at load). Default off. No counterpart in the
 * reference, whose CPU engine multiplies in f32. */
int ditch_cuda_set_f32_split(ditch_cuda_device *dev, int enabled);

/* ---- peer groups and expert parallelism (one process per GPU of one node;
 * no counterpart in ditch, which runs on one host) ---- */
typedef struct ditch_cuda_group ditch_cuda_group;
/* Bytes of one rank's IPC handle; the host gathers `world` of them in rank
 * order and gives the array to ditch_cuda_group_open on every rank. */
size_t ditch_cuda_peer_handle_bytes(void);
/* Allocates this rank's region of a peer group (`bytes` of data after a flag
 * block) on the device and writes its IPC handle to `handle`. world <= 8. */
int ditch_cuda_group_create(ditch_cuda_device *dev, int rank, int world, size_t bytes, ditch_cuda_group **out,
                            void *handle);
/* Maps every peer's region (handles: world x handle bytes, rank order). */
int ditch_cuda_group_open(ditch_cuda_group *g, const void *handles);
void ditch_cuda_group_free(ditch_cuda_group *g);
/* A device-side barrier over the group (bounded: returns
 * DITCH_CUDA_DEVICE_FAILED when a peer does not arrive within the group's
 * wait budget). */
int ditch_cuda_group_barrier(ditch_cuda_group *g);
/* The budget of every wait of the group's exchanges (barrier, expert and
 * tensor-parallel layers, data-parallel reductions, the full-mode
 * collectives): 30 s by default, (0, 600]. A wait that runs out sets the
 * device's status word; the call returns DITCH_CUDA_DEVICE_FAILED, its
 * later waits return at once, and no result of the call is kept (cached
 * row norms included). The ranks' epochs then disagree: free the models
 * and the group on every rank and build them again. */
int ditch_cuda_group_set_wait_budget(ditch_cuda_group *g, double seconds);
/* Region bytes that a model loaded with ep_world > 1 or tp_world > 1 needs
 * for forwards of at most max_tokens tokens per rank (0 without either). */
size_t ditch_cuda_model_group_bytes(const ditch_cuda_model *m, size_t max_tokens);
/* Tensor parallel (tp_world > 1): every rank runs the same tokens on its
 * shard of the attention heads and MLP columns, and the o_proj / down_proj
 * partial sums are all-reduced over the group (rank-ordered sums read over
 * NVLink), so every rank holds the same residual stream and logits.
 * Expert parallel (ep_world > 1): runs the model's routed-expert layers over the group: each
 * rank routes its own tokens, sends every (token, expert) row to the expert's
 * owner over NVLink, runs its experts' grouped GEMMs on every rank's rows and
 * returns the outputs; the combine then equals the single-GPU one bit for
 * bit. Expert scoring gathers every rank's scores, so the selective edit picks
 * the same experts on all ranks. Every rank must make the same calls in the
 * same order (forward, residual sums, edits, KL). */
int ditch_cuda_model_set_group(ditch_cuda_model *m, ditch_cuda_group *g, size_t max_tokens);
/* Data parallel (the prompt batches of src/engine.zig:383-435 split over the
 * ranks, every rank holding the same weights and making the same edits):
 * once a model has a data-parallel group, ditch_cuda_residual_sums returns
 * the sums and the prompt count of every rank's prompts (each call's sums
 * added over the ranks, in rank order), and ditch_cuda_kl_score /
 * ditch_cuda_kl_score_prompts return the mean KL over every rank's prompts,
 * the per-prompt values added in rank order and then prompt order, as
 * src/scorers.zig:385-400 adds them for the concatenated prompts. The sums
 * run on the device over NVLink (one exchange each); every rank gets the same
 * bits. Every rank must make the same calls in the same order. The group must
 * not be the model's tensor- or expert-parallel group; its region needs
 * ditch_cuda_model_dp_group_bytes(m, most prompts per KL call) bytes. NULL
 * detaches it. Replaces the host's own loops over prompt batches
 * (src/engine.zig:314-438) and prompts (src/scorers.zig:378-402) when the
 * prompts are spread over GPUs; no counterpart in the reference. */
size_t ditch_cuda_model_dp_group_bytes(const ditch_cuda_model *m, size_t max_prompts);
int ditch_cuda_model_set_dp_group(ditch_cuda_model *m, ditch_cuda_group *g);
/* data[i] <- the sum over the group's ranks of data[i] (host f64 arrays, n
 * values; added in rank order on the device, the same bits on every rank): a
 * host-side counter or score summed over the ranks (a refusal count of
 * src/scorers.zig:95-155, for instance). Every rank calls it with the same n. */
int ditch_cuda_group_allreduce_f64(ditch_cuda_group *g, double *data, size_t n);

/* ---- timing support (CUDA events on the device's stream) ---- */
/* Accumulated device time and launch count of the weight GEMMs since the
 * last reset (when enabled), for roofline reporting. */
int ditch_cuda_set_profiling(ditch_cuda_device *dev, int enabled);
int ditch_cuda_gemm_stats(ditch_cuda_device *dev, double *ms, uint64_t *launches, double *flops);
int ditch_cuda_reset_stats(ditch_cuda_device *dev);
/* Number of kernels this library launched since the last reset. */
uint64_t ditch_cuda_launches(const ditch_cuda_device *dev);
/* Records an event pair around work issued between start and stop. */
int ditch_cuda_timer_start(ditch_cuda_device *dev);
int ditch_cuda_timer_stop(ditch_cuda_device *dev, float *ms);
int ditch_cuda_synchronize(ditch_cuda_device *dev);

#ifdef __cplusplus
}
#endif
#endif
