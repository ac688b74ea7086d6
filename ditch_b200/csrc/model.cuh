// The resident model: weights in HBM in their GEMM-ready storage, the
// forward's workspace, the per-layer rank-1 edits, the refusal directions and
// the KL prompts with their baseline log-probabilities.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "device.cuh"
#include "peer.cuh"

namespace ditch {

// A weight matrix (or a stack of `slabs` expert matrices) in the storage the
// GEMM reads: bf16, or a quantised format decoded inside the GEMM.
struct Mat {
    int fmt = kFmtBf16;
    int rows = 0, cols = 0, slabs = 1;  // rows per slab
    long long row_bytes = 0;
    DevBuf data;    // bf16 [slabs*rows][cols] | E4M3 codes | MXFP4 nibbles | INT4 words
    DevBuf scales;  // FP8 f32 [slabs*srows][scols] | MXFP4 u8 [slabs*rows][cols/32] | INT4 f32 [slabs*rows][groups]
    DevBuf zeros;   // INT4 packed zero points [slabs*rows/8][groups]
    int br = 0, bc = 0, scols = 0, groups = 0, group = 0;
    // Rows [decoded_row0, decoded_row0 + decoded_rows) decoded to bf16 by a
    // staged GEMM and kept (the weights never change: edits are deltas).
    mutable DevBuf decoded;
    mutable int decoded_row0 = -1, decoded_rows = 0;
    // f32-level products (a model loaded in split mode): the weight as
    // [hi | lo | hi] bf16 segments of split_k columns each, [rows][3 split_k],
    // the operand the GEMM reads; `data` keeps the hi part for the rest
    DevBuf split;
    int split_k = 0;
    bool empty() const { return data.ptr == nullptr; }
    size_t bytes() const { return data.bytes + scales.bytes + zeros.bytes; }
};

struct Layer {
    DevBuf input_norm, post_norm, q_norm, k_norm;  // f32
    Mat qkv;                                       // [qd + 2 kvd][H]
    DevBuf qkv_bias;                               // f32 [qd + 2 kvd] or empty
    Mat o;                                         // [H][qd]
    Mat gate_up;                                   // [2 I][H]: gate rows then up rows
    Mat down;                                      // [H][I]
    bool moe = false;
    Mat router;                                    // [E][H] (bf16)
    Mat router3;                                   // [E][3 cp]: split-bf16 [hi | lo | hi] of the router
    Mat e_gate_up;                                 // [E][2 mi][H]: per expert gate rows then up rows
    Mat e_down;                                    // [E][H][mi]
    // none-mode deltas (src/abliterate.zig:270-280): out += (x . a) b
    bool o_edit = false, down_edit = false;
    int o_rank = 1, down_rank = 1;                 // terms of the delta (full row normalisation: up to kMaxDeltaRank)
    DevBuf o_a, o_b, down_a, down_b;               // f32 [rank][qd], [H][rank], [rank][I], [H][rank]
    std::vector<uint8_t> e_edit;                   // per expert
    std::vector<float> e_fro;                      // ||W_down_e||_F per expert (computed once)
    DevBuf e_proj;                                 // f32 [E][mi]: v^T W_down_e of the last scoring
    int e_rank = 1;                                // terms of the expert deltas (full row normalisation: up to kMaxDeltaRank)
    DevBuf e_a, e_b;                               // f32 [E][e_rank][mi], [E][H][e_rank]
    DevBuf e_edit_dev;                             // int [E]
    // row norms ||W_i|| for the pre-normalised edit (computed once; the base weights never change)
    DevBuf o_rn, down_rn, e_rn;                    // f32 [H], [H], [E][H]
    // rn_pending: computed by the call in progress; rn_valid: by a call whose
    // device status came back clean (only then are they reused)
    bool rn_pending = false, rn_valid = false;
};

struct Config {
    int n_layers, hidden, heads, kv_heads, head_dim, inter, vocab;
    float eps;
    double rope_theta;
    int rope_scaling;
    double rope_factor, rope_low_ff, rope_high_ff, rope_orig_max;
    std::vector<float> rope_factors;  // per-frequency divisors (rope_scaling 4)
    double rope_attention_factor = 1.0, rope_beta_fast = 32.0, rope_beta_slow = 1.0;
    int rope_truncate = 1;
    int qk_norm;
    int n_experts, top_k, moe_inter, norm_topk;
    std::vector<uint8_t> moe_layers;
    int max_seq;
    int ep_rank = 0, ep_world = 1;  // expert parallelism: this rank's routed experts are [e0, e0 + e_loc)
    int e_loc = 0, e0 = 0;
    int tp_rank = 0, tp_world = 1;  // tensor parallelism: heads, kv_heads and inter above are this rank's
    int qd() const { return heads * head_dim; }
    int kvd() const { return kv_heads * head_dim; }
    int qkv_width() const { return qd() + 2 * kvd(); }
};

// One flattened batch of prompts on the device.
struct Batch {
    int n = 0, prompts = 0;
    DevBuf tokens, seq_start, seq_len, cap_slot, logit_rows;
    DevBuf row_b, row_pos;  // per row: KV-cache slot and position (generation only)
    std::vector<int> h_start, h_len;
};

// What a forward does with the KV cache: nothing (prompts attend within the
// call), store the prompts' keys and values (a generation's prefill), or run
// single-token rows against the cache (a decode step).
enum FwdMode { kFwdPrompts = 0, kFwdPromptsCache = 1, kFwdDecode = 2 };

}  // namespace ditch

struct ditch_cuda_model {
    ditch_cuda_device *dev = nullptr;
    ditch::Config cfg;
    ditch::DevBuf embed;
    bool embed_bf16 = true;
    ditch::DevBuf final_norm;
    ditch::Mat lm_head;
    std::vector<ditch::Layer> layers;
    ditch::DevBuf rope_cos, rope_sin;
    int rope_len = 0;
    // workspace
    int ws_tokens = 0;
    ditch::DevBuf x, h, qkv, att, act, xa;
    // split mode (f32-level products for f32 / f16 weights): h, att, act and
    // hl hold [hi | hi | lo] operand rows; att32 / gu32 / act32 the f32 values
    bool split3 = false;
    ditch::DevBuf att32, gu32, act32;
    ditch::DevBuf res, hl, logits;
    // MoE workspace
    ditch::DevBuf moe_h3, moe_logits, moe_sel, moe_w, moe_counts, moe_offsets, moe_perm, moe_pw, moe_pexp, moe_slot,
        moe_xg, moe_act, moe_eo, moe_xa, moe_sched_gu, moe_sched_d, moe_nsched, moe_cc;
    // directions
    ditch::DevBuf dirs;
    std::vector<float> h_dirs;
    int dir_entries = 0;
    ditch::DevBuf vtmp;  // interpolated direction
    ditch::DevBuf gemv_part;  // partial sums of the deterministic GEMV-T
    // KL prompts
    ditch::Batch kl;
    ditch::DevBuf kl_base, kl_vals, kl_part;  // kl_part: the row pieces' log-sum-exp and KL sums
    bool kl_ready = false;
    std::vector<size_t> kl_offsets;
    std::vector<uint32_t> kl_tokens_host;
    // data parallelism: residual sums and KL combined over this group's ranks
    ditch_cuda_group *dp_group = nullptr;
    ditch::DevBuf dp_buf;  // f64 [2] reduced KL sum and count / [1 + entries * H] sums to reduce
    // expert parallelism: the peer group and this rank's receive-side scratch
    ditch_cuda_group *group = nullptr;
    size_t group_tokens = 0;  // most tokens per rank per forward
    ditch::DevBuf ep_dst, ep_rcnt, ep_roff, ep_pexp, ep_act, ep_eo, ep_xa, ep_sched_gu, ep_sched_d, ep_nsched,
        ep_scores;
    int ep_score_parity = 0;
    // greedy generation: KV cache f32 [layers][slots][kv_len][kvd] for keys and for values
    ditch::DevBuf kv_k, kv_v, gen_next;
    int kv_slots = 0, kv_len = 0;
    int row_norm = 0;    // edit row normalisation: 0 none, 1 pre, 2 full (src/abliterate.zig:283-350)
    int lora_rank = 3;   // full: rank of the delta (Options.lora_rank)
    uint64_t edit_seed = 0, seed_counter = 0;  // full: the sketch seed of each matrix is seed + its index
    ditch::DevBuf vn;    // f32 [H]: v / ||W_i|| of the pre-normalised edit
    ditch::DevBuf fn_act, fn_out, fn_y, fn_x, fn_a, fn_s;  // full-mode scratch
    ditch::DevBuf fn_red;                                  // full mode under TP: the group reductions' f64 values
    ditch::Batch work;   // scratch batch for forward / residual passes
    ditch::DevBuf sums;       // f64 residual sums
    ditch::DevBuf sums_part;  // the prompt runs' partial sums of one batch
    uint64_t bytes = 0;
};

namespace ditch {

// Builds a device batch from flattened prompts (tokens + offsets); capture
// rows = the last `window` tokens of every prompt (window 0 = none); logit
// rows = each prompt's last token when `logits` is set.
int make_batch(ditch_cuda_model *m, Batch &b, const uint32_t *tokens, const size_t *offsets, size_t n_prompts,
               size_t window, bool logits, std::vector<int> *first_capture, std::vector<int> *take);

// The forward over a device batch: residual capture into m->res ([L+1][nc][H])
// when nc > 0, logits of the batch's logit rows into m->logits when nl > 0.
// `mode` (FwdMode) says how attention uses the KV cache (b.row_b / b.row_pos
// and m->kv_* must be set for the cache modes).
int forward_batch(ditch_cuda_model *m, Batch &b, int nc, int nl, int mode = kFwdPrompts);

int ensure_workspace(ditch_cuda_model *m, int n_tokens, int nc, int nl);

// out[cols] = v^T W over rows [row0, row0 + rows) of a resident weight in its
// stored format (v device f32 [rows]); out is overwritten.
int gemv_t_mat(ditch_cuda_model *m, const Mat &w, int row0, int rows, const float *v, float *out);

// row_normalization = full (src/abliterate.zig:324-350): the rank-`*rank_out`
// delta (a_out [rank][cols], b_out [rows][rank], device) of the H-row weight
// at row0 for direction v (device f32 [H]) with row norms rn (device).
int full_norm_delta(ditch_cuda_model *m, const Mat &w, int row0, const float *rn, const float *v_dev, float lambda,
                    int lora_rank, uint64_t seed, float *a_out, float *b_out, int *rank_out);

// Rows [row0, row0 + rows) of a weight decoded to the bf16 operand the GEMM
// sees (quantised formats), and their row norms ||W_i|| in f32.
cudaError_t decode_rows_bf16(ditch_cuda_device *dev, const Mat &w, int row0, int rows, uint16_t *out);
int mat_row_norms(ditch_cuda_device *dev, const Mat &w, int row0, int rows, float *out);

// MoE MLP of layer `li`: post-norm of x, routing, experts, combine into x.
int moe_mlp(ditch_cuda_model *m, Layer &L, int li, int n);

// Tensor parallelism: region bytes per rank, this rank's send rows (where the
// row-parallel GEMMs write their partial sums) and the all-reduce that adds
// the summed partials of the first n rows into x.
size_t tp_group_bytes(const Config &c, size_t max_tokens);
float *tp_send_rows(ditch_cuda_model *m);
int tp_allreduce_add(ditch_cuda_model *m, int n, float *x);
int tp_row_norms(ditch_cuda_model *m, const Mat &w, float *out);

// Expert scores of this rank's routed experts (`local` [e_loc]) gathered from
// every rank of the model's peer group into `all` [n_experts].
int ep_allgather_scores(ditch_cuda_model *m, const std::vector<float> &local, std::vector<float> &all);
// Whether any rank of the model's expert-parallel group still has prompts to
// decode (one exchange; every rank calls it at the same step).
int ep_any_active(ditch_cuda_model *m, size_t local_active, bool *any);

// The split-bf16 router operand from f32 router weights [E][hidden] (device).
int build_router_split(ditch_cuda_device *dev, const float *router_f32, int E, int hidden, Mat &out);

// GEMM with a resident weight as the A operand.
int gemm_weight(ditch_cuda_model *m, const Mat &w, int slab_row0, int m_rows, const uint16_t *act, int n_tok,
                void *out, long long ldo, int flags, const float *bias, const float *xa, const float *db,
                int a2_row_offset, int delta_rank = 1);

// Options beyond the dense single-matrix product: split-K, or the grouped
// (per-expert) tile schedule of the routed-expert path.
struct GemmExtra {
    int k_splits = 1;
    const int4 *sched = nullptr;
    const int *n_sched = nullptr;
    int slab_rows = 0;
    const int *e_flags = nullptr;
    long long db_stride = 0;
    int bn = 0;
};

// A routed-expert stack in a quantised format (MXFP4, FP8, INT4) decoded once
// to bf16 and kept (while the decode cache is on, staging is not off and
// more than 4 GiB stays free): grouped products then run the bf16 GEMM over
// the copy, as ditch holds its experts (decoded at load, src/dequant.zig).
// Returns whether the copy exists (decoding it on first use).
bool expert_stack_cached(ditch_cuda_device *dev, const Mat &w);

int gemm_mat(ditch_cuda_device *dev, const Mat &w, int slab_row0, int m_rows, const uint16_t *act, int n_tok,
             void *out, long long ldo, int flags, const float *bias, const float *xa, const float *db,
             int a2_row_offset, const GemmExtra *ex, int delta_rank = 1);

// Builds a GEMM operand from one tensor of the C ABI (quantised formats the
// GEMM decodes stay quantised; others are decoded to bf16 once).
int build_weight(ditch_cuda_device *dev, const ditch_cuda_tensor *t, Mat &out);

}  // namespace ditch
