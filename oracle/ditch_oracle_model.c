/* CPU restatement of ditch's batched forward (src/model.zig, src/moe.zig), the
 * none-mode edit (src/abliterate.zig), residual capture (src/engine.zig) and
 * the KL scorer (src/scorers.zig). TEST INFRASTRUCTURE only. */
#include "ditch_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* `axpy` (src/tensor.zig:561-570): y += alpha * x, unfused. */
static void axpy(float *y, float alpha, const float *x, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] = y[i] + alpha * x[i];
}

static void add_bias(float *buf, size_t n, size_t width, const float *b) {
    if (!b) return;
    for (size_t i = 0; i < n; i++) axpy(buf + i * width, 1.0f, b, width);
}

/* attentionScores / attentionValues (src/tensor.zig:1126-1160) for a
 * vectorised head (hd % 16 == 0), else the scalar path of attentionWorker
 * (src/model.zig:2935-2986). */
static void attend(const float *q, const float *kbase, const float *vbase, size_t stride,
                   size_t n_keys, size_t hd, float scale, float *scores, float *out) {
    int vec = hd % 16 == 0;
    for (size_t p = 0; p < n_keys; p++) {
        if (vec) {
            /* per key: VL-lane FMA accumulation then an ordered reduction */
            scores[p] = or_dot(q, kbase + p * stride, hd) * scale;
        } else {
            scores[p] = or_dot(q, kbase + p * stride, hd) * scale;
        }
    }
    or_softmax_inplace(scores, n_keys);
    if (vec) {
        for (size_t j = 0; j < hd; j += 16) {
            float a[4][16];
            memset(a, 0, sizeof a);
            size_t p = 0;
            for (; p + 4 <= n_keys; p += 4)
                for (int kk = 0; kk < 4; kk++)
                    for (int l = 0; l < 16; l++)
                        a[kk][l] = fmaf(vbase[(p + kk) * stride + j + l], scores[p + kk], a[kk][l]);
            for (; p < n_keys; p++)
                for (int l = 0; l < 16; l++) a[0][l] = fmaf(vbase[p * stride + j + l], scores[p], a[0][l]);
            for (int l = 0; l < 16; l++) out[j + l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
        }
    } else {
        memset(out, 0, sizeof(float) * hd);
        for (size_t p = 0; p < n_keys; p++) axpy(out, scores[p], vbase + p * stride, hd);
    }
}

/* topk (src/moe.zig:971-985): the first maximum wins ties. */
/* A weight product: f32 weights, or (m->w_bf16) bf16 bit arrays through
 * ditch's half-precision path; `off` elements into the weight (expert slabs). */
static void mm(const or_model *m, float *out, const float *x, size_t n, const float *w, size_t off, size_t rows,
               size_t cols, const float *da, const float *db, size_t rank) {
    if (m->w_bf16)
        or_matmul_t_bf16(out, x, n, (const uint16_t *)(const void *)w + off, rows, cols, da, db, rank);
    else
        or_matmul_t(out, x, n, w + off, rows, cols, da, db, rank);
}

static void topk(const float *scores, float *sel, size_t ne, size_t k, size_t *idx, float *wts) {
    for (size_t j = 0; j < k; j++) {
        size_t best = 0;
        float bv = -INFINITY;
        for (size_t e = 0; e < ne; e++)
            if (sel[e] > bv) { bv = sel[e]; best = e; }
        idx[j] = best;
        wts[j] = scores[best];
        sel[best] = -INFINITY;
    }
}

/* moe.forward softmax / top-k / index-order union path (src/moe.zig:998-1228). */
static void moe_forward(const or_model *m, const or_layer *L, const float *h, size_t n, float *out) {
    const or_config *c = &m->c;
    size_t H = (size_t)c->hidden, E = (size_t)c->n_experts, k = (size_t)c->top_k, mi = (size_t)c->moe_inter;
    float *logits = malloc(sizeof(float) * n * E);
    mm(m, logits, h, n, L->router, 0, E, H, NULL, NULL, 0);
    size_t *sel = malloc(sizeof(size_t) * n * k);
    float *selw = malloc(sizeof(float) * n * k), *choice = malloc(sizeof(float) * E);
    for (size_t t = 0; t < n; t++) {
        float *row = logits + t * E;
        or_softmax_inplace(row, E);
        for (size_t e = 0; e < E; e++) choice[e] = row[e];
        topk(row, choice, E, k, sel + t * k, selw + t * k);
        float sum = 0;
        for (size_t j = 0; j < k; j++) sum += selw[t * k + j];
        if (c->norm_topk && sum > 0)
            for (size_t j = 0; j < k; j++) selw[t * k + j] /= sum;
    }
    memset(out, 0, sizeof(float) * n * H);
    float *xg = malloc(sizeof(float) * n * H), *g = malloc(sizeof(float) * n * mi);
    float *u = malloc(sizeof(float) * n * mi), *eo = malloc(sizeof(float) * n * H);
    size_t *tok = malloc(sizeof(size_t) * n);
    float *w = malloc(sizeof(float) * n);
    for (size_t e = 0; e < E; e++) {
        size_t ne = 0;
        for (size_t t = 0; t < n; t++)
            for (size_t j = 0; j < k; j++)
                if (sel[t * k + j] == e) { tok[ne] = t; w[ne] = selw[t * k + j]; ne++; }
        if (ne == 0) continue;
        for (size_t j = 0; j < ne; j++) memcpy(xg + j * H, h + tok[j] * H, sizeof(float) * H);
        mm(m, g, xg, ne, L->e_gate, e * mi * H, mi, H, NULL, NULL, 0);
        mm(m, u, xg, ne, L->e_up, e * mi * H, mi, H, NULL, NULL, 0);
        or_gated_silu(g, g, u, ne, mi, mi, mi);
        const float *da = L->e_down_da ? L->e_down_da[e] : NULL;
        const float *db = L->e_down_db ? L->e_down_db[e] : NULL;
        const size_t dr = L->e_down_rank ? L->e_down_rank[e] : 1;
        mm(m, eo, g, ne, L->e_down, e * H * mi, H, mi, da, db, da && db ? dr : 0);
        for (size_t j = 0; j < ne; j++) axpy(out + tok[j] * H, w[j], eo + j * H, H);
    }
    free(logits); free(sel); free(selw); free(choice); free(xg); free(g); free(u); free(eo);
    free(tok); free(w);
}

/* forward (src/model.zig:4619-4853) with layerBlock (4880-4959), attention
 * (4147-4219), attentionTail (4226-4374) and mlpBlock (4430-4486) for the
 * Llama / Qwen2 / Qwen3 / Qwen3-MoE layout. */
int or_forward(const or_model *m, const uint32_t *tokens, const uint32_t *row_b,
               const uint32_t *row_pos, size_t n, const size_t *capture_rows, size_t nc,
               float *residuals, const size_t *logit_rows, size_t nl, float *logits) {
    const or_config *c = &m->c;
    size_t H = (size_t)c->hidden, hd = (size_t)c->head_dim, nh = (size_t)c->heads, nkv = (size_t)c->kv_heads;
    size_t qd = nh * hd, kvd = nkv * hd, I = (size_t)c->inter, V = (size_t)c->vocab;
    size_t B = 0, maxp = 0;
    for (size_t i = 0; i < n; i++) {
        if (row_b[i] + 1 > B) B = row_b[i] + 1;
        if (row_pos[i] + 1 > maxp) maxp = row_pos[i] + 1;
    }
    float *x = malloc(sizeof(float) * n * H), *h = malloc(sizeof(float) * n * H);
    float *q = malloc(sizeof(float) * n * qd), *kk = malloc(sizeof(float) * n * kvd);
    float *vv = malloc(sizeof(float) * n * kvd), *att = malloc(sizeof(float) * n * qd);
    float *o = malloc(sizeof(float) * n * H);
    size_t mw = I > (size_t)c->moe_inter ? I : (size_t)c->moe_inter;
    float *gate = malloc(sizeof(float) * n * (mw ? mw : 1)), *up = malloc(sizeof(float) * n * (mw ? mw : 1));
    float *mo = malloc(sizeof(float) * n * H);
    float *kc = malloc(sizeof(float) * B * maxp * kvd), *vc = malloc(sizeof(float) * B * maxp * kvd);
    float *cos_t = malloc(sizeof(float) * maxp * hd / 2), *sin_t = malloc(sizeof(float) * maxp * hd / 2);
    {
        or_rope r = {c->rope_scaling, c->rope_factor, c->rope_low_ff, c->rope_high_ff, c->rope_orig_max,
                     c->rope_factors, c->n_rope_factors,
                     c->rope_attention_factor != 0 ? c->rope_attention_factor : 1.0, c->rope_beta_fast,
                     c->rope_beta_slow, c->rope_truncate};
        or_rope_table_ex(cos_t, sin_t, maxp, hd, c->rope_theta, &r);
    }
    float scale = 1.0f / sqrtf((float)hd);

    for (size_t i = 0; i < n; i++) {
        if (tokens[i] >= V) return -1; /* embedRowIndex: out of range is an error */
        for (size_t j = 0; j < H; j++) x[i * H + j] = m->embed[(size_t)tokens[i] * H + j];
    }
    if (residuals)
        for (size_t ci = 0; ci < nc; ci++) memcpy(residuals + ci * H, x + capture_rows[ci] * H, sizeof(float) * H);

    for (int li = 0; li < c->n_layers; li++) {
        const or_layer *L = &m->layers[li];
        for (size_t i = 0; i < n; i++) or_rmsnorm(h + i * H, x + i * H, L->input_norm, H, c->eps);
        mm(m, q, h, n, L->q, 0, qd, H, NULL, NULL, 0);
        add_bias(q, n, qd, L->qb);
        mm(m, kk, h, n, L->k, 0, kvd, H, NULL, NULL, 0);
        mm(m, vv, h, n, L->v, 0, kvd, H, NULL, NULL, 0);
        add_bias(kk, n, kvd, L->kb);
        add_bias(vv, n, kvd, L->vb);
        for (size_t i = 0; i < n; i++) {
            size_t pos = row_pos[i];
            const float *cr = cos_t + pos * hd / 2, *sr = sin_t + pos * hd / 2;
            for (size_t hh = 0; hh < nh; hh++) {
                float *qh = q + i * qd + hh * hd;
                if (c->qk_norm && L->q_norm) or_rmsnorm(qh, qh, L->q_norm, hd, c->eps);
                or_apply_rope(qh, cr, sr, hd);
            }
            for (size_t hh = 0; hh < nkv; hh++) {
                float *kh = kk + i * kvd + hh * hd;
                if (c->qk_norm && L->k_norm) or_rmsnorm(kh, kh, L->k_norm, hd, c->eps);
                or_apply_rope(kh, cr, sr, hd);
            }
            memcpy(kc + ((size_t)row_b[i] * maxp + pos) * kvd, kk + i * kvd, sizeof(float) * kvd);
            memcpy(vc + ((size_t)row_b[i] * maxp + pos) * kvd, vv + i * kvd, sizeof(float) * kvd);
        }
#pragma omp parallel num_threads(or_get_threads())
        {
            float *scores = malloc(sizeof(float) * maxp);
#pragma omp for schedule(dynamic)
            for (long t = 0; t < (long)(n * nh); t++) {
                size_t i = (size_t)t / nh, hh = (size_t)t % nh, kvh = hh / (nh / nkv);
                size_t pos = row_pos[i], b = row_b[i];
                attend(q + i * qd + hh * hd, kc + b * maxp * kvd + kvh * hd, vc + b * maxp * kvd + kvh * hd,
                       kvd, pos + 1, hd, scale, scores, att + i * qd + hh * hd);
            }
            free(scores);
        }
        mm(m, o, att, n, L->o, 0, H, qd, L->o_da, L->o_db, L->o_rank);
        for (size_t i = 0; i < n; i++) axpy(x + i * H, 1.0f, o + i * H, H);
        for (size_t i = 0; i < n; i++) or_rmsnorm(h + i * H, x + i * H, L->post_norm, H, c->eps);
        if (L->router) {
            moe_forward(m, L, h, n, mo);
        } else {
            mm(m, gate, h, n, L->gate, 0, I, H, NULL, NULL, 0);
            mm(m, up, h, n, L->up, 0, I, H, NULL, NULL, 0);
            or_gated_silu(gate, gate, up, n, I, I, I);
            mm(m, mo, gate, n, L->down, 0, H, I, L->down_da, L->down_db, L->down_rank);
        }
        for (size_t i = 0; i < n; i++) axpy(x + i * H, 1.0f, mo + i * H, H);
        if (residuals)
            for (size_t ci = 0; ci < nc; ci++)
                memcpy(residuals + ((size_t)(li + 1) * nc + ci) * H, x + capture_rows[ci] * H, sizeof(float) * H);
    }
    if (nl > 0 && logits) {
        float *hl = malloc(sizeof(float) * nl * H);
        for (size_t i = 0; i < nl; i++) or_rmsnorm(hl + i * H, x + logit_rows[i] * H, m->final_norm, H, c->eps);
        mm(m, logits, hl, nl, m->lm_head, 0, V, H, NULL, NULL, 0);
        free(hl);
    }
    free(x); free(h); free(q); free(kk); free(vv); free(att); free(o); free(gate); free(up);
    free(mo); free(kc); free(vc); free(cos_t); free(sin_t);
    return 0;
}

/* ---- abliteration: src/abliterate.zig ---- */

/* kernelWeight: src/abliterate.zig:134-140 */
int or_kernel_weight(or_params p, size_t layer, float *out) {
    float distance = fabsf((float)layer - p.max_weight_position);
    if (distance > p.min_weight_distance) return 0;
    float w = p.max_weight + (distance / p.min_weight_distance) * (p.min_weight - p.max_weight);
    if (w == 0) return 0;
    *out = w;
    return 1;
}

static void normalize(float *x, size_t n) {
    float nr = sqrtf(or_dot(x, x, n));
    if (nr > 1e-12f) {
        float s = 1.0f / nr;
        for (size_t i = 0; i < n; i++) x[i] *= s;
    }
}

/* computeDirections: src/abliterate.zig:88-109 */
void or_compute_directions(const float *good, const float *bad, size_t entries, size_t hidden,
                           int orthogonalize, float *dirs) {
    float *gd = malloc(sizeof(float) * hidden);
    for (size_t e = 0; e < entries; e++) {
        float *d = dirs + e * hidden;
        const float *g = good + e * hidden, *b = bad + e * hidden;
        for (size_t i = 0; i < hidden; i++) d[i] = b[i] - g[i];
        normalize(d, hidden);
        if (orthogonalize) {
            memcpy(gd, g, sizeof(float) * hidden);
            normalize(gd, hidden);
            float proj = or_dot(d, gd, hidden);
            axpy(d, -proj, gd, hidden);
            normalize(d, hidden);
        }
    }
    free(gd);
}

/* computeOutputDelta, row_normalization none: src/abliterate.zig:270-280 */
void or_compute_delta_none(const float *w, size_t rows, size_t cols, const float *v,
                           float lambda, float *a, float *b) {
    or_matvec_t_multi(a, w, rows, cols, v, 1);
    for (size_t i = 0; i < rows; i++) b[i] = -lambda * v[i];
}

/* materialize (test helper): src/abliterate.zig:544-552 */
void or_materialize(const float *w, size_t rows, size_t cols, const float *a, const float *b,
                    size_t rank, float *out) {
    for (size_t i = 0; i < rows; i++)
        for (size_t j = 0; j < cols; j++) {
            float acc = 0;
            for (size_t k = 0; k < rank; k++) acc += b[i * rank + k] * a[k * cols + j];
            out[i * cols + j] = w[i * cols + j] + acc;
        }
}

/* scoreDown: src/moe.zig:1239-1250 */
float or_score_down(const float *w, size_t rows, size_t cols, const float *v) {
    float *proj = malloc(sizeof(float) * cols), *norms = malloc(sizeof(float) * rows);
    or_matvec_t_multi(proj, w, rows, cols, v, 1);
    or_row_norms(norms, w, rows, cols);
    float fro = sqrtf(or_dot(norms, norms, rows));
    float r = fro > 0 ? sqrtf(or_dot(proj, proj, cols)) / fro : 0;
    free(proj);
    free(norms);
    return r;
}

/* rankScores: descending, ties by index (src/moe.zig:1296-1306) */
void or_rank_scores(const float *s, size_t n, uint32_t *order) {
    for (size_t i = 0; i < n; i++) order[i] = (uint32_t)i;
    for (size_t i = 1; i < n; i++) { /* stable insertion sort */
        uint32_t cur = order[i];
        size_t j = i;
        while (j > 0) {
            uint32_t p = order[j - 1];
            int before = s[cur] != s[p] ? s[cur] > s[p] : cur < p;
            if (!before) break;
            order[j] = p;
            j--;
        }
        order[j] = cur;
    }
}

/* ---- engine and scorers ---- */

/* forEachResidual + Acc.add (src/engine.zig:314-336, 414-431), no winsorising
 * (the default quantile 1.0 disables it, src/config.zig:169). */
void or_residual_sums(const float *res, size_t entries, size_t nc, size_t hidden,
                      const size_t *first_capture, const size_t *take, size_t prompts,
                      double *sums) {
    float *v = malloc(sizeof(float) * hidden);
    for (size_t b = 0; b < prompts; b++) {
        size_t tk = take[b];
        float inv = 1.0f / (float)(tk > 0 ? tk : 1);
        for (size_t l = 0; l < entries; l++) {
            memset(v, 0, sizeof(float) * hidden);
            for (size_t t = 0; t < tk; t++) axpy(v, inv, res + (l * nc + first_capture[b] + t) * hidden, hidden);
            for (size_t i = 0; i < hidden; i++) sums[l * hidden + i] += v[i];
        }
    }
    free(v);
}

/* KlDivergence.score with kl_tokens = 1: src/scorers.zig:378-402 */
double or_kl_first_token(const float *base, const float *logits, size_t prompts, size_t vocab,
                         double *per_prompt) {
    double total = 0;
#pragma omp parallel for reduction(+ : total) schedule(static) num_threads(or_get_threads())
    for (long p = 0; p < (long)prompts; p++) {
        float *tmp = malloc(sizeof(float) * vocab);
        or_log_softmax(tmp, logits + (size_t)p * vocab, vocab);
        const float *lb = base + (size_t)p * vocab;
        double kl = 0;
        for (size_t j = 0; j < vocab; j++) kl += exp((double)lb[j]) * ((double)lb[j] - (double)tmp[j]);
        if (per_prompt) per_prompt[p] = kl;
        total += kl;
        free(tmp);
    }
    return total / (double)(prompts > 0 ? prompts : 1);
}
