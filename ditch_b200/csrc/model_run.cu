// Resident-model execution: batches, the forward (src/model.zig:4619-4959),
// the residual pass and directions, the none-mode edit and the KL scorer.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <array>
#include <numeric>

#include "model.cuh"

using namespace ditch;

namespace {

#define REQUIRE(cond, ...)             \
    do {                               \
        if (!(cond)) {                 \
            set_error(__VA_ARGS__);    \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)

__global__ void k_capture_rows(const float *x, const int *cap_slot, int n, int hidden, float *res) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    const int slot = cap_slot[row];
    if (slot < 0) return;
    for (int i = lane; i < hidden; i += 32) res[(long long)slot * hidden + i] = x[(long long)row * hidden + i];
}

template <class T>
cudaError_t upload_vec(DevBuf &buf, const std::vector<T> &v, cudaStream_t st) {
    cudaError_t e = buf.reserve(std::max<size_t>(v.size() * sizeof(T), 4));
    if (e != cudaSuccess || v.empty()) return e;
    return cudaMemcpyAsync(buf.ptr, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, st);
}

// kernelWeight (src/abliterate.zig:134-140), f32 arithmetic as the reference.
bool kernel_weight(const ditch_cuda_params &p, size_t layer, float *out) {
    const float distance = std::fabs((float)layer - p.max_weight_position);
    if (distance > p.min_weight_distance) return false;
    const float w = p.max_weight + (distance / p.min_weight_distance) * (p.min_weight - p.max_weight);
    if (w == 0.0f) return false;
    *out = w;
    return true;
}

// GEMV-T over one slab of a resident weight: out[cols] = v^T W (out zeroed here).

// interpolateBasis with k = 1 (src/abliterate.zig:119-131, orthonormalize 409-423).
std::vector<float> interpolate(const std::vector<float> &dirs, int entries, int hidden, float di) {
    const float shifted = di + 1.0f;
    const int idx = (int)std::floor(shifted);
    const float frac = shifted - std::floor(shifted);
    const float *a = dirs.data() + (size_t)std::min(idx, entries - 1) * hidden;
    const float *b = dirs.data() + (size_t)std::min(idx + 1, entries - 1) * hidden;
    std::vector<float> out(hidden);
    for (int i = 0; i < hidden; i++) out[i] = a[i] + frac * (b[i] - a[i]);
    double s = 0;
    for (float x : out) s += (double)x * x;
    const float nrm = (float)std::sqrt(s);
    for (float &x : out) x = nrm > 1e-20f ? x * (1.0f / nrm) : 0.0f;
    return out;
}

}  // namespace

namespace ditch {

int gemv_t_mat(ditch_cuda_model *m, const Mat &w, int row0, int rows, const float *v, float *out) {
    ditch_cuda_device *dev = m->dev;
    if (w.split.ptr) {
        // v^T (hi + lo): the GEMV-T over the split operand's segments, then
        // the hi and lo sums added (the third segment repeats hi)
        const int kp = w.split_k;
        DITCH_CUDA(m->gemv_part.reserve((size_t)3 * kp * 4));
        DITCH_CUDA(cudaMemsetAsync(m->gemv_part.ptr, 0, (size_t)3 * kp * 4, dev->stream));
        DITCH_LAUNCH(dev, gemv_t_bf16(w.split.as<uint16_t>() + (size_t)row0 * 3 * kp, rows, 3 * kp, v,
                                      m->gemv_part.as<float>(), dev->stream));
        DITCH_LAUNCH(dev, add_split_halves(m->gemv_part.as<float>(), kp, out, dev->stream));
        return DITCH_CUDA_OK;
    }
    DITCH_CUDA(cudaMemsetAsync(out, 0, (size_t)w.cols * 4, dev->stream));
    switch (w.fmt) {
    case kFmtBf16:
        DITCH_LAUNCH(dev, gemv_t_bf16(w.data.as<uint16_t>() + (size_t)row0 * w.cols, rows, w.cols, v, out, dev->stream));
        break;
    case kFmtFp8:
        DITCH_LAUNCH(dev, gemv_t_fp8(w.data.as<uint8_t>() + (size_t)row0 * w.cols,
                                     w.scales.as<float>() + (size_t)(row0 / w.br) * w.scols, rows, w.cols, w.br, w.bc,
                                     v, out, dev->stream));
        break;
    case kFmtMxfp4:
        DITCH_CUDA(m->gemv_part.reserve(gemv_t_mxfp4_scratch(1, rows, w.cols) * 4));
        DITCH_LAUNCH(dev, gemv_t_mxfp4(w.data.as<uint8_t>() + (size_t)row0 * w.cols / 2,
                                       w.scales.as<uint8_t>() + (size_t)row0 * w.cols / 32, rows, w.cols, v, out,
                                       m->gemv_part.as<float>(), dev->stream));
        break;
    case kFmtInt4: {
        DevBuf tmp;
        DITCH_CUDA(tmp.reserve((size_t)rows * w.cols * 2));
        DITCH_LAUNCH(dev, dequant_int_bf16(w.data.as<uint32_t>() + (size_t)row0 * w.cols / 8, w.cols / 8,
                                           w.scales.as<float>() + (size_t)row0 * w.groups,
                                           w.zeros.as<uint32_t>() + (size_t)(row0 / 8) * w.groups, nullptr, w.groups,
                                           rows, w.cols, 4, w.group, tmp.as<uint16_t>(), dev->stream));
        DITCH_LAUNCH(dev, gemv_t_bf16(tmp.as<uint16_t>(), rows, w.cols, v, out, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        break;
    }
    case kFmtQ8_0: {  // the f32 values d * q, as ditch's A = v^T W reads them
        DevBuf tmp;
        DITCH_CUDA(tmp.reserve((size_t)rows * w.cols * 4));
        DITCH_LAUNCH(dev, q8_0_f32(w.data.as<int8_t>() + (size_t)row0 * w.cols, w.scales.as<float>() + (size_t)row0 * w.scols,
                                   (long long)rows * w.cols, tmp.as<float>(), dev->stream));
        DITCH_LAUNCH(dev, gemv_t_f32(tmp.as<float>(), rows, w.cols, v, out, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        break;
    }
    case kFmtQ4K: {  // the f32 values d1 * q - m1
        DevBuf tmp;
        DITCH_CUDA(tmp.reserve((size_t)rows * w.cols * 4));
        DITCH_LAUNCH(dev, q4_k_f32(w.data.as<uint8_t>() + (size_t)row0 * w.cols / 2,
                                   w.scales.as<float>() + (size_t)row0 * w.scols * 2, (long long)rows * w.cols,
                                   tmp.as<float>(), dev->stream));
        DITCH_LAUNCH(dev, gemv_t_f32(tmp.as<float>(), rows, w.cols, v, out, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        break;
    }
    default:
        set_error("edit: weight format %d not supported", w.fmt);
        return DITCH_CUDA_UNSUPPORTED;
    }
    return DITCH_CUDA_OK;
}

int ensure_workspace(ditch_cuda_model *m, int n, int nc, int nl) {
    const Config &c = m->cfg;
    const size_t N = (size_t)std::max(n, 1), H = c.hidden;
    const size_t inter = (std::max(c.inter, 1) + 7) / 8 * 8;
    // split mode: GEMM inputs are [hi | hi | lo] rows of 8-aligned segments
    const size_t sf = m->split3 ? 3 : 1;
    const size_t hk = m->split3 ? (H + 7) / 8 * 8 : H, qk = m->split3 ? ((size_t)c.qd() + 7) / 8 * 8 : c.qd();
    DITCH_CUDA(m->x.reserve(N * H * 4));
    DITCH_CUDA(m->h.reserve(N * hk * sf * 2));
    DITCH_CUDA(m->qkv.reserve(N * c.qkv_width() * 4));
    DITCH_CUDA(m->att.reserve(N * qk * sf * 2));
    DITCH_CUDA(m->act.reserve(N * inter * sf * 2));
    DITCH_CUDA(m->xa.reserve(N * 4 * kMaxDeltaRank));
    if (m->split3) {
        DITCH_CUDA(m->att32.reserve(N * c.qd() * 4));
        DITCH_CUDA(m->gu32.reserve(N * 2 * (size_t)c.inter * 4));
        DITCH_CUDA(m->act32.reserve(N * inter * 4));
    }
    if (nc > 0) DITCH_CUDA(m->res.reserve((size_t)(c.n_layers + 1) * nc * H * 4));
    if (nl > 0) {
        DITCH_CUDA(m->hl.reserve((size_t)nl * hk * sf * 2));
        DITCH_CUDA(m->logits.reserve((size_t)nl * c.vocab * 4));
    }
    return DITCH_CUDA_OK;
}

int make_batch(ditch_cuda_model *m, Batch &b, const uint32_t *tokens, const size_t *offsets, size_t n_prompts,
               size_t window, bool logits, std::vector<int> *first_capture, std::vector<int> *take) {
    REQUIRE(tokens && offsets, "null prompts");
    const size_t n = offsets[n_prompts] - offsets[0];
    REQUIRE(n < (1u << 30), "too many tokens");
    b.n = (int)n;
    b.prompts = (int)n_prompts;
    b.h_start.resize(n_prompts);
    b.h_len.resize(n_prompts);
    std::vector<int> cap(n, -1), lrows;
    int slot = 0;
    if (first_capture) first_capture->assign(n_prompts, 0);
    if (take) take->assign(n_prompts, 0);
    for (size_t p = 0; p < n_prompts; p++) {
        REQUIRE(offsets[p + 1] > offsets[p], "prompt %zu is empty", p);
        const int start = (int)(offsets[p] - offsets[0]), len = (int)(offsets[p + 1] - offsets[p]);
        REQUIRE(len <= m->rope_len, "prompt %zu has %d tokens; the model was loaded for %d", p, len, m->rope_len);
        b.h_start[p] = start;
        b.h_len[p] = len;
        const int tk = (int)std::min<size_t>(window, (size_t)len);
        if (first_capture) (*first_capture)[p] = slot;
        if (take) (*take)[p] = tk;
        for (int pos = len - tk; pos < len; pos++) cap[start + pos] = slot++;
        if (logits) lrows.push_back(start + len - 1);
    }
    cudaStream_t st = m->dev->stream;
    DITCH_CUDA(b.tokens.reserve(std::max<size_t>(n * 4, 4)));
    DITCH_CUDA(cudaMemcpyAsync(b.tokens.ptr, tokens + offsets[0], n * 4, cudaMemcpyHostToDevice, st));
    DITCH_CUDA(upload_vec(b.seq_start, b.h_start, st));
    DITCH_CUDA(upload_vec(b.seq_len, b.h_len, st));
    DITCH_CUDA(upload_vec(b.cap_slot, cap, st));
    DITCH_CUDA(upload_vec(b.logit_rows, lrows, st));
    return DITCH_CUDA_OK;
}

cudaError_t decode_rows_bf16(ditch_cuda_device *dev, const Mat &w, int row0, int rows, uint16_t *out) {
    StageArgs sa{};
    sa.fmt = w.fmt;
    sa.data = w.data.as<uint8_t>();
    sa.row_bytes = w.row_bytes;
    sa.row0 = row0;
    sa.rows = rows;
    sa.cols = w.cols;
    sa.out = out;
    if (w.fmt == kFmtFp8) {
        sa.scales = w.scales.as<float>();
        sa.blk_rows = w.br;
        sa.blk_cols = w.bc;
        sa.scale_cols = w.scols;
    } else if (w.fmt == kFmtMxfp4) {
        sa.scales_u8 = w.scales.as<uint8_t>();
    } else if (w.fmt == kFmtQ8_0 || w.fmt == kFmtQ4K) {
        sa.scales = w.scales.as<float>();
        sa.scale_cols = w.scols;
    } else {
        sa.scales = w.scales.as<float>();
        sa.zeros = w.zeros.as<uint32_t>();
        sa.blk_cols = w.group;
        sa.scale_cols = w.groups;
    }
    return launch_stage_decode(sa, dev->sms, dev->stream);
}

int mat_row_norms(ditch_cuda_device *dev, const Mat &w, int row0, int rows, float *out) {
    if (w.split.ptr) {  // the norms of hi + lo
        DevBuf f;
        DITCH_CUDA(f.reserve((size_t)rows * w.split_k * 4));
        DITCH_LAUNCH(dev, merge_split_rows(w.split.as<uint16_t>() + (size_t)row0 * 3 * w.split_k, rows, w.split_k,
                                           f.as<float>(), dev->stream));
        DITCH_LAUNCH(dev, row_norms_f32(f.as<float>(), rows, w.split_k, out, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));  // f is freed on return
        return DITCH_CUDA_OK;
    }
    if (w.fmt == kFmtBf16) {
        DITCH_LAUNCH(dev, row_norms_bf16(w.data.as<uint16_t>() + (size_t)row0 * w.cols, rows, w.cols, out, dev->stream));
        return DITCH_CUDA_OK;
    }
    if (w.fmt == kFmtMxfp4) {
        DITCH_LAUNCH(dev, row_norms_mxfp4(w.data.as<uint8_t>() + (size_t)row0 * w.row_bytes,
                                          w.scales.as<uint8_t>() + (size_t)row0 * (w.cols / 32), rows, w.cols, out,
                                          dev->stream));
        return DITCH_CUDA_OK;
    }
    // other formats: the bf16 operand the GEMM sees, then its norms
    DevBuf tmp;
    DITCH_CUDA(tmp.reserve((size_t)rows * w.cols * 2));
    DITCH_LAUNCH(dev, decode_rows_bf16(dev, w, row0, rows, tmp.as<uint16_t>()));
    DITCH_LAUNCH(dev, row_norms_bf16(tmp.as<uint16_t>(), rows, w.cols, out, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));  // tmp is freed on return
    return DITCH_CUDA_OK;
}

int gemm_weight(ditch_cuda_model *m, const Mat &w, int slab_row0, int m_rows, const uint16_t *act, int n_tok,
                void *out, long long ldo, int flags, const float *bias, const float *xa, const float *db,
                int a2_row_offset, int delta_rank) {
    return gemm_mat(m->dev, w, slab_row0, m_rows, act, n_tok, out, ldo, flags, bias, xa, db, a2_row_offset, nullptr,
                    delta_rank);
}

bool expert_stack_cached(ditch_cuda_device *dev, const Mat &w) {
    if (w.fmt == kFmtBf16 || !dev->decode_cache || dev->stage_min_tokens <= 0) return false;
    const int rows = w.rows * w.slabs;
    if (w.decoded.ptr) return w.decoded_row0 == 0 && w.decoded_rows == rows;
    const size_t bytes = (size_t)rows * w.cols * 2;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess || free_b <= bytes + (4ull << 30)) return false;
    if (w.decoded.reserve(bytes) != cudaSuccess) return false;
    if (decode_rows_bf16(dev, w, 0, rows, w.decoded.as<uint16_t>()) != cudaSuccess) {
        w.decoded.release();
        return false;
    }
    dev->launches.fetch_add(1, std::memory_order_relaxed);
    w.decoded_row0 = 0;
    w.decoded_rows = rows;
    return true;
}

int gemm_mat(ditch_cuda_device *dev, const Mat &w, int slab_row0, int m_rows, const uint16_t *act, int n_tok,
             void *out, long long ldo, int flags, const float *bias, const float *xa, const float *db,
             int a2_row_offset, const GemmExtra *ex, int delta_rank) {
    if (n_tok <= 0 || m_rows <= 0) return DITCH_CUDA_OK;
    if (delta_rank < 1 || delta_rank > kMaxDeltaRank) {
        set_error("delta rank %d is not within 1..%d", delta_rank, kMaxDeltaRank);
        return DITCH_CUDA_INVALID;
    }
    // split mode: the weight's [hi | lo | hi] operand against [hi | hi | lo]
    // activation rows, K three segments long
    const bool split = w.split.ptr != nullptr;
    const int K = split ? 3 * w.split_k : w.cols;
    GemmOperand A{split ? w.split.ptr : w.data.ptr, w.rows * w.slabs, K, split ? (long long)K * 2 : w.row_bytes};
    GemmOperand B{act, n_tok, K, (long long)K * 2};
    int fmt = w.fmt;
    const bool dual = (flags & kEpiSwiglu) != 0;
    // Staged decode. The fused transform decodes every weight element once per
    // token tile; past a few tiles, decoding the rows once to bf16 scratch (one
    // more pass over the weight: codes in, 2 bytes out, 2 bytes back in) and
    // running the bf16 GEMM costs less. Both build the same bf16 operand.
    // A bf16 copy kept by an earlier staged call also serves the products
    // below the staging threshold (the decode steps of generation after the
    // prefill): past 16 tokens the bf16 GEMM over it runs faster than
    // decoding the stored format tile by tile (same operand bits).
    const int st_rows = (dual ? a2_row_offset : 0) + m_rows;
    const bool cached = fmt != kFmtBf16 && !(ex && ex->sched) && w.decoded.ptr && w.decoded_row0 == slab_row0 &&
                        w.decoded_rows == st_rows;
    const bool stack_cached = fmt != kFmtBf16 && ex && ex->sched && w.decoded.ptr && w.decoded_row0 == 0 &&
                              w.decoded_rows == w.rows * w.slabs;
    if (stack_cached) {
        // the grouped (routed-expert) product over the kept bf16 copy of the
        // whole expert stack (expert_stack_cached): the same slab rows
        A = GemmOperand{w.decoded.ptr, w.rows * w.slabs, w.cols, (long long)w.cols * 2};
        fmt = kFmtBf16;
    } else if (cached && n_tok > 16 && n_tok < dev->stage_min_tokens) {
        A = GemmOperand{w.decoded.ptr, st_rows, w.cols, (long long)w.cols * 2};
        fmt = kFmtBf16;
        slab_row0 = 0;
    } else if (fmt != kFmtBf16 && !(ex && ex->sched) && dev->stage_min_tokens > 0 && n_tok >= dev->stage_min_tokens) {
        const int rows = st_rows;
        const size_t bytes = (size_t)rows * w.cols * 2;
        const void *dec = nullptr;
        if (w.decoded.ptr && w.decoded_row0 == slab_row0 && w.decoded_rows == rows) {
            dec = w.decoded.ptr;  // decoded by an earlier call
        } else if (dev->decode_cache && !w.decoded.ptr) {
            // keep the bf16 copy when memory allows (4 GiB left for everything else)
            size_t free_b = 0, total_b = 0;
            if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && free_b > bytes + (4ull << 30) &&
                w.decoded.reserve(bytes) == cudaSuccess) {
                DITCH_LAUNCH(dev, decode_rows_bf16(dev, w, slab_row0, rows, w.decoded.as<uint16_t>()));
                w.decoded_row0 = slab_row0;
                w.decoded_rows = rows;
                dec = w.decoded.ptr;
            }
        }
        if (!dec) {
            DITCH_CUDA(dev->stage.reserve(bytes));
            DITCH_LAUNCH(dev, decode_rows_bf16(dev, w, slab_row0, rows, dev->stage.as<uint16_t>()));
            dec = dev->stage.ptr;
        }
        A = GemmOperand{dec, rows, w.cols, (long long)w.cols * 2};
        fmt = kFmtBf16;
        slab_row0 = 0;
    }
    GemmParams p{};
    p.m_w = m_rows;
    p.n_tok = n_tok;
    p.k = K;
    p.k_splits = 1;
    if (ex) {
        p.k_splits = ex->k_splits > 0 ? ex->k_splits : 1;
        p.sched = ex->sched;
        p.n_sched = ex->n_sched;
        p.slab_rows = ex->slab_rows;
        p.e_flags = ex->e_flags;
        p.db_stride = ex->db_stride;
        p.bn = ex->bn;
    }
    // 1..16 tokens: the weight-streaming product, K split over the grid: the
    // partial sums are added atomically, or in deterministic mode left in
    // sk_ws and added in split order by the last block of each row block
    const int sk = skinny_chunk(fmt);
    if (!p.sched && p.k_splits == 1 && !dual && !(flags & kEpiOutBf16) && n_tok <= 16 && sk && K % sk == 0 &&
        !(fmt == kFmtFp8 && w.bc % 16) && !(fmt == kFmtInt4 && w.group % 32)) {
        const int bx = (m_rows + 15) / 16, chunks = K / sk;
        const int ks = std::max(1, std::min(chunks, (2 * dev->sms + bx - 1) / bx));  // about one wave
        if (ks > 1 && !dev->deterministic) {
            if (!(flags & kEpiResidual))
                DITCH_CUDA(cudaMemset2DAsync(out, (size_t)ldo * 4, 0, (size_t)m_rows * 4, n_tok, dev->stream));
            flags = (flags & ~kEpiResidual) | kEpiAtomic;
        } else if (ks > 1) {
            const int per = (chunks + ks - 1) / ks, splits = (chunks + per - 1) / per;
            DITCH_CUDA(dev->sk_ws.reserve(skinny_split_bytes(m_rows, splits)));
            if (dev->sk_tiles < bx) {
                DITCH_CUDA(dev->sk_cnt.reserve((size_t)bx * sizeof(int)));
                DITCH_CUDA(cudaMemsetAsync(dev->sk_cnt.ptr, 0, (size_t)bx * sizeof(int), dev->stream));
                dev->sk_tiles = bx;
            }
            p.sk_ws = dev->sk_ws.as<float>();
            p.sk_cnt = dev->sk_cnt.as<int>();
        }
        p.a_row0 = slab_row0;
        p.out = out;
        p.ldo = ldo;
        p.flags = flags;
        p.bias = bias;
        p.xa = xa;
        p.db = db;
        p.delta_rank = delta_rank;
        if (fmt == kFmtFp8) {
            p.scales = w.scales.as<float>();
            p.blk_rows = w.br;
            p.blk_cols = w.bc;
            p.scale_cols = w.scols;
        } else if (fmt == kFmtMxfp4) {
            p.scales_u8 = w.scales.as<uint8_t>();
        } else if (fmt == kFmtQ8_0 || fmt == kFmtQ4K) {
            p.scales = w.scales.as<float>();
            p.scale_cols = w.scols;
        } else if (fmt == kFmtInt4) {
            p.scales = w.scales.as<float>();
            p.zeros = w.zeros.as<uint32_t>();
            p.blk_cols = w.group;
            p.scale_cols = w.groups;
        }
        cudaError_t e = run_skinny(dev, fmt, A, B, p, ks);
        if (e != cudaSuccess) return cuda_status(e, "skinny product");
        return DITCH_CUDA_OK;
    }
    // Few output tiles (few weight rows and few tokens) leave SMs idle: split
    // K. By default the splits are fixed and add their partial sums
    // atomically (linear epilogues only); in deterministic mode the GEMM runs
    // stream-K, where a tile split between CTAs is summed in k order by the
    // CTA that brings its last part, for any epilogue.
    const int bn = gemm_token_tile(n_tok, dual, fmt != kFmtBf16);
    const long long tiles = (long long)((m_rows + 127) / 128) * ((n_tok + bn - 1) / bn);
    const int k_tiles = (K + 63) / 64;
    if (!dev->deterministic && !p.sched && p.k_splits == 1 && !dual && !(flags & kEpiOutBf16) &&
        tiles < dev->sms && k_tiles >= 8) {
        // as many splits as still fit one wave: a second, nearly empty wave
        // would double the time of the streaming-bound product
        const int ks = std::min((int)(dev->sms / tiles), k_tiles / 4);
        if (ks > 1) {
            p.k_splits = ks;
            if (!(flags & kEpiResidual))
                DITCH_CUDA(cudaMemset2DAsync(out, (size_t)ldo * 4, 0, (size_t)m_rows * 4, n_tok, dev->stream));
            flags = (flags & ~kEpiResidual) | kEpiAtomic;
        }
    }
    if (dev->deterministic && !p.sched && p.k_splits == 1) {
        if (gemm_wants_stream_k(tiles, k_tiles, dev->sms)) {
            DITCH_CUDA(dev->sk_ws.reserve(gemm_stream_k_bytes(dev->sms, bn, dual)));
            if (dev->sk_tiles < tiles) {
                DITCH_CUDA(dev->sk_cnt.reserve((size_t)tiles * sizeof(int)));
                DITCH_CUDA(cudaMemsetAsync(dev->sk_cnt.ptr, 0, (size_t)tiles * sizeof(int), dev->stream));
                dev->sk_tiles = tiles;
            }
            p.stream_k = 1;
            p.sk_ws = dev->sk_ws.as<float>();
            p.sk_cnt = dev->sk_cnt.as<int>();
        }
    }
    p.a2_row_offset = a2_row_offset;
    p.a_row0 = slab_row0;
    p.out = out;
    p.ldo = ldo;
    p.flags = flags;
    p.bias = bias;
    p.xa = xa;
    p.db = db;
    p.delta_rank = delta_rank;
    if (fmt == kFmtFp8) {
        p.scales = w.scales.as<float>();
        p.blk_rows = w.br;
        p.blk_cols = w.bc;
        p.scale_cols = w.scols;
    } else if (fmt == kFmtMxfp4) {
        p.scales_u8 = w.scales.as<uint8_t>();
    } else if (fmt == kFmtQ8_0 || fmt == kFmtQ4K) {
        p.scales = w.scales.as<float>();
        p.scale_cols = w.scols;
    } else if (fmt == kFmtInt4) {
        p.scales = w.scales.as<float>();
        p.zeros = w.zeros.as<uint32_t>();
        p.blk_cols = w.group;
        p.scale_cols = w.groups;
    }
    cudaError_t e = run_gemm(dev, fmt, A, (flags & kEpiSwiglu) ? &A : nullptr, B, p);
    if (e != cudaSuccess) return cuda_status(e, "gemm");
    return DITCH_CUDA_OK;
}

int forward_batch(ditch_cuda_model *m, Batch &b, int nc, int nl, int mode) {
    const Config &c = m->cfg;
    ditch_cuda_device *dev = m->dev;
    cudaStream_t st = dev->stream;
    const int n = b.n, H = c.hidden, qd = c.qd(), W = c.qkv_width();
    int s;
    if (m->group && c.tp_world > 1 && (size_t)n > m->group_tokens) {
        set_error("%d tokens exceed the %zu the peer group was sized for", n, m->group_tokens);
        return DITCH_CUDA_INVALID;
    }
    if ((s = ensure_workspace(m, n, nc, nl))) return s;
    float *x = m->x.as<float>();
    uint16_t *h = m->h.as<uint16_t>();
    float *res = nc > 0 ? m->res.as<float>() : nullptr;
    const int *cap = nc > 0 ? b.cap_slot.as<int>() : nullptr;
    const size_t entry = (size_t)nc * H;
    DITCH_LAUNCH(dev, embed_rows(m->embed.ptr, m->embed_bf16 ? 1 : 0, b.tokens.as<uint32_t>(), n, H, x, cap, res,
                                 dev->status, c.vocab, st));
    // split mode: the norms write [hi | hi | lo] operand rows of kh columns a
    // segment; attention and SwiGLU go through f32 first
    const bool sp = m->split3;
    const int kh = sp ? (H + 7) / 8 * 8 : 0;
    for (int li = 0; li < c.n_layers; li++) {
        Layer &L = m->layers[li];
        // input norm; entry li (the previous layer's output) is captured here
        DITCH_LAUNCH(dev, rmsnorm_rows_bf16(x, L.input_norm.as<float>(), n, H, c.eps, h, li > 0 ? cap : nullptr,
                                            li > 0 && res ? res + (size_t)li * entry : nullptr, nullptr, st, kh));
        if ((s = gemm_weight(m, L.qkv, 0, W, h, n, m->qkv.ptr, W, 0, L.qkv_bias.as<float>(), nullptr, nullptr, 0)))
            return s;
        AttnParams ap{};
        ap.qkv = m->qkv.as<float>();
        ap.out = m->att.as<uint16_t>();
        ap.out_f32 = sp ? m->att32.as<float>() : nullptr;
        ap.seq_start = b.seq_start.as<int>();
        ap.seq_len = b.seq_len.as<int>();
        ap.n_prompts = b.prompts;
        ap.heads = c.heads;
        ap.kv_heads = c.kv_heads;
        ap.head_dim = c.head_dim;
        ap.rope_cos = m->rope_cos.as<float>();
        ap.rope_sin = m->rope_sin.as<float>();
        ap.q_norm = c.qk_norm ? L.q_norm.as<float>() : nullptr;
        ap.k_norm = c.qk_norm ? L.k_norm.as<float>() : nullptr;
        ap.eps = c.eps;
        ap.scale = 1.0f / std::sqrt((float)c.head_dim);
        ap.status = dev->status;
        ap.max_len = b.h_len.empty() ? 1 : *std::max_element(b.h_len.begin(), b.h_len.end());
        ap.tc = dev->attn_tc;
        if (mode == kFwdPrompts) {
            DITCH_LAUNCH(dev, attention_prefill(ap, st));
        } else {
            // the cache of this layer; decode rows store their key and value
            // first, so each attends to its own key as well
            const size_t per_layer = (size_t)m->kv_slots * m->kv_len * c.kvd();
            KvParams kp{};
            kp.qkv = m->qkv.as<float>();
            kp.row_b = b.row_b.as<int>();
            kp.row_pos = b.row_pos.as<int>();
            kp.n = n;
            kp.slots = m->kv_slots;
            kp.max_len = m->kv_len;
            kp.heads = c.heads;
            kp.kv_heads = c.kv_heads;
            kp.head_dim = c.head_dim;
            kp.rope_cos = ap.rope_cos;
            kp.rope_sin = ap.rope_sin;
            kp.q_norm = ap.q_norm;
            kp.k_norm = ap.k_norm;
            kp.eps = c.eps;
            kp.cache_k = m->kv_k.as<float>() + li * per_layer;
            kp.cache_v = m->kv_v.as<float>() + li * per_layer;
            kp.status = dev->status;
            if (mode == kFwdDecode) {
                kp.prep_k = kp.prep_q = 1;
                DITCH_LAUNCH(dev, kv_store(kp, st));
                DecodeAttnParams dp{};
                dp.qkv = m->qkv.as<float>();
                dp.out = m->att.as<uint16_t>();
                dp.out_f32 = ap.out_f32;
                dp.row_b = kp.row_b;
                dp.row_pos = kp.row_pos;
                dp.n = n;
                dp.max_len = m->kv_len;
                dp.heads = c.heads;
                dp.kv_heads = c.kv_heads;
                dp.head_dim = c.head_dim;
                dp.cache_k = kp.cache_k;
                dp.cache_v = kp.cache_v;
                dp.scale = ap.scale;
                DITCH_LAUNCH(dev, attention_decode(dp, st));
            } else {
                DITCH_LAUNCH(dev, attention_prefill(ap, st));
                kp.prep_k = attention_prefill_preps_in_place(c.head_dim, 0) ? 0 : 1;
                DITCH_LAUNCH(dev, kv_store(kp, st));
            }
        }
        if (sp) DITCH_LAUNCH(dev, split_act_rows(m->att32.as<float>(), n, qd, L.o.split_k, m->att.as<uint16_t>(), st));
        if (L.o_edit)
            for (int t = 0; t < L.o_rank; t++) {
                if (sp)
                    DITCH_LAUNCH(dev, rowdot_f32_strided(m->att32.as<float>(), L.o_a.as<float>() + (size_t)t * qd, n, qd,
                                                         m->xa.as<float>() + t, L.o_rank, st));
                else
                    DITCH_LAUNCH(dev, rowdot_bf16_strided(m->att.as<uint16_t>(), L.o_a.as<float>() + (size_t)t * qd, n,
                                                          qd, m->xa.as<float>() + t, L.o_rank, st));
            }
        // tensor parallel: the partial sum goes to the group's send rows, then the all-reduce adds it to x
        const bool tp = m->group && c.tp_world > 1;
        if ((s = gemm_weight(m, L.o, 0, H, m->att.as<uint16_t>(), n, tp ? tp_send_rows(m) : x, H, tp ? 0 : kEpiResidual,
                             nullptr, L.o_edit ? m->xa.as<float>() : nullptr, L.o_edit ? L.o_b.as<float>() : nullptr, 0,
                             L.o_edit ? L.o_rank : 1)))
            return s;
        if (tp && (s = tp_allreduce_add(m, n, x))) return s;
        if (L.moe) {
            if ((s = moe_mlp(m, L, li, n))) return s;
        } else {
            DITCH_LAUNCH(dev, rmsnorm_rows_bf16(x, L.post_norm.as<float>(), n, H, c.eps, h, nullptr, nullptr, nullptr, st,
                                                kh));
            const int I = c.inter, Ip = L.down.cols;  // Ip: the stored (8-aligned) width
            if (sp) {
                // the gate | up product in f32, then silu(gate) * up and its split operand
                if ((s = gemm_weight(m, L.gate_up, 0, 2 * I, h, n, m->gu32.ptr, 2 * I, 0, nullptr, nullptr, nullptr, 0)))
                    return s;
                DITCH_LAUNCH(dev, swiglu_split(m->gu32.as<float>(), n, I, L.down.split_k, m->act32.as<float>(),
                                               m->act.as<uint16_t>(), st));
            } else {
                if (Ip != I) DITCH_CUDA(cudaMemsetAsync(m->act.ptr, 0, (size_t)n * Ip * 2, st));
                if ((s = gemm_weight(m, L.gate_up, 0, I, h, n, m->act.ptr, Ip, kEpiSwiglu, nullptr, nullptr, nullptr, I)))
                    return s;
            }
            if (L.down_edit)
                for (int t = 0; t < L.down_rank; t++) {
                    if (sp)
                        DITCH_LAUNCH(dev, rowdot_f32_strided(m->act32.as<float>(), L.down_a.as<float>() + (size_t)t * Ip,
                                                             n, Ip, m->xa.as<float>() + t, L.down_rank, st));
                    else
                        DITCH_LAUNCH(dev, rowdot_bf16_strided(m->act.as<uint16_t>(),
                                                              L.down_a.as<float>() + (size_t)t * Ip, n, Ip,
                                                              m->xa.as<float>() + t, L.down_rank, st));
                }
            if ((s = gemm_weight(m, L.down, 0, H, m->act.as<uint16_t>(), n, tp ? tp_send_rows(m) : x, H,
                                 tp ? 0 : kEpiResidual, nullptr, L.down_edit ? m->xa.as<float>() : nullptr,
                                 L.down_edit ? L.down_b.as<float>() : nullptr, 0, L.down_edit ? L.down_rank : 1)))
                return s;
            if (tp && (s = tp_allreduce_add(m, n, x))) return s;
        }
    }
    if (res) {
        k_capture_rows<<<(n + 7) / 8, 256, 0, st>>>(x, cap, n, H, res + (size_t)c.n_layers * entry);
        DITCH_LAUNCH(dev, cudaGetLastError());
    }
    if (nl > 0) {
        DITCH_LAUNCH(dev, gather_rmsnorm_bf16(x, b.logit_rows.as<int>(), nl, H, c.eps, m->final_norm.as<float>(),
                                              m->hl.as<uint16_t>(), st, kh));
        if ((s = gemm_weight(m, m->lm_head, 0, c.vocab, m->hl.as<uint16_t>(), nl, m->logits.ptr, c.vocab, 0, nullptr,
                             nullptr, nullptr, 0)))
            return s;
    }
    return DITCH_CUDA_OK;
}

}  // namespace ditch

namespace {

// The rank-1 delta (a, b) of one matrix whose rows are the H outputs:
// none mode a = v^T W, b = -lambda v; pre mode a = (v / n)^T W, b = -lambda v n
// with n the row norms (src/abliterate.zig:264-323).
int rank1_delta(ditch_cuda_model *m, const Mat &w, int row0, DevBuf &rn_cache, size_t rn_off, const float *v,
                float lambda, float *a, float *b) {
    ditch_cuda_device *dev = m->dev;
    const int H = m->cfg.hidden;
    if (m->row_norm == 0) {
        int s;
        if ((s = gemv_t_mat(m, w, row0, H, v, a))) return s;
        DITCH_LAUNCH(dev, scale_vec(v, lambda, H, b, dev->stream));
        return DITCH_CUDA_OK;
    }
    DITCH_CUDA(m->vn.reserve((size_t)H * 4));
    DITCH_LAUNCH(dev, prenorm_vec(v, rn_cache.as<float>() + rn_off, lambda, H, m->vn.as<float>(), b, dev->stream));
    return gemv_t_mat(m, w, row0, H, m->vn.as<float>(), a);
}

// Row norms of o_proj, down_proj and the routed experts' down projections of
// one layer (under tensor parallelism summed over the ranks' column shards:
// a collective). Marked pending; settle_row_norms marks them valid once the
// call's device status is known to be clean.
int compute_row_norms(ditch_cuda_model *m, Layer &L) {
    ditch_cuda_device *dev = m->dev;
    const int H = m->cfg.hidden;
    int s;
    L.rn_valid = false;
    L.rn_pending = true;
    DITCH_CUDA(L.o_rn.reserve((size_t)H * 4));
    if ((s = tp_row_norms(m, L.o, L.o_rn.as<float>()))) return s;
    if (!L.moe) {
        DITCH_CUDA(L.down_rn.reserve((size_t)H * 4));
        if ((s = tp_row_norms(m, L.down, L.down_rn.as<float>()))) return s;
    } else {
        const int E = m->cfg.e_loc;
        DITCH_CUDA(L.e_rn.reserve((size_t)E * H * 4));
        if ((s = mat_row_norms(dev, L.e_down, 0, E * H, L.e_rn.as<float>()))) return s;
    }
    return DITCH_CUDA_OK;
}

// Pending row norms become valid when the call that computed them ended with
// a clean status (`ok`); otherwise (a peer wait that ran out, a failed step)
// they are dropped and the next edit computes them again.
void settle_row_norms(ditch_cuda_model *m, bool ok) {
    for (Layer &L : m->layers)
        if (L.rn_pending) {
            L.rn_pending = false;
            L.rn_valid = ok;
        }
}

// The row norms of layer li, computed on first use. On a tensor-parallel
// model they are a collective, so ditch_cuda_set_row_normalization computes
// every layer's at once (every rank calls it once, in the same order) and an
// edit never starts one.
int ensure_row_norms(ditch_cuda_model *m, Layer &L) {
    if (L.rn_valid || L.rn_pending) return DITCH_CUDA_OK;
    if (m->cfg.tp_world > 1) {
        set_error("row norms of this tensor-parallel model are missing: call set_row_normalization again");
        return DITCH_CUDA_INVALID;
    }
    return compute_row_norms(m, L);
}

int apply_component_edit(ditch_cuda_model *m, int li, bool is_o, const float *v, float lambda) {
    Layer &L = m->layers[li];
    int s;
    if (m->row_norm && (s = ensure_row_norms(m, L))) return s;
    if (m->row_norm == 2) {  // full: a rank-r delta from a randomised SVD
        const Mat &w = is_o ? L.o : L.down;
        int rank = 1;
        if ((s = full_norm_delta(m, w, 0, (is_o ? L.o_rn : L.down_rn).as<float>(), v, lambda, m->lora_rank,
                                 m->edit_seed + m->seed_counter++, (is_o ? L.o_a : L.down_a).as<float>(),
                                 (is_o ? L.o_b : L.down_b).as<float>(), &rank)))
            return s;
        if (is_o) {
            L.o_rank = rank;
            L.o_edit = true;
        } else {
            L.down_rank = rank;
            L.down_edit = true;
        }
        return DITCH_CUDA_OK;
    }
    if (is_o) {
        if ((s = rank1_delta(m, L.o, 0, L.o_rn, 0, v, lambda, L.o_a.as<float>(), L.o_b.as<float>()))) return s;
        L.o_edit = true;
    } else {
        if ((s = rank1_delta(m, L.down, 0, L.down_rn, 0, v, lambda, L.down_a.as<float>(), L.down_b.as<float>())))
            return s;
        L.down_edit = true;
    }
    return DITCH_CUDA_OK;
}

int upload_expert_flags(ditch_cuda_model *m) {
    for (Layer &L : m->layers) {
        if (!L.moe) continue;
        std::vector<int> f(L.e_edit.begin(), L.e_edit.end());
        DITCH_CUDA(cudaMemcpyAsync(L.e_edit_dev.ptr, f.data(), f.size() * 4, cudaMemcpyHostToDevice, m->dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(m->dev->stream));
    }
    return DITCH_CUDA_OK;
}

void clear_edits(ditch_cuda_model *m) {
    for (Layer &L : m->layers) {
        L.o_edit = L.down_edit = false;
        L.o_rank = L.down_rank = L.e_rank = 1;
        std::fill(L.e_edit.begin(), L.e_edit.end(), 0);
    }
}

// The direction for layer li: dirs[li + 1] or the interpolated one.
const float *direction_for(ditch_cuda_model *m, int li, bool use_di) {
    return use_di ? m->vtmp.as<float>() : m->dirs.as<float>() + (size_t)(li + 1) * m->cfg.hidden;
}

int prepare_direction(ditch_cuda_model *m, float di, bool use_di) {
    REQUIRE(m->dir_entries >= (use_di ? 1 : m->cfg.n_layers + 1), "directions not set (need %d entries)",
            m->cfg.n_layers + 1);
    if (use_di) {
        std::vector<float> v = interpolate(m->h_dirs, m->dir_entries, m->cfg.hidden, di);
        DITCH_CUDA(cudaMemcpyAsync(m->vtmp.ptr, v.data(), v.size() * 4, cudaMemcpyHostToDevice, m->dev->stream));
    }
    return DITCH_CUDA_OK;
}

// A_e = v^T W_down_e for every routed expert of `li` into L.e_proj [E][mi]
// (v device f32 [H]); one launch over the whole MXFP4 stack.
int expert_projections(ditch_cuda_model *m, int li, const float *v) {
    ditch_cuda_device *dev = m->dev;
    Layer &L = m->layers[li];
    const int E = m->cfg.e_loc, H = m->cfg.hidden, mi = L.e_down.cols;  // this rank's experts; stored width
    DITCH_CUDA(L.e_proj.reserve((size_t)E * mi * 4));
    float *proj = L.e_proj.as<float>();
    if (L.e_down.fmt == kFmtMxfp4) {
        DITCH_CUDA(cudaMemsetAsync(proj, 0, (size_t)E * mi * 4, dev->stream));
        DITCH_CUDA(m->gemv_part.reserve(gemv_t_mxfp4_scratch(E, H, mi) * 4));
        DITCH_LAUNCH(dev, gemv_t_mxfp4_stack(L.e_down.data.as<uint8_t>(), L.e_down.scales.as<uint8_t>(), E, H, mi, v,
                                             proj, m->gemv_part.as<float>(), dev->stream));
        return DITCH_CUDA_OK;
    }
    int s;
    for (int e = 0; e < E; e++)
        if ((s = gemv_t_mat(m, L.e_down, e * H, H, v, proj + (size_t)e * mi))) return s;
    return DITCH_CUDA_OK;
}

// ||W_down_e||_F of every routed expert of `li`, once per model (the base
// weights never change; edits are kept as separate deltas).
int expert_frobenius(ditch_cuda_model *m, int li) {
    ditch_cuda_device *dev = m->dev;
    Layer &L = m->layers[li];
    const int E = m->cfg.e_loc, H = m->cfg.hidden, mi = L.e_down.cols;  // this rank's experts
    if ((int)L.e_fro.size() == E) return DITCH_CUDA_OK;
    DevBuf norms;
    DITCH_CUDA(norms.reserve((size_t)E * H * 4));
    const Mat &w = L.e_down;
    if (w.fmt == kFmtBf16) {
        DITCH_LAUNCH(dev, row_norms_bf16(w.data.as<uint16_t>(), E * H, mi, norms.as<float>(), dev->stream));
    } else if (w.fmt == kFmtMxfp4) {
        DITCH_LAUNCH(dev, row_norms_mxfp4(w.data.as<uint8_t>(), w.scales.as<uint8_t>(), E * H, mi, norms.as<float>(),
                                          dev->stream));
    } else {
        DevBuf tmp;
        DITCH_CUDA(tmp.reserve((size_t)H * mi * 2));
        for (int e = 0; e < E; e++) {
            if (w.fmt == kFmtFp8) {
                DITCH_LAUNCH(dev, dequant_fp8_bf16(w.data.as<uint8_t>() + (size_t)e * H * mi,
                                                   w.scales.as<float>() + (size_t)(e * H / w.br) * w.scols, H, mi, w.br,
                                                   w.bc, tmp.as<uint16_t>(), dev->stream));
            } else {
                DITCH_LAUNCH(dev, dequant_int_bf16(w.data.as<uint32_t>() + (size_t)e * H * mi / 8, mi / 8,
                                                   w.scales.as<float>() + (size_t)e * H * w.groups,
                                                   w.zeros.as<uint32_t>() + (size_t)(e * H / 8) * w.groups, nullptr,
                                                   w.groups, H, mi, 4, w.group, tmp.as<uint16_t>(), dev->stream));
            }
            DITCH_LAUNCH(dev, row_norms_bf16(tmp.as<uint16_t>(), H, mi, norms.as<float>() + (size_t)e * H, dev->stream));
        }
    }
    std::vector<float> hn((size_t)E * H);
    DITCH_CUDA(cudaMemcpyAsync(hn.data(), norms.ptr, hn.size() * 4, cudaMemcpyDeviceToHost, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    L.e_fro.assign(E, 0.0f);
    for (int e = 0; e < E; e++) {
        float fro = 0.0f;
        for (int r = 0; r < H; r++) fro = std::fma(hn[(size_t)e * H + r], hn[(size_t)e * H + r], fro);
        L.e_fro[e] = std::sqrt(fro);
    }
    return DITCH_CUDA_OK;
}

// Scores of every routed expert of `li` against v (device f32 [H]):
// ||v^T W_down_e|| / ||W_down_e||_F (src/moe.zig:1239-1283). Leaves the
// projections in L.e_proj for the edit of the selected experts. With expert
// parallelism each rank scores its own experts and the group gathers them.
int expert_scores(ditch_cuda_model *m, int li, const float *v, std::vector<float> &scores) {
    ditch_cuda_device *dev = m->dev;
    Layer &L = m->layers[li];
    const int E = m->cfg.e_loc, mi = L.e_down.cols;
    int s;
    if ((s = expert_frobenius(m, li))) return s;
    if ((s = expert_projections(m, li, v))) return s;
    std::vector<float> hp((size_t)E * mi);
    DITCH_CUDA(cudaMemcpyAsync(hp.data(), L.e_proj.ptr, hp.size() * 4, cudaMemcpyDeviceToHost, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    scores.assign(E, 0.0f);
    for (int e = 0; e < E; e++) {
        float pn = 0.0f;
        for (int j = 0; j < mi; j++) pn = std::fma(hp[(size_t)e * mi + j], hp[(size_t)e * mi + j], pn);
        const float fro = L.e_fro[e];
        scores[e] = fro > 0 ? std::sqrt(pn) / fro : 0.0f;
    }
    if (m->group) {
        std::vector<float> all;
        if ((s = ep_allgather_scores(m, scores, all))) return s;
        scores.swap(all);
    }
    return DITCH_CUDA_OK;
}

// The none-mode delta of expert e from its projection in L.e_proj:
// a = v^T W_down_e, b = -lambda v, stored as (a, lambda v) for the epilogue.
// seed_index: this matrix's running index in the edit as one device would
// count it (full mode seeds its sketch with edit_seed plus it, so every rank
// of an expert-parallel model draws the same sketch for the same expert).
int expert_delta_from_proj(ditch_cuda_model *m, int li, int e, const float *v, float lambda, uint64_t seed_index) {
    ditch_cuda_device *dev = m->dev;
    Layer &L = m->layers[li];
    const int H = m->cfg.hidden, mi = L.e_down.cols;
    if (m->row_norm == 2) {  // full: expert e's rank-r delta, [E][r][mi] and [E][H][r]
        int s;
        if ((s = ensure_row_norms(m, L))) return s;
        const int r = m->lora_rank;
        int got = 0;
        if ((s = full_norm_delta(m, L.e_down, e * H, L.e_rn.as<float>() + (size_t)e * H, v, lambda, r,
                                 m->edit_seed + seed_index, L.e_a.as<float>() + (size_t)e * r * mi,
                                 L.e_b.as<float>() + (size_t)e * H * r, &got)))
            return s;
        REQUIRE(got == r, "expert %d: a rank-%d delta where the layer's experts take rank %d", e, got, r);
        L.e_rank = r;
        L.e_edit[e] = 1;
        return DITCH_CUDA_OK;
    }
    if (m->row_norm) {  // pre-normalised: the projection of v / n_e, not of v
        int s;
        if ((s = ensure_row_norms(m, L))) return s;
        if ((s = rank1_delta(m, L.e_down, e * H, L.e_rn, (size_t)e * H, v, lambda, L.e_a.as<float>() + (size_t)e * mi,
                             L.e_b.as<float>() + (size_t)e * H)))
            return s;
        L.e_edit[e] = 1;
        return DITCH_CUDA_OK;
    }
    DITCH_CUDA(cudaMemcpyAsync(L.e_a.as<float>() + (size_t)e * mi, L.e_proj.as<float>() + (size_t)e * mi,
                               (size_t)mi * 4, cudaMemcpyDeviceToDevice, dev->stream));
    DITCH_LAUNCH(dev, scale_vec(v, lambda, H, L.e_b.as<float>() + (size_t)e * H, dev->stream));
    L.e_edit[e] = 1;
    return DITCH_CUDA_OK;
}

std::vector<uint32_t> rank(const std::vector<float> &s) {
    std::vector<uint32_t> order(s.size());
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        if (s[a] != s[b]) return s[a] > s[b];
        return a < b;
    });
    return order;
}

int edit_body(ditch_cuda_model *m, const ditch_cuda_params *attn_o, const ditch_cuda_params *mlp_down, float di,
              int use_di, bool selective, size_t n_experts, float strength) {
    const Config &c = m->cfg;
    clear_edits(m);
    m->seed_counter = 0;
    int s;
    if ((s = prepare_direction(m, di, use_di != 0))) return s;
    for (int li = 0; li < c.n_layers; li++) {
        const float *v = direction_for(m, li, use_di != 0);
        float lambda;
        if (attn_o && kernel_weight(*attn_o, li, &lambda))
            if ((s = apply_component_edit(m, li, true, v, lambda))) return s;
        if (!mlp_down || !kernel_weight(*mlp_down, li, &lambda)) continue;
        Layer &L = m->layers[li];
        if (!L.moe) {
            if ((s = apply_component_edit(m, li, false, v, lambda))) return s;
            continue;
        }
        const int E = c.n_experts;
        if (!selective || n_experts == 0) {
            if (!m->row_norm && (s = expert_projections(m, li, v))) return s;  // every expert's v^T W_e at once
            for (int e = 0; e < c.e_loc; e++)  // this rank's experts
                if ((s = expert_delta_from_proj(m, li, e, v, lambda, m->seed_counter + c.e0 + e))) return s;
            m->seed_counter += E;  // every expert of the layer counts, wherever it lives
            continue;
        }
        const float weight = std::max(0.0f, lambda * strength);
        const size_t n = std::min<size_t>(n_experts, (size_t)E);
        if (weight == 0.0f || n == 0) continue;
        std::vector<float> scores;
        if ((s = expert_scores(m, li, v, scores))) return s;
        std::vector<uint32_t> order = rank(scores);
        for (size_t j = 0; j < n; j++) {
            const int e = (int)order[j] - c.e0;  // edited by the rank that owns it
            if (e >= 0 && e < c.e_loc)
                if ((s = expert_delta_from_proj(m, li, e, v, weight, m->seed_counter + j))) return s;
        }
        m->seed_counter += n;
    }
    if ((s = upload_expert_flags(m))) return s;
    return check_status(m->dev, "apply_edit");
}

int edit_common(ditch_cuda_model *m, const ditch_cuda_params *attn_o, const ditch_cuda_params *mlp_down, float di,
                int use_di, bool selective, size_t n_experts, float strength) {
    const int s = edit_body(m, attn_o, mlp_down, di, use_di, selective, n_experts, strength);
    settle_row_norms(m, s == DITCH_CUDA_OK);
    return s;
}

int kl_score_impl(ditch_cuda_model *m, double *kl) {
    ditch_cuda_device *dev = m->dev;
    const int P = m->kl.prompts, V = m->cfg.vocab;
    int s;
    if ((s = forward_batch(m, m->kl, 0, P))) return s;
    DITCH_CUDA(m->kl_vals.reserve((size_t)P * 8));
    DITCH_CUDA(m->kl_part.reserve(kl_scratch_bytes(P, V)));
    DITCH_LAUNCH(dev, kl_rows(m->kl_base.as<float>(), m->logits.as<float>(), P, V, m->kl_vals.as<double>(),
                              m->kl_part.ptr, dev->stream));
    if (m->dp_group) {
        // data parallel: every rank's per-prompt values summed in rank order,
        // then prompt order (one device's order over the concatenated prompts)
        double tot[2] = {0.0, 0.0};
        DITCH_CUDA(m->dp_buf.reserve(2 * 8));
        if ((s = dp_ordered_sum(dev, m->dp_group, m->kl_vals.as<double>(), (size_t)P, m->dp_buf.as<double>())))
            return s;
        DITCH_CUDA(cudaMemcpyAsync(tot, m->dp_buf.ptr, 2 * 8, cudaMemcpyDeviceToHost, dev->stream));
        if ((s = check_status(dev, "kl_score"))) return s;
        *kl = tot[0] / std::max(tot[1], 1.0);
        return DITCH_CUDA_OK;
    }
    std::vector<double> per(P);
    DITCH_CUDA(cudaMemcpyAsync(per.data(), m->kl_vals.ptr, (size_t)P * 8, cudaMemcpyDeviceToHost, dev->stream));
    if ((s = check_status(dev, "kl_score"))) return s;
    double total = 0.0;
    for (int p = 0; p < P; p++) total += per[p];  // prompt order, as src/scorers.zig:385-400
    *kl = total / (double)std::max(P, 1);
    return DITCH_CUDA_OK;
}

}  // namespace

extern "C" {

int ditch_cuda_forward(ditch_cuda_model *m, const uint32_t *tokens, const uint32_t *row_b, const uint32_t *row_pos,
                       size_t n, const size_t *capture_rows, size_t nc, float *residuals, const size_t *logit_rows,
                       size_t nl, float *logits) {
    clear_error();
    REQUIRE(m && tokens && row_b && row_pos, "null argument");
    REQUIRE(nc == 0 || (capture_rows && residuals), "capture rows without an output");
    REQUIRE(nl == 0 || (logit_rows && logits), "logit rows without an output");
    if (n == 0) return DITCH_CUDA_OK;
    ditch_cuda_device *dev = m->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    // The device forward reads each prompt's keys from the call itself: rows
    // of a batch slot must be contiguous with positions 0, 1, ... (the layout
    // src/engine.zig:392-410 builds). Anything else is left to the CPU.
    std::vector<size_t> offsets{0};
    for (size_t i = 0; i < n; i++) {
        const bool new_prompt = i == 0 || row_b[i] != row_b[i - 1];
        if (new_prompt && i > 0) offsets.push_back(i);
        if ((new_prompt && row_pos[i] != 0) || (!new_prompt && row_pos[i] != row_pos[i - 1] + 1)) {
            set_error("rows are not contiguous prompts starting at position 0");
            return DITCH_CUDA_UNSUPPORTED;
        }
    }
    offsets.push_back(n);
    const size_t P = offsets.size() - 1;
    for (size_t i = 1; i < P; i++)
        for (size_t j = 0; j < i; j++)
            if (row_b[offsets[i]] == row_b[offsets[j]]) {
                set_error("a batch slot appears twice");
                return DITCH_CUDA_UNSUPPORTED;
            }
    for (size_t i = 0; i < nc; i++) REQUIRE(capture_rows[i] < n, "capture row out of range");
    for (size_t i = 0; i < nl; i++) REQUIRE(logit_rows[i] < n, "logit row out of range");
    Batch &b = m->work;
    int s;
    if ((s = make_batch(m, b, tokens, offsets.data(), P, 0, false, nullptr, nullptr))) return s;
    std::vector<int> cap(n, -1), lr(nl);
    for (size_t i = 0; i < nc; i++) cap[capture_rows[i]] = (int)i;
    for (size_t i = 0; i < nl; i++) lr[i] = (int)logit_rows[i];
    DITCH_CUDA(upload_vec(b.cap_slot, cap, dev->stream));
    DITCH_CUDA(upload_vec(b.logit_rows, lr, dev->stream));
    if ((s = forward_batch(m, b, (int)nc, (int)nl))) return s;
    const Config &c = m->cfg;
    if (nc) {
        // a row captured twice keeps one slot: fill duplicates from it
        std::vector<float> res((size_t)(c.n_layers + 1) * nc * c.hidden);
        DITCH_CUDA(cudaMemcpyAsync(res.data(), m->res.ptr, res.size() * 4, cudaMemcpyDeviceToHost, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        for (int l = 0; l <= c.n_layers; l++)
            for (size_t i = 0; i < nc; i++) {
                const int slot = cap[capture_rows[i]];
                memcpy(residuals + ((size_t)l * nc + i) * c.hidden, res.data() + ((size_t)l * nc + slot) * c.hidden,
                       (size_t)c.hidden * 4);
            }
    }
    if (nl) DITCH_CUDA(cudaMemcpyAsync(logits, m->logits.ptr, nl * (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, dev->stream));
    return check_status(dev, "forward");
}

int ditch_cuda_residual_sums(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets,
                             size_t n_prompts, size_t window, size_t batch_size, double *sums, uint64_t *count) {
    clear_error();
    REQUIRE(m && tokens && prompt_offsets && sums && count, "null argument");
    ditch_cuda_device *dev = m->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const Config &c = m->cfg;
    const size_t entries = c.n_layers + 1, H = c.hidden;
    const size_t w = std::max<size_t>(window, 1);
    const size_t bs = batch_size ? batch_size : std::max<size_t>(n_prompts, 1);
    DITCH_CUDA(m->sums.reserve(entries * H * 8));
    DITCH_CUDA(cudaMemsetAsync(m->sums.ptr, 0, entries * H * 8, dev->stream));
    DevBuf dfirst, dtake;
    int s;
    for (size_t start = 0; start < n_prompts; start += bs) {
        const size_t np = std::min(bs, n_prompts - start);
        std::vector<int> first, take;
        if ((s = make_batch(m, m->work, tokens, prompt_offsets + start, np, w, false, &first, &take))) return s;
        int nc = 0;
        for (int t : take) nc += t;
        if ((s = forward_batch(m, m->work, nc, 0))) return s;
        DITCH_CUDA(upload_vec(dfirst, first, dev->stream));
        DITCH_CUDA(upload_vec(dtake, take, dev->stream));
        DITCH_CUDA(m->sums_part.reserve(residual_scratch_bytes((int)entries, (int)H, (int)np)));
        DITCH_LAUNCH(dev, residual_sums(m->res.as<float>(), (int)entries, nc, (int)H, dfirst.as<int>(), dtake.as<int>(),
                                        (int)np, m->sums.as<double>(), m->sums_part.as<double>(), dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    }
    const size_t n = entries * H;
    std::vector<double> hs(n + 1);
    if (m->dp_group) {
        // data parallel: [sums, prompt count] summed over the group's ranks
        DITCH_CUDA(m->dp_buf.reserve((2 * n + 2) * 8));
        double *src = m->dp_buf.as<double>(), *dst = src + n + 1;
        const double np = (double)n_prompts;
        DITCH_CUDA(cudaMemcpyAsync(src, m->sums.ptr, n * 8, cudaMemcpyDeviceToDevice, dev->stream));
        DITCH_CUDA(cudaMemcpyAsync(src + n, &np, 8, cudaMemcpyHostToDevice, dev->stream));
        if ((s = dp_allreduce_sum(dev, m->dp_group, src, n + 1, dst))) return s;
        DITCH_CUDA(cudaMemcpyAsync(hs.data(), dst, (n + 1) * 8, cudaMemcpyDeviceToHost, dev->stream));
    } else {
        DITCH_CUDA(cudaMemcpyAsync(hs.data(), m->sums.ptr, n * 8, cudaMemcpyDeviceToHost, dev->stream));
        hs[n] = (double)n_prompts;
    }
    if ((s = check_status(dev, "residual_sums"))) return s;
    for (size_t i = 0; i < n; i++) sums[i] += hs[i];
    *count += (uint64_t)hs[n];
    return DITCH_CUDA_OK;
}

int ditch_cuda_directions(ditch_cuda_model *m, const double *good_sums, uint64_t good_count, const double *bad_sums,
                          uint64_t bad_count, int orthogonalize, float *dirs) {
    clear_error();
    REQUIRE(m && good_sums && bad_sums, "null argument");
    ditch_cuda_device *dev = m->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const Config &c = m->cfg;
    const size_t entries = c.n_layers + 1, H = c.hidden;
    DevBuf g, b;
    DITCH_CUDA(g.reserve(entries * H * 8));
    DITCH_CUDA(b.reserve(entries * H * 8));
    DITCH_CUDA(cudaMemcpyAsync(g.ptr, good_sums, entries * H * 8, cudaMemcpyHostToDevice, dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(b.ptr, bad_sums, entries * H * 8, cudaMemcpyHostToDevice, dev->stream));
    DITCH_LAUNCH(dev, directions_from_sums(g.as<double>(), (double)good_count, b.as<double>(), (double)bad_count,
                                           (int)entries, (int)H, orthogonalize, m->dirs.as<float>(), nullptr, nullptr,
                                           dev->stream));
    m->h_dirs.resize(entries * H);
    DITCH_CUDA(cudaMemcpyAsync(m->h_dirs.data(), m->dirs.ptr, entries * H * 4, cudaMemcpyDeviceToHost, dev->stream));
    int s = check_status(dev, "directions");
    if (s) return s;
    m->dir_entries = (int)entries;
    if (dirs) memcpy(dirs, m->h_dirs.data(), entries * H * 4);
    return DITCH_CUDA_OK;
}

int ditch_cuda_set_directions(ditch_cuda_model *m, const float *dirs, size_t entries) {
    clear_error();
    REQUIRE(m && dirs && entries > 0, "bad argument");
    ditch_cuda_device *dev = m->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const size_t H = m->cfg.hidden;
    DITCH_CUDA(m->dirs.reserve(entries * H * 4));
    DITCH_CUDA(cudaMemcpyAsync(m->dirs.ptr, dirs, entries * H * 4, cudaMemcpyHostToDevice, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    m->h_dirs.assign(dirs, dirs + entries * H);
    m->dir_entries = (int)entries;
    return DITCH_CUDA_OK;
}

int ditch_cuda_apply_edit(ditch_cuda_model *m, const ditch_cuda_params *attn_o, const ditch_cuda_params *mlp_down,
                          float direction_index, int use_direction_index) {
    clear_error();
    REQUIRE(m, "null model");
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    return edit_common(m, attn_o, mlp_down, direction_index, use_direction_index, false, 0, 1.0f);
}

int ditch_cuda_apply_expert_edit(ditch_cuda_model *m, const ditch_cuda_params *attn_o, const ditch_cuda_params *mlp_down,
                                 float direction_index, int use_direction_index, size_t n_experts, float strength) {
    clear_error();
    REQUIRE(m, "null model");
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    return edit_common(m, attn_o, mlp_down, direction_index, use_direction_index, true, n_experts, strength);
}

int ditch_cuda_reset_edits(ditch_cuda_model *m) {
    clear_error();
    REQUIRE(m, "null model");
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    clear_edits(m);
    return upload_expert_flags(m);
}

int ditch_cuda_rank_experts(ditch_cuda_model *m, size_t layer, const float *v, uint32_t *order, float *scores) {
    clear_error();
    REQUIRE(m && v, "null argument");
    REQUIRE(layer < (size_t)m->cfg.n_layers && m->layers[layer].moe, "layer %zu is not an MoE layer", layer);
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    DITCH_CUDA(cudaMemcpyAsync(m->vtmp.ptr, v, (size_t)m->cfg.hidden * 4, cudaMemcpyHostToDevice, m->dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(m->dev->stream));
    std::vector<float> s;
    int st = expert_scores(m, (int)layer, m->vtmp.as<float>(), s);
    if (st) return st;
    std::vector<uint32_t> o = rank(s);
    if (order) memcpy(order, o.data(), o.size() * 4);
    if (scores) memcpy(scores, s.data(), s.size() * 4);
    return DITCH_CUDA_OK;
}

int ditch_cuda_kl_init(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets, size_t n_prompts) {
    clear_error();
    REQUIRE(m && tokens && prompt_offsets && n_prompts > 0, "bad argument");
    ditch_cuda_device *dev = m->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    int s;
    if ((s = make_batch(m, m->kl, tokens, prompt_offsets, n_prompts, 0, true, nullptr, nullptr))) return s;
    m->kl_offsets.assign(prompt_offsets, prompt_offsets + n_prompts + 1);
    m->kl_tokens_host.assign(tokens + prompt_offsets[0], tokens + prompt_offsets[n_prompts]);
    // the baseline is the unedited model: suspend edits for this forward
    std::vector<std::array<bool, 2>> flags;
    for (Layer &L : m->layers) flags.push_back({L.o_edit, L.down_edit});
    std::vector<std::vector<uint8_t>> eflags;
    for (Layer &L : m->layers) eflags.push_back(L.e_edit);
    clear_edits(m);
    if ((s = upload_expert_flags(m))) return s;
    const int P = (int)n_prompts, V = m->cfg.vocab;
    s = forward_batch(m, m->kl, 0, P);
    for (size_t i = 0; i < m->layers.size(); i++) {
        m->layers[i].o_edit = flags[i][0];
        m->layers[i].down_edit = flags[i][1];
        m->layers[i].e_edit = eflags[i];
    }
    if (s) return s;
    if ((s = upload_expert_flags(m))) return s;
    DITCH_CUDA(m->kl_base.reserve((size_t)P * V * 4));
    DITCH_CUDA(m->kl_part.reserve(kl_scratch_bytes(P, V)));
    DITCH_LAUNCH(dev, log_softmax_rows(m->logits.as<float>(), P, V, m->kl_base.as<float>(), m->kl_part.ptr, dev->stream));
    if ((s = check_status(dev, "kl_init"))) return s;
    m->kl_ready = true;
    return DITCH_CUDA_OK;
}

int ditch_cuda_kl_score(ditch_cuda_model *m, double *kl) {
    clear_error();
    REQUIRE(m && kl, "null argument");
    REQUIRE(m->kl_ready, "ditch_cuda_kl_init has not run");
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    return kl_score_impl(m, kl);
}

int ditch_cuda_kl_score_prompts(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets,
                                size_t n_prompts, double *kl) {
    clear_error();
    REQUIRE(m && kl && tokens && prompt_offsets, "null argument");
    REQUIRE(m->kl_ready, "ditch_cuda_kl_init has not run");
    REQUIRE(n_prompts + 1 == m->kl_offsets.size(), "prompt count differs from ditch_cuda_kl_init");
    for (size_t i = 0; i <= n_prompts; i++)
        REQUIRE(prompt_offsets[i] - prompt_offsets[0] == m->kl_offsets[i] - m->kl_offsets[0],
                "prompt lengths differ from ditch_cuda_kl_init");
    std::lock_guard<std::mutex> lk(m->dev->mu);
    DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
    const size_t n = prompt_offsets[n_prompts] - prompt_offsets[0];
    DITCH_CUDA(cudaMemcpyAsync(m->kl.tokens.ptr, tokens + prompt_offsets[0], n * 4, cudaMemcpyHostToDevice,
                               m->dev->stream));
    return kl_score_impl(m, kl);
}

int ditch_cuda_set_row_normalization(ditch_cuda_model *m, int mode, size_t lora_rank, uint64_t seed) {
    clear_error();
    REQUIRE(m, "null model");
    REQUIRE(mode >= 0 && mode <= 2, "row normalisation %d is not none (0), pre (1) or full (2)", mode);
    if (mode == 2) {
        REQUIRE(lora_rank >= 1 && lora_rank <= (size_t)kMaxDeltaRank, "lora_rank %zu is not within 1..%d", lora_rank,
                kMaxDeltaRank);
    }
    std::lock_guard<std::mutex> lk(m->dev->mu);
    if (mode >= 1 && m->cfg.tp_world > 1) {
        // the shards' norms are summed over the group: every layer's now, in
        // one call that every rank makes, so no edit issues a collective
        DITCH_CUDA(cudaSetDevice(m->dev->ordinal));
        int s = DITCH_CUDA_OK;
        for (Layer &L : m->layers)
            if (!L.rn_valid && (s = compute_row_norms(m, L))) break;
        if (!s) s = check_status(m->dev, "set_row_normalization");
        settle_row_norms(m, s == DITCH_CUDA_OK);
        if (s) return s;
    }
    m->row_norm = mode;
    if (mode == 2) {
        m->lora_rank = (int)lora_rank;
        m->edit_seed = seed;
    }
    return DITCH_CUDA_OK;
}

int ditch_cuda_generate(ditch_cuda_model *m, const uint32_t *tokens, const size_t *prompt_offsets, size_t n_prompts,
                        size_t max_new_tokens, const uint32_t *eos_ids, size_t n_eos, uint32_t *out_tokens,
                        size_t *out_counts) {
    clear_error();
    REQUIRE(m && tokens && prompt_offsets && out_tokens && out_counts, "null argument");
    REQUIRE(n_prompts > 0 && n_prompts < (1u << 20), "bad prompt count %zu", n_prompts);
    REQUIRE(!n_eos || eos_ids, "null eos ids");
    ditch_cuda_device *dev = m->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const Config &c = m->cfg;
    // Expert parallelism: every rank generates for its own prompts, and every
    // MoE layer of every step exchanges rows with every rank, so all ranks
    // take the same number of decode steps: before each step they agree
    // whether any rank still has an active prompt, and a rank whose prompts
    // have all finished runs the step on one placeholder row (slot 0,
    // position 0, token 0; its cache entry and logits are never read).
    const bool ep = c.ep_world > 1;
    REQUIRE(!ep || m->group, "expert parallelism without a peer group (ditch_cuda_model_set_group)");
    const size_t P = n_prompts;
    size_t longest = 0;
    for (size_t p = 0; p < P; p++) {
        REQUIRE(prompt_offsets[p + 1] > prompt_offsets[p], "prompt %zu is empty", p);
        longest = std::max(longest, prompt_offsets[p + 1] - prompt_offsets[p]);
    }
    REQUIRE(longest + max_new_tokens <= (size_t)m->rope_len,
            "%zu prompt tokens plus %zu new ones exceed the %d positions the model was loaded for", longest,
            max_new_tokens, m->rope_len);
    // KvCache.initFor(model, prompts, longest + max_new + 1) (src/engine.zig:254-260)
    const size_t max_len = longest + max_new_tokens + 1;
    const size_t cache_bytes = (size_t)c.n_layers * P * max_len * c.kvd() * 4;
    DITCH_CUDA(m->kv_k.reserve(cache_bytes));
    DITCH_CUDA(m->kv_v.reserve(cache_bytes));
    DITCH_CUDA(m->gen_next.reserve(P * 4));
    m->kv_slots = (int)P;
    m->kv_len = (int)max_len;
    cudaStream_t st = dev->stream;
    const int V = c.vocab;
    int s;

    // prefill: the prompts' keys and values go to their slots, the last row
    // of every prompt gives the first token (src/model.zig:5292-5357)
    Batch &b = m->work;
    if ((s = make_batch(m, b, tokens, prompt_offsets, P, 0, true, nullptr, nullptr))) return s;
    std::vector<int> rb, rp;
    rb.reserve(b.n);
    rp.reserve(b.n);
    for (size_t p = 0; p < P; p++)
        for (int pos = 0; pos < b.h_len[p]; pos++) {
            rb.push_back((int)p);
            rp.push_back(pos);
        }
    DITCH_CUDA(upload_vec(b.row_b, rb, st));
    DITCH_CUDA(upload_vec(b.row_pos, rp, st));
    if ((s = forward_batch(m, b, 0, (int)P, kFwdPromptsCache))) return s;
    std::vector<uint32_t> next(P);
    DITCH_LAUNCH(dev, argmax_rows(m->logits.as<float>(), (int)P, V, m->gen_next.as<uint32_t>(), st));
    DITCH_CUDA(cudaMemcpyAsync(next.data(), m->gen_next.ptr, P * 4, cudaMemcpyDeviceToHost, st));
    DITCH_CUDA(cudaStreamSynchronize(st));

    auto is_eos = [&](uint32_t t) {
        for (size_t e = 0; e < n_eos; e++)
            if (eos_ids[e] == t) return true;
        return false;
    };
    const size_t stride = std::max<size_t>(max_new_tokens, 1);
    std::vector<size_t> pos(P), count(P, 1);
    std::vector<char> active(P, 0);
    size_t n_active = 0;
    for (size_t i = 0; i < P; i++) {
        out_tokens[i * stride] = next[i];
        pos[i] = (size_t)b.h_len[i];
        if (!(is_eos(next[i]) || max_new_tokens <= 1 || pos[i] >= max_len)) {
            active[i] = 1;
            n_active++;
        }
    }
    // decode steps over the active prompts, one row each at its next position
    std::vector<uint32_t> toks;
    std::vector<int> lr;
    for (size_t step = 1; step < max_new_tokens; step++) {
        if (ep) {
            bool any = false;
            if ((s = ep_any_active(m, n_active, &any))) return s;
            if (!any) break;
        } else if (n_active == 0) {
            break;
        }
        toks.clear();
        rb.clear();
        rp.clear();
        lr.clear();
        for (size_t i = 0; i < P; i++) {
            if (!active[i]) continue;
            lr.push_back((int)toks.size());
            toks.push_back(out_tokens[i * stride + count[i] - 1]);
            rb.push_back((int)i);
            rp.push_back((int)pos[i]);
        }
        if (toks.empty()) {  // expert parallelism: the placeholder row
            lr.push_back(0);
            toks.push_back(0);
            rb.push_back(0);
            rp.push_back(0);
        }
        const int n = (int)toks.size();
        b.n = n;
        b.prompts = n;
        b.h_start.clear();
        b.h_len.clear();
        DITCH_CUDA(upload_vec(b.tokens, toks, st));
        DITCH_CUDA(upload_vec(b.row_b, rb, st));
        DITCH_CUDA(upload_vec(b.row_pos, rp, st));
        DITCH_CUDA(upload_vec(b.logit_rows, lr, st));
        if ((s = forward_batch(m, b, 0, n, kFwdDecode))) return s;
        DITCH_LAUNCH(dev, argmax_rows(m->logits.as<float>(), n, V, m->gen_next.as<uint32_t>(), st));
        DITCH_CUDA(cudaMemcpyAsync(next.data(), m->gen_next.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
        DITCH_CUDA(cudaStreamSynchronize(st));
        if (n_active == 0) continue;  // the placeholder's token is dropped
        int j = 0;
        for (size_t i = 0; i < P; i++) {
            if (!active[i]) continue;
            const uint32_t t = next[j++];
            pos[i]++;
            out_tokens[i * stride + count[i]++] = t;
            if (is_eos(t) || pos[i] >= max_len) {
                active[i] = 0;
                n_active--;
            }
        }
    }
    for (size_t i = 0; i < P; i++) out_counts[i] = count[i];
    return check_status(dev, "generate");
}

}  // extern "C"
