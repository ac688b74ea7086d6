// row_normalization = full (src/abliterate.zig:324-350, randomizedSvd
// 473-538): the edit W' = diag(n) rownorm(Wn + B A^T) of the row-normalised
// weight, as a low-rank delta found by a randomised SVD of the implicit
// operator D = W' - W = diag(c) W + d a^T, never materialised.
//
// The weight products run on the device over the stored format: D X uses the
// GEMM with X split into bf16 high and low parts (an f32-accurate product,
// about 2^-16 relative), D^T Y one GEMV-T per vector. The small dense steps
// (Gram-Schmidt, the q x q eigenproblem, the row coefficients) run on the
// host in f32 in the reference's order. The random test matrix is seeded
// (SplitMix64 and Box-Muller) but is not the reference's random sequence: the
// two sketches give the same delta up to the randomised SVD's accuracy.
//
// Under tensor parallelism a rank holds a column shard of the matrix (o_proj
// and down_proj are split by columns). The products over columns (W a, D X,
// a . x) are partial sums on each rank, summed over the group in rank order;
// the column-space vectors (a, the D^T Y sketches) are gathered whole, so
// Gram-Schmidt, the Gram matrices and the eigenproblem run on full vectors,
// the same on every rank; each rank keeps its columns of the delta's A and
// all of B. The random test matrix is drawn for all columns, so the sketch
// is the one a single GPU draws; the results agree with one GPU up to the
// order of the partial sums.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <vector>

#include "model.cuh"

namespace ditch {

namespace {

// f32 to bf16 bits, round to nearest even (finite inputs: the split of an
// orthonormal sketch).
uint16_t f32_to_bf16_host(float x) {
    uint32_t b;
    std::memcpy(&b, &x, 4);
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

// f32 dot product in eight interleaved partial sums (the shape of ditch's
// vector-lane dot, src/tensor.zig:550-558, and one the host compiler
// vectorises), then the partials in order and the tail.
float dotf(const float *a, const float *b, size_t n) {
    float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    size_t i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) p[l] += a[i + l] * b[i + l];
    float s = 0.0f;
    for (int l = 0; l < 8; l++) s += p[l];
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

void axpyf(float *y, float a, const float *x, size_t n) {
    for (size_t i = 0; i < n; i++) y[i] += a * x[i];
}

// Modified Gram-Schmidt with two passes, rows of `vecs` (orthonormalize,
// src/abliterate.zig:409-423).
void orthonormalize(std::vector<float> &vecs, int q, size_t n) {
    for (int i = 0; i < q; i++) {
        float *vi = vecs.data() + (size_t)i * n;
        for (int pass = 0; pass < 2; pass++)
            for (int j = 0; j < i; j++) {
                const float *vj = vecs.data() + (size_t)j * n;
                axpyf(vi, -dotf(vi, vj, n), vj, n);
            }
        const float nrm = std::sqrt(dotf(vi, vi, n));
        if (nrm > 1e-20f) {
            const float inv = 1.0f / nrm;
            for (size_t k = 0; k < n; k++) vi[k] *= inv;
        } else {
            std::fill(vi, vi + n, 0.0f);
        }
    }
}

// Cyclic Jacobi eigen-decomposition of the symmetric n x n matrix m (in
// place; eigenvalues on its diagonal), eigenvectors in the columns of vecs
// (jacobiEigen, src/abliterate.zig:427-470).
void jacobi_eigen(std::vector<float> &m, std::vector<float> &vecs, int n) {
    vecs.assign((size_t)n * n, 0.0f);
    for (int i = 0; i < n; i++) vecs[(size_t)i * n + i] = 1.0f;
    for (int sweep = 0; sweep < 50; sweep++) {
        double off = 0.0;
        for (int i = 0; i < n; i++)
            for (int j = 0; j < n; j++)
                if (i != j) off += (double)m[(size_t)i * n + j] * m[(size_t)i * n + j];
        if (off < 1e-18) break;
        for (int p = 0; p < n; p++)
            for (int qi = p + 1; qi < n; qi++) {
                const float apq = m[(size_t)p * n + qi];
                if (std::fabs(apq) < 1e-20f) continue;
                const float app = m[(size_t)p * n + p], aqq = m[(size_t)qi * n + qi];
                const float theta = (aqq - app) / (2.0f * apq);
                const float sg = theta > 0.0f ? 1.0f : theta < 0.0f ? -1.0f : 0.0f;
                const float t = sg / (std::fabs(theta) + std::sqrt(theta * theta + 1.0f));
                const float tf = theta == 0.0f ? 1.0f : t;
                const float cs = 1.0f / std::sqrt(tf * tf + 1.0f), sn = tf * cs;
                for (int k = 0; k < n; k++) {
                    const float akp = m[(size_t)k * n + p], akq = m[(size_t)k * n + qi];
                    m[(size_t)k * n + p] = cs * akp - sn * akq;
                    m[(size_t)k * n + qi] = sn * akp + cs * akq;
                }
                for (int k = 0; k < n; k++) {
                    const float apk = m[(size_t)p * n + k], aqk = m[(size_t)qi * n + k];
                    m[(size_t)p * n + k] = cs * apk - sn * aqk;
                    m[(size_t)qi * n + k] = sn * apk + cs * aqk;
                }
                for (int k = 0; k < n; k++) {
                    const float vkp = vecs[(size_t)k * n + p], vkq = vecs[(size_t)k * n + qi];
                    vecs[(size_t)k * n + p] = cs * vkp - sn * vkq;
                    vecs[(size_t)k * n + qi] = sn * vkp + cs * vkq;
                }
            }
    }
}

// Seeded standard normals: SplitMix64 then Box-Muller.
struct Normal {
    uint64_t s;
    bool have = false;
    float spare = 0.0f;
    uint64_t next() {
        uint64_t z = (s += 0x9e3779b97f4a7c15ull);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        return z ^ (z >> 31);
    }
    float operator()() {
        if (have) {
            have = false;
            return spare;
        }
        const double u1 = ((next() >> 11) + 1.0) * 0x1p-53, u2 = (next() >> 11) * 0x1p-53;
        const double r = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586 * u2;
        spare = (float)(r * std::sin(th));
        have = true;
        return (float)(r * std::cos(th));
    }
};

// The implicit operator D = diag(c) W + d a^T over rows [row0, row0 + rows)
// of a resident weight (DeltaOperator, src/abliterate.zig:355-400).
struct Operator {
    ditch_cuda_model *m;
    const Mat &w;
    int row0, rows, cols;
    const std::vector<float> &a, &c, &d;
    DevBuf &act, &out, &ybuf, &xbuf;  // the model's scratch (kept between matrices)

    // out[q][rows] = (D X)^T for x[q][cols]
    int apply(const std::vector<float> &x, int q, std::vector<float> &y) {
        ditch_cuda_device *dev = m->dev;
        std::vector<uint16_t> split((size_t)2 * q * cols);
        for (size_t i = 0; i < (size_t)q * cols; i++) {
            const uint16_t hi = f32_to_bf16_host(x[i]);
            const uint32_t hb = (uint32_t)hi << 16;
            float hf;
            std::memcpy(&hf, &hb, 4);
            split[i] = hi;
            split[(size_t)q * cols + i] = f32_to_bf16_host(x[i] - hf);
        }
        DITCH_CUDA(act.reserve(split.size() * 2));
        DITCH_CUDA(out.reserve((size_t)2 * q * rows * 4));
        DITCH_CUDA(cudaMemcpyAsync(act.ptr, split.data(), split.size() * 2, cudaMemcpyHostToDevice, dev->stream));
        int s;
        if ((s = gemm_mat(dev, w, row0, rows, act.as<uint16_t>(), 2 * q, out.ptr, rows, 0, nullptr, nullptr, nullptr, 0,
                          nullptr)))
            return s;
        std::vector<float> both((size_t)2 * q * rows);
        DITCH_CUDA(cudaMemcpyAsync(both.data(), out.ptr, both.size() * 4, cudaMemcpyDeviceToHost, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        y.assign((size_t)q * rows, 0.0f);
        for (int j = 0; j < q; j++) {
            float *o = y.data() + (size_t)j * rows;
            const float *h = both.data() + (size_t)j * rows, *l = both.data() + (size_t)(q + j) * rows;
            for (int i = 0; i < rows; i++) o[i] = (h[i] + l[i]) * c[i];
            axpyf(o, dotf(a.data(), x.data() + (size_t)j * cols, cols), d.data(), rows);
        }
        return DITCH_CUDA_OK;
    }

    // out[q][cols] = (D^T Y)^T for y[q][rows]
    int apply_t(const std::vector<float> &y, int q, std::vector<float> &x) {
        ditch_cuda_device *dev = m->dev;
        std::vector<float> cy((size_t)q * rows);
        for (int j = 0; j < q; j++)
            for (int i = 0; i < rows; i++) cy[(size_t)j * rows + i] = c[i] * y[(size_t)j * rows + i];
        DITCH_CUDA(ybuf.reserve(cy.size() * 4));
        DITCH_CUDA(xbuf.reserve((size_t)q * cols * 4));
        DITCH_CUDA(cudaMemcpyAsync(ybuf.ptr, cy.data(), cy.size() * 4, cudaMemcpyHostToDevice, dev->stream));
        int s;
        for (int j = 0; j < q; j++)
            if ((s = gemv_t_mat(m, w, row0, rows, ybuf.as<float>() + (size_t)j * rows, xbuf.as<float>() + (size_t)j * cols)))
                return s;
        x.assign((size_t)q * cols, 0.0f);
        DITCH_CUDA(cudaMemcpyAsync(x.data(), xbuf.ptr, x.size() * 4, cudaMemcpyDeviceToHost, dev->stream));
        DITCH_CUDA(cudaStreamSynchronize(dev->stream));
        for (int j = 0; j < q; j++)
            axpyf(x.data() + (size_t)j * cols, dotf(d.data(), y.data() + (size_t)j * rows, rows), a.data(), cols);
        return DITCH_CUDA_OK;
    }
};

// Tensor-parallel helpers: the sum of every rank's `v` in rank order (f32
// widened to f64 for the group's reduction, the same bits on every rank),
// and the concatenation of every rank's column slice.
int tp_sum(ditch_cuda_model *m, std::vector<float> &v) {
    ditch_cuda_device *dev = m->dev;
    std::vector<double> h(v.begin(), v.end());
    DITCH_CUDA(m->fn_red.reserve(2 * h.size() * 8));
    double *src = m->fn_red.as<double>(), *dst = src + h.size();
    DITCH_CUDA(cudaMemcpyAsync(src, h.data(), h.size() * 8, cudaMemcpyHostToDevice, dev->stream));
    int s;
    if ((s = dp_allreduce_sum(dev, m->group, src, h.size(), dst))) return s;
    DITCH_CUDA(cudaMemcpyAsync(h.data(), dst, h.size() * 8, cudaMemcpyDeviceToHost, dev->stream));
    if ((s = check_status(dev, "tensor-parallel full normalisation"))) return s;
    for (size_t i = 0; i < v.size(); i++) v[i] = (float)h[i];
    return DITCH_CUDA_OK;
}

// local [q][cols] (columns [rank cols, (rank + 1) cols) of the whole) to
// full [q][world cols]
int tp_gather(ditch_cuda_model *m, const std::vector<float> &local, int q, int cols, std::vector<float> &full) {
    const int W = m->cfg.tp_world, r = m->cfg.tp_rank;
    full.assign((size_t)q * cols * W, 0.0f);
    for (int j = 0; j < q; j++)
        std::memcpy(&full[((size_t)j * W + r) * cols], &local[(size_t)j * cols], (size_t)cols * 4);
    return tp_sum(m, full);
}

void tp_slice(const std::vector<float> &full, int q, int cols, int W, int r, std::vector<float> &local) {
    local.resize((size_t)q * cols);
    for (int j = 0; j < q; j++)
        std::memcpy(&local[(size_t)j * cols], &full[((size_t)j * W + r) * cols], (size_t)cols * 4);
}

}  // namespace

int full_norm_delta(ditch_cuda_model *m, const Mat &w, int row0, const float *rn, const float *v_dev, float lambda,
                    int lora_rank, uint64_t seed, float *a_out, float *b_out, int *rank_out) {
    ditch_cuda_device *dev = m->dev;
    const int rows = m->cfg.hidden, cols = w.cols;
    const bool tp = m->cfg.tp_world > 1;
    const int W = tp ? m->cfg.tp_world : 1, tr = tp ? m->cfg.tp_rank : 0, cols_all = cols * W;
    int s;
    if (tp) {
        if (!m->group) {
            set_error("tensor-parallel model without its peer group");
            return DITCH_CUDA_INVALID;
        }
        // every peer has finished reading the region (the forward's last reduction)
        if ((s = group_exchange(dev, m->group, m->group->wait_s))) return s;
    }
    // a = (v / n)^T W on the device, then n, v, a on the host
    DITCH_CUDA(m->vn.reserve((size_t)rows * 4));
    DevBuf &scratch = m->fn_s, &adev = m->fn_a;
    DITCH_CUDA(scratch.reserve((size_t)rows * 4));
    DITCH_CUDA(adev.reserve((size_t)cols * 4));
    DITCH_LAUNCH(dev, prenorm_vec(v_dev, rn, lambda, rows, m->vn.as<float>(), scratch.as<float>(), dev->stream));
    if ((s = gemv_t_mat(m, w, row0, rows, m->vn.as<float>(), adev.as<float>()))) return s;
    std::vector<float> n(rows), v(rows), a(cols);
    DITCH_CUDA(cudaMemcpyAsync(n.data(), rn, (size_t)rows * 4, cudaMemcpyDeviceToHost, dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(v.data(), v_dev, (size_t)rows * 4, cudaMemcpyDeviceToHost, dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(a.data(), adev.ptr, (size_t)cols * 4, cudaMemcpyDeviceToHost, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    // wa = W a (through the operator with c = 1, d = 0), gram = a . a
    std::vector<float> ones(rows, 1.0f), zeros(rows, 0.0f), c(rows), d(rows);
    std::vector<float> wa, a_all;
    {
        Operator plain{m, w, row0, rows, cols, a, ones, zeros, m->fn_act, m->fn_out, m->fn_y, m->fn_x};
        if ((s = plain.apply(a, 1, wa))) return s;
    }
    if (tp) {
        if ((s = tp_sum(m, wa))) return s;
        if ((s = tp_gather(m, a, 1, cols, a_all))) return s;
    }
    const std::vector<float> &af = tp ? a_all : a;
    const float gram = dotf(af.data(), af.data(), cols_all);
    for (int i = 0; i < rows; i++) {
        const float bij = -lambda * v[i];
        const float wn_dot_a = n[i] > 0.0f ? wa[i] / n[i] : 0.0f;
        float s2 = 1.0f;
        s2 += 2.0f * bij * wn_dot_a;
        s2 += bij * (-lambda * v[i]) * gram;
        const float sq = std::sqrt(std::max(s2, 1e-12f));
        c[i] = 1.0f / sq - 1.0f;
        d[i] = n[i] * (-lambda * v[i]) / sq;
    }
    // randomised SVD of D (q sketch vectors, 6 power iterations)
    const int r = std::max(lora_rank, 1);
    const int q = std::min(2 * r + 4, std::min(rows, cols_all));
    Operator op{m, w, row0, rows, cols, a, c, d, m->fn_act, m->fn_out, m->fn_y, m->fn_x};
    Normal rng{seed};
    std::vector<float> omega((size_t)q * cols_all), qy, qx, bt, full;
    for (float &x : omega) x = rng();
    // D X over this rank's columns, summed over the group
    auto apply = [&](const std::vector<float> &x_all, std::vector<float> &y) -> int {
        int st;
        if (!tp) return op.apply(x_all, q, y);
        std::vector<float> x;
        tp_slice(x_all, q, cols, W, tr, x);
        if ((st = op.apply(x, q, y))) return st;
        return tp_sum(m, y);
    };
    // D^T Y, this rank's columns gathered whole
    auto apply_t = [&](const std::vector<float> &y, std::vector<float> &x_all) -> int {
        int st;
        if (!tp) return op.apply_t(y, q, x_all);
        std::vector<float> x;
        if ((st = op.apply_t(y, q, x))) return st;
        return tp_gather(m, x, q, cols, x_all);
    };
    if ((s = apply(omega, qy))) return s;
    orthonormalize(qy, q, rows);
    for (int it = 0; it < 6; it++) {
        if ((s = apply_t(qy, qx))) return s;
        orthonormalize(qx, q, cols_all);
        if ((s = apply(qx, qy))) return s;
        orthonormalize(qy, q, rows);
    }
    if ((s = apply_t(qy, bt))) return s;  // B^T = D^T Q
    std::vector<float> bbt((size_t)q * q), evecs;
    for (int i = 0; i < q; i++)
        for (int j = 0; j < q; j++)
            bbt[(size_t)i * q + j] = dotf(&bt[(size_t)i * cols_all], &bt[(size_t)j * cols_all], cols_all);
    jacobi_eigen(bbt, evecs, q);
    std::vector<int> order(q);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int x, int y) { return bbt[(size_t)x * q + x] > bbt[(size_t)y * q + y]; });
    const int rank = std::min(r, q);
    std::vector<float> la((size_t)rank * cols_all, 0.0f), lb((size_t)rows * rank, 0.0f), uk(rows), vk(cols_all);
    for (int k = 0; k < rank; k++) {
        const int src = order[k];
        const float sk = std::sqrt(std::max(bbt[(size_t)src * q + src], 0.0f));
        std::fill(uk.begin(), uk.end(), 0.0f);
        std::fill(vk.begin(), vk.end(), 0.0f);
        for (int i = 0; i < q; i++) {
            axpyf(uk.data(), evecs[(size_t)i * q + src], &qy[(size_t)i * rows], rows);
            axpyf(vk.data(), evecs[(size_t)i * q + src], &bt[(size_t)i * cols_all], cols_all);
        }
        if (sk > 1e-12f) {
            const float inv = 1.0f / sk;
            for (float &x : vk) x *= inv;
        } else {
            std::fill(vk.begin(), vk.end(), 0.0f);
        }
        const float sq = std::sqrt(std::max(sk, 0.0f));
        for (int j = 0; j < cols_all; j++) la[(size_t)k * cols_all + j] = sq * vk[j];
        for (int i = 0; i < rows; i++) lb[(size_t)i * rank + k] = uk[i] * sq;
    }
    if (tp) {
        std::vector<float> mine;
        tp_slice(la, rank, cols, W, tr, mine);
        la.swap(mine);
        // every peer has finished reading the region before the next forward writes it
        if ((s = group_exchange(dev, m->group, m->group->wait_s))) return s;
    }
    DITCH_CUDA(cudaMemcpyAsync(a_out, la.data(), la.size() * 4, cudaMemcpyHostToDevice, dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(b_out, lb.data(), lb.size() * 4, cudaMemcpyHostToDevice, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    *rank_out = rank;
    return DITCH_CUDA_OK;
}

}  // namespace ditch
