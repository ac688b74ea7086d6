// Tensor parallelism: the all-reduce of the row-parallel o_proj / down_proj
// partial sums over the model's peer group, in two exchanges and without any
// copy of the partials:
//   1. every rank's GEMM writes its partial [n][H] f32 into its own region
//      (the `send` rows); exchange;
//   2. rank r sums chunk r of every rank's send rows, reading the peers' over
//      NVLink, in rank order (so every element has one well-defined sum), into
//      its own `red` rows; exchange;
//   3. every rank adds all chunks of the peers' red rows into its residual
//      stream x (the same values on every rank).
// Reuse is safe single-buffered: a rank rewrites its send rows only after
// the second exchange of the previous all-reduce (every peer has finished
// reading them), and its red rows only after the first exchange of the next
// one (every peer has finished step 3 of the previous).
#include "model.cuh"

namespace ditch {

namespace {

inline size_t align256(size_t x) { return (x + 255) / 256 * 256; }

__global__ void k_tp_reduce(PeerPtrs pp, int world, int rank, size_t send_off, size_t red_off, long long total4,
                            long long chunk4) {
    const long long c0 = (long long)rank * chunk4, c1 = min(total4, c0 + chunk4);
    float4 *red = reinterpret_cast<float4 *>(pp.p[rank] + kPeerFlagBytes + red_off);
    for (long long i = c0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < c1;
         i += (long long)gridDim.x * blockDim.x) {
        float4 a = reinterpret_cast<const float4 *>(pp.p[0] + kPeerFlagBytes + send_off)[i];
        for (int s = 1; s < world; s++) {
            const float4 b = reinterpret_cast<const float4 *>(pp.p[s] + kPeerFlagBytes + send_off)[i];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        red[i] = a;
    }
    __threadfence_system();
}

__global__ void k_tp_gather_add(PeerPtrs pp, size_t red_off, long long total4, long long chunk4, float4 *x) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total4;
         i += (long long)gridDim.x * blockDim.x) {
        const int owner = (int)(i / chunk4);
        const float4 r = reinterpret_cast<const float4 *>(pp.p[owner] + kPeerFlagBytes + red_off)[i];
        float4 v = x[i];
        v.x += r.x;
        v.y += r.y;
        v.z += r.z;
        v.w += r.w;
        x[i] = v;
    }
}

__global__ void k_square(const float *x, float *y, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) y[i] = x[i] * x[i];
}

__global__ void k_sqrt(float *x, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] = sqrtf(x[i]);
}

}  // namespace

// Row norms of a row-parallel weight (o_proj, down_proj: each rank holds a
// column shard of every row): the shard's norms, squared, summed over the
// ranks, then the root. Every rank of the group calls this in the same order.
int tp_row_norms(ditch_cuda_model *m, const Mat &w, float *out) {
    ditch_cuda_device *dev = m->dev;
    const int H = m->cfg.hidden;
    int s;
    if ((s = mat_row_norms(dev, w, 0, H, out))) return s;
    if (m->cfg.tp_world <= 1) return DITCH_CUDA_OK;
    if (!m->group || H % 4) {
        set_error("row norms of a tensor-parallel model need its peer group (and hidden a multiple of 4)");
        return DITCH_CUDA_INVALID;
    }
    const int grid = std::min((H + 255) / 256, 4 * dev->sms);
    k_square<<<grid, 256, 0, dev->stream>>>(out, tp_send_rows(m), H);
    DITCH_LAUNCH(dev, cudaGetLastError());
    DITCH_CUDA(cudaMemsetAsync(out, 0, (size_t)H * 4, dev->stream));
    if ((s = tp_allreduce_add(m, 1, out))) return s;
    k_sqrt<<<grid, 256, 0, dev->stream>>>(out, H);
    DITCH_LAUNCH(dev, cudaGetLastError());
    return DITCH_CUDA_OK;
}

size_t tp_group_bytes(const Config &c, size_t max_tokens) {
    return 2 * align256(max_tokens * (size_t)c.hidden * 4);
}

float *tp_send_rows(ditch_cuda_model *m) { return reinterpret_cast<float *>(peer_data(m->group->base)); }

int tp_allreduce_add(ditch_cuda_model *m, int n, float *x) {
    ditch_cuda_device *dev = m->dev;
    ditch_cuda_group *g = m->group;
    cudaStream_t st = dev->stream;
    const size_t send_off = 0, red_off = align256(m->group_tokens * (size_t)m->cfg.hidden * 4);
    const long long total4 = (long long)n * m->cfg.hidden / 4;
    const long long chunk4 = (total4 + g->world - 1) / g->world;
    int s;
    if ((s = group_exchange(dev, g, g->wait_s))) return s;
    const int grid = (int)std::min<long long>((chunk4 + 255) / 256, 2 * dev->sms);
    k_tp_reduce<<<std::max(grid, 1), 256, 0, st>>>(g->peers, g->world, g->rank, send_off, red_off, total4, chunk4);
    DITCH_LAUNCH(dev, cudaGetLastError());
    if ((s = group_exchange(dev, g, g->wait_s))) return s;
    const int grid2 = (int)std::min<long long>((total4 + 255) / 256, 4 * dev->sms);
    k_tp_gather_add<<<std::max(grid2, 1), 256, 0, st>>>(g->peers, red_off, total4, chunk4,
                                                         reinterpret_cast<float4 *>(x));
    DITCH_LAUNCH(dev, cudaGetLastError());
    return DITCH_CUDA_OK;
}

}  // namespace ditch
