// Data parallelism over a peer group: every rank evaluates its own prompts
// with the same weights and edits, and the prompt-indexed results are
// combined over the group on the device's stream, with no host transport.
// ditch sums the residuals of every prompt (src/engine.zig:383-435) and the
// per-prompt KL in prompt order (src/scorers.zig:385-400); over a group the
// prompts are the concatenation of the ranks' prompts in rank order.
//
// A reduction writes this rank's values into its own region, runs one
// exchange (signal + bounded wait, peer.cu), and every rank then reads every
// rank's values over NVLink and adds them in rank order, so all ranks get
// the same bits. The data area is split in two halves used by alternate
// reductions: a rank only rewrites a half after an exchange that every peer
// signals once it has finished reading that half (the reduction in between),
// so one exchange per reduction suffices.
#include <algorithm>

#include "model.cuh"

namespace ditch {
namespace {

__device__ __forceinline__ const double *rank_half(const PeerPtrs &pp, int r, size_t half_off) {
    return reinterpret_cast<const double *>(pp.p[r] + kPeerFlagBytes + half_off);
}

__global__ void k_dp_sum(PeerPtrs pp, int world, size_t half_off, long long n, double *out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        double s = 0.0;
        for (int r = 0; r < world; r++) s += rank_half(pp, r, half_off)[i];
        out[i] = s;
    }
}

__global__ void k_dp_put(double *dst, const double *vals, long long count) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i <= count; i += (long long)gridDim.x * blockDim.x)
        dst[i] = i == 0 ? (double)count : vals[i - 1];
}

// One block: each rank's block [count, v0, v1, ...] is staged through shared
// memory (coalesced loads over NVLink) and thread 0 adds the values one by
// one, ranks in order.
constexpr int kOrderedChunk = 1024;

__global__ void __launch_bounds__(256) k_dp_ordered_sum(PeerPtrs pp, int world, size_t half_off, double *out) {
    __shared__ double sh[kOrderedChunk];
    double total = 0.0, n = 0.0;
    for (int r = 0; r < world; r++) {
        const double *src = rank_half(pp, r, half_off);
        const long long c = (long long)src[0];
        for (long long base = 0; base < c; base += kOrderedChunk) {
            const int len = (int)min((long long)kOrderedChunk, c - base);
            for (int j = threadIdx.x; j < len; j += blockDim.x) sh[j] = src[1 + base + j];
            __syncthreads();
            if (threadIdx.x == 0)
                for (int j = 0; j < len; j++) total += sh[j];
            __syncthreads();
        }
        n += (double)c;
    }
    if (threadIdx.x == 0) {
        out[0] = total;
        out[1] = n;
    }
}

size_t half_bytes(const ditch_cuda_group *g) { return (g->bytes / 2) & ~(size_t)255; }

}  // namespace

size_t dp_ordered_bytes(size_t count) { return 2 * (((count + 1) * 8 + 255) & ~(size_t)255); }

int dp_allreduce_sum(ditch_cuda_device *dev, ditch_cuda_group *g, const double *src, size_t n, double *dst) {
    const size_t cap = half_bytes(g) / 8;
    if (cap == 0) {
        set_error("the peer group's region (%zu bytes) is too small for a reduction", g->bytes);
        return DITCH_CUDA_INVALID;
    }
    cudaStream_t st = dev->stream;
    int s;
    for (size_t off = 0; off < n; off += cap) {
        const size_t len = std::min(cap, n - off);
        const size_t half_off = (g->dp_calls++ & 1) * half_bytes(g);
        DITCH_CUDA(cudaMemcpyAsync(peer_data(g->base) + half_off, src + off, len * 8, cudaMemcpyDeviceToDevice, st));
        if ((s = group_exchange(dev, g, g->wait_s))) return s;
        const int grid = (int)std::min<size_t>((len + 255) / 256, (size_t)dev->sms * 2);
        k_dp_sum<<<std::max(grid, 1), 256, 0, st>>>(g->peers, g->world, half_off, (long long)len, dst + off);
        DITCH_LAUNCH(dev, cudaGetLastError());
    }
    return DITCH_CUDA_OK;
}

int dp_ordered_sum(ditch_cuda_device *dev, ditch_cuda_group *g, const double *vals, size_t count, double *out) {
    if (dp_ordered_bytes(count) > g->bytes) {
        set_error("the peer group's region (%zu bytes) is too small for %zu values (needs %zu)", g->bytes, count,
                  dp_ordered_bytes(count));
        return DITCH_CUDA_INVALID;
    }
    cudaStream_t st = dev->stream;
    const size_t half_off = (g->dp_calls++ & 1) * half_bytes(g);
    double *own = reinterpret_cast<double *>(peer_data(g->base) + half_off);
    const int grid = (int)std::min<size_t>((count + 256) / 256, (size_t)dev->sms);
    k_dp_put<<<std::max(grid, 1), 256, 0, st>>>(own, vals, (long long)count);
    DITCH_LAUNCH(dev, cudaGetLastError());
    int s;
    if ((s = group_exchange(dev, g, g->wait_s))) return s;
    k_dp_ordered_sum<<<1, 256, 0, st>>>(g->peers, g->world, half_off, out);
    DITCH_LAUNCH(dev, cudaGetLastError());
    return DITCH_CUDA_OK;
}

}  // namespace ditch

using namespace ditch;

namespace {
#define REQUIRE(cond, ...)             \
    do {                               \
        if (!(cond)) {                 \
            set_error(__VA_ARGS__);    \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)
}  // namespace

extern "C" {

size_t ditch_cuda_model_dp_group_bytes(const ditch_cuda_model *m, size_t max_prompts) {
    if (!m) return 0;
    const size_t sums = 2 * (((1 + (size_t)(m->cfg.n_layers + 1) * m->cfg.hidden) * 8 + 255) & ~(size_t)255);
    return std::max(sums, dp_ordered_bytes(max_prompts));
}

int ditch_cuda_model_set_dp_group(ditch_cuda_model *m, ditch_cuda_group *g) {
    clear_error();
    REQUIRE(m, "null model");
    std::lock_guard<std::mutex> lk(m->dev->mu);
    if (g) {
        REQUIRE(g->opened, "group not opened");
        REQUIRE(g->dev == m->dev, "the group belongs to another device handle");
        REQUIRE(g != m->group, "the data-parallel group must not be the model's tensor- or expert-parallel group");
        REQUIRE(g->bytes >= 2 * 256, "the group's region is too small (ditch_cuda_model_dp_group_bytes)");
    }
    m->dp_group = g;
    return DITCH_CUDA_OK;
}

int ditch_cuda_group_allreduce_f64(ditch_cuda_group *g, double *data, size_t n) {
    clear_error();
    REQUIRE(g && (data || n == 0), "null argument");
    REQUIRE(g->opened, "group not opened");
    if (n == 0) return DITCH_CUDA_OK;
    ditch_cuda_device *dev = g->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(dev->bx.reserve(n * 8));
    DITCH_CUDA(dev->bo.reserve(n * 8));
    DITCH_CUDA(cudaMemcpyAsync(dev->bx.ptr, data, n * 8, cudaMemcpyHostToDevice, dev->stream));
    int s;
    if ((s = dp_allreduce_sum(dev, g, dev->bx.as<double>(), n, dev->bo.as<double>()))) return s;
    DITCH_CUDA(cudaMemcpyAsync(data, dev->bo.ptr, n * 8, cudaMemcpyDeviceToHost, dev->stream));
    return check_status(dev, "group_allreduce_f64");
}

}  // extern "C"
