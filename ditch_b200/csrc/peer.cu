// Peer groups over CUDA IPC mappings: allocation and handle export, opening
// the peers' regions, and the signal / bounded-wait kernels of an exchange.
#include "peer.cuh"

#include <cstring>
#include <memory>

using namespace ditch;

namespace {

#define REQUIRE(cond, ...)             \
    do {                               \
        if (!(cond)) {                 \
            set_error(__VA_ARGS__);    \
            return DITCH_CUDA_INVALID; \
        }                              \
    } while (0)

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Thread s < world stores `epoch` into rank s's flag slot for `rank`.
__global__ void k_peer_signal(PeerPtrs pp, int rank, int world, uint64_t epoch) {
    const int s = threadIdx.x;
    if (s >= world) return;
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint64_t *>(pp.p[s]) + rank, epoch);
}

// Thread s < world waits until this rank's slot s holds at least `epoch`.
// Once a wait of the current call has run out (the status word says so),
// the later waits of that call return at once: the call fails anyway.
__global__ void k_peer_wait(uint8_t *own, int world, uint64_t epoch, int *status, uint64_t budget_ns) {
    const int s = threadIdx.x;
    if (s >= world) return;
    if (status && *reinterpret_cast<volatile int *>(status) == kKernelWaitTimeout) return;
    const uint64_t *flag = reinterpret_cast<const uint64_t *>(own) + s;
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys(flag) < epoch) {
        if (global_ns() - t0 > budget_ns) {
            if (status) atomicExch(status, kKernelWaitTimeout);
            return;
        }
        __nanosleep(200);
    }
    __threadfence_system();
}

}  // namespace

namespace ditch {

cudaError_t peer_signal(const PeerPtrs &pp, int rank, int world, uint64_t epoch, cudaStream_t st) {
    k_peer_signal<<<1, 32, 0, st>>>(pp, rank, world, epoch);
    return cudaGetLastError();
}

cudaError_t peer_wait(uint8_t *own, int world, uint64_t epoch, int *status, double budget_s, cudaStream_t st) {
    k_peer_wait<<<1, 32, 0, st>>>(own, world, epoch, status, (uint64_t)(budget_s * 1e9));
    return cudaGetLastError();
}

int group_exchange(ditch_cuda_device *dev, ditch_cuda_group *g, double budget_s) {
    const uint64_t ep = ++g->epoch;
    DITCH_LAUNCH(dev, peer_signal(g->peers, g->rank, g->world, ep, dev->stream));
    DITCH_LAUNCH(dev, peer_wait(g->base, g->world, ep, dev->status, budget_s, dev->stream));
    return DITCH_CUDA_OK;
}

}  // namespace ditch

extern "C" {

size_t ditch_cuda_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int ditch_cuda_group_create(ditch_cuda_device *dev, int rank, int world, size_t bytes, ditch_cuda_group **out,
                            void *handle) {
    clear_error();
    REQUIRE(dev && out && handle, "null argument");
    REQUIRE(world >= 1 && world <= kMaxPeers, "world must be 1..%d", kMaxPeers);
    REQUIRE(rank >= 0 && rank < world, "rank out of range");
    *out = nullptr;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    std::unique_ptr<ditch_cuda_group> g(new ditch_cuda_group());
    g->dev = dev;
    g->rank = rank;
    g->world = world;
    g->bytes = bytes;
    void *p = nullptr;
    DITCH_CUDA(cudaMalloc(&p, kPeerFlagBytes + bytes));
    g->base = static_cast<uint8_t *>(p);
    DITCH_CUDA(cudaMemset(g->base, 0, kPeerFlagBytes));
    DITCH_CUDA(cudaDeviceSynchronize());
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, g->base);
    if (e != cudaSuccess) {
        cudaFree(g->base);
        return cuda_status(e, "cudaIpcGetMemHandle");
    }
    std::memcpy(handle, &h, sizeof(h));
    for (int s = 0; s < kMaxPeers; s++) g->peers.p[s] = nullptr;
    g->peers.p[rank] = g->base;
    *out = g.release();
    return DITCH_CUDA_OK;
}

int ditch_cuda_group_open(ditch_cuda_group *g, const void *handles) {
    clear_error();
    REQUIRE(g && handles, "null argument");
    REQUIRE(!g->opened, "group already opened");
    ditch_cuda_device *dev = g->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    for (int s = 0; s < g->world; s++) {
        if (s == g->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hb + (size_t)s * sizeof(h), sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle (peer rank)");
        g->peers.p[s] = static_cast<uint8_t *>(p);
    }
    g->opened = true;
    return DITCH_CUDA_OK;
}

void ditch_cuda_group_free(ditch_cuda_group *g) {
    if (!g) return;
    ditch_cuda_device *dev = g->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    cudaSetDevice(dev->ordinal);
    cudaStreamSynchronize(dev->stream);
    for (int s = 0; s < g->world; s++)
        if (s != g->rank && g->peers.p[s]) cudaIpcCloseMemHandle(g->peers.p[s]);
    if (g->base) cudaFree(g->base);
    delete g;
}

int ditch_cuda_group_barrier(ditch_cuda_group *g) {
    clear_error();
    REQUIRE(g && g->opened, "group not opened");
    ditch_cuda_device *dev = g->dev;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const uint64_t ep = ++g->epoch;
    DITCH_LAUNCH(dev, peer_signal(g->peers, g->rank, g->world, ep, dev->stream));
    DITCH_LAUNCH(dev, peer_wait(g->base, g->world, ep, dev->status, g->wait_s, dev->stream));
    DITCH_CUDA(cudaStreamSynchronize(dev->stream));
    return check_status(dev, "group barrier");
}

int ditch_cuda_group_set_wait_budget(ditch_cuda_group *g, double seconds) {
    clear_error();
    REQUIRE(g, "null group");
    REQUIRE(seconds > 0.0 && seconds <= 600.0, "wait budget %g s is not within (0, 600]", seconds);
    g->wait_s = seconds;
    return DITCH_CUDA_OK;
}

}  // extern "C"
