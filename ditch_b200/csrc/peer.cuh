// Peer groups: the GPUs of one node exchanging data through each other's
// memory over NVLink (CUDA IPC mappings), with flag-based signalling.
//
// Every rank allocates one region of the same layout and exports its IPC
// handle; the host exchanges the handles; each rank maps its peers' regions.
// An exchange is: kernels write into peers' regions (plain P2P stores), each
// writing thread ends with a system-scope fence, then `signal` stores this
// exchange's epoch into every peer's flag slot for this rank (release, system
// scope), and `wait` spins, bounded, until every peer's slot in this rank's
// own flags holds at least the epoch (acquire, system scope). Epochs only grow
// and every rank runs the same exchanges in the same order, so a fast peer
// that has already signalled a later exchange also satisfies the wait.
//
// Each kind of exchange has its own region and is single-buffered: a rank
// only writes exchange k + 1 into a peer after waiting on an exchange that the
// peer signals after it has finished reading exchange k (the callers' order
// guarantees it; see moe.cu). No TMA and no multicast touch peer memory.
#pragma once

#include "device.cuh"

namespace ditch {

constexpr int kMaxPeers = 8;

struct PeerPtrs {
    uint8_t *p[kMaxPeers];  // every rank's region base, mapped in this process (own rank included)
};

// Device-side helpers.
__device__ __forceinline__ void st_release_sys(uint64_t *addr, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *addr) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// Host side.
cudaError_t peer_signal(const PeerPtrs &pp, int rank, int world, uint64_t epoch, cudaStream_t st);
// Bounded: after about `budget_s` seconds without every peer's epoch the
// status word gets kKernelWaitTimeout and the kernel returns.
cudaError_t peer_wait(uint8_t *own, int world, uint64_t epoch, int *status, double budget_s, cudaStream_t st);

}  // namespace ditch

struct ditch_cuda_group {
    ditch_cuda_device *dev = nullptr;
    int rank = 0, world = 1;
    size_t bytes = 0;               // data bytes after the flag block
    uint8_t *base = nullptr;        // own region (flags, then data)
    ditch::PeerPtrs peers{};        // every rank's region in this process
    bool opened = false;
    uint64_t epoch = 0;             // last exchange started
    uint64_t dp_calls = 0;          // data-parallel reductions so far (their half of the region alternates)
    double wait_s = 30.0;           // budget of every wait of an exchange (ditch_cuda_group_set_wait_budget)
};

namespace ditch {
// Flag block at the head of every region: [kMaxPeers] u64, slot s written by rank s.
constexpr size_t kPeerFlagBytes = 256;
inline uint8_t *peer_data(uint8_t *region) { return region + kPeerFlagBytes; }

// One exchange on the device's stream: signal the next epoch to every peer,
// then wait (bounded by budget_s; then the status word reports a timeout)
// until every peer has signalled it.
int group_exchange(ditch_cuda_device *dev, ditch_cuda_group *g, double budget_s);

// Data-parallel reductions over a group (dp.cu), on the device's stream.
// dst[i] = sum over ranks, in rank order, of every rank's src[i] (device
// pointers, n doubles; the same bits on every rank).
int dp_allreduce_sum(ditch_cuda_device *dev, ditch_cuda_group *g, const double *src, size_t n, double *dst);
// out[0] = the sum of every rank's `count` values taken one after another in
// rank order, then in each rank's own order (the order one device would sum
// the concatenated prompts in); out[1] = the total count.
int dp_ordered_sum(ditch_cuda_device *dev, ditch_cuda_group *g, const double *vals, size_t count, double *out);
// Region bytes a group needs for dp_ordered_sum of `count` values.
size_t dp_ordered_bytes(size_t count);
}  // namespace ditch
