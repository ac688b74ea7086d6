// Internal state of a device handle and shared host-side helpers of the
// C ABI (include/ditch_cuda.h).
#pragma once

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/ditch_cuda.h"
#include "gemm.cuh"
#include "kernels.cuh"

namespace ditch {

// Thread-local text of the last failure (ditch_cuda_last_error).
void set_error(const char *fmt, ...);
void clear_error();

// A growable device allocation.
struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    DevBuf(DevBuf &&o) noexcept : ptr(o.ptr), bytes(o.bytes) {
        o.ptr = nullptr;
        o.bytes = 0;
    }
    DevBuf &operator=(DevBuf &&o) noexcept {
        if (this != &o) {
            release();
            ptr = o.ptr;
            bytes = o.bytes;
            o.ptr = nullptr;
            o.bytes = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
    // Ensures at least n bytes (contents are not kept on growth).
    cudaError_t reserve(size_t n) {
        if (n <= bytes) return cudaSuccess;
        release();
        cudaError_t e = cudaMalloc(&ptr, n < 256 ? 256 : n);
        if (e == cudaSuccess) bytes = n < 256 ? 256 : n;
        return e;
    }
    template <class T>
    T *as() const { return static_cast<T *>(ptr); }
};

// One resident weight tile of the per-op seam (compute.Residency entry).
struct ResidentTile {
    uint64_t sig;
    size_t bytes;
    uint64_t used_at;
    void *split;     // split-bf16 GEMM operand [rows][kseg * cp]
    void *f32;       // decoded f32 copy for GEMV-T / row norms (may be null)
};

struct GemmEvent {
    cudaEvent_t start, stop;
    double flops;
};

}  // namespace ditch

struct ditch_cuda_device {
    int ordinal = 0;
    int sms = 148;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    uint64_t budget = 0;
    bool weights_stable = false;
    std::atomic<uint64_t> served{0};
    std::atomic<uint64_t> launches{0};
    int *status = nullptr;  // device status word written by kernels
    // residency cache, keyed by (host address, length)
    std::unordered_map<std::string, ditch::ResidentTile> tiles;
    uint64_t used_bytes = 0, clock = 0;
    // per-op scratch
    ditch::DevBuf bx, bw, bo, by, braw;
    // staged decode: quantised weights of GEMMs with at least this many tokens
    // are decoded once to bf16 here and multiplied by the bf16 GEMM (0 = never)
    ditch::DevBuf stage;
    ditch::DevBuf sk_ws, sk_cnt;  // stream-K partial sums and per-tile arrival counters
    long long sk_tiles = 0;      // counters zeroed so far
    int stage_min_tokens = 1024;
    bool deterministic = false;  // K splits summed in a fixed order (no atomics)
    bool decode_cache = true;    // staged GEMMs keep their weight's bf16 copy
    bool f32_split = false;      // models loaded next run f32-level split-bf16 products
    int cta_pairs = 2;           // wide dense bf16 GEMMs on CTA pairs (cta_group::2): 1 single-accumulator, 2 + SwiGLU
    int attn_tc = 2;             // prefill attention on tcgen05: 0 off, 1 one CTA per item, 2 two per SM (<= 64 tokens)
    // profiling of GEMMs
    bool profiling = false;
    std::vector<ditch::GemmEvent> events;
    size_t n_events = 0;
    double gemm_ms_done = 0.0, gemm_flops_done = 0.0;
    uint64_t gemm_launches = 0;
    cudaEvent_t t0 = nullptr, t1 = nullptr;
};

namespace ditch {

// Maps a CUDA error to a status code and records its text.
int cuda_status(cudaError_t e, const char *what);

// Launch bookkeeping: counts a kernel launch and converts errors.
#define DITCH_LAUNCH(dev, expr)                                   \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        (dev)->launches.fetch_add(1, std::memory_order_relaxed);  \
        if (_e != cudaSuccess) return ::ditch::cuda_status(_e, #expr); \
    } while (0)

#define DITCH_CUDA(expr)                                          \
    do {                                                          \
        cudaError_t _e = (expr);                                  \
        if (_e != cudaSuccess) return ::ditch::cuda_status(_e, #expr); \
    } while (0)

// Runs one weight GEMM on the device's stream, with event timing when the
// device profiles. flops = 2 * m * n * k (algorithmic).
cudaError_t run_gemm(ditch_cuda_device *dev, int fmt, const GemmOperand &a, const GemmOperand *a2,
                     const GemmOperand &b, const GemmParams &p);
// The weight-streaming product for 1..16 tokens (same bookkeeping).
cudaError_t run_skinny(ditch_cuda_device *dev, int fmt, const GemmOperand &a, const GemmOperand &b,
                       const GemmParams &p, int k_splits);

// Reads and clears the device status word; returns DITCH_CUDA_OK or a failure.
int check_status(ditch_cuda_device *dev, const char *what);

}  // namespace ditch
