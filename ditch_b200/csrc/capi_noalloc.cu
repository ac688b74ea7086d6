// An allocation-free variant of the in-place rank-1 weight edit.
//
// Some callers cannot allocate device memory while they edit weights: a host
// that has handed every byte of HBM to its own pool allocator (an inference
// server that reserved the GPU at start-up), code that must not stall other
// streams (cudaMalloc and cudaFree can synchronise the whole device), or a
// caller that never created a ditch_cuda_device handle (creating one allocates
// its stream and status word). For them this entry point keeps its scratch,
// the vectors a = r^T W and b = -alpha r, in a fixed array that is part of the
// library image on the GPU, so a call allocates nothing.
#include <mutex>

#include "device.cuh"

namespace {

// Largest matrix the allocation-free edit takes (512 KiB of scratch in all).
constexpr size_t kNoAllocMaxCols = 65536;
constexpr size_t kNoAllocMaxRows = 65536;

// The scratch: a [cols] then b [rows]. Every GPU that loads the library holds
// this array until the process exits. Every call shares it and it keeps the
// last call's contents, so calls that overlap on the GPU (on different
// streams, or from different threads) race on it.
static __device__ __align__(256) float g_edit_scratch[kNoAllocMaxCols + kNoAllocMaxRows];

std::mutex g_mu;
constexpr int kMaxDevices = 64;
float *g_scratch[kMaxDevices] = {};

// The device address of the scratch on the current device. In host code the
// array's name only stands for it, so the address is looked up once per
// device, with that device current.
int scratch_for_current_device(float **out) {
    int d = 0;
    cudaError_t e = cudaGetDevice(&d);
    if (e != cudaSuccess) return ditch::cuda_status(e, "edit_weight_bf16_noalloc: cudaGetDevice");
    if (d < 0 || d >= kMaxDevices) {
        ditch::set_error("edit_weight_bf16_noalloc: device %d out of range", d);
        return DITCH_CUDA_INVALID;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch[d]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_edit_scratch);
        if (e != cudaSuccess) return ditch::cuda_status(e, "edit_weight_bf16_noalloc: cudaGetSymbolAddress");
        g_scratch[d] = static_cast<float *>(p);
    }
    *out = g_scratch[d];
    return DITCH_CUDA_OK;
}

}  // namespace

extern "C" {

int ditch_cuda_edit_weight_bf16_noalloc(void *w, size_t rows, size_t cols, const float *r, float alpha,
                                        void *stream) {
    ditch::clear_error();
    if (!w || !r) {
        ditch::set_error("edit_weight_bf16_noalloc: null argument");
        return DITCH_CUDA_INVALID;
    }
    // bf16 elements and f32 entries must sit on their own size; rows that are
    // not 16-byte aligned take the kernels' 2-byte path
    if ((reinterpret_cast<uintptr_t>(w) & 1) || (reinterpret_cast<uintptr_t>(r) & 3)) {
        ditch::set_error("edit_weight_bf16_noalloc: w must be 2-byte and r 4-byte aligned");
        return DITCH_CUDA_INVALID;
    }
    if (rows == 0 || cols == 0) return DITCH_CUDA_OK;
    if (rows > kNoAllocMaxRows || cols > kNoAllocMaxCols) {
        ditch::set_error("edit_weight_bf16_noalloc: %zu x %zu exceeds the fixed scratch (at most %zu rows and %zu "
                         "columns); use ditch_cuda_edit_weight_bf16",
                         rows, cols, kNoAllocMaxRows, kNoAllocMaxCols);
        return DITCH_CUDA_INVALID;
    }
    float *scratch = nullptr;
    int st = scratch_for_current_device(&scratch);
    if (st) return st;
    float *a = scratch, *b = scratch + kNoAllocMaxCols;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // a accumulates partial sums, so it starts from zero on every call
    DITCH_CUDA(cudaMemsetAsync(a, 0, cols * sizeof(float), s));
    DITCH_CUDA(ditch::gemv_t_bf16(static_cast<const uint16_t *>(w), (int)rows, (int)cols, r, a, s));
    DITCH_CUDA(ditch::scale_vec(r, alpha, (int)rows, b, s));
    DITCH_CUDA(ditch::rank1_update_bf16(static_cast<uint16_t *>(w), (int)rows, (int)cols, b, a, s));
    return DITCH_CUDA_OK;
}

}  // extern "C"
