// C ABI: device handles, the per-op entries of ditch's compute seam
// (src/compute.zig:90-117), the standalone decoders and timing support.
#include <algorithm>
#include <cstring>

#include "device.cuh"

using namespace ditch;

namespace ditch {

static thread_local std::string g_last_error;

void set_error(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

int cuda_status(cudaError_t e, const char *what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return DITCH_CUDA_OUT_OF_MEMORY;
    }
    if (e == cudaErrorNotSupported) return DITCH_CUDA_UNSUPPORTED;
    if (e == cudaErrorInvalidValue) return DITCH_CUDA_INVALID;
    return DITCH_CUDA_DEVICE_FAILED;
}

int check_status(ditch_cuda_device *dev, const char *what) {
    int st = 0;
    cudaError_t e = cudaMemcpyAsync(&st, dev->status, sizeof(int), cudaMemcpyDeviceToHost, dev->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(dev->stream);
    if (e != cudaSuccess) return cuda_status(e, what);
    if (st != 0) {
        cudaMemsetAsync(dev->status, 0, sizeof(int), dev->stream);
        cudaStreamSynchronize(dev->stream);
        if (st == kKernelWaitTimeout) {
            set_error("%s: a kernel wait ran out of time", what);
            return DITCH_CUDA_DEVICE_FAILED;
        }
        set_error("%s: invalid input (e.g. a token id outside the embedding table)", what);
        return DITCH_CUDA_INVALID;
    }
    return DITCH_CUDA_OK;
}

cudaError_t run_skinny(ditch_cuda_device *dev, int fmt, const GemmOperand &a, const GemmOperand &b,
                       const GemmParams &p0, int k_splits) {
    GemmParams p = p0;
    p.status = dev->status;
    p.cta_pairs = dev->cta_pairs;
    GemmEvent *ev = nullptr;
    if (dev->profiling) {
        if (dev->n_events == dev->events.size()) {
            GemmEvent g;
            cudaEventCreate(&g.start);
            cudaEventCreate(&g.stop);
            dev->events.push_back(g);
        }
        ev = &dev->events[dev->n_events++];
        ev->flops = 2.0 * p.m_w * (double)p.n_tok * p.k;
        cudaEventRecord(ev->start, dev->stream);
    }
    cudaError_t e = launch_skinny(fmt, a, b, p, k_splits, dev->stream);
    dev->launches.fetch_add(1, std::memory_order_relaxed);
    if (ev) cudaEventRecord(ev->stop, dev->stream);
    return e;
}

cudaError_t run_gemm(ditch_cuda_device *dev, int fmt, const GemmOperand &a, const GemmOperand *a2,
                     const GemmOperand &b, const GemmParams &p0) {
    GemmParams p = p0;
    p.status = dev->status;
    p.cta_pairs = dev->cta_pairs;
    GemmEvent *ev = nullptr;
    if (dev->profiling) {
        if (dev->n_events == dev->events.size()) {
            GemmEvent g;
            cudaEventCreate(&g.start);
            cudaEventCreate(&g.stop);
            dev->events.push_back(g);
        }
        ev = &dev->events[dev->n_events++];
        ev->flops = 2.0 * p.m_w * (double)p.n_tok * p.k * ((p.flags & kEpiSwiglu) ? 2 : 1);
        cudaEventRecord(ev->start, dev->stream);
    }
    cudaError_t e = launch_gemm(fmt, a, a2, b, p, dev->sms, dev->stream);
    dev->launches.fetch_add(1, std::memory_order_relaxed);
    if (ev) cudaEventRecord(ev->stop, dev->stream);
    return e;
}

}  // namespace ditch

namespace {

// Rejects a null handle or pointer with DITCH_CUDA_INVALID.
#define REQUIRE(cond, msg)                       \
    do {                                         \
        if (!(cond)) {                           \
            set_error("%s", msg);                \
            return DITCH_CUDA_INVALID;           \
        }                                        \
    } while (0)

size_t dtype_row_bytes(int dtype, size_t cols) {
    switch (dtype) {
    case DITCH_DTYPE_F32: return cols * 4;
    case DITCH_DTYPE_F16:
    case DITCH_DTYPE_BF16: return cols * 2;
    case DITCH_DTYPE_Q8_0: return cols % 32 ? 0 : cols / 32 * 34;
    case DITCH_DTYPE_Q4_0: return cols % 32 ? 0 : cols / 32 * 18;
    case DITCH_DTYPE_Q4_1: return cols % 32 ? 0 : cols / 32 * 20;
    case DITCH_DTYPE_Q5_0: return cols % 32 ? 0 : cols / 32 * 22;
    case DITCH_DTYPE_Q5_1: return cols % 32 ? 0 : cols / 32 * 24;
    case DITCH_DTYPE_Q4_K: return cols % 256 ? 0 : cols / 256 * 144;
    case DITCH_DTYPE_Q6_K: return cols % 256 ? 0 : cols / 256 * 210;
    case DITCH_DTYPE_Q8_K: return cols % 256 ? 0 : cols / 256 * 292;
    }
    return 0;
}

// Splits rows of f32 values into bf16 segments of width cp: segment s holds
// the high part (pattern bit s = 0) or the low residual bf16(v - hi) (1).
__global__ void k_split(const float *src, int rows, int cols, int cp, int nseg, int pattern, uint16_t *dst) {
    const long long total = (long long)rows * cp;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(e / cp), c = (int)(e % cp);
        uint16_t hi = 0, lo = 0;
        if (c < cols) {
            const float v = src[(long long)r * cols + c];
            hi = f32_to_bf16_bits(v);
            lo = f32_to_bf16_bits(v - bf16_bits_to_f32(hi));
        }
        for (int s = 0; s < nseg; s++)
            dst[(long long)r * nseg * cp + (long long)s * cp + c] = ((pattern >> s) & 1) ? lo : hi;
    }
}

int grid_for(long long n) { return (int)std::min<long long>(std::max<long long>((n + 255) / 256, 1), 148LL * 32); }

// Decodes a host weight of any seam dtype into device f32 [rows][cols].
int upload_weight_f32(ditch_cuda_device *dev, const uint8_t *w, size_t w_len, int dtype, size_t rows, size_t cols,
                      float *out_f32) {
    const size_t rb = dtype_row_bytes(dtype, cols);
    if (rb == 0) {
        set_error("dtype %d with %zu columns is not supported", dtype, cols);
        return DITCH_CUDA_UNSUPPORTED;
    }
    REQUIRE(w_len >= rb * rows, "weight slice shorter than rows * row bytes");
    const size_t n = rows * cols;
    if (dtype == DITCH_DTYPE_F32) {
        DITCH_CUDA(cudaMemcpyAsync(out_f32, w, n * 4, cudaMemcpyHostToDevice, dev->stream));
        return DITCH_CUDA_OK;
    }
    DITCH_CUDA(dev->braw.reserve(rb * rows));
    DITCH_CUDA(cudaMemcpyAsync(dev->braw.ptr, w, rb * rows, cudaMemcpyHostToDevice, dev->stream));
    if (dtype == DITCH_DTYPE_BF16) {
        DITCH_LAUNCH(dev, bf16_to_f32(dev->braw.as<uint16_t>(), out_f32, n, dev->stream));
    } else if (dtype == DITCH_DTYPE_F16) {
        DITCH_LAUNCH(dev, f16_to_f32(dev->braw.as<uint16_t>(), out_f32, n, dev->stream));
    } else {
        DITCH_LAUNCH(dev, dequant_ggml_f32(dtype, dev->braw.as<uint8_t>(), (long long)n, out_f32, dev->stream));
    }
    return DITCH_CUDA_OK;
}

uint64_t signature(const uint8_t *data, size_t len) {
    // FNV-1a over up to four 64-byte samples (start, two interior points, end),
    // the sampling of compute.Residency.signature (src/compute.zig:617-627).
    uint64_t h = 1469598103934665603ull ^ len;
    auto mix = [&](const uint8_t *p, size_t k) {
        for (size_t i = 0; i < k; i++) h = (h ^ p[i]) * 1099511628211ull;
    };
    const size_t k = 64;
    if (len <= 4 * k) {
        mix(data, len);
    } else {
        const size_t at[4] = {0, len / 3, 2 * (len / 3), len - k};
        for (size_t a : at) mix(data + a, k);
    }
    return h;
}

void evict_oldest(ditch_cuda_device *dev) {
    auto oldest = dev->tiles.end();
    for (auto it = dev->tiles.begin(); it != dev->tiles.end(); ++it)
        if (oldest == dev->tiles.end() || it->second.used_at < oldest->second.used_at) oldest = it;
    if (oldest == dev->tiles.end()) return;
    cudaFree(oldest->second.split);
    if (oldest->second.f32) cudaFree(oldest->second.f32);
    dev->used_bytes -= std::min(dev->used_bytes, (uint64_t)oldest->second.bytes);
    dev->tiles.erase(oldest);
}

void forget_all(ditch_cuda_device *dev) {
    cudaStreamSynchronize(dev->stream);
    for (auto &kv : dev->tiles) {
        cudaFree(kv.second.split);
        if (kv.second.f32) cudaFree(kv.second.f32);
    }
    dev->tiles.clear();
    dev->used_bytes = 0;
}

}  // namespace

extern "C" {

const char *ditch_cuda_last_error(void) { return g_last_error.c_str(); }

const char *ditch_cuda_version(void) { return "ditch_cuda 0.1 (sm_100a)"; }

int ditch_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int ditch_cuda_open(int ordinal, uint64_t memory_budget, ditch_cuda_device **out) {
    clear_error();
    REQUIRE(out, "out is null");
    *out = nullptr;
    int n = ditch_cuda_device_count();
    if (ordinal < 0 || ordinal >= n) {
        set_error("no CUDA device %d (%d present)", ordinal, n);
        return DITCH_CUDA_UNSUPPORTED;
    }
    DITCH_CUDA(cudaSetDevice(ordinal));
    cudaDeviceProp prop;
    DITCH_CUDA(cudaGetDeviceProperties(&prop, ordinal));
    if (prop.major != 10) {
        set_error("device %d is sm_%d%d; this build targets sm_100a", ordinal, prop.major, prop.minor);
        return DITCH_CUDA_UNSUPPORTED;
    }
    auto *dev = new ditch_cuda_device();
    dev->ordinal = ordinal;
    dev->sms = prop.multiProcessorCount;
    dev->budget = memory_budget;
    cudaError_t e = cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&dev->status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemsetAsync(dev->status, 0, sizeof(int), dev->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(dev->stream);
    if (e == cudaSuccess) e = cudaEventCreate(&dev->t0);
    if (e == cudaSuccess) e = cudaEventCreate(&dev->t1);
    if (e != cudaSuccess) {
        int st = cuda_status(e, "ditch_cuda_open");
        delete dev;
        return st;
    }
    *out = dev;
    return DITCH_CUDA_OK;
}

void ditch_cuda_close(ditch_cuda_device *dev) {
    if (!dev) return;
    cudaSetDevice(dev->ordinal);
    forget_all(dev);
    for (auto &g : dev->events) {
        cudaEventDestroy(g.start);
        cudaEventDestroy(g.stop);
    }
    if (dev->t0) cudaEventDestroy(dev->t0);
    if (dev->t1) cudaEventDestroy(dev->t1);
    dev->bx.release();
    dev->bw.release();
    dev->bo.release();
    dev->by.release();
    dev->braw.release();
    if (dev->status) cudaFree(dev->status);
    if (dev->stream) cudaStreamDestroy(dev->stream);
    delete dev;
}

void ditch_cuda_forget_weights(ditch_cuda_device *dev) {
    if (!dev) return;
    std::lock_guard<std::mutex> lk(dev->mu);
    cudaSetDevice(dev->ordinal);
    forget_all(dev);
}

uint64_t ditch_cuda_served(const ditch_cuda_device *dev) { return dev ? dev->served.load() : 0; }

void ditch_cuda_set_weights_stable(ditch_cuda_device *dev, int stable) {
    if (!dev) return;
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->weights_stable = stable != 0;
    if (!dev->weights_stable) forget_all(dev);
}

// matmulT (src/compute.zig:343-357 device branch): out[n][rows] = x . W^T as
// a split-bf16 product: x = xh + xl and W = Wh + Wl (Wl = 0 for bf16), so
// x.W^T ~ xh.Wh + xh.Wl + xl.Wh, computed as one tcgen05 GEMM over
// concatenated K segments [xh | xh | xl] . [Wh | Wl | Wh]^T.
int ditch_cuda_matmul_t(ditch_cuda_device *dev, float *out, const float *x, size_t n, const uint8_t *w, size_t w_len,
                        int dtype, size_t rows, size_t cols) {
    clear_error();
    REQUIRE(dev && out && x && w, "null argument");
    if (n == 0 || rows == 0) return DITCH_CUDA_OK;
    if (rows > (1u << 30) || cols > (1u << 24) || n > (1u << 30)) return DITCH_CUDA_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    const int cp = (int)((cols + 63) / 64 * 64);
    const int nseg = dtype == DITCH_DTYPE_BF16 ? 2 : 3;
    const int wpat = nseg == 2 ? 0 /* [W | W] */ : 2 /* [Wh | Wl | Wh] */;
    const int xpat = nseg == 2 ? 2 /* [xh | xl] */ : 4 /* [xh | xh | xl] */;
    const long long kk = (long long)nseg * cp;
    // Scratch is sized once up front: a growth mid-call would free a buffer
    // that queued kernels still read.
    DITCH_CUDA(dev->by.reserve(std::max(n * rows * 4, rows * cols * 4)));
    DITCH_CUDA(dev->bo.reserve(n * cols * 4));
    DITCH_CUDA(dev->bx.reserve((size_t)n * kk * 2));
    DITCH_CUDA(dev->bw.reserve((size_t)rows * kk * 2));
    // weight operand: resident or uploaded for this call
    void *wsplit = nullptr;
    std::string key;
    uint64_t sig = 0;
    const bool cache = dev->budget > 0 && dev->weights_stable;
    if (cache) {
        char kb[64];
        snprintf(kb, sizeof kb, "%p:%zu:%d", (const void *)w, w_len, dtype);
        key = kb;
        sig = signature(w, w_len);
        auto it = dev->tiles.find(key);
        if (it != dev->tiles.end()) {
            if (it->second.sig == sig) {
                it->second.used_at = ++dev->clock;
                wsplit = it->second.split;
            } else {
                cudaStreamSynchronize(dev->stream);
                cudaFree(it->second.split);
                if (it->second.f32) cudaFree(it->second.f32);
                dev->used_bytes -= std::min(dev->used_bytes, (uint64_t)it->second.bytes);
                dev->tiles.erase(it);
            }
        }
    }
    if (!wsplit) {
        DITCH_CUDA(dev->by.reserve(rows * cols * 4));
        int st = upload_weight_f32(dev, w, w_len, dtype, rows, cols, dev->by.as<float>());
        if (st) return st;
        const size_t sbytes = (size_t)rows * kk * 2;
        bool owned = false;
        if (cache && sbytes <= dev->budget) {
            while (dev->used_bytes + sbytes > dev->budget && !dev->tiles.empty()) {
                cudaStreamSynchronize(dev->stream);
                evict_oldest(dev);
            }
            if (cudaMalloc(&wsplit, sbytes) == cudaSuccess) {
                owned = true;
                dev->tiles[key] = ResidentTile{sig, sbytes, ++dev->clock, wsplit, nullptr};
                dev->used_bytes += sbytes;
            } else {
                cudaGetLastError();
                wsplit = nullptr;
            }
        }
        if (!owned) {
            DITCH_CUDA(dev->bw.reserve(sbytes));
            wsplit = dev->bw.ptr;
        }
        DITCH_LAUNCH(dev, (k_split<<<grid_for((long long)rows * cp), 256, 0, dev->stream>>>(
                               dev->by.as<float>(), (int)rows, (int)cols, cp, nseg, wpat, (uint16_t *)wsplit),
                           cudaGetLastError()));
    }
    // input operand
    DITCH_CUDA(dev->bo.reserve(n * cols * 4));
    DITCH_CUDA(cudaMemcpyAsync(dev->bo.ptr, x, n * cols * 4, cudaMemcpyHostToDevice, dev->stream));
    DITCH_CUDA(dev->bx.reserve((size_t)n * kk * 2));
    DITCH_LAUNCH(dev, (k_split<<<grid_for((long long)n * cp), 256, 0, dev->stream>>>(
                           dev->bo.as<float>(), (int)n, (int)cols, cp, nseg, xpat, dev->bx.as<uint16_t>()),
                       cudaGetLastError()));
    // output (reuses the f32 input buffer region after the split)
    DITCH_CUDA(dev->by.reserve(std::max(n * rows * 4, rows * cols * 4)));
    GemmOperand A{wsplit, (int)rows, (int)kk, kk * 2};
    GemmOperand B{dev->bx.ptr, (int)n, (int)kk, kk * 2};
    GemmParams p{};
    p.m_w = (int)rows;
    p.n_tok = (int)n;
    p.k = (int)kk;
    p.k_splits = 1;
    p.out = dev->by.ptr;
    p.ldo = (long long)rows;
    DITCH_CUDA(run_gemm(dev, kFmtBf16, A, nullptr, B, p));
    DITCH_CUDA(cudaMemcpyAsync(out, dev->by.ptr, n * rows * 4, cudaMemcpyDeviceToHost, dev->stream));
    int st = check_status(dev, "matmul_t");
    if (st == DITCH_CUDA_OK) dev->served.fetch_add(1);
    return st;
}

int ditch_cuda_matvec_t_multi(ditch_cuda_device *dev, float *out, const uint8_t *w, size_t w_len, int dtype,
                              size_t rows, size_t cols, const float *y, size_t q) {
    clear_error();
    REQUIRE(dev && out && w && y, "null argument");
    if (q == 0 || rows == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(dev->by.reserve(rows * cols * 4));
    int st = upload_weight_f32(dev, w, w_len, dtype, rows, cols, dev->by.as<float>());
    if (st) return st;
    DITCH_CUDA(dev->bx.reserve(q * rows * 4));
    DITCH_CUDA(dev->bo.reserve(q * cols * 4));
    DITCH_CUDA(cudaMemcpyAsync(dev->bx.ptr, y, q * rows * 4, cudaMemcpyHostToDevice, dev->stream));
    DITCH_CUDA(cudaMemsetAsync(dev->bo.ptr, 0, q * cols * 4, dev->stream));
    for (size_t j = 0; j < q; j++)
        DITCH_LAUNCH(dev, gemv_t_f32(dev->by.as<float>(), (int)rows, (int)cols, dev->bx.as<float>() + j * rows,
                                     dev->bo.as<float>() + j * cols, dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(out, dev->bo.ptr, q * cols * 4, cudaMemcpyDeviceToHost, dev->stream));
    st = check_status(dev, "matvec_t_multi");
    if (st == DITCH_CUDA_OK) dev->served.fetch_add(1);
    return st;
}

int ditch_cuda_row_norms(ditch_cuda_device *dev, float *out, const uint8_t *w, size_t w_len, int dtype, size_t rows,
                         size_t cols) {
    clear_error();
    REQUIRE(dev && out && w, "null argument");
    if (rows == 0) return DITCH_CUDA_OK;
    std::lock_guard<std::mutex> lk(dev->mu);
    DITCH_CUDA(cudaSetDevice(dev->ordinal));
    DITCH_CUDA(dev->by.reserve(rows * cols * 4));
    int st = upload_weight_f32(dev, w, w_len, dtype, rows, cols, dev->by.as<float>());
    if (st) return st;
    DITCH_CUDA(dev->bo.reserve(rows * 4));
    DITCH_LAUNCH(dev, row_norms_f32(dev->by.as<float>(), (int)rows, (int)cols, dev->bo.as<float>(), dev->stream));
    DITCH_CUDA(cudaMemcpyAsync(out, dev->bo.ptr, rows * 4, cudaMemcpyDeviceToHost, dev->stream));
    st = check_status(dev, "row_norms");
    if (st == DITCH_CUDA_OK) dev->served.fetch_add(1);
    return st;
}

}  // extern "C"
