// Bandwidth-bound kernels of the edit, the scorers and the residual
// reduction: GEMV-T (A = v^T W), row norms, the in-place rank-1 update, the
// fused log-softmax / KL, and the f64 residual sums and directions.
#include <algorithm>

#include "kernels.cuh"

namespace ditch {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions (blockDim.x a multiple of 32, <= 1024).
__device__ float block_sum(float v, float *sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float t = lane < nw ? sh[lane] : 0.0f;
    return warp_sum(t);
}

__device__ double block_sum_d(double v, double *sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum_d(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    double t = lane < nw ? sh[lane] : 0.0;
    return warp_sum_d(t);
}

__device__ float block_max(float v, float *sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float t = lane < nw ? sh[lane] : -INFINITY;
    return warp_max(t);
}

constexpr int kGemvThreads = 256;

// Row splits of a GEMV-T: about two blocks per SM in all, at least
// `min_rows` rows each (every split adds its partial sums atomically).
inline int row_splits(int rows, int col_blocks, int min_rows = 64) {
    const int target = 2 * 148;
    int s = (target + col_blocks - 1) / col_blocks;
    s = s < 1 ? 1 : s;
    const int max_s = (rows + min_rows - 1) / min_rows;
    return s > max_s ? (max_s < 1 ? 1 : max_s) : s;
}

// out[c] += sum_{r in split} v[r] W[r][c]; thread = 8 consecutive bf16
// columns, 2-byte loads: the form for rows that are not 16-byte aligned (the
// piece kernel below takes the rest). Rows with v[r] == 0 are skipped, as
// src/tensor.zig:1065-1068.
__global__ void k_gemv_t_bf16(const uint16_t *w, int rows, int cols, const float *v, float *out, int rows_per) {
    const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
    if (c0 >= cols) return;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = r0; r < r1; r++) {
        const float vr = v[r];
        if (vr == 0.0f) continue;
        for (int j = 0; j < 8 && c0 + j < cols; j++)
            acc[j] = fmaf(vr, bf16_bits_to_f32(w[(long long)r * cols + c0 + j]), acc[j]);
    }
    for (int j = 0; j < 8 && c0 + j < cols; j++) atomicAdd(out + c0 + j, acc[j]);
}

__global__ void k_gemv_t_f32(const float *w, int rows, int cols, const float *v, float *out, int rows_per) {
    const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
    if (c0 >= cols) return;
    float acc[4] = {0, 0, 0, 0};
    for (int r = r0; r < r1; r++) {
        const float vr = v[r];
        if (vr == 0.0f) continue;
        if (c0 + 4 <= cols && (cols & 3) == 0) {
            float4 q = __ldg(reinterpret_cast<const float4 *>(w + (long long)r * cols + c0));
            acc[0] = fmaf(vr, q.x, acc[0]);
            acc[1] = fmaf(vr, q.y, acc[1]);
            acc[2] = fmaf(vr, q.z, acc[2]);
            acc[3] = fmaf(vr, q.w, acc[3]);
        } else {
            for (int j = 0; j < 4 && c0 + j < cols; j++) acc[j] = fmaf(vr, w[(long long)r * cols + c0 + j], acc[j]);
        }
    }
    for (int j = 0; j < 4 && c0 + j < cols; j++) atomicAdd(out + c0 + j, acc[j]);
}

__device__ __forceinline__ void e4m3x4(uint32_t w, float *f) {
    uint32_t h01, h23;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
        : "=r"(h01), "=r"(h23)
        : "r"(w));
    float2 a = __half22float2(*reinterpret_cast<__half2 *>(&h01));
    float2 b = __half22float2(*reinterpret_cast<__half2 *>(&h23));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

// FP8 weights: each element is the decoded bf16 value bf16(code * scale),
// as the reference's materialised weight (src/dequant.zig:505-511). The
// byte-wise form, for shapes the piece kernel below does not take (columns or
// column blocks not a multiple of 16, or codes not 16-byte aligned).
__global__ void k_gemv_t_fp8(const uint8_t *codes, const float *scales, int rows, int cols, int br, int bc,
                             int scols, const float *v, float *out, int rows_per) {
    const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 16;
    const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
    if (c0 >= cols) return;
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; j++) acc[j] = 0.0f;
    for (int r = r0; r < r1; r++) {
        const float vr = v[r];
        const float *srow = scales + (long long)(r / br) * scols;
        for (int j = 0; j < 16 && c0 + j < cols; j++) {
            float f[4];
            e4m3x4(codes[(long long)r * cols + c0 + j], f);
            acc[j] = fmaf(vr, bf16_bits_to_f32(f32_to_bf16_bits(f[0] * srow[(c0 + j) / bc])), acc[j]);
        }
    }
    for (int j = 0; j < 16 && c0 + j < cols; j++) atomicAdd(out + c0 + j, acc[j]);
}



// ---- streaming GEMV-T over 16-byte row pieces ----
// out[c] += sum_{r in the block's rows} v[r] W[r][c] for bf16 weights (8
// columns per 16-byte piece) or FP8 block-scaled ones (16 columns, each
// element the decoded bf16(code * scale) of src/dequant.zig:505-511, the
// operand the reference multiplies). Block = 32 column lanes (x) by 8 row
// lanes (y): a warp reads 512 contiguous bytes of one row; row lane y takes
// rows r0 + y, r0 + y + 8, ..., four of them per step with the next four
// loaded before this step's math. The 8 row lanes are added in shared memory
// in lane order and the block adds each column's sum to out with one atomic
// (a block covers 256 / 512 columns and a run of rows; the runs are sized for
// the blocks one SM holds at once: three bf16 ones, two FP8 ones). Needs 16-byte aligned rows (w aligned, cols a
// multiple of the piece) and, for FP8, column blocks a multiple of 16. Rows
// with v[r] == 0 are not skipped (the reference skips them,
// src/tensor.zig:1065-1068): for finite weights they add exactly zero, and
// the stream keeps its loads in flight without a data-dependent branch.
constexpr int kRowLanes = 8;

template <bool FP8>
__global__ void __launch_bounds__(32 * kRowLanes, FP8 ? 2 : 3)
    k_gemv_t_pieces(const uint8_t *w, const float *scales, int rows, int cols, int br, int bc, int scols,
                    const float *v, float *out, int rows_per) {
    constexpr int E = FP8 ? 16 : 8;        // columns per piece
    constexpr int kBytes = FP8 ? 1 : 2;    // per element
    __shared__ float red[kRowLanes][E][33];
    const int x = threadIdx.x, y = threadIdx.y;
    const int cblk = blockIdx.x * 32 * E;
    const int c0 = cblk + x * E;
    const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
    float acc[E];
#pragma unroll
    for (int j = 0; j < E; j++) acc[j] = 0.0f;
    if (c0 < cols) {
        const uint8_t *base = w + (long long)c0 * kBytes;
        const long long pitch = (long long)cols * kBytes;
        const int sc = FP8 ? c0 / bc : 0;
        uint4 qn[4];
        float vn[4], sn[4];
        auto fetch = [&](int rb) {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int r = rb + kRowLanes * u;
                const bool ok = r < r1;
                qn[u] = ok ? __ldg(reinterpret_cast<const uint4 *>(base + (long long)r * pitch)) : make_uint4(0, 0, 0, 0);
                vn[u] = ok ? __ldg(v + r) : 0.0f;
                sn[u] = (FP8 && ok) ? __ldg(scales + (long long)(r / br) * scols + sc) : 0.0f;
            }
        };
        fetch(r0 + y);
        for (int rb = r0 + y; rb < r1; rb += 4 * kRowLanes) {
            uint4 q[4];
            float vr[4], s4[4];
#pragma unroll
            for (int u = 0; u < 4; u++) q[u] = qn[u], vr[u] = vn[u], s4[u] = sn[u];
            if (rb + 4 * kRowLanes < r1) fetch(rb + 4 * kRowLanes);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t wd[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (FP8) {
                        const uint32_t p0 = scale_pack(e4m3x2_f32(wd[j] & 0xffff), s4[u]);
                        const uint32_t p1 = scale_pack(e4m3x2_f32(wd[j] >> 16), s4[u]);
                        acc[4 * j] = fmaf(vr[u], __uint_as_float(p0 << 16), acc[4 * j]);
                        acc[4 * j + 1] = fmaf(vr[u], __uint_as_float(p0 & 0xffff0000u), acc[4 * j + 1]);
                        acc[4 * j + 2] = fmaf(vr[u], __uint_as_float(p1 << 16), acc[4 * j + 2]);
                        acc[4 * j + 3] = fmaf(vr[u], __uint_as_float(p1 & 0xffff0000u), acc[4 * j + 3]);
                    } else {
                        acc[2 * j] = fmaf(vr[u], __uint_as_float(wd[j] << 16), acc[2 * j]);
                        acc[2 * j + 1] = fmaf(vr[u], __uint_as_float(wd[j] & 0xffff0000u), acc[2 * j + 1]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < E; j++) red[y][j][x] = acc[j];
    __syncthreads();
    for (int cc = y * 32 + x; cc < 32 * E; cc += 32 * kRowLanes) {
        const int col = cblk + cc;
        if (col >= cols) break;
        const int xx = cc / E, j = cc % E;
        float t = 0.0f;
#pragma unroll
        for (int l = 0; l < kRowLanes; l++) t += red[l][j][xx];
        atomicAdd(out + col, t);
    }
}

__device__ __constant__ float kE2M1e[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                            -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

__device__ __forceinline__ float mx_scale(uint32_t b) { return __uint_as_float(b == 0 ? 0x00400000u : (b << 23)); }

// Two E2M1 nibbles (one byte, low nibble first) to two f32, exactly.
__device__ __forceinline__ float2 e2m1x2(uint32_t byte) {
    uint32_t h;
    asm("{\n\t.reg .b8 b;\n\tcvt.u8.u32 b, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b;\n\t}" : "=r"(h) : "r"(byte));
    return __half22float2(*reinterpret_cast<__half2 *>(&h));
}

// MXFP4 (natural layout) over a stack of `slabs` matrices [rows][cols]:
// out[e][c] = sum_r v[r] W_e[r][c] (the decoded value e2m1 * 2^(b - 127) is
// exact in bf16, src/dequant.zig:643-673). Block = 32 column blocks (x) by 8
// row lanes (y); grid = (column-block groups, row chunks of kMxChunk rows,
// slabs). Each thread streams one 32-element block of its rows, four rows of
// loads in flight; the 8 row lanes are summed in shared memory and each
// chunk's partial sums are stored, then k_sum_parts adds the chunks in order.
// The chunking depends only on the matrix shape, so every matrix of a stack
// gets the same sums whatever the stack size (no atomics, deterministic).
constexpr int kMxLanes = 8;
constexpr int kMxChunk = 256;
__global__ void __launch_bounds__(32 * kMxLanes) k_gemv_t_mxfp4(const uint8_t *blocks, const uint8_t *scales,
                                                                int rows, int cols, const float *v, float *part,
                                                                int rows_per) {
    __shared__ float lanes[kMxLanes][32][33];
    const int nblk = cols / 32;
    const int blk = blockIdx.x * 32 + threadIdx.x;
    const int e = blockIdx.z;
    const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
    const uint8_t *bl = blocks + (long long)e * rows * (cols / 2);
    const uint8_t *sc = scales + (long long)e * rows * nblk;
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; j++) acc[j] = 0.0f;
    if (blk < nblk) {
        int r = r0 + threadIdx.y;
        for (; r + 3 * kMxLanes < r1; r += 4 * kMxLanes) {
            uint4 q[4];
            float vr[4], s[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int rr = r + u * kMxLanes;
                q[u] = __ldg(reinterpret_cast<const uint4 *>(bl + (long long)rr * (cols / 2) + blk * 16));
                vr[u] = __ldg(v + rr);
                s[u] = mx_scale(__ldg(sc + (long long)rr * nblk + blk));
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t wd[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
                const float vs = vr[u];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float2 f = e2m1x2((wd[j / 4] >> (8 * (j & 3))) & 0xff);
                    acc[2 * j] = fmaf(vs, f.x * s[u], acc[2 * j]);
                    acc[2 * j + 1] = fmaf(vs, f.y * s[u], acc[2 * j + 1]);
                }
            }
        }
        for (; r < r1; r += kMxLanes) {
            const uint4 q = __ldg(reinterpret_cast<const uint4 *>(bl + (long long)r * (cols / 2) + blk * 16));
            const float vs = __ldg(v + r), s = mx_scale(__ldg(sc + (long long)r * nblk + blk));
            const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float2 f = e2m1x2((wd[j / 4] >> (8 * (j & 3))) & 0xff);
                acc[2 * j] = fmaf(vs, f.x * s, acc[2 * j]);
                acc[2 * j + 1] = fmaf(vs, f.y * s, acc[2 * j + 1]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 32; j++) lanes[threadIdx.y][threadIdx.x][j] = acc[j];
    __syncthreads();
    // thread (x, y) sums columns y, y + 8, y + 16, y + 24 of column block x
    if (blk < nblk) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int j = threadIdx.y + kMxLanes * k;
            float t = 0.0f;
#pragma unroll
            for (int l = 0; l < kMxLanes; l++) t += lanes[l][threadIdx.x][j];
            part[((long long)e * gridDim.y + blockIdx.y) * cols + blk * 32 + j] = t;
        }
    }
}

// out[e][c] = sum over chunks q (in order) of part[e][q][c].
__global__ void k_sum_parts(const float *part, int chunks, int slabs, int cols, float *out) {
    const long long n = (long long)slabs * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long e = i / cols, c = i % cols;
        float t = 0.0f;
        for (int q = 0; q < chunks; q++) t += part[(e * chunks + q) * cols + c];
        out[i] = t;
    }
}

template <typename LOAD>
__global__ void k_row_norms(int rows, int cols, float *out, LOAD load) {
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) {
        const float x = load(row, c);
        s = fmaf(x, x, s);
    }
    s = warp_sum(s);
    if (lane == 0) out[row] = sqrtf(s);
}

struct LoadBf16 {
    const uint16_t *w;
    int cols;
    __device__ float operator()(int r, int c) const { return bf16_bits_to_f32(w[(long long)r * cols + c]); }
};
struct LoadF32 {
    const float *w;
    int cols;
    __device__ float operator()(int r, int c) const { return w[(long long)r * cols + c]; }
};
struct LoadMxfp4 {
    const uint8_t *b, *s;
    int cols;
    __device__ float operator()(int r, int c) const {
        const uint8_t byte = b[(long long)r * (cols / 2) + c / 2];
        return kE2M1e[(c & 1) ? (byte >> 4) : (byte & 0xf)] * mx_scale(s[(long long)r * (cols / 32) + c / 32]);
    }
};

// Block = a strip of 8 * blockDim columns over a range of rows: the strip's
// a values stay in registers, each row is one 16-byte read and write per
// thread, four rows in flight.
__global__ void k_rank1_bf16(uint16_t *w, int rows, int cols, const float *b, const float *a, int rows_per) {
    const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
    if (c0 >= cols) return;
    float av[8];
    {
        const float4 a0 = *reinterpret_cast<const float4 *>(a + c0), a1 = *reinterpret_cast<const float4 *>(a + c0 + 4);
        av[0] = a0.x, av[1] = a0.y, av[2] = a0.z, av[3] = a0.w, av[4] = a1.x, av[5] = a1.y, av[6] = a1.z, av[7] = a1.w;
    }
    uint16_t *base = w + c0;
    int r = r0;
    for (; r + 4 <= r1; r += 4) {
        uint4 q[4];
        float br[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            q[u] = *reinterpret_cast<const uint4 *>(base + (long long)(r + u) * cols);
            br[u] = __ldg(b + r + u);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            uint32_t wd[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float lo = fmaf(br[u], av[2 * j], __uint_as_float(wd[j] << 16));
                const float hi = fmaf(br[u], av[2 * j + 1], __uint_as_float(wd[j] & 0xffff0000u));
                wd[j] = pack_bf16x2(lo, hi);
            }
            *reinterpret_cast<uint4 *>(base + (long long)(r + u) * cols) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
    }
    for (; r < r1; r++) {
        uint4 q = *reinterpret_cast<const uint4 *>(base + (long long)r * cols);
        const float br = __ldg(b + r);
        uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; j++)
            wd[j] = pack_bf16x2(fmaf(br, av[2 * j], __uint_as_float(wd[j] << 16)),
                                fmaf(br, av[2 * j + 1], __uint_as_float(wd[j] & 0xffff0000u)));
        *reinterpret_cast<uint4 *>(base + (long long)r * cols) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
}

__global__ void k_rank1_bf16_scalar(uint16_t *w, int rows, int cols, const float *b, const float *a) {
    const long long total = (long long)rows * cols;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(e / cols), c = (int)(e % cols);
        w[e] = f32_to_bf16_bits(fmaf(b[r], a[c], bf16_bits_to_f32(w[e])));
    }
}

__global__ void k_scale_vec(const float *v, float lambda, int n, float *b) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b[i] = -lambda * v[i];
}

// ---- scoring ----
// ---- log-softmax and KL over row pieces ----
// A vocabulary row (C2: 128256 logits) is split into pieces of kKlPiece
// logits, one block each (16 per thread, read once and kept in registers for
// both the maximum and the sum): piece (row, c) finds its maximum m_c and
// s_c = sum exp(x - m_c) in f64; the row's log-sum-exp combines the pieces in
// order, lse = m + log(sum_c s_c exp(m_c - m)) with m = max m_c, as
// src/tensor.zig:1203-1210 (the f32 difference, its exp and the sum in f64,
// the result in f32). The exp stays in f64: the KL moves one for one with
// the f32 lse, so an f32 exp (6e-8 relative per term) would flip the lse's
// last bit on some rows and move a small KL by a few 1e-4 relative.
// The KL pieces then add exp(b)(b - (x - lse)) in f64 (src/scorers.zig:
// 385-400: the reference forms each term in f64; here the term is an f32
// product of f32 expf and the f32 difference, widened before the f64 sum)
// and one thread per row adds the pieces in order. The pieces depend only on the vocabulary size, so the sums
// are the same for any batch.
constexpr int kKlThreads = 256, kKlEach = 16, kKlPiece = kKlThreads * kKlEach;

// this thread's 16 logits of a piece (out-of-row slots get `fill`): four
// 16-byte loads when rows are 16-byte aligned (vocab a multiple of 4 on an
// aligned base), else strided scalar loads.
__device__ __forceinline__ void kl_load(const float *xr, int lo, int vocab, bool vec, float fill,
                                        float (&v)[kKlEach]) {
    if (vec) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int j = lo + (k * kKlThreads + (int)threadIdx.x) * 4;
            float4 q = make_float4(fill, fill, fill, fill);
            if (j < vocab) q = __ldg(reinterpret_cast<const float4 *>(xr + j));  // j + 3 < vocab
            v[4 * k] = q.x, v[4 * k + 1] = q.y, v[4 * k + 2] = q.z, v[4 * k + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int k = 0; k < kKlEach; k++) {
            const int j = lo + k * kKlThreads + (int)threadIdx.x;
            v[k] = j < vocab ? __ldg(xr + j) : fill;
        }
    }
}

// the column of slot k of this thread (the layout kl_load reads)
__device__ __forceinline__ int kl_col(int lo, bool vec, int k) {
    return vec ? lo + ((k >> 2) * kKlThreads + (int)threadIdx.x) * 4 + (k & 3) : lo + k * kKlThreads + (int)threadIdx.x;
}

__global__ void __launch_bounds__(kKlThreads) k_lse_part(const float *x, int vocab, bool vec, double2 *part) {
    __shared__ float shf[32];
    __shared__ double shd[32];
    const int row = blockIdx.y, c = blockIdx.x, chunks = gridDim.x;
    const float *xr = x + (long long)row * vocab;
    float v[kKlEach];
    kl_load(xr, c * kKlPiece, vocab, vec, -INFINITY, v);
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kKlEach; k++) m = fmaxf(m, v[k]);
    m = block_max(m, shf);
    double s = 0.0;
    if (m > -INFINITY) {
#pragma unroll
        for (int k = 0; k < kKlEach; k++) s += exp((double)(v[k] - m));
    }
    s = block_sum_d(s, shd);
    if (threadIdx.x == 0) part[(long long)row * chunks + c] = make_double2((double)m, s);
}

// The row's log-sum-exp from its pieces, by one whole warp (each lane a
// stride of the pieces, then shuffles): the same bits wherever it is called,
// so the baseline's log-probs and the KL's see the same value.
__device__ __forceinline__ float row_lse_warp(const double2 *part, int chunks) {
    const int lane = threadIdx.x & 31;
    float m = -INFINITY;
    for (int c = lane; c < chunks; c += 32) m = fmaxf(m, (float)part[c].x);
    m = warp_max(m);
    double s = 0.0;
    for (int c = lane; c < chunks; c += 32)
        if (part[c].x > -INFINITY) s += part[c].y * exp(part[c].x - (double)m);
    s = warp_sum_d(s);
    return m + (float)log(s);
}

__global__ void __launch_bounds__(kKlThreads) k_log_softmax_part(const float *x, int vocab, bool vec,
                                                                 const double2 *part, float *out) {
    __shared__ float s_lse;
    const int row = blockIdx.y, c = blockIdx.x, chunks = gridDim.x;
    if (threadIdx.x < 32) {
        const float l = row_lse_warp(part + (long long)row * chunks, chunks);
        if (threadIdx.x == 0) s_lse = l;
    }
    __syncthreads();
    const float lse = s_lse;
    const float *xr = x + (long long)row * vocab;
    float *o = out + (long long)row * vocab;
    const int lo = c * kKlPiece;
    if (vec) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int j = lo + (k * kKlThreads + (int)threadIdx.x) * 4;
            if (j < vocab) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(xr + j));
                *reinterpret_cast<float4 *>(o + j) = make_float4(q.x - lse, q.y - lse, q.z - lse, q.w - lse);
            }
        }
    } else {
        for (int k = 0; k < kKlEach; k++) {
            const int j = lo + k * kKlThreads + (int)threadIdx.x;
            if (j < vocab) o[j] = xr[j] - lse;
        }
    }
}

__global__ void __launch_bounds__(kKlThreads) k_kl_part(const float *base, const float *logits, int vocab, bool vec,
                                                        const double2 *part, double *kl_part) {
    __shared__ float s_lse;
    __shared__ double shd[32];
    const int row = blockIdx.y, c = blockIdx.x, chunks = gridDim.x;
    if (threadIdx.x < 32) {
        const float l = row_lse_warp(part + (long long)row * chunks, chunks);
        if (threadIdx.x == 0) s_lse = l;
    }
    const int lo = c * kKlPiece;
    float x[kKlEach], b[kKlEach];
    kl_load(logits + (long long)row * vocab, lo, vocab, vec, 0.0f, x);
    kl_load(base + (long long)row * vocab, lo, vocab, vec, 0.0f, b);
    __syncthreads();
    const float lse = s_lse;
    double s = 0.0;
#pragma unroll
    for (int k = 0; k < kKlEach; k++) {
        if (kl_col(lo, vec, k) < vocab) {
            // b - lt is exact in f32 wherever the two are within a factor of
            // two (Sterbenz), i.e. wherever the edit moved the log-prob by
            // less than that; the product takes one f32 rounding (about
            // 6e-8 relative) before the f64 sum
            const float lt = x[k] - lse;
            s += (double)(expf(b[k]) * (b[k] - lt));
        }
    }
    s = block_sum_d(s, shd);
    if (threadIdx.x == 0) kl_part[(long long)row * chunks + c] = s;
}

__global__ void k_kl_rows_sum(const double *kl_part, int rows, int chunks, double *kl) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    double s = 0.0;
    for (int c = 0; c < chunks; c++) s += kl_part[(long long)row * chunks + c];
    kl[row] = s;
}

// ---- capture and directions ----
// Prompt b's mean over its take[b] captures is an f32 running sum of
// (1 / take) * r in token order, added to the entry's f64 sum in prompt order
// (src/engine.zig:414-431). The prompts are split into `groups` consecutive
// runs (blockIdx.y): a thread handles one (entry, 4 hidden coordinates) of
// one run, its prompts in order, and stores the run's f64 sum; a second pass
// adds the runs in order. Every prompt's f32 mean is the reference's; only
// the f64 additions are grouped (runs, then their totals).
__global__ void k_residual_sums(const float *res, int entries, int nc, int hidden, const int *first, const int *take,
                                int prompts, int per_group, double *part) {
    const int h4 = hidden / 4;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    const bool vec = (hidden & 3) == 0;
    const int per_entry = vec ? h4 : hidden;
    if (idx >= entries * per_entry) return;
    const int l = idx / per_entry, j = idx % per_entry;
    const int b0 = blockIdx.y * per_group, b1 = min(prompts, b0 + per_group);
    double *o = part + ((long long)blockIdx.y * entries + l) * hidden;
    if (vec) {
        double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        for (int b = b0; b < b1; b++) {
            const int tk = take[b];
            const float inv = 1.0f / (float)(tk > 0 ? tk : 1);
            const float4 *src = reinterpret_cast<const float4 *>(res + ((long long)l * nc + first[b]) * hidden) + j;
            float v0 = 0, v1 = 0, v2 = 0, v3 = 0;
#pragma unroll 4
            for (int t = 0; t < tk; t++) {
                const float4 r = __ldg(src + (long long)t * h4);
                v0 = v0 + inv * r.x;
                v1 = v1 + inv * r.y;
                v2 = v2 + inv * r.z;
                v3 = v3 + inv * r.w;
            }
            s0 += v0;
            s1 += v1;
            s2 += v2;
            s3 += v3;
        }
        *reinterpret_cast<double2 *>(o + 4 * j) = make_double2(s0, s1);
        *reinterpret_cast<double2 *>(o + 4 * j + 2) = make_double2(s2, s3);
    } else {
        double s = 0;
        for (int b = b0; b < b1; b++) {
            const int tk = take[b];
            const float inv = 1.0f / (float)(tk > 0 ? tk : 1);
            float v = 0;
            for (int t = 0; t < tk; t++) v = v + inv * res[((long long)l * nc + first[b] + t) * hidden + j];
            s += v;
        }
        o[j] = s;
    }
}

// sums[i] += the runs' sums in run order
__global__ void k_residual_groups_sum(const double *part, long long n, int groups, double *sums) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    double s = 0;
    for (int g = 0; g < groups; g++) s += part[(long long)g * n + i];
    sums[i] += s;
}

// One block per entry: means, difference, normalisation, orthogonalisation.
__global__ void k_directions(const double *gs, double gc, const double *bs, double bc, int hidden, int ortho,
                             float *dirs, float *gmean, float *bmean) {
    __shared__ float sh[32];
    const int e = blockIdx.x;
    float *d = dirs + (long long)e * hidden;
    const double *g = gs + (long long)e * hidden, *b = bs + (long long)e * hidden;
    const double gcn = gc > 1 ? gc : 1, bcn = bc > 1 ? bc : 1;
    float ss = 0.0f, gg = 0.0f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float gm = (float)(g[i] / gcn), bm = (float)(b[i] / bcn);
        if (gmean) gmean[(long long)e * hidden + i] = gm;
        if (bmean) bmean[(long long)e * hidden + i] = bm;
        const float v = bm - gm;
        d[i] = v;
        ss = fmaf(v, v, ss);
        gg = fmaf(gm, gm, gg);
    }
    const float nd = sqrtf(block_sum(ss, sh));
    const float ng = sqrtf(block_sum(gg, sh));
    const float sd = nd > 1e-12f ? 1.0f / nd : 1.0f;
    const float sg = ng > 1e-12f ? 1.0f / ng : 1.0f;
    if (!ortho) {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) d[i] = d[i] * sd;
        return;
    }
    float pr = 0.0f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        d[i] = d[i] * sd;
        pr = fmaf(d[i], (float)(g[i] / gcn) * sg, pr);
    }
    const float proj = block_sum(pr, sh);
    float s2 = 0.0f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float v = d[i] + (-proj) * ((float)(g[i] / gcn) * sg);
        d[i] = v;
        s2 = fmaf(v, v, s2);
    }
    const float n2 = sqrtf(block_sum(s2, sh));
    const float s3 = n2 > 1e-12f ? 1.0f / n2 : 1.0f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) d[i] = d[i] * s3;
}

}  // namespace

// Row runs for the piece kernels: at most one wave of `per_sm` blocks per SM
// (a partial second wave would double the time), at least 64 rows (8 per
// row lane) per block.
static int piece_splits(int rows, int col_blocks, int per_sm) {
    int s = (per_sm * 148) / col_blocks;
    s = std::min(s, (rows + 63) / 64);
    return std::max(1, std::min(s, 65535));
}

cudaError_t gemv_t_bf16(const uint16_t *w, int rows, int cols, const float *v, float *out, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    const bool vec = (cols & 7) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
    if (vec) {
        const int cb = (cols + 255) / 256;
        const int sp = piece_splits(rows, cb, 3);
        const int per = (rows + sp - 1) / sp;
        k_gemv_t_pieces<false><<<dim3(cb, (rows + per - 1) / per), dim3(32, kRowLanes), 0, st>>>(
            reinterpret_cast<const uint8_t *>(w), nullptr, rows, cols, 1, 1, 1, v, out, per);
        return cudaGetLastError();
    }
    const int cb = (cols + kGemvThreads * 8 - 1) / (kGemvThreads * 8);
    const int sp = row_splits(rows, cb);
    const int per = (rows + sp - 1) / sp;
    k_gemv_t_bf16<<<dim3(cb, (rows + per - 1) / per), kGemvThreads, 0, st>>>(w, rows, cols, v, out, per);
    return cudaGetLastError();
}

cudaError_t gemv_t_f32(const float *w, int rows, int cols, const float *v, float *out, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    const int cb = (cols + kGemvThreads * 4 - 1) / (kGemvThreads * 4);
    const int sp = row_splits(rows, cb);
    const int per = (rows + sp - 1) / sp;
    k_gemv_t_f32<<<dim3(cb, (rows + per - 1) / per), kGemvThreads, 0, st>>>(w, rows, cols, v, out, per);
    return cudaGetLastError();
}

cudaError_t gemv_t_fp8(const uint8_t *codes, const float *scales, int rows, int cols, int br, int bc,
                       const float *v, float *out, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    const int scols = (cols + bc - 1) / bc;
    if ((cols & 15) == 0 && (bc & 15) == 0 && (reinterpret_cast<uintptr_t>(codes) & 15) == 0) {
        const int cb = (cols + 511) / 512;
        const int sp = piece_splits(rows, cb, 2);
        const int per = (rows + sp - 1) / sp;
        k_gemv_t_pieces<true><<<dim3(cb, (rows + per - 1) / per), dim3(32, kRowLanes), 0, st>>>(
            codes, scales, rows, cols, br, bc, scols, v, out, per);
        return cudaGetLastError();
    }
    const int cb = (cols + kGemvThreads * 16 - 1) / (kGemvThreads * 16);
    const int sp = row_splits(rows, cb, 16);
    const int per = (rows + sp - 1) / sp;
    k_gemv_t_fp8<<<dim3(cb, (rows + per - 1) / per), kGemvThreads, 0, st>>>(codes, scales, rows, cols, br, bc, scols,
                                                                          v, out, per);
    return cudaGetLastError();
}

size_t gemv_t_mxfp4_scratch(int slabs, int rows, int cols) {
    return (size_t)slabs * ((rows + kMxChunk - 1) / kMxChunk) * cols;
}

cudaError_t gemv_t_mxfp4(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, const float *v,
                         float *out, float *scratch, cudaStream_t st) {
    return gemv_t_mxfp4_stack(blocks, scales, 1, rows, cols, v, out, scratch, st);
}

cudaError_t gemv_t_mxfp4_stack(const uint8_t *blocks, const uint8_t *scales, int slabs, int rows, int cols,
                               const float *v, float *out, float *scratch, cudaStream_t st) {
    if (rows <= 0 || cols <= 0 || slabs <= 0) return cudaSuccess;
    if (cols % 32 || slabs > 65535 || !scratch) return cudaErrorInvalidValue;
    const int gx = (cols / 32 + 31) / 32;
    const int chunks = (rows + kMxChunk - 1) / kMxChunk;
    k_gemv_t_mxfp4<<<dim3(gx, chunks, slabs), dim3(32, kMxLanes), 0, st>>>(blocks, scales, rows, cols, v, scratch,
                                                                         kMxChunk);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long n = (long long)slabs * cols;
    k_sum_parts<<<(int)std::min<long long>((n + 255) / 256, 4096), 256, 0, st>>>(scratch, chunks, slabs, cols, out);
    return cudaGetLastError();
}

cudaError_t row_norms_bf16(const uint16_t *w, int rows, int cols, float *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_row_norms<<<(rows + 7) / 8, 256, 0, st>>>(rows, cols, out, LoadBf16{w, cols});
    return cudaGetLastError();
}

cudaError_t row_norms_f32(const float *w, int rows, int cols, float *out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_row_norms<<<(rows + 7) / 8, 256, 0, st>>>(rows, cols, out, LoadF32{w, cols});
    return cudaGetLastError();
}

cudaError_t row_norms_mxfp4(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, float *out,
                            cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    k_row_norms<<<(rows + 7) / 8, 256, 0, st>>>(rows, cols, out, LoadMxfp4{blocks, scales, cols});
    return cudaGetLastError();
}

cudaError_t rank1_update_bf16(uint16_t *w, int rows, int cols, const float *b, const float *a, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    // 16-byte accesses need every row of w (and a) on a 16-byte boundary
    if ((cols & 7) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
        const int cb = (cols + 2047) / 2048;
        int sp = std::max(1, (8 * 148 + cb - 1) / cb);
        sp = std::min(sp, std::max(1, rows / 16));
        const int per = (rows + sp - 1) / sp;
        k_rank1_bf16<<<dim3(cb, (rows + per - 1) / per), 256, 0, st>>>(w, rows, cols, b, a, per);
    } else {
        const long long n = (long long)rows * cols;
        const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
        k_rank1_bf16_scalar<<<blocks, 256, 0, st>>>(w, rows, cols, b, a);
    }
    return cudaGetLastError();
}

__global__ void k_prenorm_vec(const float *v, const float *n, float lambda, int len, float *vn, float *b) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= len) return;
    const float ni = n[i];
    vn[i] = ni > 0.0f ? v[i] / ni : 0.0f;
    b[i] = -lambda * v[i] * ni;
}

cudaError_t prenorm_vec(const float *v, const float *n, float lambda, int len, float *vn, float *b, cudaStream_t st) {
    if (len <= 0) return cudaSuccess;
    k_prenorm_vec<<<(len + 255) / 256, 256, 0, st>>>(v, n, lambda, len, vn, b);
    return cudaGetLastError();
}

cudaError_t scale_vec(const float *v, float lambda, int n, float *b, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_scale_vec<<<(n + 255) / 256, 256, 0, st>>>(v, lambda, n, b);
    return cudaGetLastError();
}

int kl_chunks(int rows, int vocab) {
    (void)rows;
    return std::max(1, (vocab + kKlPiece - 1) / kKlPiece);
}

size_t kl_scratch_bytes(int rows, int vocab) {
    const size_t n = (size_t)std::max(rows, 1) * kl_chunks(rows, vocab);
    return n * sizeof(double2) + n * sizeof(double);
}

static bool kl_vec(const void *a, const void *b, int vocab) {
    return (vocab & 3) == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0;
}

cudaError_t log_softmax_rows(const float *x, int rows, int vocab, float *out, void *scratch, cudaStream_t st) {
    if (rows <= 0 || vocab <= 0) return cudaSuccess;
    if (rows > 65535) return cudaErrorInvalidValue;  // rows are the grid's y
    const int chunks = kl_chunks(rows, vocab);
    const bool vec = kl_vec(x, out, vocab);
    double2 *part = static_cast<double2 *>(scratch);
    k_lse_part<<<dim3(chunks, rows), kKlThreads, 0, st>>>(x, vocab, vec, part);
    k_log_softmax_part<<<dim3(chunks, rows), kKlThreads, 0, st>>>(x, vocab, vec, part, out);
    return cudaGetLastError();
}

cudaError_t kl_rows(const float *baseline, const float *logits, int rows, int vocab, double *kl, void *scratch,
                    cudaStream_t st) {
    if (rows <= 0 || vocab <= 0) return cudaSuccess;
    if (rows > 65535) return cudaErrorInvalidValue;  // rows are the grid's y
    const int chunks = kl_chunks(rows, vocab);
    const bool vec = kl_vec(baseline, logits, vocab);
    double2 *part = static_cast<double2 *>(scratch);
    double *kl_part = reinterpret_cast<double *>(part + (size_t)rows * chunks);
    k_lse_part<<<dim3(chunks, rows), kKlThreads, 0, st>>>(logits, vocab, vec, part);
    k_kl_part<<<dim3(chunks, rows), kKlThreads, 0, st>>>(baseline, logits, vocab, vec, part, kl_part);
    k_kl_rows_sum<<<(rows + 127) / 128, 128, 0, st>>>(kl_part, rows, chunks, kl);
    return cudaGetLastError();
}

// Runs of at least four prompts, enough of them for about 2048 threads per SM.
static int residual_groups(int entries, int hidden, int prompts) {
    const long long threads = (long long)entries * ((hidden & 3) == 0 ? hidden / 4 : hidden);
    long long g = (148LL * 2048 + threads - 1) / std::max(threads, 1LL);
    g = std::min<long long>(g, (prompts + 3) / 4);
    return (int)std::max(1LL, std::min(g, 65535LL));
}

size_t residual_scratch_bytes(int entries, int hidden, int prompts) {
    return (size_t)residual_groups(entries, hidden, prompts) * std::max(entries, 0) * std::max(hidden, 0) * 8;
}

cudaError_t residual_sums(const float *res, int entries, int nc, int hidden, const int *first, const int *take,
                          int prompts, double *sums, double *scratch, cudaStream_t st) {
    const int per = (hidden & 3) == 0 ? hidden / 4 : hidden;
    const int total = entries * per;
    if (total <= 0 || prompts <= 0) return cudaSuccess;
    if ((hidden & 3) == 0 && (reinterpret_cast<uintptr_t>(res) & 15)) return cudaErrorInvalidValue;
    const int groups = residual_groups(entries, hidden, prompts);
    const int per_group = (prompts + groups - 1) / groups;
    const int used = (prompts + per_group - 1) / per_group;
    k_residual_sums<<<dim3((total + 127) / 128, used), 128, 0, st>>>(res, entries, nc, hidden, first, take, prompts,
                                                                     per_group, scratch);
    const long long n = (long long)entries * hidden;
    k_residual_groups_sum<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(scratch, n, used, sums);
    return cudaGetLastError();
}

cudaError_t directions_from_sums(const double *good_sums, double good_count, const double *bad_sums,
                                 double bad_count, int entries, int hidden, int orthogonalize, float *dirs,
                                 float *good_mean, float *bad_mean, cudaStream_t st) {
    if (entries <= 0) return cudaSuccess;
    k_directions<<<entries, 256, 0, st>>>(good_sums, good_count, bad_sums, bad_count, hidden, orthogonalize, dirs,
                                          good_mean, bad_mean);
    return cudaGetLastError();
}

}  // namespace ditch
