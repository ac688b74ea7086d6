// Standalone weight decoders, bit-exact against ditch's decode rules:
// src/dequant.zig (FP8 block, pack-quantized INT, MXFP4 in both layouts) and
// src/quant.zig (ggml blocks). Also the plain dtype conversions.
#include "kernels.cuh"

namespace ditch {

namespace {

constexpr int kThreads = 256;

// A block per row, at most eight per SM at a time (grid-stride over rows).
inline int row_grid(int rows) { return rows < 148 * 8 ? (rows < 1 ? 1 : rows) : 148 * 8; }

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int blocks_for(long long n, int per_thread) {
    long long t = (n + per_thread - 1) / per_thread;
    long long b = (t + kThreads - 1) / kThreads;
    return static_cast<int>(b < 1 ? 1 : (b > 1048576 ? 1048576 : b));
}

// fp8Table(4) of src/dequant.zig:281-304 (E4M3 "fn": no infinities, 0x7f / 0xff NaN).
__device__ __forceinline__ float e4m3_value(uint32_t code) {
    const uint32_t sign = code >> 7, exp = (code >> 3) & 0xf, man = code & 7;
    float v;
    if (exp == 0) v = (float)man * 0.125f * 0.015625f;  // man / 8 * 2^-6
    else v = (1.0f + (float)man * 0.125f) * __uint_as_float((exp - 7 + 127) << 23);
    return sign ? -v : v;
}

// bf16 bits of the reference's NaN for an E4M3 NaN code: the table's quiet
// NaN (sign kept) times a finite scale stays that NaN on the host.
__device__ __forceinline__ uint16_t e4m3_nan_bf16(uint32_t code) { return (code & 0x80) ? 0xffc0 : 0x7fc0; }

__device__ __forceinline__ uint16_t fp8_elem(uint32_t code, float s) {
    if ((code & 0x7f) == 0x7f) return e4m3_nan_bf16(code);
    return f32_to_bf16_bits(e4m3_value(code) * s);
}

__global__ void k_dequant_fp8(const uint8_t *codes, const float *scales, int rows, int cols, int br, int bc,
                              int scols, uint16_t *out) {
    const long long total16 = (long long)rows * cols / 16;
    const bool vec = (cols % 16) == 0;
    if (vec) {
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total16;
             i += (long long)gridDim.x * blockDim.x) {
            const long long e0 = i * 16;
            const int r = (int)(e0 / cols), c0 = (int)(e0 % cols);
            uint4 q = *reinterpret_cast<const uint4 *>(codes + e0);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
            uint32_t o[8];
            const float *srow = scales + (long long)(r / br) * scols;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int c = c0 + 2 * j;
                const uint32_t b0 = (w[j / 2] >> (16 * (j & 1))) & 0xff, b1 = (w[j / 2] >> (16 * (j & 1) + 8)) & 0xff;
                const uint16_t lo = fp8_elem(b0, srow[c / bc]), hi = fp8_elem(b1, srow[(c + 1) / bc]);
                o[j] = (uint32_t)lo | ((uint32_t)hi << 16);
            }
            uint4 *dst = reinterpret_cast<uint4 *>(out + e0);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
    } else {
        const long long total = (long long)rows * cols;
        for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
             e += (long long)gridDim.x * blockDim.x) {
            const int r = (int)(e / cols), c = (int)(e % cols);
            out[e] = fp8_elem(codes[e], scales[(long long)(r / br) * scols + c / bc]);
        }
    }
}

// ---- streaming decoders: a block per row (grid-stride over rows); a row is
// cut into pieces of 8 elements (16 bytes of bf16 out) and thread t of the
// block takes pieces t, t + 256, t + 512, t + 768 of each run of 1024, so
// every warp store writes 512 contiguous bytes and every warp load reads 256
// (FP8: 8 codes) or 128 (MXFP4 / INT4: 4 bytes) contiguous bytes; the four
// loads of a run are issued before any conversion. The values come from the
// exact packed conversions (cvt e4m3x2 / e2m1x2 to f16x2), the f32 product
// with the scale and one round to bf16, as the rules above; the codes the
// packed path does not follow (E4M3 NaN codes, the E8M0 255 scale) take the
// element rules.

// true when one of the word's four E4M3 codes is a NaN (0x7f or 0xff)
__device__ __forceinline__ bool e4m3_nan_in(uint32_t w) {
    const uint32_t t = (w & 0x7f7f7f7fu) ^ 0x7f7f7f7fu;  // a zero byte marks a NaN code
    return ((t - 0x01010101u) & ~t & 0x80808080u) != 0;
}

// four E4M3 codes of one word with one block scale to two bf16x2 words
__device__ __forceinline__ void fp8_word(uint32_t w, float s, uint32_t &o0, uint32_t &o1) {
    o0 = scale_pack(e4m3x2_f32(w & 0xffff), s);
    o1 = scale_pack(e4m3x2_f32(w >> 16), s);
    if (e4m3_nan_in(w)) {
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const uint32_t code = (w >> (8 * b)) & 0xff;
            if ((code & 0x7f) == 0x7f) {
                uint32_t &word = (b >> 1) ? o1 : o0;
                const int sh = 16 * (b & 1);
                word = (word & ~(0xffffu << sh)) | ((uint32_t)e4m3_nan_bf16(code) << sh);
            }
        }
    }
}

__device__ __forceinline__ uint16_t mxfp4_elem(uint32_t nib, uint32_t b);

// eight E2M1 nibbles (one word, low nibble first) with E8M0 scale b
__device__ __forceinline__ uint4 mxfp4_word(uint32_t w, uint32_t b) {
    if (b == 255) {  // the +inf scale: the element rule's NaN / inf
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t byte = (w >> (8 * e)) & 0xff;
            o[e] = (uint32_t)mxfp4_elem(byte & 0xf, b) | ((uint32_t)mxfp4_elem(byte >> 4, b) << 16);
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
    }
    const float s = e8m0_scale(b);
    return make_uint4(scale_pack(e2m1x2_f32(w & 0xff), s), scale_pack(e2m1x2_f32((w >> 8) & 0xff), s),
                      scale_pack(e2m1x2_f32((w >> 16) & 0xff), s), scale_pack(e2m1x2_f32(w >> 24), s));
}

constexpr int kPieceSlots = 4;

// FP8 block-scaled; cols and the column block a multiple of 8
__global__ void __launch_bounds__(kThreads) k_dequant_fp8_rows(const uint8_t *codes, const float *scales, int rows,
                                                               int cols, int br, int bc, int scols, uint16_t *out) {
    const int pieces = cols / 8;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint2 *crow = reinterpret_cast<const uint2 *>(codes + (long long)r * cols);
        const float *srow = scales + (long long)(r / br) * scols;
        uint4 *orow = reinterpret_cast<uint4 *>(out + (long long)r * cols);
        for (int p0 = threadIdx.x; p0 < pieces; p0 += kPieceSlots * kThreads) {
            uint2 q[kPieceSlots];
            float sc[kPieceSlots];
#pragma unroll
            for (int k = 0; k < kPieceSlots; k++) {
                const int p = p0 + k * kThreads;
                q[k] = p < pieces ? __ldg(crow + p) : make_uint2(0, 0);
                sc[k] = p < pieces ? __ldg(srow + (p * 8) / bc) : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < kPieceSlots; k++) {
                const int p = p0 + k * kThreads;
                if (p >= pieces) break;
                uint4 o;
                fp8_word(q[k].x, sc[k], o.x, o.y);
                fp8_word(q[k].y, sc[k], o.z, o.w);
                orow[p] = o;
            }
        }
    }
}

// MXFP4 natural layout; cols a multiple of 32 (a piece lies in one scale block)
__global__ void __launch_bounds__(kThreads) k_dequant_mxfp4_rows(const uint8_t *blocks, const uint8_t *scales, int rows,
                                                                 int cols, uint16_t *out) {
    const int pieces = cols / 8;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint32_t *brow = reinterpret_cast<const uint32_t *>(blocks + (long long)r * (cols / 2));
        const uint8_t *srow = scales + (long long)r * (cols / 32);
        uint4 *orow = reinterpret_cast<uint4 *>(out + (long long)r * cols);
        for (int p0 = threadIdx.x; p0 < pieces; p0 += kPieceSlots * kThreads) {
            uint32_t q[kPieceSlots], b[kPieceSlots];
#pragma unroll
            for (int k = 0; k < kPieceSlots; k++) {
                const int p = p0 + k * kThreads;
                q[k] = p < pieces ? __ldg(brow + p) : 0u;
                b[k] = p < pieces ? __ldg(srow + p / 4) : 0u;
            }
#pragma unroll
            for (int k = 0; k < kPieceSlots; k++) {
                const int p = p0 + k * kThreads;
                if (p >= pieces) break;
                orow[p] = mxfp4_word(q[k], b[k]);
            }
        }
    }
}

// INT4 pack-quantized without g_idx, groups a multiple of 8: the 8 fields of
// a word share a group's scale and zero point; bf16(f32(q - zq) * scale)
// with q, zq the raw fields (the offset cancels).
__global__ void __launch_bounds__(kThreads) k_dequant_int4_rows(const uint32_t *packed, long long wpr,
                                                                const float *scales, const uint32_t *zeros,
                                                                int groups, int rows, int cols, int group,
                                                                uint16_t *out) {
    const int pieces = cols / 8;
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const uint32_t *prow = packed + (long long)r * wpr;
        const float *srow = scales + (long long)r * groups;
        const uint32_t *zrow = zeros ? zeros + (long long)(r >> 3) * groups : nullptr;
        const int zsh = (r & 7) * 4;
        uint4 *orow = reinterpret_cast<uint4 *>(out + (long long)r * cols);
        for (int p0 = threadIdx.x; p0 < pieces; p0 += kPieceSlots * kThreads) {
            uint32_t q[kPieceSlots];
            float sc[kPieceSlots];
            int zq[kPieceSlots];
#pragma unroll
            for (int k = 0; k < kPieceSlots; k++) {
                const int p = p0 + k * kThreads;
                const int g = (p * 8) / group;
                q[k] = p < pieces ? __ldg(prow + p) : 0u;
                sc[k] = p < pieces ? __ldg(srow + g) : 0.0f;
                zq[k] = (zrow && p < pieces) ? (int)((__ldg(zrow + g) >> zsh) & 0xf) : 8;
            }
#pragma unroll
            for (int k = 0; k < kPieceSlots; k++) {
                const int p = p0 + k * kThreads;
                if (p >= pieces) break;
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int lo = (int)((q[k] >> (8 * e)) & 0xf) - zq[k], hi = (int)((q[k] >> (8 * e + 4)) & 0xf) - zq[k];
                    o[e] = scale_pack(make_float2((float)lo, (float)hi), sc[k]);
                }
                orow[p] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
}

// unpackField (src/dequant.zig:313-321): field i of `bits` bits in a
// little-endian u32 word stream.
__device__ __forceinline__ uint32_t unpack_field(const uint32_t *words, long long i, int bits) {
    const long long start = i * bits;
    const long long w = start >> 5;
    const int off = (int)(start & 31);
    const int lo = min(32 - off, bits);
    uint32_t v = (words[w] >> off) & (lo >= 32 ? 0xffffffffu : ((1u << lo) - 1));
    if (lo < bits) v |= (words[w + 1] & ((1u << (bits - lo)) - 1)) << lo;
    return v;
}

__global__ void k_dequant_int(const uint32_t *packed, long long wpr, const float *scales, const uint32_t *zeros,
                              const uint32_t *g_idx, int groups, int rows, int cols, int bits, int group,
                              uint16_t *out) {
    const long long total = (long long)rows * cols;
    const int offset = 1 << (bits - 1);
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(e / cols), c = (int)(e % cols);
        const int g = g_idx ? (int)g_idx[c] : c / group;
        int zp = 0;
        if (zeros) {
            // field r of column g's word stream; words laid out [words][groups]
            const long long start = (long long)r * bits, w = start >> 5;
            const int off = (int)(start & 31), lo = min(32 - off, bits);
            uint32_t v = (zeros[w * groups + g] >> off) & (lo >= 32 ? 0xffffffffu : ((1u << lo) - 1));
            if (lo < bits) v |= (zeros[(w + 1) * groups + g] & ((1u << (bits - lo)) - 1)) << lo;
            zp = (int)v - offset;
        }
        const int q = (int)unpack_field(packed + (long long)r * wpr, c, bits) - offset;
        out[e] = f32_to_bf16_bits((float)(q - zp) * scales[(long long)r * groups + g]);
    }
}

__device__ __constant__ float kE2M1v[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                                            -0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

// bf16(e2m1[nib] * 2^(b - 127)) (src/dequant.zig:259-261). For b = 255 the
// scale is +inf: the host's 0 * inf is the x86 default NaN (sign set).
__device__ __forceinline__ uint16_t mxfp4_elem(uint32_t nib, uint32_t b) {
    if (b == 255) {
        if ((nib & 7) == 0) return 0xffc0;
        return (nib & 8) ? 0xff80 : 0x7f80;
    }
    const float s = __uint_as_float(b == 0 ? 0x00400000u : (b << 23));
    return f32_to_bf16_bits(kE2M1v[nib] * s);
}

__global__ void k_dequant_mxfp4(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, uint16_t *out) {
    const long long total = (long long)rows * cols / 2;  // one byte -> two elements
    const int nblk = cols / 32;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long e = 2 * i;
        const int r = (int)(e / cols), c = (int)(e % cols);
        const uint32_t byte = blocks[i], b = scales[(long long)r * nblk + c / 32];
        const uint32_t v = (uint32_t)mxfp4_elem(byte & 0xf, b) | ((uint32_t)mxfp4_elem(byte >> 4, b) << 16);
        *reinterpret_cast<uint32_t *>(out + e) = v;
    }
}

// Source [src_rows][src_cols/32][16] bytes + [src_rows][src_cols/32] scales;
// out [src_cols][src_rows] (the transpose, src/dequant.zig:603-637).
__global__ void k_dequant_mxfp4t(const uint8_t *blocks, const uint8_t *scales, int src_rows, int src_cols,
                                 uint16_t *out) {
    const long long total = (long long)src_rows * src_cols;
    const int nblk = src_cols / 32;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        // output element (h, j): h = source column, j = source row; j fastest
        const int h = (int)(e / src_rows), j = (int)(e % src_rows);
        const int k = h / 32, i = (h % 32) / 2;
        const uint32_t byte = blocks[((long long)j * nblk + k) * 16 + i];
        const uint32_t nib = (h & 1) ? (byte >> 4) : (byte & 0xf);
        out[e] = mxfp4_elem(nib, scales[(long long)j * nblk + k]);
    }
}

// ---- ggml blocks (src/quant.zig:57-209) ----
__device__ __forceinline__ float rd_f16(const uint8_t *b) {
    return __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
}

__device__ float ggml_elem(int dt, const uint8_t *blk, int j) {
    switch (dt) {
    case 5: return (float)(int8_t)blk[2 + j] * rd_f16(blk);  // q8_0
    case 6: {                                                 // q4_0
        const int b = blk[2 + (j & 15)];
        const int x = (j < 16 ? (b & 0xf) : (b >> 4)) - 8;
        return (float)x * rd_f16(blk);
    }
    case 7: {  // q4_1
        const int b = blk[4 + (j & 15)];
        return (float)(j < 16 ? (b & 0xf) : (b >> 4)) * rd_f16(blk) + rd_f16(blk + 2);
    }
    case 8: {  // q5_0
        const uint32_t qh = blk[2] | (blk[3] << 8) | (blk[4] << 16) | ((uint32_t)blk[5] << 24);
        const int jj = j & 15, b = blk[6 + jj];
        int x;
        if (j < 16) x = ((b & 0xf) | (int)(((qh >> jj) << 4) & 0x10)) - 16;
        else x = ((b >> 4) | (int)((qh >> (jj + 12)) & 0x10)) - 16;
        return (float)x * rd_f16(blk);
    }
    case 9: {  // q5_1
        const uint32_t qh = blk[4] | (blk[5] << 8) | (blk[6] << 16) | ((uint32_t)blk[7] << 24);
        const int jj = j & 15, b = blk[8 + jj];
        int x;
        if (j < 16) x = (b & 0xf) | (int)(((qh >> jj) << 4) & 0x10);
        else x = (b >> 4) | (int)((qh >> (jj + 12)) & 0x10);
        return (float)x * rd_f16(blk) + rd_f16(blk + 2);
    }
    case 10: {  // q4_k: 4 groups of 64, each 32 low nibbles then 32 high nibbles
        const float d = rd_f16(blk), mn = rd_f16(blk + 2);
        const uint8_t *q = blk + 4;
        const int grp = j / 64, within = j % 64, is = 2 * grp + (within >= 32 ? 1 : 0);
        uint32_t sc, m;
        if (is < 4) {
            sc = q[is] & 63;
            m = q[is + 4] & 63;
        } else {
            sc = (q[is + 4] & 0xf) | ((q[is - 4] >> 6) << 4);
            m = (q[is + 4] >> 4) | ((q[is] >> 6) << 4);
        }
        const uint8_t b = blk[16 + grp * 32 + (within & 31)];
        const uint32_t nib = within < 32 ? (b & 0xf) : (b >> 4);
        return d * (float)sc * (float)nib - mn * (float)m;
    }
    case 11: {  // q6_k
        const int half = j / 128, l = j % 128, part = l / 32, ll = l % 32, is = ll / 16;
        const uint8_t *ql = blk + 64 * half, *qh = blk + 128 + 32 * half;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * half);
        const float d = rd_f16(blk + 208);
        int q;
        switch (part) {
        case 0: q = (int)((ql[ll] & 0xf) | (((qh[ll] >> 0) & 3) << 4)) - 32; break;
        case 1: q = (int)((ql[ll + 32] & 0xf) | (((qh[ll] >> 2) & 3) << 4)) - 32; break;
        case 2: q = (int)((ql[ll] >> 4) | (((qh[ll] >> 4) & 3) << 4)) - 32; break;
        default: q = (int)((ql[ll + 32] >> 4) | (((qh[ll] >> 6) & 3) << 4)) - 32; break;
        }
        return d * (float)sc[is + 2 * part] * (float)q;
    }
    case 12: {  // q8_k
        const uint32_t bits = blk[0] | (blk[1] << 8) | (blk[2] << 16) | ((uint32_t)blk[3] << 24);
        return __uint_as_float(bits) * (float)(int8_t)blk[4 + j];
    }
    }
    return 0.0f;
}

__host__ __device__ inline int ggml_bs(int dt) { return dt >= 10 ? 256 : 32; }
__host__ __device__ inline int ggml_bb(int dt) {
    switch (dt) {
    case 5: return 34;
    case 6: return 18;
    case 7: return 20;
    case 8: return 22;
    case 9: return 24;
    case 10: return 144;
    case 11: return 210;
    case 12: return 292;
    }
    return 0;
}

template <bool BF16>
__global__ void k_dequant_ggml(int dt, const uint8_t *src, long long n, void *out) {
    const int bs = ggml_bs(dt), bb = ggml_bb(dt);
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const float v = ggml_elem(dt, src + (e / bs) * bb, (int)(e % bs));
        if (BF16) reinterpret_cast<uint16_t *>(out)[e] = f32_to_bf16_bits(v);
        else reinterpret_cast<float *>(out)[e] = v;
    }
}

// Q8_0 blocks (f16 d, 32 x int8; src/quant.zig:81-85) of `rows` rows to the
// GEMM's layout: int8 codes [rows][cols] and f32 scales [rows][cols / 32].
__global__ void k_repack_q8_0(const uint8_t *src, long long blocks, int8_t *codes, float *scales) {
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < blocks;
         b += (long long)gridDim.x * blockDim.x) {
        const uint8_t *blk = src + b * 34;
        const uint16_t dbits = (uint16_t)blk[0] | ((uint16_t)blk[1] << 8);
        scales[b] = __half2float(__ushort_as_half(dbits));
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            w[i] = (uint32_t)blk[2 + 4 * i] | ((uint32_t)blk[3 + 4 * i] << 8) | ((uint32_t)blk[4 + 4 * i] << 16) |
                   ((uint32_t)blk[5 + 4 * i] << 24);
        uint4 *dst = reinterpret_cast<uint4 *>(codes + b * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// Q4_K super-blocks (f16 d, f16 dmin, 12 bytes of 6-bit scales / mins, 128
// bytes of nibbles; src/quant.zig:140-173) to the GEMM's layout: 4-bit codes
// in element order (byte i: elements 2i, 2i + 1, low nibble first) and per
// 32-element sub-block the f32 pair (d * scale, dmin * min), both products
// exact. One thread per output byte; sub-block is = e / 32 of the super-block.
__global__ void k_repack_q4_k(const uint8_t *src, long long n_bytes, uint8_t *codes, float2 *dm) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_bytes;
         i += (long long)gridDim.x * blockDim.x) {
        const long long b = i / 128;
        const int e = (int)(i % 128) * 2;  // first element of the pair in the super-block
        const uint8_t *blk = src + b * 144, *sc = blk + 4, *qs = blk + 16;
        const int grp = e / 64, l = e % 32;
        const bool high = (e % 64) >= 32;
        const uint8_t b0 = qs[grp * 32 + l], b1 = qs[grp * 32 + l + 1];
        codes[i] = high ? (uint8_t)((b0 >> 4) | (b1 & 0xf0)) : (uint8_t)((b0 & 0xf) | ((b1 & 0xf) << 4));
        if ((e & 31) == 0) {
            const int is = e / 32;
            uint32_t s, m;
            if (is < 4) {
                s = sc[is] & 63;
                m = sc[is + 4] & 63;
            } else {
                s = (sc[is + 4] & 0xf) | ((sc[is - 4] >> 6) << 4);
                m = (sc[is + 4] >> 4) | ((sc[is] >> 6) << 4);
            }
            const float d = rd_f16(blk), dmin = rd_f16(blk + 2);
            dm[b * 8 + is] = make_float2(__fmul_rn(d, (float)s), __fmul_rn(dmin, (float)m));
        }
    }
}

// The repacked Q4_K values as f32 (d1 * q - m1, src/quant.zig:148-173).
__global__ void k_q4_k_f32(const uint8_t *codes, const float2 *dm, long long n, float *out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const uint32_t q = (codes[i / 2] >> (4 * (i & 1))) & 0xf;
        const float2 v = dm[i / 32];
        out[i] = __fsub_rn(__fmul_rn(v.x, (float)q), v.y);
    }
}

// The repacked Q8_0 values as f32 (d * q, exact as src/quant.zig:81-85).
__global__ void k_q8_0_f32(const int8_t *codes, const float *scales, long long n, float *out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = scales[i / 32] * (float)codes[i];
}

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

__global__ void k_f32_to_bf16(const float *src, uint16_t *dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = f32_to_bf16_bits(src[i]);
}

__global__ void k_bf16_to_f32(const uint16_t *src, float *dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = bf16_bits_to_f32(src[i]);
}

__global__ void k_f16_to_f32(const uint16_t *src, float *dst, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = __half2float(__ushort_as_half(src[i]));
}

}  // namespace

cudaError_t repack_q8_0(const uint8_t *src, long long blocks, int8_t *codes, float *scales, cudaStream_t st) {
    if (blocks <= 0) return cudaSuccess;
    k_repack_q8_0<<<blocks_for(blocks, 1), kThreads, 0, st>>>(src, blocks, codes, scales);
    return cudaGetLastError();
}

cudaError_t repack_q4_k(const uint8_t *src, long long super_blocks, uint8_t *codes, float *dm, cudaStream_t st) {
    if (super_blocks <= 0) return cudaSuccess;
    k_repack_q4_k<<<blocks_for(super_blocks * 128, 1), kThreads, 0, st>>>(src, super_blocks * 128, codes,
                                                                         reinterpret_cast<float2 *>(dm));
    return cudaGetLastError();
}

cudaError_t q4_k_f32(const uint8_t *codes, const float *dm, long long n, float *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_q4_k_f32<<<blocks_for(n, 4), kThreads, 0, st>>>(codes, reinterpret_cast<const float2 *>(dm), n, out);
    return cudaGetLastError();
}

cudaError_t q8_0_f32(const int8_t *codes, const float *scales, long long n, float *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    k_q8_0_f32<<<blocks_for(n, 4), kThreads, 0, st>>>(codes, scales, n, out);
    return cudaGetLastError();
}

cudaError_t dequant_fp8_bf16(const uint8_t *codes, const float *scales, int rows, int cols, int br, int bc,
                             uint16_t *out, cudaStream_t st) {
    if (br <= 0 || bc <= 0) return cudaErrorInvalidValue;
    const int scols = (cols + bc - 1) / bc;
    const long long n = (long long)rows * cols;
    if (cols % 8 == 0 && bc % 8 == 0 && aligned16(codes) && aligned16(out)) {
        k_dequant_fp8_rows<<<row_grid(rows), kThreads, 0, st>>>(codes, scales, rows, cols, br, bc, scols, out);
        return cudaGetLastError();
    }
    k_dequant_fp8<<<blocks_for(n, (cols % 16) ? 1 : 16), kThreads, 0, st>>>(codes, scales, rows, cols, br, bc, scols,
                                                                            out);
    return cudaGetLastError();
}

cudaError_t dequant_int_bf16(const uint32_t *packed, long long wpr, const float *scales, const uint32_t *zeros,
                             const uint32_t *g_idx, int groups, int rows, int cols, int bits, int group,
                             uint16_t *out, cudaStream_t st) {
    if (bits < 1 || bits > 8 || (!g_idx && group <= 0)) return cudaErrorInvalidValue;
    if (bits == 4 && !g_idx && group % 8 == 0 && cols % 8 == 0 && wpr == cols / 8 && aligned16(packed) &&
        aligned16(out)) {
        k_dequant_int4_rows<<<row_grid(rows), kThreads, 0, st>>>(packed, wpr, scales, zeros, groups, rows, cols, group,
                                                                 out);
        return cudaGetLastError();
    }
    k_dequant_int<<<blocks_for((long long)rows * cols, 1), kThreads, 0, st>>>(packed, wpr, scales, zeros, g_idx, groups,
                                                                            rows, cols, bits, group, out);
    return cudaGetLastError();
}

cudaError_t dequant_mxfp4_bf16(const uint8_t *blocks, const uint8_t *scales, int rows, int cols, uint16_t *out,
                               cudaStream_t st) {
    if (cols % 32) return cudaErrorInvalidValue;
    if (aligned16(blocks) && aligned16(out)) {
        k_dequant_mxfp4_rows<<<row_grid(rows), kThreads, 0, st>>>(blocks, scales, rows, cols, out);
        return cudaGetLastError();
    }
    k_dequant_mxfp4<<<blocks_for((long long)rows * cols / 2, 1), kThreads, 0, st>>>(blocks, scales, rows, cols, out);
    return cudaGetLastError();
}

cudaError_t dequant_mxfp4t_bf16(const uint8_t *blocks, const uint8_t *scales, int src_rows, int src_cols,
                                uint16_t *out, cudaStream_t st) {
    if (src_cols % 32) return cudaErrorInvalidValue;
    k_dequant_mxfp4t<<<blocks_for((long long)src_rows * src_cols, 1), kThreads, 0, st>>>(blocks, scales, src_rows,
                                                                                       src_cols, out);
    return cudaGetLastError();
}

cudaError_t dequant_ggml_f32(int dtype, const uint8_t *src, long long n, float *out, cudaStream_t st) {
    if (dtype < 5 || dtype > 12 || n % ggml_bs(dtype)) return cudaErrorInvalidValue;
    k_dequant_ggml<false><<<blocks_for(n, 1), kThreads, 0, st>>>(dtype, src, n, out);
    return cudaGetLastError();
}

cudaError_t dequant_ggml_bf16(int dtype, const uint8_t *src, long long n, uint16_t *out, cudaStream_t st) {
    if (dtype < 5 || dtype > 12 || n % ggml_bs(dtype)) return cudaErrorInvalidValue;
    k_dequant_ggml<true><<<blocks_for(n, 1), kThreads, 0, st>>>(dtype, src, n, out);
    return cudaGetLastError();
}

cudaError_t split_bf16(const float *src, int rows, int cols, int cp, int nseg, int pattern, uint16_t *dst,
                       cudaStream_t st) {
    if (rows <= 0 || cp <= 0) return cudaSuccess;
    k_split<<<blocks_for((long long)rows * cp, 1), kThreads, 0, st>>>(src, rows, cols, cp, nseg, pattern, dst);
    return cudaGetLastError();
}

cudaError_t f32_to_bf16(const float *src, uint16_t *dst, long long n, cudaStream_t st) {
    k_f32_to_bf16<<<blocks_for(n, 1), kThreads, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t bf16_to_f32(const uint16_t *src, float *dst, long long n, cudaStream_t st) {
    k_bf16_to_f32<<<blocks_for(n, 1), kThreads, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t f16_to_f32(const uint16_t *src, float *dst, long long n, cudaStream_t st) {
    k_f16_to_f32<<<blocks_for(n, 1), kThreads, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

}  // namespace ditch
