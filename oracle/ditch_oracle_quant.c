/* CPU restatement of ditch's weight decoders: ggml blocks (src/quant.zig) and
 * the safetensors dequantisers (src/dequant.zig). TEST INFRASTRUCTURE: the
 * bit-exact checker for the CUDA decoders. */
#include "ditch_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- ggml block layouts: src/quant.zig:17-42 ---- */
size_t or_ggml_block_size(int dt) {
    switch (dt) {
    case 5: case 6: case 7: case 8: case 9: return 32;
    case 10: case 11: case 12: return 256;
    default: return 1;
    }
}

size_t or_ggml_block_bytes(int dt) {
    switch (dt) {
    case 5: return 34;
    case 6: return 18;
    case 7: return 20;
    case 8: return 22;
    case 9: return 24;
    case 10: return 144;
    case 11: return 210;
    case 12: return 292;
    default: return 0;
    }
}

static float rd_f16(const uint8_t *b) { return or_f16_to_f32((uint16_t)(b[0] | (b[1] << 8))); }

static uint32_t rd_u32(const uint8_t *b) {
    return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

/* src/quant.zig:81-85 */
static void deq_q8_0(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    for (int j = 0; j < 32; j++) y[j] = (float)(int8_t)b[2 + j] * d;
}

/* src/quant.zig:87-96 */
static void deq_q4_0(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    for (int j = 0; j < 16; j++) {
        y[j] = (float)((int)(b[2 + j] & 0x0f) - 8) * d;
        y[j + 16] = (float)((int)(b[2 + j] >> 4) - 8) * d;
    }
}

/* src/quant.zig:98-106 */
static void deq_q4_1(const uint8_t *b, float *y) {
    float d = rd_f16(b), m = rd_f16(b + 2);
    for (int j = 0; j < 16; j++) {
        y[j] = (float)(b[4 + j] & 0x0f) * d + m;
        y[j + 16] = (float)(b[4 + j] >> 4) * d + m;
    }
}

/* src/quant.zig:108-121 */
static void deq_q5_0(const uint8_t *b, float *y) {
    float d = rd_f16(b);
    uint32_t qh = rd_u32(b + 2);
    const uint8_t *qs = b + 6;
    for (int j = 0; j < 16; j++) {
        uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10);
        uint8_t xh1 = (uint8_t)((qh >> (j + 12)) & 0x10);
        y[j] = (float)((int)((qs[j] & 0x0f) | xh0) - 16) * d;
        y[j + 16] = (float)((int)((qs[j] >> 4) | xh1) - 16) * d;
    }
}

/* src/quant.zig:123-137 */
static void deq_q5_1(const uint8_t *b, float *y) {
    float d = rd_f16(b), m = rd_f16(b + 2);
    uint32_t qh = rd_u32(b + 4);
    const uint8_t *qs = b + 8;
    for (int j = 0; j < 16; j++) {
        uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10);
        uint8_t xh1 = (uint8_t)((qh >> (j + 12)) & 0x10);
        y[j] = (float)((qs[j] & 0x0f) | xh0) * d + m;
        y[j + 16] = (float)((qs[j] >> 4) | xh1) * d + m;
    }
}

/* get_scale_min_k4: src/quant.zig:140-146 */
static void scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xf) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* src/quant.zig:148-173 */
static void deq_q4_k(const uint8_t *b, float *y) {
    float d = rd_f16(b), mn = rd_f16(b + 2);
    const uint8_t *sc = b + 4, *q = b + 16;
    int is = 0;
    for (int j = 0; j < 256; j += 64) {
        uint8_t s1, m1, s2, m2;
        scale_min_k4(is, sc, &s1, &m1);
        scale_min_k4(is + 1, sc, &s2, &m2);
        float d1 = d * (float)s1, mm1 = mn * (float)m1;
        float d2 = d * (float)s2, mm2 = mn * (float)m2;
        for (int l = 0; l < 32; l++) y[j + l] = d1 * (float)(q[l] & 0xf) - mm1;
        for (int l = 0; l < 32; l++) y[j + 32 + l] = d2 * (float)(q[l] >> 4) - mm2;
        q += 32;
        is += 2;
    }
}

/* src/quant.zig:175-199 */
static void deq_q6_k(const uint8_t *b, float *y) {
    const uint8_t *ql = b, *qh = b + 128;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = rd_f16(b + 208);
    for (int n = 0; n < 256; n += 128) {
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = (int)((ql[l] & 0xf) | (((qh[l] >> 0) & 3) << 4)) - 32;
            int q2 = (int)((ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[n + l] = d * (float)sc[is] * (float)q1;
            y[n + l + 32] = d * (float)sc[is + 2] * (float)q2;
            y[n + l + 64] = d * (float)sc[is + 4] * (float)q3;
            y[n + l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
        ql += 64;
        qh += 32;
        sc += 8;
    }
}

/* src/quant.zig:203-207 */
static void deq_q8_k(const uint8_t *b, float *y) {
    uint32_t bits = rd_u32(b);
    float d;
    memcpy(&d, &bits, 4);
    for (int j = 0; j < 256; j++) y[j] = d * (float)(int8_t)b[4 + j];
}

/* src/quant.zig:57-79 */
int or_dequant_ggml(int dt, const uint8_t *src, float *out, size_t n) {
    size_t bs = or_ggml_block_size(dt), bb = or_ggml_block_bytes(dt);
    if (bb == 0 || n % bs) return -1;
    size_t nb = n / bs;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = src + i * bb;
        float *y = out + i * bs;
        switch (dt) {
        case 5: deq_q8_0(b, y); break;
        case 6: deq_q4_0(b, y); break;
        case 7: deq_q4_1(b, y); break;
        case 8: deq_q5_0(b, y); break;
        case 9: deq_q5_1(b, y); break;
        case 10: deq_q4_k(b, y); break;
        case 11: deq_q6_k(b, y); break;
        case 12: deq_q8_k(b, y); break;
        default: return -1;
        }
    }
    return 0;
}

/* quantQ8_0: src/quant.zig:245-255 */
void or_quant_q8_0(const float *x, uint8_t *out, size_t n) {
    for (size_t blk = 0; blk < n / 32; blk++) {
        const float *xb = x + blk * 32;
        uint8_t *b = out + blk * 34;
        float amax = 0;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(xb[j]));
        float d = amax / 127.0f;
        float id = d != 0 ? 1.0f / d : 0.0f;
        uint16_t h = or_f32_to_f16(d);
        b[0] = (uint8_t)(h & 0xff);
        b[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 32; j++) b[2 + j] = (uint8_t)(int8_t)roundf(xb[j] * id);
    }
}

/* A simple, valid Q4_K encoder (min/max per 32-element sub-block, 6-bit
 * scale and min codes against the super-block's f16 d and dmin).  The
 * reference ships no Q4_K quantiser; this only produces test blocks whose
 * decode (the part under test) follows src/quant.zig:148-173. */
void or_quant_q4_k(const float *x, uint8_t *out, size_t n) {
    for (size_t blk = 0; blk < n / 256; blk++) {
        const float *xb = x + blk * 256;
        uint8_t *b = out + blk * 144;
        float sc[8], mn[8], max_sc = 0, max_mn = 0;
        for (int s = 0; s < 8; s++) {
            float lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                float v = xb[s * 32 + l];
                lo = fminf(lo, v);
                hi = fmaxf(hi, v);
            }
            sc[s] = (hi - lo) / 15.0f;
            mn[s] = -lo;
            max_sc = fmaxf(max_sc, sc[s]);
            max_mn = fmaxf(max_mn, mn[s]);
        }
        float d = max_sc / 63.0f, dmin = max_mn / 63.0f;
        uint16_t hd = or_f32_to_f16(d), hm = or_f32_to_f16(dmin);
        d = or_f16_to_f32(hd);
        dmin = or_f16_to_f32(hm);
        b[0] = (uint8_t)(hd & 0xff); b[1] = (uint8_t)(hd >> 8);
        b[2] = (uint8_t)(hm & 0xff); b[3] = (uint8_t)(hm >> 8);
        uint8_t ls[8], lm[8];
        for (int s = 0; s < 8; s++) {
            int a = d > 0 ? (int)lrintf(sc[s] / d) : 0, c = dmin > 0 ? (int)lrintf(mn[s] / dmin) : 0;
            ls[s] = (uint8_t)(a < 0 ? 0 : a > 63 ? 63 : a);
            lm[s] = (uint8_t)(c < 0 ? 0 : c > 63 ? 63 : c);
        }
        uint8_t *q = b + 4;
        memset(q, 0, 12);
        for (int j = 0; j < 4; j++) {
            q[j] = (uint8_t)(ls[j] | ((ls[j + 4] >> 4) << 6));
            q[j + 4] = (uint8_t)(lm[j] | ((lm[j + 4] >> 4) << 6));
            q[j + 8] = (uint8_t)((ls[j + 4] & 0xf) | ((lm[j + 4] & 0xf) << 4));
        }
        uint8_t *qs = b + 16;
        for (int s = 0; s < 8; s++) {
            float ds = d * (float)ls[s], ms = dmin * (float)lm[s];
            for (int l = 0; l < 32; l++) {
                int v = ds > 0 ? (int)lrintf((xb[s * 32 + l] + ms) / ds) : 0;
                v = v < 0 ? 0 : v > 15 ? 15 : v;
                int byte = (s / 2) * 32 + l;
                if (s % 2 == 0) qs[byte] = (uint8_t)((qs[byte] & 0xf0) | v);
                else qs[byte] = (uint8_t)((qs[byte] & 0x0f) | (v << 4));
            }
        }
    }
}

/* ---- safetensors decoders: src/dequant.zig ---- */

/* fp8Table(4): src/dequant.zig:281-304 */
float or_e4m3_value(uint8_t code) {
    int sign = code >> 7, exp = (code >> 3) & 0xf, man = code & 7;
    float v;
    if (exp == 0) v = (float)man * 0.125f * ldexpf(1.0f, 1 - 7);
    else if (exp == 15 && man == 7) v = NAN;
    else v = (1.0f + (float)man * 0.125f) * ldexpf(1.0f, exp - 7);
    return sign ? -v : v;
}

/* e8m0Scale: src/dequant.zig:259-261 */
float or_e8m0_scale(uint8_t b) {
    uint32_t bits = b == 0 ? 0x00400000u : ((uint32_t)b << 23);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static const float e2m1[16] = {0, 0.5f, 1, 1.5f, 2, 3, 4, 6, -0.0f, -0.5f, -1, -1.5f, -2, -3, -4, -6};

/* readFp8 per element: bf16(table[code] * scale), src/dequant.zig:505-511 */
void or_dequant_fp8(const uint8_t *codes, const float *scales, size_t rows, size_t cols,
                    size_t br, size_t bc, uint16_t *out) {
    size_t scols = (cols + bc - 1) / bc;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long r = 0; r < (long)rows; r++)
        for (size_t c = 0; c < cols; c++)
            out[r * cols + c] = or_f32_to_bf16(or_e4m3_value(codes[r * cols + c]) * scales[(r / br) * scols + c / bc]);
}

/* unpackField: src/dequant.zig:313-321 */
uint32_t or_unpack_field(const uint32_t *words, size_t i, int bits) {
    size_t start = i * (size_t)bits;
    size_t w = start / 32;
    unsigned off = (unsigned)(start % 32);
    unsigned lo = 32 - off < (unsigned)bits ? 32 - off : (unsigned)bits;
    uint32_t mask_lo = lo >= 32 ? 0xffffffffu : ((1u << lo) - 1);
    uint32_t v = (words[w] >> off) & mask_lo;
    if (lo < (unsigned)bits) {
        unsigned hi = (unsigned)bits - lo;
        v |= (words[w + 1] & ((1u << hi) - 1)) << lo;
    }
    return v;
}

/* readPacked: src/dequant.zig:518-597 */
void or_dequant_int_packed(const uint32_t *packed, size_t wpr, const float *scales,
                           const uint32_t *zeros, const uint32_t *g_idx, size_t rows,
                           size_t cols, int bits, size_t group, uint16_t *out) {
    int offset = 1 << (bits - 1);
    size_t groups = g_idx ? 0 : (cols + group - 1) / group;
    if (g_idx) {
        for (size_t c = 0; c < cols; c++)
            if (g_idx[c] + 1 > groups) groups = g_idx[c] + 1;
    }
    for (size_t r = 0; r < rows; r++) {
        const uint32_t *rw = packed + r * wpr;
        for (size_t c = 0; c < cols; c++) {
            size_t g = g_idx ? g_idx[c] : c / group;
            int zp = 0;
            if (zeros) {
                /* field `r` of column g's word stream, words laid out [words][groups] */
                size_t start = r * (size_t)bits, w = start / 32;
                unsigned off = (unsigned)(start % 32);
                unsigned lo = 32 - off < (unsigned)bits ? 32 - off : (unsigned)bits;
                uint32_t v = (zeros[w * groups + g] >> off) & ((lo >= 32) ? 0xffffffffu : ((1u << lo) - 1));
                if (lo < (unsigned)bits) v |= (zeros[(w + 1) * groups + g] & ((1u << (bits - lo)) - 1)) << lo;
                zp = (int)v - offset;
            }
            int q = (int)or_unpack_field(rw, c, bits) - offset;
            out[r * cols + c] = or_f32_to_bf16((float)(q - zp) * scales[r * groups + g]);
        }
    }
}

/* readMxfp4Packed: src/dequant.zig:643-673 */
void or_dequant_mxfp4_packed(const uint8_t *blocks, const uint8_t *scales, size_t rows,
                             size_t cols, uint16_t *out) {
    size_t nblk = cols / 32, rb = cols / 2;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long r = 0; r < (long)rows; r++)
        for (size_t k = 0; k < nblk; k++) {
            float sc = or_e8m0_scale(scales[r * nblk + k]);
            for (int j = 0; j < 16; j++) {
                uint8_t b = blocks[r * rb + k * 16 + j];
                out[r * cols + k * 32 + 2 * j] = or_f32_to_bf16(e2m1[b & 0xf] * sc);
                out[r * cols + k * 32 + 2 * j + 1] = or_f32_to_bf16(e2m1[b >> 4] * sc);
            }
        }
}

/* decodeMxfp4Slab: src/dequant.zig:603-637 (transposed gpt-oss layout) */
void or_dequant_mxfp4_transposed(const uint8_t *blocks, const uint8_t *scales,
                                 size_t src_rows, size_t src_cols, uint16_t *out) {
    size_t nblk = src_cols / 32;
    for (size_t j = 0; j < src_rows; j++)
        for (size_t k = 0; k < nblk; k++) {
            const uint8_t *b = blocks + (j * nblk + k) * 16;
            float sc = or_e8m0_scale(scales[j * nblk + k]);
            for (int i = 0; i < 16; i++) {
                out[(k * 32 + 2 * i) * src_rows + j] = or_f32_to_bf16(e2m1[b[i] & 0xf] * sc);
                out[(k * 32 + 2 * i + 1) * src_rows + j] = or_f32_to_bf16(e2m1[b[i] >> 4] * sc);
            }
        }
}

/* ---- synthetic-data quantisers: tools/make_fixture.py ---- */
/* The nearest code with the first code winning a tie, as an argmin over all
 * 256 codes in code order gives: the magnitudes of codes 0..126 ascend and
 * the negative codes 128..254 mirror them, so |x| is placed among the 127
 * magnitudes (a tie goes to the smaller one, the lower code) and the sign
 * bit is added for x < 0 unless the nearest magnitude is zero (+0, code 0,
 * comes before -0). |x - t| is sign-symmetric in float, so the distances are
 * the ones the full scan compares. */
static float g_e4m3_mag[127];
static int g_e4m3_ready = 0;

static void e4m3_table(void) {
    if (g_e4m3_ready) return;
    for (int c = 0; c < 127; c++) g_e4m3_mag[c] = or_e4m3_value((uint8_t)c);
    g_e4m3_ready = 1;
}

static uint8_t nearest_e4m3(float x) {
    const float a = fabsf(x);
    int lo = 0, hi = 126;  /* first k with mag[k] >= a, or 126 */
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (g_e4m3_mag[mid] >= a) hi = mid; else lo = mid + 1;
    }
    int k = lo;
    if (k > 0 && fabsf(a - g_e4m3_mag[k - 1]) <= fabsf(a - g_e4m3_mag[k])) k--;
    return (uint8_t)(x < 0 && k > 0 ? (0x80 | k) : k);
}

/* quant_fp8_block: make_fixture.py:109-127 (scale = max(amax, 1e-12) / 448). */
void or_quant_fp8_block(const float *w, size_t rows, size_t cols, size_t br, size_t bc,
                        uint8_t *codes, float *scales) {
    size_t nb0 = (rows + br - 1) / br, nb1 = (cols + bc - 1) / bc;
    e4m3_table();
#pragma omp parallel for schedule(dynamic) num_threads(or_get_threads())
    for (long bi = 0; bi < (long)(nb0 * nb1); bi++) {
        size_t i = (size_t)bi / nb1, j = (size_t)bi % nb1;
        size_t r1 = (i + 1) * br < rows ? (i + 1) * br : rows, c1 = (j + 1) * bc < cols ? (j + 1) * bc : cols;
        float amax = 0;
        for (size_t r = i * br; r < r1; r++)
            for (size_t c = j * bc; c < c1; c++) amax = fmaxf(amax, fabsf(w[r * cols + c]));
        float s = (float)((double)fmaxf(amax, 1e-12f) / 448.0);
        scales[i * nb1 + j] = s;
        for (size_t r = i * br; r < r1; r++)
            for (size_t c = j * bc; c < c1; c++) codes[r * cols + c] = nearest_e4m3(w[r * cols + c] / s);
    }
}

static uint8_t nearest_e2m1(float x) {
    float best = INFINITY;
    int bi = 0;
    for (int c = 0; c < 16; c++) {
        float d = fabsf(x - e2m1[c]);
        if (d < best) { best = d; bi = c; }
    }
    return (uint8_t)bi;
}

/* quant_mxfp4_packed: make_fixture.py:210-224 (scale floor(log2(amax / 6))). */
void or_quant_mxfp4_packed(const float *w, size_t rows, size_t cols, uint8_t *blocks,
                           uint8_t *scales) {
    size_t nblk = cols / 32;
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long r = 0; r < (long)rows; r++)
        for (size_t k = 0; k < nblk; k++) {
            const float *x = w + r * cols + k * 32;
            float amax = 0;
            for (int l = 0; l < 32; l++) amax = fmaxf(amax, fabsf(x[l]));
            int e = amax > 0 ? (int)floor(log2((double)fmaxf(amax, 1e-30f) / 6.0)) : 0;
            e = e < -127 ? -127 : e > 127 ? 127 : e;
            scales[r * nblk + k] = (uint8_t)(e + 127);
            double p = ldexp(1.0, e);
            for (int j = 0; j < 16; j++) {
                float a = (float)fmin(fmax(x[2 * j] / p, -6.0), 6.0);
                float b = (float)fmin(fmax(x[2 * j + 1] / p, -6.0), 6.0);
                blocks[r * (cols / 2) + k * 16 + j] = (uint8_t)(nearest_e2m1(a) | (nearest_e2m1(b) << 4));
            }
        }
}

/* quant_int_packed (asymmetric, contiguous groups): make_fixture.py:156-194.
 * packed [rows][ceil(cols*bits/32)], scales f32 (bf16-rounded) [rows][groups],
 * zeros [ceil(rows*bits/32)][groups]. */
void or_quant_int_packed(const float *w, size_t rows, size_t cols, int bits, size_t group,
                         uint32_t *packed, float *scales, uint32_t *zeros) {
    int qmin = -(1 << (bits - 1)), qmax = (1 << (bits - 1)) - 1, offset = 1 << (bits - 1);
    size_t groups = cols / group, wpr = (cols * bits + 31) / 32, zrows = (rows * bits + 31) / 32;
    memset(packed, 0, sizeof(uint32_t) * rows * wpr);
    memset(zeros, 0, sizeof(uint32_t) * zrows * groups);
    for (size_t r = 0; r < rows; r++)
        for (size_t g = 0; g < groups; g++) {
            const float *x = w + r * cols + g * group;
            float mn = 0, mx = 0;
            for (size_t l = 0; l < group; l++) {
                mn = fminf(mn, x[l]);
                mx = fmaxf(mx, x[l]);
            }
            float s = or_bf16_to_f32(or_f32_to_bf16(fmaxf(mx - mn, 1e-8f) / (float)(qmax - qmin)));
            scales[r * groups + g] = s;
            double zd = nearbyint((double)qmin - (double)mn / (double)s);
            int zp = (int)(zd < qmin ? qmin : zd > qmax ? qmax : zd);
            for (size_t l = 0; l < group; l++) {
                double qd = nearbyint((double)(x[l] / s)) + zp;
                int q = (int)(qd < qmin ? qmin : qd > qmax ? qmax : qd);
                uint32_t u = (uint32_t)(q + offset);
                size_t i = g * group + l, start = i * bits, wd = start / 32, off = start % 32;
                packed[r * wpr + wd] |= u << off;
                if (off + bits > 32) packed[r * wpr + wd + 1] |= u >> (32 - off);
            }
            uint32_t uz = (uint32_t)(zp + offset);
            size_t start = r * bits, wd = start / 32, off = start % 32;
            zeros[wd * groups + g] |= uz << off;
            if (off + bits > 32) zeros[(wd + 1) * groups + g] |= uz >> (32 - off);
        }
}

/* f32 -> bf16 bits over an array (src/tensor.zig:423-430 per element). */
void or_f32_to_bf16_array(const float *x, size_t n, uint16_t *out) {
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long i = 0; i < (long)n; i++) out[i] = or_f32_to_bf16(x[i]);
}
