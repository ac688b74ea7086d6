/* CPU restatement of ditch's f32 kernels (src/tensor.zig). TEST INFRASTRUCTURE:
 * the parity checker and CPU baseline for the CUDA product; never shipped in
 * the product path.  Compiled with -ffp-contract=off so that a multiply-add is
 * fused exactly where the reference fuses it (its `fma` helper,
 * src/tensor.zig:685-687), and nowhere else. */
#include "ditch_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define VL 16 /* src/tensor.zig:653-655, the AVX-512 shape */

static int g_threads = 0;

void or_set_threads(int n) { g_threads = n; }

int or_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- conversions: src/tensor.zig:419-440 ---- */
float or_bf16_to_f32(uint16_t v) {
    uint32_t b = (uint32_t)v << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

uint16_t or_f32_to_bf16(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40); /* NaN */
    uint32_t lsb = (bits >> 16) & 1u;
    return (uint16_t)((bits + 0x7fffu + lsb) >> 16);
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t or_f32_to_f16(float v) {
    /* round to nearest even, as Zig's @floatCast */
    _Float16 h = (_Float16)v;
    uint16_t r;
    memcpy(&r, &h, 2);
    return r;
}

void or_bf16_to_f32_n(const uint16_t *src, float *dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = or_bf16_to_f32(src[i]);
}

void or_f32_to_bf16_n(const float *src, uint16_t *dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = or_f32_to_bf16(src[i]);
}

/* ---- dot: src/tensor.zig:550-558 ----
 * VL lanes of fused multiply-adds over whole blocks, one ordered reduction,
 * then the tail with scalar fused multiply-adds. */
static inline float reduce16(const float *acc) {
    float s = acc[0];
    for (int l = 1; l < VL; l++) s += acc[l];
    return s;
}

float or_dot(const float *a, const float *b, size_t n) {
    float acc[VL] = {0};
    size_t i = 0;
    for (; i + VL <= n; i += VL)
        for (int l = 0; l < VL; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s = reduce16(acc);
    for (; i < n; i++) s = fmaf(a[i], b[i], s);
    return s;
}

#if defined(__x86_64__)
/* The same per-output arithmetic as or_dot with four weight rows against four
 * inputs at once (the register tile of src/tensor.zig:889-913); every output
 * is bit-identical to or_dot of its two rows. */
__attribute__((target("avx512f,fma"))) static void tile4x4_avx512(
    const float *w, const float *x, size_t cols, size_t ldo, float *out) {
    __m512 acc[4][4];
    for (int i = 0; i < 4; i++)
        for (int k = 0; k < 4; k++) acc[i][k] = _mm512_setzero_ps();
    size_t c = 0;
    for (; c + VL <= cols; c += VL) {
        __m512 wv0 = _mm512_loadu_ps(w + 0 * cols + c), wv1 = _mm512_loadu_ps(w + 1 * cols + c);
        __m512 wv2 = _mm512_loadu_ps(w + 2 * cols + c), wv3 = _mm512_loadu_ps(w + 3 * cols + c);
        for (int i = 0; i < 4; i++) {
            __m512 xv = _mm512_loadu_ps(x + i * cols + c);
            acc[i][0] = _mm512_fmadd_ps(wv0, xv, acc[i][0]);
            acc[i][1] = _mm512_fmadd_ps(wv1, xv, acc[i][1]);
            acc[i][2] = _mm512_fmadd_ps(wv2, xv, acc[i][2]);
            acc[i][3] = _mm512_fmadd_ps(wv3, xv, acc[i][3]);
        }
    }
    for (int i = 0; i < 4; i++)
        for (int k = 0; k < 4; k++) {
            float lanes[VL];
            _mm512_storeu_ps(lanes, acc[i][k]);
            float s = reduce16(lanes);
            for (size_t t = c; t < cols; t++) s = fmaf(w[k * cols + t], x[i * cols + t], s);
            out[i * ldo + k] = s;
        }
}

static int have_avx512(void) {
    static int v = -1;
    if (v < 0) {
        __builtin_cpu_init();
        v = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("fma");
    }
    return v;
}
#endif

/* matmulT: src/tensor.zig:1023-1045 (+ matmulWorker 827-883 for the delta
 * order: out += sum_j b[r][j] * xa[i][j], xa = dot(a_j, x_i)). */
void or_matmul_t(float *out, const float *x, size_t n, const float *w, size_t rows,
                 size_t cols, const float *da, const float *db, size_t rank) {
    if (rows == 0 || n == 0) return;
    const int fast =
#if defined(__x86_64__)
        have_avx512();
#else
        0;
#endif
    const long rblocks = (long)((rows + 3) / 4);
#pragma omp parallel for schedule(dynamic, 4) num_threads(or_get_threads())
    for (long rb = 0; rb < rblocks; rb++) {
        size_t r0 = (size_t)rb * 4;
        size_t nr = rows - r0 < 4 ? rows - r0 : 4;
        size_t i = 0;
#if defined(__x86_64__)
        if (fast && nr == 4)
            for (; i + 4 <= n; i += 4) tile4x4_avx512(w + r0 * cols, x + i * cols, cols, rows, out + i * rows + r0);
#endif
        for (; i < n; i++)
            for (size_t k = 0; k < nr; k++)
                out[i * rows + r0 + k] = or_dot(w + (r0 + k) * cols, x + i * cols, cols);
    }
    if (da && db && rank > 0) {
        float *xa = (float *)malloc(sizeof(float) * n * rank);
        for (size_t i = 0; i < n; i++)
            for (size_t j = 0; j < rank; j++) xa[i * rank + j] = or_dot(da + j * cols, x + i * cols, cols);
        for (size_t i = 0; i < n; i++)
            for (size_t r = 0; r < rows; r++) {
                float v = 0;
                for (size_t j = 0; j < rank; j++) v += db[r * rank + j] * xa[i * rank + j];
                out[i * rows + r] += v;
            }
        free(xa);
    }
}

void or_matmul_t_bf16(float *out, const float *x, size_t n, const uint16_t *w, size_t rows,
                      size_t cols, const float *da, const float *db, size_t rank) {
    if (rows == 0 || n == 0) return;
    const int fast =
#if defined(__x86_64__)
        have_avx512();
#else
        0;
#endif
    const long rblocks = (long)((rows + 3) / 4);
#pragma omp parallel num_threads(or_get_threads())
    {
        float *buf = (float *)malloc(sizeof(float) * 4 * cols);  /* this task's rows as f32 */
#pragma omp for schedule(dynamic, 4)
        for (long rb = 0; rb < rblocks; rb++) {
            size_t r0 = (size_t)rb * 4;
            size_t nr = rows - r0 < 4 ? rows - r0 : 4;
            for (size_t k = 0; k < nr; k++)
                for (size_t c = 0; c < cols; c++) buf[k * cols + c] = or_bf16_to_f32(w[(r0 + k) * cols + c]);
            size_t i = 0;
#if defined(__x86_64__)
            if (fast && nr == 4)
                for (; i + 4 <= n; i += 4) tile4x4_avx512(buf, x + i * cols, cols, rows, out + i * rows + r0);
#endif
            for (; i < n; i++)
                for (size_t k = 0; k < nr; k++) out[i * rows + r0 + k] = or_dot(buf + k * cols, x + i * cols, cols);
        }
        free(buf);
    }
    if (da && db && rank > 0) {
        float *xa = (float *)malloc(sizeof(float) * n * rank);
        for (size_t i = 0; i < n; i++)
            for (size_t j = 0; j < rank; j++) xa[i * rank + j] = or_dot(da + j * cols, x + i * cols, cols);
        for (size_t i = 0; i < n; i++)
            for (size_t r = 0; r < rows; r++) {
                float v = 0;
                for (size_t j = 0; j < rank; j++) v += db[r * rank + j] * xa[i * rank + j];
                out[i * rows + r] += v;
            }
        free(xa);
    }
}

/* matvecTMulti with one accumulator slot: out[j] = sum_r y[j][r] * W_r,
 * rows with y == 0 skipped, `axpy` unfused (src/tensor.zig:560-570,
 * 1056-1094). The column range is split across threads; each column keeps
 * the reference's row order. */
void or_matvec_t_multi(float *out, const float *w, size_t rows, size_t cols, const float *y,
                       size_t q) {
    memset(out, 0, sizeof(float) * q * cols);
    const long cblocks = (long)((cols + 255) / 256);
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long cb = 0; cb < cblocks; cb++) {
        size_t c0 = (size_t)cb * 256, c1 = c0 + 256 < cols ? c0 + 256 : cols;
        for (size_t r = 0; r < rows; r++)
            for (size_t j = 0; j < q; j++) {
                float yr = y[j * rows + r];
                if (yr == 0) continue;
                const float *wr = w + r * cols;
                float *o = out + j * cols;
                for (size_t c = c0; c < c1; c++) o[c] = o[c] + yr * wr[c];
            }
    }
}

void or_row_norms(float *out, const float *w, size_t rows, size_t cols) {
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long r = 0; r < (long)rows; r++) out[r] = sqrtf(or_dot(w + r * cols, w + r * cols, cols));
}

/* ---- element-wise: src/tensor.zig:1167-1294 ---- */
void or_rmsnorm(float *out, const float *x, const float *w, size_t len, float eps) {
    float ss = 0;
    for (size_t i = 0; i < len; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)len + eps);
    if (!w) {
        for (size_t i = 0; i < len; i++) out[i] = x[i] * inv;
    } else {
        for (size_t i = 0; i < len; i++) out[i] = x[i] * inv * w[i];
    }
}

/* expVec (src/tensor.zig:1280-1294): Cephes expf, a published method. */
void or_exp_vec16(const float *xin, float *out) {
    for (int l = 0; l < VL; l++) {
        float x = xin[l];
        x = fminf(fmaxf(x, -87.3f), 88.0f);
        /* Zig's @round rounds half away from zero, as roundf */
        float fx = roundf(x * 1.44269504088896341f);
        float r = fmaf(fx, 2.12194440e-4f, fmaf(fx, -0.693359375f, x));
        float y = 1.9875691500e-4f;
        y = fmaf(y, r, 1.3981999507e-3f);
        y = fmaf(y, r, 8.3334519073e-3f);
        y = fmaf(y, r, 4.1665795894e-2f);
        y = fmaf(y, r, 1.6666665459e-1f);
        y = fmaf(y, r, 5.0000001201e-1f);
        y = fmaf(y, r * r, r + 1.0f);
        int32_t e = (int32_t)fx;
        uint32_t bits = (uint32_t)(e + 127) << 23;
        float s;
        memcpy(&s, &bits, 4);
        out[l] = y * s;
    }
}

void or_softmax_inplace(float *x, size_t n) {
    float mv[VL];
    for (int l = 0; l < VL; l++) mv[l] = -INFINITY;
    size_t i = 0;
    for (; i + VL <= n; i += VL)
        for (int l = 0; l < VL; l++) mv[l] = fmaxf(mv[l], x[i + l]);
    float m = mv[0];
    for (int l = 1; l < VL; l++) m = fmaxf(m, mv[l]);
    for (; i < n; i++) m = fmaxf(m, x[i]);
    float sv[VL] = {0};
    i = 0;
    for (; i + VL <= n; i += VL) {
        float t[VL], e[VL];
        for (int l = 0; l < VL; l++) t[l] = x[i + l] - m;
        or_exp_vec16(t, e);
        for (int l = 0; l < VL; l++) {
            x[i + l] = e[l];
            sv[l] += e[l];
        }
    }
    float s = reduce16(sv);
    for (; i < n; i++) {
        x[i] = expf(x[i] - m);
        s += x[i];
    }
    float inv = 1.0f / s;
    for (size_t k = 0; k < n; k++) x[k] *= inv;
}

void or_log_softmax(float *out, const float *x, size_t n) {
    float m = -INFINITY;
    for (size_t i = 0; i < n; i++) m = fmaxf(m, x[i]);
    double s = 0;
    for (size_t i = 0; i < n; i++) s += exp((double)(x[i] - m));
    float lse = m + (float)log(s);
    for (size_t i = 0; i < n; i++) out[i] = x[i] - lse;
}

float or_silu(float x) { return x / (1.0f + expf(-x)); }

void or_gated_silu(float *out, const float *gate, const float *up, size_t n, size_t len,
                   size_t in_stride, size_t out_stride) {
#pragma omp parallel for schedule(static) num_threads(or_get_threads())
    for (long i = 0; i < (long)n; i++) {
        const float *g = gate + i * in_stride;
        const float *u = up ? up + i * in_stride : NULL;
        float *o = out + i * out_stride;
        size_t j = 0;
        for (; j + VL <= len; j += VL) {
            float t[VL], e[VL];
            for (int l = 0; l < VL; l++) t[l] = -g[j + l];
            or_exp_vec16(t, e);
            for (int l = 0; l < VL; l++) {
                float v = g[j + l] / (1.0f + e[l]);
                if (u) v *= u[j + l];
                o[j + l] = v;
            }
        }
        for (; j < len; j++) {
            float v = or_silu(g[j]);
            if (u) v *= u[j];
            o[j] = v;
        }
    }
}

void or_apply_rope(float *x, const float *c, const float *s, size_t dim) {
    size_t half = dim / 2;
    for (size_t i = 0; i < half; i++) {
        float x1 = x[i], x2 = x[i + half];
        x[i] = x1 * c[i] - x2 * s[i];
        x[i + half] = x2 * c[i] + x1 * s[i];
    }
}

/* fillRope (src/model.zig:2200-2282): inverse frequencies theta^(-2i/dim),
 * scaled per r->scaling, then cos / sin of the f64 angles times the
 * attention factor, cast to f32. */
void or_rope_table_ex(float *cos_t, float *sin_t, size_t len, size_t dim, double theta, const or_rope *r) {
    size_t half = dim / 2;
    double *inv = (double *)malloc(sizeof(double) * (half ? half : 1));
    double attn = 1.0;
    for (size_t i = 0; i < half; i++) inv[i] = 1.0 / pow(theta, (double)(2 * i) / (double)dim);
    if (r->scaling == 1) { /* llama3 */
        double low_wavelen = r->orig_max / r->low_ff, high_wavelen = r->orig_max / r->high_ff;
        for (size_t i = 0; i < half; i++) {
            double wavelen = 2.0 * M_PI / inv[i];
            if (wavelen < high_wavelen) {
            } else if (wavelen > low_wavelen) {
                inv[i] /= r->factor;
            } else {
                double smooth = (r->orig_max / wavelen - r->low_ff) / (r->high_ff - r->low_ff);
                inv[i] = (1.0 - smooth) * inv[i] / r->factor + smooth * inv[i];
            }
        }
    } else if (r->scaling == 2) { /* linear */
        for (size_t i = 0; i < half; i++) inv[i] /= r->factor;
    } else if (r->scaling == 3) { /* yarn: ramp between the correction dims */
        double d = (double)dim;
        double lo = d * log(r->orig_max / (r->beta_fast * 2.0 * M_PI)) / (2.0 * log(theta));
        double hi = d * log(r->orig_max / (r->beta_slow * 2.0 * M_PI)) / (2.0 * log(theta));
        if (r->truncate) {
            lo = floor(lo);
            hi = ceil(hi);
        }
        if (lo < 0) lo = 0;
        if (hi > d - 1) hi = d - 1;
        if (lo == hi) hi += 0.001;
        for (size_t i = 0; i < half; i++) {
            double ramp = ((double)i - lo) / (hi - lo);
            ramp = ramp < 0 ? 0 : (ramp > 1 ? 1 : ramp);
            double keep = 1.0 - ramp;
            inv[i] = inv[i] / r->factor * (1.0 - keep) + inv[i] * keep;
        }
        attn = r->attention_factor;
    } else if (r->scaling == 4) { /* per-frequency divisors */
        for (size_t i = 0; i < half && i < r->n_factors; i++) inv[i] /= (double)r->factors[i];
        attn = r->attention_factor;
    }
    for (size_t p = 0; p < len; p++)
        for (size_t i = 0; i < half; i++) {
            double a = (double)p * inv[i];
            cos_t[p * half + i] = (float)(cos(a) * attn);
            sin_t[p * half + i] = (float)(sin(a) * attn);
        }
    free(inv);
}

void or_rope_table(float *cos_t, float *sin_t, size_t len, size_t dim, double theta,
                   int scaling, double factor, double low_ff, double high_ff, double orig_max) {
    or_rope r = {scaling, factor, low_ff, high_ff, orig_max, NULL, 0, 1.0, 32.0, 1.0, 1};
    or_rope_table_ex(cos_t, sin_t, len, dim, theta, &r);
}
