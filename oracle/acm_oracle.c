/*
 * acm_oracle.c -- CPU ORACLE (test infrastructure only).
 *
 * A plain-C restatement of the reference's token loop (Quad4-Software/
 * auto-commit-msg, package internal/infer plus internal/gguf).  It exists to
 * CHECK the CUDA engine and to time the reference algorithm on host cores.
 * Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline and
 * --impl reference legs) may load it.  The product never calls it.
 *
 * Parity status: the reference is Go and no Go toolchain exists here, so the
 * restatement cannot be run against the reference binary.  The dequantizers
 * are pinned against an independent implementation of the same ggml block
 * formats (gguf-py 0.19.0 `gguf.quants`, fixtures in tests/golden/); the
 * Forward/sampler restatement is pinned only by its own tests ("parity
 * unpinned" against the Go binary).
 *
 * Citations are internal/<pkg>/<file>:<line> in the reference tree.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#ifdef __AVX2__
#include <immintrin.h>
#endif

#define OR_API __attribute__((visibility("default")))

/* ggml tensor types, gguf/gguf.go:31-40 */
enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

/* BlockSize, gguf/gguf.go:70-90: (elements per block, bytes per block) */
OR_API int or_block_size(uint32_t typ, int *bs, int *ts) {
    switch (typ) {
    case T_F32: *bs = 1; *ts = 4; return 1;
    case T_F16: *bs = 1; *ts = 2; return 1;
    case T_Q4_0: *bs = 32; *ts = 18; return 1;
    case T_Q5_0: *bs = 32; *ts = 22; return 1;
    case T_Q8_0: *bs = 32; *ts = 34; return 1;
    case T_Q4_K: *bs = 256; *ts = 144; return 1;
    case T_Q5_K: *bs = 256; *ts = 176; return 1;
    case T_Q6_K: *bs = 256; *ts = 210; return 1;
    }
    *bs = 0; *ts = 0;
    return 0;
}

/* ------------------------------------------------------------------ */
/* f16 / dequant: infer/tensor.go:17-226 (the scalar path, the one     */
/* ACM_NO_ASM_DEQUANT=1 selects, tensor.go:45-53)                       */
/* ------------------------------------------------------------------ */

static inline uint16_t rd16(const uint8_t *b) { return (uint16_t)(b[0] | (b[1] << 8)); }
static inline uint32_t rd32(const uint8_t *b) {
    return (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
}

/* f16, tensor.go:17-40 */
OR_API float or_f16(uint16_t h) {
    uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    float f;
    if (e == 0) {
        f = (float)m * 0x1p-24f;
    } else if (e == 31) {
        f = m ? NAN : INFINITY;
    } else {
        f = (float)m * 0x1p-10f;
        f += 1.0f;
        f *= (float)ldexp(1.0, (int)e - 15);
    }
    return s ? -f : f;
}

static inline float f32le(const uint8_t *b) {
    uint32_t u = rd32(b);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* dequantQ80, tensor.go:83-92 */
static void dq_q8_0(const uint8_t *row, float *dst, int64_t n) {
    for (int64_t b = 0; b * 32 < n; b++) {
        float d = or_f16(rd16(row));
        const uint8_t *qs = row + 2;
        for (int j = 0; j < 32; j++) dst[b * 32 + j] = d * (float)(int8_t)qs[j];
        row += 34;
    }
}

/* dequantQ40, tensor.go:94-105 */
static void dq_q4_0(const uint8_t *row, float *dst, int64_t n) {
    for (int64_t b = 0; b * 32 < n; b++) {
        float d = or_f16(rd16(row));
        const uint8_t *qs = row + 2;
        for (int j = 0; j < 16; j++) {
            dst[b * 32 + j] = d * (float)((int)(qs[j] & 0x0f) - 8);
            dst[b * 32 + j + 16] = d * (float)((int)(qs[j] >> 4) - 8);
        }
        row += 18;
    }
}

/* dequantQ50, tensor.go:106-122 */
static void dq_q5_0(const uint8_t *row, float *dst, int64_t n) {
    for (int64_t b = 0; b * 32 < n; b++) {
        const uint8_t *blk = row + b * 22;
        float d = or_f16(rd16(blk));
        uint32_t qh = rd32(blk + 2);
        const uint8_t *qs = blk + 6;
        for (int j = 0; j < 16; j++) {
            int x0 = (int)(qs[j] & 0x0f) | (int)((qh >> j) & 1) << 4;
            int x1 = (int)(qs[j] >> 4) | (int)((qh >> (j + 16)) & 1) << 4;
            dst[b * 32 + j] = d * (float)(x0 - 16);
            dst[b * 32 + j + 16] = d * (float)(x1 - 16);
        }
    }
}

/* scaleMinK4, tensor.go:123-130 */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* dequantQ4K, tensor.go:132-158 */
static void dq_q4_k(const uint8_t *row, float *dst, int64_t n) {
    for (int64_t nb = 0; nb * 256 < n; nb++) {
        const uint8_t *blk = row + nb * 144;
        float d = or_f16(rd16(blk)), dmin = or_f16(rd16(blk + 2));
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        float *y = dst + nb * 256;
        int yi = 0, is = 0;
        for (int j = 0; j < 256; j += 64) {
            const uint8_t *q = qs + j / 2;
            uint8_t sc, m;
            scale_min_k4(is, scales, &sc, &m);
            float d1 = d * (float)sc, m1 = dmin * (float)m;
            scale_min_k4(is + 1, scales, &sc, &m);
            float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) y[yi++] = d1 * (float)(q[l] & 0x0f) - m1;
            for (int l = 0; l < 32; l++) y[yi++] = d2 * (float)(q[l] >> 4) - m2;
            is += 2;
        }
    }
}

/* dequantQ5K, tensor.go:160-198 */
static void dq_q5_k(const uint8_t *row, float *dst, int64_t n) {
    for (int64_t nb = 0; nb * 256 < n; nb++) {
        const uint8_t *blk = row + nb * 176;
        float d = or_f16(rd16(blk)), dmin = or_f16(rd16(blk + 2));
        const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
        float *y = dst + nb * 256;
        int yi = 0, is = 0;
        uint8_t u1 = 1, u2 = 2;
        for (int j = 0; j < 256; j += 64) {
            const uint8_t *ql = qs + j / 2;
            uint8_t sc, m;
            scale_min_k4(is, scales, &sc, &m);
            float d1 = d * (float)sc, m1 = dmin * (float)m;
            scale_min_k4(is + 1, scales, &sc, &m);
            float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) {
                float add = (qh[l] & u1) ? 16.0f : 0.0f;
                y[yi++] = d1 * ((float)(ql[l] & 0x0f) + add) - m1;
            }
            for (int l = 0; l < 32; l++) {
                float add = (qh[l] & u2) ? 16.0f : 0.0f;
                y[yi++] = d2 * ((float)(ql[l] >> 4) + add) - m2;
            }
            is += 2;
            u1 = (uint8_t)(u1 << 2);
            u2 = (uint8_t)(u2 << 2);
        }
    }
}

/* dequantQ6K, tensor.go:200-226 */
static void dq_q6_k(const uint8_t *row, float *dst, int64_t n) {
    for (int64_t nb = 0; nb * 256 < n; nb++) {
        const uint8_t *blk = row + nb * 210;
        const uint8_t *ql = blk, *qh = blk + 128;
        const int8_t *scales = (const int8_t *)(blk + 192);
        float d = or_f16(rd16(blk + 208));
        for (int nn = 0; nn < 256; nn += 128) {
            int i = nn / 128;
            const uint8_t *qlb = ql + 64 * i, *qhb = qh + 32 * i;
            const int8_t *sc = scales + 8 * i;
            float *y = dst + nb * 256 + nn;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int8_t q1 = (int8_t)((qlb[l] & 0x0f) | ((qhb[l] & 3) << 4)) - 32;
                int8_t q2 = (int8_t)((qlb[l + 32] & 0x0f) | (((qhb[l] >> 2) & 3) << 4)) - 32;
                int8_t q3 = (int8_t)((qlb[l] >> 4) | (((qhb[l] >> 4) & 3) << 4)) - 32;
                int8_t q4 = (int8_t)((qlb[l + 32] >> 4) | (((qhb[l] >> 6) & 3) << 4)) - 32;
                y[l] = d * (float)sc[is] * (float)q1;
                y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                y[l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
        }
    }
}

/* dequantRowSlow, tensor.go:55-81.  Returns 0 on an unsupported type where
 * the reference panics (tensor.go:79). */
OR_API int or_dequant_row(uint32_t typ, const uint8_t *row, float *dst, int64_t n) {
    switch (typ) {
    case T_F32: for (int64_t i = 0; i < n; i++) dst[i] = f32le(row + 4 * i); return 1;
    case T_F16: for (int64_t i = 0; i < n; i++) dst[i] = or_f16(rd16(row + 2 * i)); return 1;
    case T_Q8_0: dq_q8_0(row, dst, n); return 1;
    case T_Q4_0: dq_q4_0(row, dst, n); return 1;
    case T_Q5_0: dq_q5_0(row, dst, n); return 1;
    case T_Q4_K: dq_q4_k(row, dst, n); return 1;
    case T_Q5_K: dq_q5_k(row, dst, n); return 1;
    case T_Q6_K: dq_q6_k(row, dst, n); return 1;
    }
    return 0;
}

static int64_t row_bytes_of(uint32_t typ, int64_t k) {
    int bs, ts;
    if (!or_block_size(typ, &bs, &ts)) return 0;
    return k / bs * ts; /* Tensor.RowBytes, gguf.go:52-59 */
}

/* Dequantize nrows consecutive rows of K elements. */
OR_API int or_dequant_rows(uint32_t typ, const uint8_t *data, int64_t nrows, int64_t k, float *dst) {
    int64_t rb = row_bytes_of(typ, k);
    if (!rb) return 0;
    for (int64_t r = 0; r < nrows; r++)
        if (!or_dequant_row(typ, data + r * rb, dst + r * k, k)) return 0;
    return 1;
}

/* ------------------------------------------------------------------ */
/* dot / dot4 / axpy: infer/dot.go:6-31, dot_amd64.s:33-181             */
/* The AVX2 bodies keep the reference's accumulator structure: dot uses */
/* four 8-lane accumulators over 32-element strides, dot4 two per       */
/* output over 16-element strides; scalar tails as dispatch_amd64.go.   */
/* ------------------------------------------------------------------ */

#ifdef __AVX2__
static inline float hsum8(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s);
}
#endif

static float dot(const float *a, const float *b, int64_t n) {
#ifdef __AVX2__
    int64_t n8 = n & ~(int64_t)7, i = 0;
    float s = 0;
    if (n8 > 0) {
        __m256 y0 = _mm256_setzero_ps(), y1 = y0, y2 = y0, y3 = y0;
        for (; i + 32 <= n8; i += 32) {
            y0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), y0);
            y1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), y1);
            y2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 16), _mm256_loadu_ps(b + i + 16), y2);
            y3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 24), _mm256_loadu_ps(b + i + 24), y3);
        }
        for (; i < n8; i += 8) y0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), y0);
        s = hsum8(_mm256_add_ps(_mm256_add_ps(y0, y1), _mm256_add_ps(y2, y3)));
    }
    for (; i < n; i++) s += a[i] * b[i];
    return s;
#else
    /* dotScalar, dot.go:6-19 */
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int64_t n4 = n & ~(int64_t)3, i;
    for (i = 0; i < n4; i += 4) {
        s0 += a[i] * b[i];
        s1 += a[i + 1] * b[i + 1];
        s2 += a[i + 2] * b[i + 2];
        s3 += a[i + 3] * b[i + 3];
    }
    for (; i < n; i++) s0 += a[i] * b[i];
    return s0 + s1 + s2 + s3;
#endif
}

static void dot4(const float *w, const float *a, const float *b, const float *c, const float *d, int64_t n,
                 float *r0, float *r1, float *r2, float *r3) {
    float s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int64_t i = 0;
#ifdef __AVX2__
    int64_t n8 = n & ~(int64_t)7;
    if (n8 > 0) {
        __m256 y0 = _mm256_setzero_ps(), y1 = y0, y2 = y0, y3 = y0, y4 = y0, y5 = y0, y6 = y0, y7 = y0;
        for (; i + 16 <= n8; i += 16) {
            __m256 w0 = _mm256_loadu_ps(w + i), w1 = _mm256_loadu_ps(w + i + 8);
            y0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(a + i), y0);
            y1 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(b + i), y1);
            y2 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(c + i), y2);
            y3 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(d + i), y3);
            y4 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(a + i + 8), y4);
            y5 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(b + i + 8), y5);
            y6 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(c + i + 8), y6);
            y7 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(d + i + 8), y7);
        }
        for (; i < n8; i += 8) {
            __m256 w0 = _mm256_loadu_ps(w + i);
            y0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(a + i), y0);
            y1 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(b + i), y1);
            y2 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(c + i), y2);
            y3 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(d + i), y3);
        }
        s0 = hsum8(_mm256_add_ps(y0, y4));
        s1 = hsum8(_mm256_add_ps(y1, y5));
        s2 = hsum8(_mm256_add_ps(y2, y6));
        s3 = hsum8(_mm256_add_ps(y3, y7));
    }
#endif
    for (; i < n; i++) {
        float v = w[i];
        s0 += v * a[i];
        s1 += v * b[i];
        s2 += v * c[i];
        s3 += v * d[i];
    }
    *r0 = s0; *r1 = s1; *r2 = s2; *r3 = s3;
}

static void axpy(float *dst, float w, const float *src, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] += w * src[i];
}

/* ------------------------------------------------------------------ */
/* parFor + matmul: infer/tensor.go:228-303                             */
/* ------------------------------------------------------------------ */

static int g_threads = 0; /* 0 = all host cores, runtime.NumCPU(), tensor.go:228 */

OR_API void or_set_threads(int n) { g_threads = n; }
OR_API int or_get_threads(void) {
    if (g_threads > 0) return g_threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef void (*par_fn)(void *ctx, int64_t lo, int64_t hi, int worker);
typedef struct {
    par_fn fn;
    void *ctx;
    int64_t lo, hi;
    int worker;
} par_job;

static void *par_tramp(void *p) {
    par_job *j = (par_job *)p;
    j->fn(j->ctx, j->lo, j->hi, j->worker);
    return NULL;
}

/* parFor, tensor.go:234-248: n items split into NumCPU contiguous ranges */
static void par_for(int64_t n, par_fn fn, void *ctx) {
    int procs = or_get_threads();
    if (n <= 0) return;
    int64_t step = (n + procs - 1) / procs;
    int nj = (int)((n + step - 1) / step);
    if (nj <= 1) {
        fn(ctx, 0, n, 0);
        return;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * nj);
    par_job *jobs = (par_job *)malloc(sizeof(par_job) * nj);
    int w = 0;
    for (int64_t p = 0; p < n; p += step, w++) {
        jobs[w].fn = fn;
        jobs[w].ctx = ctx;
        jobs[w].lo = p;
        jobs[w].hi = p + step < n ? p + step : n;
        jobs[w].worker = w;
    }
    for (int i = 1; i < nj; i++) pthread_create(&th[i], NULL, par_tramp, &jobs[i]);
    par_tramp(&jobs[0]);
    for (int i = 1; i < nj; i++) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
}

typedef struct {
    float *dst;
    const uint8_t *w;
    uint32_t typ;
    int64_t n, d, rb;
    const float *x;
    int m, br;
} mm_ctx;

static void mm_body(void *vc, int64_t lo, int64_t hi, int worker) {
    (void)worker;
    mm_ctx *c = (mm_ctx *)vc;
    int64_t d = c->d, n = c->n;
    int br = c->br, m = c->m;
    float *buf = (float *)malloc(sizeof(float) * (size_t)br * (size_t)d);
    for (int64_t b0 = lo * br; b0 < hi * br && b0 < n; b0 += br) {
        int rows = (int)((n - b0) < br ? (n - b0) : br);
        for (int r = 0; r < rows; r++) or_dequant_row(c->typ, c->w + (b0 + r) * c->rb, buf + (int64_t)r * d, d);
        int j = 0;
        for (; j + 4 <= m; j += 4) {
            const float *x0 = c->x + (int64_t)j * d, *x1 = x0 + d, *x2 = x1 + d, *x3 = x2 + d;
            for (int r = 0; r < rows; r++) {
                float s0, s1, s2, s3;
                dot4(buf + (int64_t)r * d, x0, x1, x2, x3, d, &s0, &s1, &s2, &s3);
                int64_t i = b0 + r;
                c->dst[(int64_t)j * n + i] = s0;
                c->dst[(int64_t)(j + 1) * n + i] = s1;
                c->dst[(int64_t)(j + 2) * n + i] = s2;
                c->dst[(int64_t)(j + 3) * n + i] = s3;
            }
        }
        for (; j < m; j++) {
            const float *xj = c->x + (int64_t)j * d;
            for (int r = 0; r < rows; r++) c->dst[(int64_t)j * n + b0 + r] = dot(buf + (int64_t)r * d, xj, d);
        }
    }
    free(buf);
}

/* matmul, tensor.go:253-298: dst[m][n] = x[m][d] . w[n][d]; weight rows in
 * tiles of br = min(256KiB/(4d), 64) (>= 4) rows, dequantized once per tile. */
OR_API int or_matmul(float *dst, uint32_t typ, const uint8_t *w, int64_t n, int64_t d, const float *x, int m) {
    int64_t rb = row_bytes_of(typ, d);
    if (!rb) return 0;
    int br = (int)(256 * 1024 / (4 * d));
    if (br > 64) br = 64;
    if (br < 4) br = 4;
    mm_ctx c = {dst, w, typ, n, d, rb, x, m, br};
    par_for((n + br - 1) / br, mm_body, &c);
    return 1;
}

/* ------------------------------------------------------------------ */
/* GGUF parse: internal/gguf/gguf.go:121-174                            */
/* ------------------------------------------------------------------ */

enum { V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64 };

typedef struct {
    char *key;
    int vtype;      /* value type tag, gguf.go:14-28 */
    int etype;      /* element type for arrays */
    uint64_t u;     /* integer payload (also bool) */
    double f;       /* float payload */
    char *s;        /* string payload */
    uint64_t alen;  /* array length */
    char **astr;    /* string array elements */
    uint64_t *aint; /* integer array elements */
} or_kv;

typedef struct {
    char *name;
    uint32_t ndims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t offset;
    int64_t numel;
    const uint8_t *data;
    uint64_t nbytes;
} or_tensor;

typedef struct or_file {
    uint32_t version;
    int nkv;
    or_kv *kv;
    int ntensors;
    or_tensor *t;
    void *map;
    size_t maplen;
    char err[256];
} or_file;

typedef struct {
    const uint8_t *b;
    size_t len, pos;
    int bad;
} rdr;

static const uint8_t *take(rdr *r, size_t n) {
    if (r->bad || r->pos + n > r->len) {
        r->bad = 1;
        return NULL;
    }
    const uint8_t *p = r->b + r->pos;
    r->pos += n;
    return p;
}
static uint32_t ru32(rdr *r) { const uint8_t *p = take(r, 4); return p ? rd32(p) : 0; }
static uint64_t ru64(rdr *r) {
    const uint8_t *p = take(r, 8);
    return p ? ((uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32)) : 0;
}
static char *rstr(rdr *r) {
    uint64_t n = ru64(r);
    const uint8_t *p = take(r, n);
    if (!p) return NULL;
    char *s = (char *)malloc(n + 1);
    memcpy(s, p, n);
    s[n] = 0;
    return s;
}

/* reader.value / valueTyped, gguf.go:279-347 */
static int read_scalar(rdr *r, int typ, uint64_t *u, double *f, char **s) {
    const uint8_t *p;
    *u = 0; *f = 0; *s = NULL;
    switch (typ) {
    case V_U8: p = take(r, 1); if (!p) return 0; *u = p[0]; return 1;
    case V_I8: p = take(r, 1); if (!p) return 0; *u = (uint64_t)(int64_t)(int8_t)p[0]; return 1;
    case V_U16: p = take(r, 2); if (!p) return 0; *u = rd16(p); return 1;
    case V_I16: p = take(r, 2); if (!p) return 0; *u = (uint64_t)(int64_t)(int16_t)rd16(p); return 1;
    case V_U32: *u = ru32(r); return !r->bad;
    case V_I32: *u = (uint64_t)(int64_t)(int32_t)ru32(r); return !r->bad;
    case V_U64: *u = ru64(r); return !r->bad;
    case V_I64: *u = ru64(r); return !r->bad;
    case V_F32: { uint32_t b = ru32(r); float x; memcpy(&x, &b, 4); *f = x; return !r->bad; }
    case V_F64: { uint64_t b = ru64(r); double x; memcpy(&x, &b, 8); *f = x; return !r->bad; }
    case V_BOOL: p = take(r, 1); if (!p) return 0; *u = p[0] != 0; return 1;
    case V_STR: *s = rstr(r); return *s != NULL;
    }
    return 0;
}

OR_API void or_gguf_close(or_file *f);

OR_API or_file *or_gguf_parse(const uint8_t *data, size_t len, char *err, int errlen) {
    rdr r = {data, len, 0, 0};
    or_file *f = (or_file *)calloc(1, sizeof(or_file));
    const uint8_t *magic = take(&r, 4);
    if (!magic || memcmp(magic, "GGUF", 4) != 0) {
        snprintf(err, errlen, "not a GGUF file");
        free(f);
        return NULL;
    }
    f->version = ru32(&r);
    if (f->version != 3 && f->version != 2) {
        snprintf(err, errlen, "unsupported GGUF version %u", f->version);
        free(f);
        return NULL;
    }
    uint64_t nt = ru64(&r), nkv = ru64(&r);
    if (r.bad || nkv > (1u << 24) || nt > (1u << 24)) {
        snprintf(err, errlen, "truncated GGUF header");
        free(f);
        return NULL;
    }
    f->kv = (or_kv *)calloc(nkv ? nkv : 1, sizeof(or_kv));
    for (uint64_t i = 0; i < nkv && !r.bad; i++) {
        or_kv *kv = &f->kv[f->nkv];
        kv->key = rstr(&r);
        kv->vtype = (int)ru32(&r);
        if (r.bad) break;
        f->nkv++;
        if (kv->vtype == V_ARR) {
            kv->etype = (int)ru32(&r);
            kv->alen = ru64(&r);
            if (r.bad || kv->alen > len) { r.bad = 1; break; }
            if (kv->etype == V_STR) kv->astr = (char **)calloc(kv->alen + 1, sizeof(char *));
            else kv->aint = (uint64_t *)calloc(kv->alen + 1, sizeof(uint64_t));
            for (uint64_t a = 0; a < kv->alen && !r.bad; a++) {
                uint64_t u; double fl; char *s;
                if (!read_scalar(&r, kv->etype, &u, &fl, &s)) { r.bad = 1; break; }
                if (kv->etype == V_STR) kv->astr[a] = s;
                else kv->aint[a] = u;
            }
        } else {
            if (!read_scalar(&r, kv->vtype, &kv->u, &kv->f, &kv->s)) r.bad = 1;
        }
    }
    if (r.bad) {
        snprintf(err, errlen, "truncated GGUF metadata");
        or_gguf_close(f);
        return NULL;
    }
    f->t = (or_tensor *)calloc(nt ? nt : 1, sizeof(or_tensor));
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        or_tensor *t = &f->t[i];
        t->name = rstr(&r);
        t->ndims = ru32(&r);
        if (t->ndims > 4) { r.bad = 1; break; }
        t->numel = 1;
        for (uint32_t j = 0; j < t->ndims; j++) {
            t->dims[j] = ru64(&r);
            t->numel *= (int64_t)t->dims[j];
        }
        t->type = ru32(&r);
        t->offset = ru64(&r);
        if (!r.bad) f->ntensors++;
    }
    if (r.bad) {
        snprintf(err, errlen, "truncated GGUF tensor index");
        or_gguf_close(f);
        return NULL;
    }
    uint64_t align = 32;
    for (int i = 0; i < f->nkv; i++)
        if (!strcmp(f->kv[i].key, "general.alignment")) align = f->kv[i].u;
    if (align == 0) align = 32;
    uint64_t start = ((uint64_t)r.pos + align - 1) / align * align;
    for (int i = 0; i < f->ntensors; i++) {
        or_tensor *t = &f->t[i];
        int bs, ts;
        if (!or_block_size(t->type, &bs, &ts)) {
            snprintf(err, errlen, "tensor %s: unsupported type %u", t->name, t->type);
            or_gguf_close(f);
            return NULL;
        }
        uint64_t size = (uint64_t)(t->numel / bs) * (uint64_t)ts;
        uint64_t abs_ = start + t->offset;
        if (abs_ + size > len) {
            snprintf(err, errlen, "tensor %s: out of bounds", t->name);
            or_gguf_close(f);
            return NULL;
        }
        t->data = data + abs_;
        t->nbytes = size;
    }
    return f;
}

OR_API or_file *or_gguf_open(const char *path, char *err, int errlen) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        snprintf(err, errlen, "open %s: %s", path, strerror(errno));
        return NULL;
    }
    struct stat st;
    fstat(fd, &st);
    void *m = mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) {
        snprintf(err, errlen, "mmap %s failed", path);
        return NULL;
    }
    or_file *f = or_gguf_parse((const uint8_t *)m, (size_t)st.st_size, err, errlen);
    if (!f) {
        munmap(m, (size_t)st.st_size);
        return NULL;
    }
    f->map = m;
    f->maplen = (size_t)st.st_size;
    return f;
}

OR_API void or_gguf_close(or_file *f) {
    if (!f) return;
    for (int i = 0; i < f->nkv; i++) {
        or_kv *kv = &f->kv[i];
        free(kv->key);
        free(kv->s);
        if (kv->astr) {
            for (uint64_t a = 0; a < kv->alen; a++) free(kv->astr[a]);
            free(kv->astr);
        }
        free(kv->aint);
    }
    free(f->kv);
    for (int i = 0; i < f->ntensors; i++) free(f->t[i].name);
    free(f->t);
    if (f->map) munmap(f->map, f->maplen);
    free(f);
}

static or_kv *find_kv(or_file *f, const char *key) {
    for (int i = 0; i < f->nkv; i++)
        if (!strcmp(f->kv[i].key, key)) return &f->kv[i];
    return NULL;
}

/* File.Str / U64 / F32 / Strs, gguf.go:199-233 */
OR_API const char *or_gguf_str(or_file *f, const char *key) {
    or_kv *kv = find_kv(f, key);
    return (kv && kv->vtype == V_STR) ? kv->s : "";
}
static int is_int_type(int t) {
    return t == V_U8 || t == V_I8 || t == V_U16 || t == V_I16 || t == V_U32 || t == V_I32 || t == V_U64 || t == V_I64;
}
OR_API uint64_t or_gguf_u64(or_file *f, const char *key, uint64_t def) {
    or_kv *kv = find_kv(f, key);
    if (!kv) return def;
    return is_int_type(kv->vtype) ? kv->u : 0; /* toU64 returns 0 for other types, gguf.go:176-196 */
}
OR_API float or_gguf_f32(or_file *f, const char *key, float def) {
    or_kv *kv = find_kv(f, key);
    if (kv && (kv->vtype == V_F32 || kv->vtype == V_F64)) return (float)kv->f;
    return def;
}
OR_API int64_t or_gguf_strs_len(or_file *f, const char *key) {
    or_kv *kv = find_kv(f, key);
    return (kv && kv->vtype == V_ARR) ? (int64_t)kv->alen : 0;
}
OR_API const char *or_gguf_strs_at(or_file *f, const char *key, int64_t i) {
    or_kv *kv = find_kv(f, key);
    if (!kv || kv->vtype != V_ARR || kv->etype != V_STR || i < 0 || (uint64_t)i >= kv->alen) return "";
    return kv->astr[i] ? kv->astr[i] : "";
}
OR_API int or_gguf_tensor_count(or_file *f) { return f->ntensors; }
OR_API const or_tensor *or_gguf_tensor_at(or_file *f, int i) { return (i >= 0 && i < f->ntensors) ? &f->t[i] : NULL; }
OR_API const or_tensor *or_gguf_tensor(or_file *f, const char *name) {
    for (int i = 0; i < f->ntensors; i++)
        if (!strcmp(f->t[i].name, name)) return &f->t[i];
    return NULL;
}
OR_API uint32_t or_gguf_version(or_file *f) { return f->version; }

/* ------------------------------------------------------------------ */
/* Config / Load: infer/model.go:14-211                                 */
/* ------------------------------------------------------------------ */

typedef struct {
    int arch; /* 0 qwen3, 1 qwen2, 2 llama */
    int n_layers, n_embd, n_head, n_head_kv, head_dim, n_ff, vocab, max_ctx, rope_dim;
    float rope_base;
    int rope_interleaved;
    int rope_scaling; /* 0 none, 1 linear, 2 llama3 */
    float rope_factor, rope_lo_f, rope_hi_f, rope_orig_ctx;
    float rms_eps;
    int bos, eos, eos2;
} or_config;

typedef struct {
    const or_tensor *q, *k, *v, *o, *qb, *kb, *vb, *gate, *up, *down;
    float *attn_nw, *ffn_nw, *q_nw, *k_nw;
} or_layer;

typedef struct or_model {
    or_config c;
    const or_tensor *embd, *out;
    float *out_nw;
    or_layer *layers;
    float **kc, **vc;   /* [layer][pos*kvd], grown in 256-position steps */
    int64_t *kv_cap;    /* positions allocated per layer */
    int pos;
    float *freqs;
    /* scratch, model.go:66-88 */
    float *x, *xb, *h, *q, *k, *v, *att, *hb, *hb2, *hf, *logits;
    int scratch_n;
    /* DebugLayer hook, model.go:231-233 */
    void (*debug_layer)(int li, const float *x, int ntok, int embd, void *ctx);
    void *debug_ctx;
} or_model;

static float *norm_weight(const or_tensor *t) {
    float *out = (float *)malloc(sizeof(float) * (size_t)t->numel);
    or_dequant_row(t->type, t->data, out, t->numel); /* normWeight, model.go:224-229 */
    return out;
}

/* ropeFreqs, model.go:253-280 */
static float *rope_freqs(const or_config *c) {
    int n = c->rope_dim / 2;
    float *f = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    for (int i = 0; i < n; i++) f[i] = 1.0f / (float)pow((double)c->rope_base, (double)(2 * i) / (double)c->rope_dim);
    if (c->rope_scaling == 1) {
        for (int i = 0; i < n; i++) f[i] /= c->rope_factor;
    } else if (c->rope_scaling == 2) {
        float lo_wl = c->rope_orig_ctx / c->rope_lo_f;
        float hi_wl = c->rope_orig_ctx / c->rope_hi_f;
        for (int i = 0; i < n; i++) {
            double wl = 2 * M_PI / (double)f[i];
            if (wl < (double)hi_wl) {
            } else if (wl > (double)lo_wl) {
                f[i] /= c->rope_factor;
            } else {
                float smooth = (c->rope_orig_ctx / (float)wl - c->rope_lo_f) / (c->rope_hi_f - c->rope_lo_f);
                f[i] = (1 - smooth) * f[i] / c->rope_factor + smooth * f[i];
            }
        }
    }
    return f;
}

OR_API void or_model_free(or_model *m);

/* Load, model.go:90-203 */
OR_API or_model *or_load(or_file *f, int max_ctx, char *err, int errlen) {
    const char *arch = or_gguf_str(f, "general.architecture");
    int a;
    if (!strcmp(arch, "qwen3")) a = 0;
    else if (!strcmp(arch, "qwen2")) a = 1;
    else if (!strcmp(arch, "llama")) a = 2;
    else {
        snprintf(err, errlen, "unsupported architecture \"%s\" (want qwen2, qwen3, or llama)", arch);
        return NULL;
    }
    char key[256];
#define K(s) (snprintf(key, sizeof key, "%s.%s", arch, s), key)
    or_config c;
    memset(&c, 0, sizeof c);
    c.arch = a;
    c.n_layers = (int)or_gguf_u64(f, K("block_count"), 0);
    c.n_embd = (int)or_gguf_u64(f, K("embedding_length"), 0);
    c.n_head = (int)or_gguf_u64(f, K("attention.head_count"), 0);
    c.n_head_kv = (int)or_gguf_u64(f, K("attention.head_count_kv"), 0);
    c.n_ff = (int)or_gguf_u64(f, K("feed_forward_length"), 0);
    c.max_ctx = (int)or_gguf_u64(f, K("context_length"), 0);
    c.rope_base = or_gguf_f32(f, K("rope.freq_base"), 10000);
    c.rms_eps = or_gguf_f32(f, K("attention.layer_norm_rms_epsilon"), 1e-6f);
    c.vocab = (int)or_gguf_strs_len(f, "tokenizer.ggml.tokens");
    c.bos = (int)or_gguf_u64(f, "tokenizer.ggml.bos_token_id", 0);
    c.eos = (int)or_gguf_u64(f, "tokenizer.ggml.eos_token_id", 0);
    int kl = (int)or_gguf_u64(f, K("attention.key_length"), 0);
    const or_tensor *tq = or_gguf_tensor(f, "blk.0.attn_q.weight");
    if (kl > 0) c.head_dim = kl;
    else if (tq && tq->ndims > 1 && c.n_head) c.head_dim = (int)tq->dims[1] / c.n_head;
    else c.head_dim = c.n_head ? c.n_embd / c.n_head : 0;
    c.rope_interleaved = (a == 2);
    c.rope_dim = (int)or_gguf_u64(f, K("rope.dimension_count"), (uint64_t)c.head_dim);
    const char *sc = or_gguf_str(f, K("rope.scaling.type"));
    c.rope_scaling = !strcmp(sc, "linear") ? 1 : !strcmp(sc, "llama3") ? 2 : 0;
    c.rope_factor = or_gguf_f32(f, K("rope.scaling.factor"), 0);
    c.rope_lo_f = or_gguf_f32(f, K("rope.scaling.low_freq_factor"), 0);
    c.rope_hi_f = or_gguf_f32(f, K("rope.scaling.high_freq_factor"), 0);
    c.rope_orig_ctx = or_gguf_f32(f, K("rope.scaling.original_context_length"), 0);
    if (a == 2 && sc[0] == 0 && c.rope_base >= 500000) {
        /* legacy Llama-3.x defaults, model.go:126-134 */
        c.rope_scaling = 2;
        c.rope_factor = 32;
        c.rope_lo_f = 1;
        c.rope_hi_f = 4;
        c.rope_orig_ctx = 8192;
    }
#undef K
    int hkv = c.n_head_kv ? c.n_head_kv : c.n_head;
    if (hkv == 0 || c.n_embd == 0 || c.n_layers == 0) {
        snprintf(err, errlen, "missing required metadata for arch %s", arch);
        return NULL;
    }
    c.n_head_kv = hkv; /* HeadKV(), model.go:205-210 */
    if (max_ctx <= 0 || max_ctx > c.max_ctx) max_ctx = c.max_ctx;
    c.max_ctx = max_ctx;
    c.eos2 = -1;
    for (int64_t i = 0; i < c.vocab; i++) {
        const char *tok = or_gguf_strs_at(f, "tokenizer.ggml.tokens", i);
        if (!strcmp(tok, "<|endoftext|>") || !strcmp(tok, "<|eot_id|>") || !strcmp(tok, "<|end_of_text|>"))
            if (i != c.eos) c.eos2 = (int)i;
    }
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->c = c;
    m->embd = or_gguf_tensor(f, "token_embd.weight");
    m->out = or_gguf_tensor(f, "output.weight");
    const or_tensor *on = or_gguf_tensor(f, "output_norm.weight");
    if (on) m->out_nw = norm_weight(on);
    if (!m->embd || !m->out_nw) {
        snprintf(err, errlen, "missing embedding or output norm tensors");
        or_model_free(m);
        return NULL;
    }
    if (!m->out) m->out = m->embd;
    m->layers = (or_layer *)calloc((size_t)c.n_layers, sizeof(or_layer));
    m->kc = (float **)calloc((size_t)c.n_layers, sizeof(float *));
    m->vc = (float **)calloc((size_t)c.n_layers, sizeof(float *));
    m->kv_cap = (int64_t *)calloc((size_t)c.n_layers, sizeof(int64_t));
    m->freqs = rope_freqs(&m->c);
    for (int i = 0; i < c.n_layers; i++) {
        char b[128];
        or_layer *l = &m->layers[i];
#define G(s) (snprintf(b, sizeof b, "blk.%d.%s", i, s), or_gguf_tensor(f, b))
        l->q = G("attn_q.weight");
        l->k = G("attn_k.weight");
        l->v = G("attn_v.weight");
        l->o = G("attn_output.weight");
        l->qb = G("attn_q.bias");
        l->kb = G("attn_k.bias");
        l->vb = G("attn_v.bias");
        l->gate = G("ffn_gate.weight");
        l->up = G("ffn_up.weight");
        l->down = G("ffn_down.weight");
        const or_tensor *t;
        if ((t = G("attn_norm.weight"))) l->attn_nw = norm_weight(t);
        if ((t = G("ffn_norm.weight"))) l->ffn_nw = norm_weight(t);
        if ((t = G("attn_q_norm.weight"))) l->q_nw = norm_weight(t);
        if ((t = G("attn_k_norm.weight"))) l->k_nw = norm_weight(t);
#undef G
        if (!l->attn_nw || !l->q || !l->k || !l->v || !l->o || !l->ffn_nw || !l->gate || !l->up || !l->down) {
            snprintf(err, errlen, "layer %d: missing tensors", i);
            or_model_free(m);
            return NULL;
        }
    }
    return m;
}

OR_API void or_model_free(or_model *m) {
    if (!m) return;
    if (m->layers) {
        for (int i = 0; i < m->c.n_layers; i++) {
            or_layer *l = &m->layers[i];
            free(l->attn_nw); free(l->ffn_nw); free(l->q_nw); free(l->k_nw);
        }
    }
    if (m->kc)
        for (int i = 0; i < m->c.n_layers; i++) { free(m->kc[i]); free(m->vc[i]); }
    free(m->kc); free(m->vc); free(m->kv_cap);
    free(m->layers); free(m->out_nw); free(m->freqs);
    free(m->x); free(m->xb); free(m->h); free(m->q); free(m->k); free(m->v);
    free(m->att); free(m->hb); free(m->hb2); free(m->hf); free(m->logits);
    free(m);
}

OR_API const or_config *or_model_config(or_model *m) { return &m->c; }
OR_API int or_model_pos(or_model *m) { return m->pos; }             /* Pos, model.go:455-456 */
OR_API void or_model_reset(or_model *m) { m->pos = 0; }             /* Reset, model.go:458-460 */
OR_API void or_model_set_debug(or_model *m, void (*fn)(int, const float *, int, int, void *), void *ctx) {
    m->debug_layer = fn;
    m->debug_ctx = ctx;
}
OR_API const float *or_model_freqs(or_model *m) { return m->freqs; }

/* rmsnorm, model.go:213-222 */
static void rmsnorm(float *dst, const float *x, const float *w, int n, float eps) {
    float ss = 0;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = 1.0f / (float)sqrt((double)(ss / (float)n) + (double)eps);
    for (int i = 0; i < n; i++) dst[i] = x[i] * ss * w[i];
}

/* rope, model.go:237-251 */
static void rope(float *x, int pos, int dim, const float *freqs, int interleaved) {
    int half = dim / 2;
    for (int i = 0; i < half; i++) {
        float c = (float)cos((double)((float)pos * freqs[i]));
        float s = (float)sin((double)((float)pos * freqs[i]));
        if (interleaved) {
            float a = x[2 * i], b = x[2 * i + 1];
            x[2 * i] = a * c - b * s;
            x[2 * i + 1] = a * s + b * c;
        } else {
            float a = x[i], b = x[i + half];
            x[i] = a * c - b * s;
            x[i + half] = a * s + b * c;
        }
    }
}

/* fastExp, model.go:282-295 */
OR_API float or_fast_exp(float x) {
    if (x < -87) return 0;
    float t = x * 1.4426950408889634f;
    int32_t i = (int32_t)floor((double)t);
    float f = t - (float)i;
    float p = 1.0000001f + f * (0.69314718f + f * (0.24022650f + f * (0.05550411f + f * (0.00961813f + f * 0.00133336f))));
    return (float)ldexp((double)p, i);
}

/* softmax, model.go:297-313 */
static void softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 0; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0;
    for (int i = 0; i < n; i++) {
        float e = or_fast_exp(x[i] - mx);
        x[i] = e;
        sum += e;
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* addBias, model.go:444-454 */
static void add_bias(float *dst, int64_t n, const or_tensor *t) {
    if (!t) return;
    float *b = (float *)malloc(sizeof(float) * (size_t)t->numel);
    or_dequant_row(t->type, t->data, b, t->numel);
    for (int64_t i = 0; i < n; i++) dst[i] += b[i % t->numel];
    free(b);
}

static void matmul_t(float *dst, const or_tensor *w, const float *x, int m) {
    or_matmul(dst, w->type, w->data, w->numel / (int64_t)w->dims[0], (int64_t)w->dims[0], x, m);
}

typedef struct {
    or_model *m;
    int ntok, li;
    float scale;
} att_ctx;

static void att_body(void *vc, int64_t lo, int64_t hi, int worker) {
    (void)worker;
    att_ctx *a = (att_ctx *)vc;
    or_model *m = a->m;
    const or_config *c = &m->c;
    int nh = c->n_head, nkv = c->n_head_kv, hd = c->head_dim, kvd = nkv * hd, qd = nh * hd;
    const float *kc = m->kc[a->li], *vc2 = m->vc[a->li];
    float *score = (float *)malloc(sizeof(float) * (size_t)(m->pos + a->ntok));
    for (int64_t idx = lo; idx < hi; idx++) {
        int j = (int)(idx / nh), head = (int)(idx % nh);
        int pos = m->pos + j;
        const float *qh = m->q + (int64_t)j * qd + head * hd;
        int kvh = head / (nh / nkv);
        int n = pos + 1;
        int kbase = kvh * hd;
        for (int p = 0; p <= pos; p++) score[p] = dot(qh, kc + (int64_t)p * kvd + kbase, hd) * a->scale;
        softmax(score, n);
        float *out = m->att + (int64_t)j * qd + head * hd;
        memset(out, 0, sizeof(float) * (size_t)hd);
        for (int p = 0; p <= pos; p++) axpy(out, score[p], vc2 + (int64_t)p * kvd + kbase, hd);
    }
    free(score);
}

static void scratch_for(or_model *m, int ntok) {
    const or_config *c = &m->c;
    if (m->scratch_n >= ntok) return;
    int qd = c->n_head * c->head_dim, kvd = c->n_head_kv * c->head_dim;
    free(m->x); free(m->xb); free(m->h); free(m->q); free(m->k); free(m->v);
    free(m->att); free(m->hb); free(m->hb2); free(m->hf);
    m->x = (float *)calloc((size_t)ntok * c->n_embd, 4);
    m->xb = (float *)calloc((size_t)ntok * c->n_embd, 4);
    m->h = (float *)calloc((size_t)ntok * c->n_embd, 4);
    m->q = (float *)calloc((size_t)ntok * qd, 4);
    m->k = (float *)calloc((size_t)ntok * kvd, 4);
    m->v = (float *)calloc((size_t)ntok * kvd, 4);
    m->att = (float *)calloc((size_t)ntok * qd, 4);
    m->hb = (float *)calloc((size_t)ntok * c->n_ff, 4);
    m->hb2 = (float *)calloc((size_t)ntok * c->n_ff, 4);
    m->hf = (float *)calloc((size_t)c->n_embd, 4);
    m->scratch_n = ntok;
}

/* Forward, model.go:315-442.  Returns the model-owned logits of the last
 * token (overwritten by the next call), or NULL with err set. */
OR_API const float *or_forward(or_model *m, const int32_t *tokens, int ntok, char *err, int errlen) {
    const or_config *c = &m->c;
    if (m->pos + ntok > c->max_ctx) {
        snprintf(err, errlen, "context length exceeded (%d > %d)", m->pos + ntok, c->max_ctx);
        return NULL;
    }
    if (ntok <= 0) {
        snprintf(err, errlen, "empty token batch");
        return NULL;
    }
    int embd = c->n_embd, nh = c->n_head, nkv = c->n_head_kv, hd = c->head_dim;
    int kvd = nkv * hd, qd = nh * hd, nff = c->n_ff;
    int64_t erows = m->embd->numel / (int64_t)m->embd->dims[0];
    for (int j = 0; j < ntok; j++)
        if (tokens[j] < 0 || tokens[j] >= erows) {
            snprintf(err, errlen, "token id %d out of range", tokens[j]);
            return NULL;
        }
    scratch_for(m, ntok);
    float *x = m->x, *xb = m->xb, *h = m->h, *q = m->q, *k = m->k, *v = m->v, *hb = m->hb, *hb2 = m->hb2;
    int64_t erb = row_bytes_of(m->embd->type, embd);
    for (int j = 0; j < ntok; j++) or_dequant_row(m->embd->type, m->embd->data + (int64_t)tokens[j] * erb, x + (int64_t)j * embd, embd);

    for (int li = 0; li < c->n_layers; li++) {
        or_layer *l = &m->layers[li];
        for (int j = 0; j < ntok; j++) rmsnorm(h + (int64_t)j * embd, x + (int64_t)j * embd, l->attn_nw, embd, c->rms_eps);
        matmul_t(q, l->q, h, ntok);
        matmul_t(k, l->k, h, ntok);
        matmul_t(v, l->v, h, ntok);
        add_bias(q, (int64_t)ntok * qd, l->qb);
        add_bias(k, (int64_t)ntok * kvd, l->kb);
        add_bias(v, (int64_t)ntok * kvd, l->vb);

        /* grow the KV cache in blocks of 256 positions, model.go:353-360 */
        int64_t need = (int64_t)(m->pos + ntok);
        if (m->kv_cap[li] < need) {
            int64_t cap = m->kv_cap[li];
            while (cap < need) cap += 256;
            m->kc[li] = (float *)realloc(m->kc[li], sizeof(float) * (size_t)(cap * kvd));
            m->vc[li] = (float *)realloc(m->vc[li], sizeof(float) * (size_t)(cap * kvd));
            memset(m->kc[li] + m->kv_cap[li] * kvd, 0, sizeof(float) * (size_t)((cap - m->kv_cap[li]) * kvd));
            memset(m->vc[li] + m->kv_cap[li] * kvd, 0, sizeof(float) * (size_t)((cap - m->kv_cap[li]) * kvd));
            m->kv_cap[li] = cap;
        }
        float *kc = m->kc[li], *vc = m->vc[li];
        for (int j = 0; j < ntok; j++) {
            int pos = m->pos + j;
            float *qj = q + (int64_t)j * qd, *kj = k + (int64_t)j * kvd;
            for (int head = 0; head < nh; head++) {
                float *hq = qj + head * hd;
                if (l->q_nw) rmsnorm(hq, hq, l->q_nw, hd, c->rms_eps);
                rope(hq, pos, c->rope_dim, m->freqs, c->rope_interleaved);
            }
            for (int head = 0; head < nkv; head++) {
                float *hk = kj + head * hd;
                if (l->k_nw) rmsnorm(hk, hk, l->k_nw, hd, c->rms_eps);
                rope(hk, pos, c->rope_dim, m->freqs, c->rope_interleaved);
            }
            memcpy(kc + (int64_t)pos * kvd, kj, sizeof(float) * (size_t)kvd);
            memcpy(vc + (int64_t)pos * kvd, v + (int64_t)j * kvd, sizeof(float) * (size_t)kvd);
        }
        att_ctx ac = {m, ntok, li, 1.0f / (float)sqrt((double)hd)};
        par_for((int64_t)ntok * nh, att_body, &ac);

        matmul_t(xb, l->o, m->att, ntok);
        for (int64_t i = 0; i < (int64_t)ntok * embd; i++) x[i] += xb[i];
        for (int j = 0; j < ntok; j++) rmsnorm(h + (int64_t)j * embd, x + (int64_t)j * embd, l->ffn_nw, embd, c->rms_eps);
        matmul_t(hb, l->gate, h, ntok);
        matmul_t(hb2, l->up, h, ntok);
        for (int64_t i = 0; i < (int64_t)ntok * nff; i++) {
            float g = hb[i];
            hb[i] = g * (1.0f / (1.0f + or_fast_exp(-g))) * hb2[i];
        }
        matmul_t(xb, l->down, hb, ntok);
        for (int64_t i = 0; i < (int64_t)ntok * embd; i++) x[i] += xb[i];
        if (m->debug_layer) m->debug_layer(li, x, ntok, embd, m->debug_ctx);
    }
    m->pos += ntok;
    const float *last = x + (int64_t)(ntok - 1) * embd;
    rmsnorm(m->hf, last, m->out_nw, embd, c->rms_eps);
    int64_t orows = m->out->numel / (int64_t)m->out->dims[0];
    if (!m->logits) m->logits = (float *)malloc(sizeof(float) * (size_t)(orows > c->vocab ? orows : c->vocab));
    if (orows < c->vocab) {
        /* the reference's matvec writes Rows() logits; a shorter output
         * tensor than the token list leaves the tail at zero */
        memset(m->logits, 0, sizeof(float) * (size_t)c->vocab);
    }
    matmul_t(m->logits, m->out, m->hf, 1);
    return m->logits;
}

/* ------------------------------------------------------------------ */
/* Sampler: infer/sampler.go:12-98, with the uniform draw supplied by a */
/* counter-based generator (Philox4x32-10, Salmon et al., SC'11) keyed  */
/* by (seed, step) instead of the reference's time-seeded PCG          */
/* (internal/app/rand.go:10-13).                                        */
/* ------------------------------------------------------------------ */

OR_API void or_philox4x32_10(uint32_t ctr[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* u in [0,1) with 53 random bits for (seed, step). */
OR_API double or_uniform(uint64_t seed, uint64_t step) {
    uint32_t ctr[4] = {(uint32_t)step, (uint32_t)(step >> 32), 0x5A4D4341u /* "ACMZ" */, 0};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t o[4];
    or_philox4x32_10(ctr, key, o);
    uint64_t u = ((uint64_t)o[1] << 32) | o[0];
    return (double)(u >> 11) * 0x1p-53;
}

/* greedy, sampler.go:19-27 */
OR_API int or_greedy(const float *logits, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* topK, sampler.go:80-98: indices of the k largest, sorted descending,
 * ties resolved towards the lower index.  Returns the count. */
OR_API int or_topk(const float *logits, int n, int k, int32_t *idx) {
    int len = 0;
    for (int i = 0; i < n; i++) {
        float l = logits[i];
        if (len == k && l <= logits[idx[k - 1]]) continue;
        int p = len;
        while (p > 0 && logits[idx[p - 1]] < l) p--;
        int upto = len < k ? len : k - 1; /* after append+truncate the list keeps k */
        for (int q = upto; q > p; q--) idx[q] = idx[q - 1];
        idx[p] = i;
        if (len < k) len++;
    }
    return len;
}

typedef struct {
    double temp;
    int32_t top_k;
    double top_p;
    uint64_t seed;
} or_sampler;

/* Sample, sampler.go:30-76, with u = the uniform draw. */
OR_API int or_sample_u(const or_sampler *s, const float *logits, int n, double u) {
    if (s->temp <= 0) return or_greedy(logits, n);
    int k = 64;
    if (s->top_k > 0 && s->top_k < k) k = s->top_k;
    int32_t idx[64];
    double p[64];
    int cnt = or_topk(logits, n, k, idx);
    double sum = 0, mx = (double)logits[idx[0]];
    for (int i = 0; i < cnt; i++) {
        p[i] = exp(((double)logits[idx[i]] - mx) / s->temp);
        sum += p[i];
    }
    int cut = cnt;
    if (s->top_p > 0 && s->top_p < 1) {
        double acc = 0;
        cut = k; /* cut := n, sampler.go:57 */
        if (cut > cnt) cut = cnt;
        for (int i = 0; i < cnt; i++) {
            acc += p[i] / sum;
            if (acc >= s->top_p) {
                cut = i + 1;
                break;
            }
        }
        sum = 0;
        for (int i = 0; i < cut; i++) sum += p[i];
    }
    double r = u * sum;
    for (int i = 0; i < cut; i++) {
        r -= p[i];
        if (r <= 0) return idx[i];
    }
    return idx[cut - 1];
}

OR_API int or_sample(const or_sampler *s, const float *logits, int n, uint64_t step) {
    return or_sample_u(s, logits, n, or_uniform(s->seed, step));
}

/* ------------------------------------------------------------------ */
/* Generate / decode, sampler.go:101-157.  Stats are wall-clock per     */
/* phase as in the reference.  stop_on_eos=0 runs exactly max_tok steps. */
/* ------------------------------------------------------------------ */

typedef struct {
    int64_t prefill_toks;
    double prefill_s;
    int64_t decode_toks;
    double decode_s;
} or_stats;

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* Runs the loop; writes generated ids to out (capacity max_tok) and returns
 * the count, or -1 on error.  If step_logits is non-NULL it receives the
 * logits each Sample call consumed ([(max_tok+1) x vocab], row i = the
 * logits sampled for output i). */
OR_API int or_generate(or_model *m, const int32_t *prompt, int nprompt, const or_sampler *s, int max_tok,
                       int stop_on_eos, int32_t *out, float *step_logits, or_stats *st, char *err, int errlen) {
    or_stats z = {0, 0, 0, 0};
    *st = z;
    int chunk = 1024;
    if (m->c.max_ctx - m->pos < chunk) chunk = m->c.max_ctx - m->pos;
    if (chunk <= 0) {
        snprintf(err, errlen, "context length exceeded");
        return -1;
    }
    const float *logits = NULL;
    for (int i = 0; i < nprompt; i += chunk) {
        int end = i + chunk < nprompt ? i + chunk : nprompt;
        double t0 = now_s();
        logits = or_forward(m, prompt + i, end - i, err, errlen);
        st->prefill_s += now_s() - t0;
        st->prefill_toks += end - i;
        if (!logits) return -1;
    }
    if (!logits) return 0;
    int n = 0;
    uint64_t step = 0;
    while (n < max_tok) {
        if (step_logits) memcpy(step_logits + (int64_t)n * m->c.vocab, logits, sizeof(float) * (size_t)m->c.vocab);
        int id = or_sample(s, logits, m->c.vocab, step++);
        if (stop_on_eos && (id == m->c.eos || id == m->c.eos2)) break;
        out[n++] = id;
        int32_t tok = id;
        double t0 = now_s();
        logits = or_forward(m, &tok, 1, err, errlen);
        st->decode_s += now_s() - t0;
        st->decode_toks++;
        if (!logits) return -1;
    }
    return n;
}
