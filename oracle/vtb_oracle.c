/*
 * vtb_oracle.c -- CPU restatement of vantablack's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA backend and the timed
 * CPU baseline.  Never part of the product library.  Build with
 * -ffp-contract=off (oracle/Makefile): the reference is Zig in its default
 * strict float mode, which never fuses a multiply and an add, so every
 * multiply and every add below is rounded separately, in the reference's
 * order.  Citations are file:line in the reference project.
 */
#define _GNU_SOURCE
#include "vtb_oracle.h"

#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#define LANES 8 /* simd.zig:10 lane_width */

/* f16BitsToF32, simd.zig:64-67: exact IEEE half -> single widening. */
float vtbo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal half -> normal single */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
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

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Ordered @reduce(.Add) over an 8-lane vector (Zig keeps float reduction
 * order unless the float mode is Optimized). */
static inline float reduce8(const float *acc) {
    float s = acc[0];
    for (int l = 1; l < LANES; l++) s += acc[l];
    return s;
}

/* dot_f32, simd.zig:13-29 */
float vtbo_dot_f32(const float *a, const float *b, size_t n) {
    float acc[LANES] = {0};
    size_t i = 0;
    for (; i + LANES <= n; i += LANES)
        for (int l = 0; l < LANES; l++) {
            float p = a[i + l] * b[i + l];
            acc[l] += p;
        }
    float sum = reduce8(acc);
    for (; i < n; i++) {
        float p = a[i] * b[i];
        sum += p;
    }
    return sum;
}

/* dot_i8, simd.zig:40-62: i8 x i8 widened to i32; integer sums are exact,
 * so the 16-lane split does not change the result. */
int32_t vtbo_dot_i8(const int8_t *a, const int8_t *b, size_t n) {
    int32_t s = 0;
    for (size_t i = 0; i < n; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

/* ---------------- Q8_0: simd.zig:145-190 ---------------- */
#define Q8_0_BYTES 34
#define Q8_0_ELEMS 32

void vtbo_dequant_q8_0_block(const uint8_t *blk, float *out) {
    float scale = vtbo_f16_to_f32(rd16(blk));
    for (int j = 0; j < Q8_0_ELEMS; j++) out[j] = scale * (float)(int8_t)blk[2 + j];
}

/* matmul_q8_0, simd.zig:159-190: per block four 8-lane chunks, each reduced
 * and added into block_dot; the scale multiplies the block dot. */
void vtbo_matmul_q8_0(float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    size_t nb = k / Q8_0_ELEMS, rb = nb * Q8_0_BYTES;
    for (size_t i = 0; i < m; i++) {
        const uint8_t *row = w + i * rb;
        float total = 0.f;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t *blk = row + b * Q8_0_BYTES;
            float scale = vtbo_f16_to_f32(rd16(blk));
            float block_dot = 0.f;
            for (int c = 0; c < 4; c++) {
                float p[LANES];
                for (int l = 0; l < LANES; l++)
                    p[l] = (float)(int8_t)blk[2 + c * LANES + l] * acts[b * Q8_0_ELEMS + c * LANES + l];
                block_dot += reduce8(p);
            }
            float t = scale * block_dot;
            total += t;
        }
        out[i] = total;
    }
}

/* ---------------- K-quants: simd.zig:192-434 ---------------- */
#define QK_K 256
#define Q4_K_BYTES 144
#define Q5_K_BYTES 176
#define Q6_K_BYTES 210

/* q4kScaleMin, simd.zig:211-219 */
static inline void q4k_scale_min(int s, const uint8_t *sc, uint8_t *d, uint8_t *m) {
    if (s < 4) {
        *d = sc[s] & 0x3f;
        *m = sc[s + 4] & 0x3f;
    } else {
        *d = (uint8_t)((sc[s + 4] & 0x0f) | ((sc[s - 4] >> 6) << 4));
        *m = (uint8_t)((sc[s + 4] >> 4) | ((sc[s] >> 6) << 4));
    }
}

/* dequantBlockQ4_K, simd.zig:221-243 */
void vtbo_dequant_q4_k_block(const uint8_t *blk, float *out) {
    float d = vtbo_f16_to_f32(rd16(blk));
    float dmin = vtbo_f16_to_f32(rd16(blk + 2));
    const uint8_t *scales = blk + 4, *qs = blk + 16;
    for (int s = 0; s < 8; s += 2) {
        uint8_t sa, ma, sb, mb;
        q4k_scale_min(s, scales, &sa, &ma);
        q4k_scale_min(s + 1, scales, &sb, &mb);
        float d1 = d * (float)sa, m1 = dmin * (float)ma;
        float d2 = d * (float)sb, m2 = dmin * (float)mb;
        const uint8_t *q = qs + (s / 2) * 32;
        for (int l = 0; l < 32; l++) {
            float a = d1 * (float)(q[l] & 0x0f);
            float b = d2 * (float)(q[l] >> 4);
            out[s * 32 + l] = a - m1;
            out[s * 32 + 32 + l] = b - m2;
        }
    }
}

/* dequantBlockQ5_K, simd.zig:290-319 */
void vtbo_dequant_q5_k_block(const uint8_t *blk, float *out) {
    float d = vtbo_f16_to_f32(rd16(blk));
    float dmin = vtbo_f16_to_f32(rd16(blk + 2));
    const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
    for (int s = 0; s < 8; s += 2) {
        uint8_t sa, ma, sb, mb;
        q4k_scale_min(s, scales, &sa, &ma);
        q4k_scale_min(s + 1, scales, &sb, &mb);
        float d1 = d * (float)sa, m1 = dmin * (float)ma;
        float d2 = d * (float)sb, m2 = dmin * (float)mb;
        const uint8_t *q = qs + (s / 2) * 32;
        uint8_t mlo = (uint8_t)(1u << s), mhi = (uint8_t)(1u << (s + 1));
        for (int l = 0; l < 32; l++) {
            int w0 = (q[l] & 0x0f) + ((qh[l] & mlo) ? 16 : 0);
            int w1 = (q[l] >> 4) + ((qh[l] & mhi) ? 16 : 0);
            float a = d1 * (float)w0;
            float b = d2 * (float)w1;
            out[s * 32 + l] = a - m1;
            out[s * 32 + 32 + l] = b - m2;
        }
    }
}

/* dequantBlockQ6_K, simd.zig:366-404: w = (d * sc) * q, left to right. */
void vtbo_dequant_q6_k_block(const uint8_t *blk, float *out) {
    float d = vtbo_f16_to_f32(rd16(blk + 208));
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    for (int half = 0; half < 2; half++) {
        const uint8_t *l_ql = ql + half * 64, *l_qh = qh + half * 32;
        const int8_t *l_sc = sc + half * 8;
        float *y = out + half * 128;
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = (int)((l_ql[l] & 0x0f) | (((l_qh[l] >> 0) & 3) << 4)) - 32;
            int q2 = (int)((l_ql[l + 32] & 0x0f) | (((l_qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((l_ql[l] >> 4) | (((l_qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((l_ql[l + 32] >> 4) | (((l_qh[l] >> 6) & 3) << 4)) - 32;
            float t;
            t = d * (float)l_sc[is + 0]; y[l + 0] = t * (float)q1;
            t = d * (float)l_sc[is + 2]; y[l + 32] = t * (float)q2;
            t = d * (float)l_sc[is + 4]; y[l + 64] = t * (float)q3;
            t = d * (float)l_sc[is + 6]; y[l + 96] = t * (float)q4;
        }
    }
}

/* dequantBlockTQ2_0, simd.zig:457-472, exactly as the reference writes it:
 * weight 64g + l of a 256-weight block is (((qs[16g + l % 16] >> 2g) & 3) - 1)
 * times the f16 scale at bytes 64..65.  (ggml's own TQ2_0 layout differs; the
 * reference's is the one restated here, pinned by its test at simd.zig:734-768.) */
#define TQ2_0_BYTES 66
void vtbo_dequant_tq2_0_block(const uint8_t *blk, float *out) {
    const float scale = vtbo_f16_to_f32((uint16_t)(blk[64] | (blk[65] << 8)));
    for (int g = 0; g < 4; g++) {
        const int shift = 2 * g, base = g * 16;
        for (int l = 0; l < 64; l++) {
            const uint8_t raw = (uint8_t)((blk[base + (l % 16)] >> shift) & 0x03u);
            const float tern = (float)(int32_t)raw - 1.0f;
            out[g * 64 + l] = scale * tern;
        }
    }
}

size_t vtbo_row_bytes(int quant, size_t k) {
    switch (quant) {
    case VTBO_F32: return k * 4;
    case VTBO_Q8_0: return (k / Q8_0_ELEMS) * Q8_0_BYTES;
    case VTBO_Q4_K: return (k / QK_K) * Q4_K_BYTES;
    case VTBO_Q5_K: return (k / QK_K) * Q5_K_BYTES;
    case VTBO_Q6_K: return (k / QK_K) * Q6_K_BYTES;
    case VTBO_TQ2_0: return (k / QK_K) * TQ2_0_BYTES;
    default: return 0;
    }
}

/* dequantToF32, forward.zig:654-736 */
int vtbo_dequant(int quant, const uint8_t *w, float *out, size_t n) {
    switch (quant) {
    case VTBO_F32: memcpy(out, w, n * 4); return 0;
    case VTBO_Q8_0:
        for (size_t b = 0; b < n / Q8_0_ELEMS; b++) vtbo_dequant_q8_0_block(w + b * Q8_0_BYTES, out + b * Q8_0_ELEMS);
        return 0;
    case VTBO_Q4_K:
        for (size_t b = 0; b < n / QK_K; b++) vtbo_dequant_q4_k_block(w + b * Q4_K_BYTES, out + b * QK_K);
        return 0;
    case VTBO_Q5_K:
        for (size_t b = 0; b < n / QK_K; b++) vtbo_dequant_q5_k_block(w + b * Q5_K_BYTES, out + b * QK_K);
        return 0;
    case VTBO_Q6_K:
        for (size_t b = 0; b < n / QK_K; b++) vtbo_dequant_q6_k_block(w + b * Q6_K_BYTES, out + b * QK_K);
        return 0;
    case VTBO_TQ2_0:
        for (size_t b = 0; b < n / QK_K; b++) vtbo_dequant_tq2_0_block(w + b * TQ2_0_BYTES, out + b * QK_K);
        return 0;
    default: return -1;
    }
}

/* matmul_q4_k / q5_k / q6_k, simd.zig:245-273, 321-347, 406-434: dequantize
 * one super-block to f32[256], 8-lane accumulate, ordered reduce, add. */
typedef void (*dq_fn)(const uint8_t *, float *);
static void matmul_kquant(dq_fn dq, size_t bbytes, float *out, const uint8_t *w,
                          const float *acts, size_t m, size_t k) {
    size_t nb = k / QK_K, rb = nb * bbytes;
    float tmp[QK_K];
    for (size_t i = 0; i < m; i++) {
        const uint8_t *row = w + i * rb;
        float total = 0.f;
        for (size_t b = 0; b < nb; b++) {
            dq(row + b * bbytes, tmp);
            const float *x = acts + b * QK_K;
            float acc[LANES] = {0};
            for (int j = 0; j < QK_K; j += LANES)
                for (int l = 0; l < LANES; l++) {
                    float p = tmp[j + l] * x[j + l];
                    acc[l] += p;
                }
            total += reduce8(acc);
        }
        out[i] = total;
    }
}

void vtbo_matmul_q4_k(float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    matmul_kquant(vtbo_dequant_q4_k_block, Q4_K_BYTES, out, w, acts, m, k);
}
/* matmul_ternary158, simd.zig:474-498: the same per-block structure. */
void vtbo_matmul_tq2_0(float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    matmul_kquant(vtbo_dequant_tq2_0_block, TQ2_0_BYTES, out, w, acts, m, k);
}
void vtbo_matmul_q5_k(float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    matmul_kquant(vtbo_dequant_q5_k_block, Q5_K_BYTES, out, w, acts, m, k);
}
void vtbo_matmul_q6_k(float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    matmul_kquant(vtbo_dequant_q6_k_block, Q6_K_BYTES, out, w, acts, m, k);
}

/* ---------------- Q8_0 x Q8_0 ----------------
 * The reference has dot_i8 (simd.zig:40-62) but no activation quantizer
 * (simd.zig:31-39 describes it as future work).  This oracle defines one,
 * following ggml's quantize_row_q8_0 rule: per 32-block d = max|x| / 127,
 * q = round-half-away-from-zero(x * (1/d)), d kept in f32.  The row result
 * is the in-order sum over blocks of (d_w * d_x) * float(dot_i8(qs_w, qs_x)). */
void vtbo_quantize_q8_0(const float *x, size_t k, int8_t *qs, float *d) {
    for (size_t b = 0; b < k / Q8_0_ELEMS; b++) {
        const float *xb = x + b * Q8_0_ELEMS;
        float amax = 0.f;
        for (int j = 0; j < Q8_0_ELEMS; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        float dd = amax / 127.0f;
        float id = dd != 0.f ? 1.0f / dd : 0.f;
        d[b] = dd;
        for (int j = 0; j < Q8_0_ELEMS; j++) {
            float v = xb[j] * id;
            qs[b * Q8_0_ELEMS + j] = (int8_t)roundf(v);
        }
    }
}

void vtbo_q8_0_block_dots(int32_t *dots, const uint8_t *w, const int8_t *xq, size_t m, size_t k) {
    size_t nb = k / Q8_0_ELEMS, rb = nb * Q8_0_BYTES;
    for (size_t i = 0; i < m; i++)
        for (size_t b = 0; b < nb; b++)
            dots[i * nb + b] = vtbo_dot_i8((const int8_t *)(w + i * rb + b * Q8_0_BYTES + 2),
                                           xq + b * Q8_0_ELEMS, Q8_0_ELEMS);
}

static void matmul_q8_0_q8_0_rows(float *out, const uint8_t *w, const int8_t *xq,
                                  const float *dx, size_t m, size_t k) {
    size_t nb = k / Q8_0_ELEMS, rb = nb * Q8_0_BYTES;
    for (size_t i = 0; i < m; i++) {
        float total = 0.f;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t *blk = w + i * rb + b * Q8_0_BYTES;
            int32_t dot = vtbo_dot_i8((const int8_t *)(blk + 2), xq + b * Q8_0_ELEMS, Q8_0_ELEMS);
            float s = vtbo_f16_to_f32(rd16(blk)) * dx[b];
            float t = s * (float)dot;
            total += t;
        }
        out[i] = total;
    }
}

/* ---------------- thread pool: pool.zig:44-114 ----------------
 * Persistent workers spin on an epoch counter (then yield, then sleep in 50 us
 * steps once idle for milliseconds), the caller runs
 * worker 0, and a matmul stripes rows as chunk = ceil(m / n_workers)
 * (forward.zig:534-550, prefill.zig:348-378). */
typedef void (*job_fn)(int wid, int nw, void *ctx);
static struct {
    int n;
    pthread_t *threads;
    _Atomic unsigned long epoch;
    unsigned long start_epoch; /* epoch value the workers start from */
    _Atomic int completed;
    _Atomic int shutdown;
    job_fn fn;
    void *ctx;
} g_pool = {.n = 1};

static void *worker_loop(void *arg) {
    int wid = (int)(intptr_t)arg;
    unsigned long seen = g_pool.start_epoch;
    for (;;) {
        unsigned long e;
        int spins = 0, yields = 0;
        while ((e = atomic_load_explicit(&g_pool.epoch, memory_order_acquire)) == seen) {
            if (++spins > 4096) {
                spins = 0;
                if (++yields < 2048) {
                    sched_yield();
                } else {  /* idle for milliseconds: sleep, so an idle pool leaves the cores to other work */
                    struct timespec ts = {0, 50000};
                    nanosleep(&ts, NULL);
                }
            }
        }
        seen = e;
        if (atomic_load(&g_pool.shutdown)) return NULL;
        g_pool.fn(wid, g_pool.n, g_pool.ctx);
        atomic_fetch_add_explicit(&g_pool.completed, 1, memory_order_release);
    }
}

void vtbo_pool_shutdown(void) {
    if (g_pool.n > 1 && g_pool.threads) {
        atomic_store(&g_pool.shutdown, 1);
        atomic_fetch_add(&g_pool.epoch, 1);
        for (int i = 0; i < g_pool.n - 1; i++) pthread_join(g_pool.threads[i], NULL);
        free(g_pool.threads);
    }
    g_pool.threads = NULL;
    g_pool.n = 1;
    atomic_store(&g_pool.shutdown, 0);
}

int vtbo_pool_init(int n) {
    vtbo_pool_shutdown();
    if (n < 1) n = 1;
    g_pool.n = n;
    g_pool.start_epoch = atomic_load(&g_pool.epoch);
    if (n > 1) {
        g_pool.threads = (pthread_t *)calloc((size_t)n - 1, sizeof(pthread_t));
        for (int i = 0; i < n - 1; i++)
            if (pthread_create(&g_pool.threads[i], NULL, worker_loop, (void *)(intptr_t)(i + 1)) != 0) return -1;
    }
    return 0;
}

int vtbo_pool_threads(void) { return g_pool.n; }

static void pool_dispatch(job_fn fn, void *ctx) {
    if (g_pool.n <= 1) { fn(0, 1, ctx); return; }
    g_pool.fn = fn;
    g_pool.ctx = ctx;
    atomic_store_explicit(&g_pool.completed, 0, memory_order_release);
    atomic_fetch_add_explicit(&g_pool.epoch, 1, memory_order_release);
    fn(0, g_pool.n, ctx);
    while (atomic_load_explicit(&g_pool.completed, memory_order_acquire) < g_pool.n - 1) {}
}

/* Internal job tag for the Q8_0 x Q8_0 rows (not a ggml type id). */
#define MM_Q8_0_Q8_0 (-8)

typedef struct {
    int quant;
    float *out;
    const uint8_t *w;
    const float *acts;
    const int8_t *xq;
    const float *dx;
    size_t m, k, B;
} mm_ctx;

static void stripe(size_t m, int wid, int nw, size_t *s, size_t *e) {
    size_t chunk = (m + (size_t)nw - 1) / (size_t)nw;
    *s = (size_t)wid * chunk;
    *e = *s + chunk < m ? *s + chunk : m;
}

static void matmul_worker(int wid, int nw, void *p) {
    mm_ctx *c = (mm_ctx *)p;
    size_t s, e;
    stripe(c->m, wid, nw, &s, &e);
    if (s >= e) return;
    size_t rb = vtbo_row_bytes(c->quant == MM_Q8_0_Q8_0 ? VTBO_Q8_0 : c->quant, c->k);
    const uint8_t *w = c->w + s * rb;
    switch (c->quant) {
    case VTBO_Q8_0: vtbo_matmul_q8_0(c->out + s, w, c->acts, e - s, c->k); break;
    case VTBO_Q4_K: vtbo_matmul_q4_k(c->out + s, w, c->acts, e - s, c->k); break;
    case VTBO_Q5_K: vtbo_matmul_q5_k(c->out + s, w, c->acts, e - s, c->k); break;
    case VTBO_Q6_K: vtbo_matmul_q6_k(c->out + s, w, c->acts, e - s, c->k); break;
    case VTBO_TQ2_0: vtbo_matmul_tq2_0(c->out + s, w, c->acts, e - s, c->k); break;
    case MM_Q8_0_Q8_0: matmul_q8_0_q8_0_rows(c->out + s, w, c->xq, c->dx, e - s, c->k); break;
    default: break;
    }
}

/* matmulRuntime, forward.zig:552-627 (CPU branch) */
int vtbo_matmul(int quant, float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    if (vtbo_row_bytes(quant, k) == 0 || quant == VTBO_F32) return -1;
    mm_ctx c = {quant, out, w, acts, NULL, NULL, m, k, 1};
    pool_dispatch(matmul_worker, &c);
    return 0;
}

int vtbo_matmul_q8_0_q8_0(float *out, const uint8_t *w, const float *acts, size_t m, size_t k) {
    if (k % Q8_0_ELEMS) return -1;
    int8_t *xq = (int8_t *)malloc(k);
    float *dx = (float *)malloc(sizeof(float) * (k / Q8_0_ELEMS));
    vtbo_quantize_q8_0(acts, k, xq, dx);
    mm_ctx c = {MM_Q8_0_Q8_0, out, w, acts, xq, dx, m, k, 1};
    pool_dispatch(matmul_worker, &c);
    free(xq);
    free(dx);
    return 0;
}

/* matmulBatchedWorker, prefill.zig:357-378: dequantize one full row into
 * f32[k] (k <= MAX_K = 32768, prefill.zig:313), then B dot_f32 calls. */
#define MAX_K 32768
static void batched_worker(int wid, int nw, void *p) {
    mm_ctx *c = (mm_ctx *)p;
    size_t s, e;
    stripe(c->m, wid, nw, &s, &e);
    if (s >= e) return;
    size_t rb = vtbo_row_bytes(c->quant, c->k);
    float *dq = (float *)malloc(sizeof(float) * c->k);
    for (size_t row = s; row < e; row++) {
        vtbo_dequant(c->quant, c->w + row * rb, dq, c->k);
        for (size_t b = 0; b < c->B; b++)
            c->out[b * c->m + row] = vtbo_dot_f32(dq, c->acts + b * c->k, c->k);
    }
    free(dq);
}

int vtbo_matmul_batched(int quant, float *out, const uint8_t *w, const float *acts,
                        size_t m, size_t k, size_t B) {
    if (k > MAX_K || vtbo_row_bytes(quant, k) == 0) return -1;
    mm_ctx c = {quant, out, w, acts, NULL, NULL, m, k, B};
    pool_dispatch(batched_worker, &c);
    return 0;
}

/* ---------------- math.zig ---------------- */

/* rmsNorm, math.zig:11-32 */
void vtbo_rms_norm(float *x, const float *w, size_t n, float eps) {
    float acc[LANES] = {0};
    size_t i = 0;
    for (; i + LANES <= n; i += LANES)
        for (int l = 0; l < LANES; l++) {
            float p = x[i + l] * x[i + l];
            acc[l] += p;
        }
    float ss = reduce8(acc);
    for (; i < n; i++) {
        float p = x[i] * x[i];
        ss += p;
    }
    float mean = ss / (float)n;
    float inv = 1.0f / sqrtf(mean + eps);
    for (i = 0; i < n; i++) {
        float t = x[i] * w[i];
        x[i] = t * inv;
    }
}

/* rope, math.zig:88-104 (interleaved pairs; GGUF llamas use this form,
 * model.zig:57 rope_half = false). */
void vtbo_rope(float *x, size_t hd, size_t pos, float base) {
    float pos_f = (float)pos;
    for (size_t i = 0; i < hd; i += 2) {
        float e = (float)i / (float)hd;
        float inv_freq = 1.0f / powf(base, e);
        float theta = pos_f * inv_freq;
        float c = cosf(theta), s = sinf(theta);
        float x0 = x[i], x1 = x[i + 1];
        float a = x0 * c, b = x1 * s, p = x0 * s, q = x1 * c;
        x[i] = a - b;
        x[i + 1] = p + q;
    }
}

/* softmax, math.zig:136-150 */
void vtbo_softmax(float *x, size_t n) {
    if (n == 0) return;
    float mx = x[0];
    for (size_t i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.f;
    for (size_t i = 0; i < n; i++) {
        float e = expf(x[i] - mx);
        x[i] = e;
        sum += e;
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) x[i] *= inv;
}

/* swiglu, math.zig:154-161 */
void vtbo_swiglu(float *g, const float *u, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float z = g[i];
        float den = 1.0f + expf(-z);
        float silu = z / den;
        g[i] = silu * u[i];
    }
}

/* gegluApprox, math.zig:166-175 */
void vtbo_geglu(float *g, const float *u, size_t n) {
    const float k0 = 0.7978845608028654f;
    for (size_t i = 0; i < n; i++) {
        float z = g[i];
        float z3 = 0.044715f * z;
        z3 = z3 * z;
        z3 = z3 * z;
        float inner = k0 * (z + z3);
        float t = 1.0f + tanhf(inner);
        float gelu = 0.5f * z;
        gelu = gelu * t;
        g[i] = gelu * u[i];
    }
}

/* addInto, math.zig:178-187 */
void vtbo_add_into(float *a, const float *b, size_t n) {
    for (size_t i = 0; i < n; i++) a[i] += b[i];
}

/* argmax, math.zig:190-201: first index of the maximum. */
size_t vtbo_argmax(const float *x, size_t n) {
    if (n == 0) return 0;
    size_t bi = 0;
    float bv = x[0];
    for (size_t i = 1; i < n; i++)
        if (x[i] > bv) { bv = x[i]; bi = i; }
    return bi;
}

/* ---------------- MLX affine quantization (src/kernels/mlx.zig) ---------------- */
/*
 * Layout (mlx.zig:3-23): per row, k*bits/32 little-endian u32 words, each
 * holding 32/bits values low bits first (the top 32 % bits bits unused);
 * per group of G columns one scale and one bias, f16 or bf16 (mlx.zig:30-52);
 * w = q * scale + bias.
 */
static uint16_t mlx_ld16(const uint8_t *p, size_t idx) { return (uint16_t)(p[2 * idx] | (p[2 * idx + 1] << 8)); }
static float mlx_scale(const uint8_t *p, size_t idx, int bf16) { /* loadScale, mlx.zig:43-50 */
    uint16_t b = mlx_ld16(p, idx);
    if (bf16) {
        uint32_t w = (uint32_t)b << 16;
        float f;
        memcpy(&f, &w, 4);
        return f;
    }
    return vtbo_f16_to_f32(b);
}
static uint32_t mlx_ld32(const uint8_t *p, size_t idx) {
    const uint8_t *q = p + 4 * idx;
    return (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16) | ((uint32_t)q[3] << 24);
}
static int mlx_bits_ok(unsigned bits) { return bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8; }

/* dequantRow / dequantRowQ4 (mlx.zig:62-135) for `rows` consecutive rows. */
int vtbo_mlx_dequant(float *out, const uint8_t *w, const uint8_t *scales, const uint8_t *biases, size_t rows,
                     size_t k, unsigned bits, size_t group, int bf16) {
    if (!mlx_bits_ok(bits)) return -1;
    const size_t el = 32 / bits, ng = k / group;
    const uint32_t mask = (1u << bits) - 1u;
    if (group == 0 || k % group || group % el) return -1;
    for (size_t r = 0; r < rows; r++) {
        const uint8_t *wr = w + r * (k / el) * 4, *sr = scales + r * ng * 2, *br = biases + r * ng * 2;
        float *o = out + r * k;
        size_t col = 0;
        for (size_t g = 0; g < ng; g++) {
            const float scale = mlx_scale(sr, g, bf16), bias = mlx_scale(br, g, bf16);
            for (size_t c = 0; c < group; c += el) {
                const uint32_t word = mlx_ld32(wr, (col + c) / el);
                for (size_t i = 0; i < el; i++) {
                    const uint32_t q = (word >> (i * bits)) & mask;
                    float v = (float)q * scale;
                    o[col + c + i] = v + bias;
                }
            }
            col += group;
        }
    }
    return 0;
}

/* matmul -> matmulGeneric / matmulQ4 (mlx.zig:139-330): per group
 * total += scale * sum(q * x) + bias * sum(x), sequential f32. */
int vtbo_mlx_matmul(float *out, const uint8_t *w, const uint8_t *scales, const uint8_t *biases, const float *x,
                    size_t m, size_t k, unsigned bits, size_t group, int bf16) {
    if (!mlx_bits_ok(bits)) return -1;
    const size_t el = 32 / bits, ng = k / group;
    const uint32_t mask = (1u << bits) - 1u;
    if (group == 0 || k % group || group % el) return -1;
    for (size_t r = 0; r < m; r++) {
        const uint8_t *wr = w + r * (k / el) * 4, *sr = scales + r * ng * 2, *br = biases + r * ng * 2;
        float total = 0.0f;
        size_t col = 0;
        for (size_t g = 0; g < ng; g++) {
            const float scale = mlx_scale(sr, g, bf16), bias = mlx_scale(br, g, bf16);
            float q_dot = 0.0f, x_sum = 0.0f;
            for (size_t c = col; c < col + group; c += el) {
                const uint32_t word = mlx_ld32(wr, c / el);
                for (size_t i = 0; i < el; i++) {
                    const uint32_t q = (word >> (i * bits)) & mask;
                    const float xv = x[c + i];
                    q_dot += (float)q * xv;
                    x_sum += xv;
                }
            }
            total += scale * q_dot + bias * x_sum;
            col += group;
        }
        out[r] = total;
    }
    return 0;
}

/* ---------------- token sampler ---------------- */
/*
 * Sampler.sample, src/runtime/sampler.zig:44-104, with the PRNG draw taken
 * as an argument: `u` stands for `self.prng.random().float(f32)` (:92), so
 * the rest of the pipeline can be compared draw for draw.  The index sorts
 * (:58, :70) are std.mem.sort, a stable sort, by descending logit: restated
 * as qsort with the index as the tie-break, which orders the same.
 * `logits` is mutated in place, as in the reference.
 */
static const float *g_sort_keys;
static int desc_stable(const void *a, const void *b) {
    size_t i = *(const size_t *)a, j = *(const size_t *)b;
    float x = g_sort_keys[i], y = g_sort_keys[j];
    if (x > y) return -1;
    if (y > x) return 1;
    return (i > j) - (i < j);
}

uint32_t vtbo_sample(float *logits, size_t n, float temperature, size_t top_k, float top_p, float u) {
    if (temperature == 0.0f) return (uint32_t)vtbo_argmax(logits, n); /* :45-47 */
    const float inv_t = 1.0f / temperature;                             /* :50-51 */
    for (size_t i = 0; i < n; i++) logits[i] *= inv_t;
    size_t *idx = NULL;
    if ((top_k > 0 && top_k < n) || (top_p > 0.0f && top_p < 1.0f)) {
        idx = (size_t *)malloc(n * sizeof *idx);
        if (!idx) return 0;
    }
    if (top_k > 0 && top_k < n) { /* :54-63 */
        for (size_t i = 0; i < n; i++) idx[i] = i;
        g_sort_keys = logits;
        qsort(idx, n, sizeof *idx, desc_stable);
        const float threshold = logits[idx[top_k - 1]];
        for (size_t i = 0; i < n; i++)
            if (logits[i] < threshold) logits[i] = -INFINITY;
    }
    vtbo_softmax(logits, n); /* :65 */
    if (top_p > 0.0f && top_p < 1.0f) { /* :68-89 */
        for (size_t i = 0; i < n; i++) idx[i] = i;
        g_sort_keys = logits;
        qsort(idx, n, sizeof *idx, desc_stable);
        float cumulative = 0.0f;
        size_t cutoff = n;
        for (size_t r = 0; r < n; r++) {
            cumulative += logits[idx[r]];
            if (cumulative >= top_p) { cutoff = r + 1; break; }
        }
        for (size_t r = cutoff; r < n; r++) logits[idx[r]] = 0.0f;
        float sum = 0.0f;
        for (size_t i = 0; i < n; i++) sum += logits[i];
        if (sum > 0.0f) {
            const float inv = 1.0f / sum;
            for (size_t i = 0; i < n; i++) logits[i] *= inv;
        }
    }
    free(idx);
    float acc = 0.0f; /* :92-97 */
    for (size_t i = 0; i < n; i++) {
        acc += logits[i];
        if (u <= acc) return (uint32_t)i;
    }
    size_t last = 0; /* :98-103 */
    for (size_t i = 0; i < n; i++)
        if (logits[i] > 0.0f) last = i;
    return (uint32_t)last;
}

/* ---------------- Llama forward ---------------- */
struct vtbo_model {
    vtbo_config c;
    vtbo_layer *layers;
    const uint8_t *token_embd, *output_w;
    const float *output_norm;
    int q_embd, q_out;
    float *k_cache, *v_cache; /* kv_cache.zig:20-73, [layer][t][kv_h][hd] */
    int64_t pos;
    /* forward.zig State, :33-113 */
    float *x, *xb, *xb2, *q, *kc, *vc, *scores, *attn_out, *gate, *up, *ffn_out;
    int q8_act; /* Q8_0 projections take Q8_0-quantized activations (int32 block dots) */
};

/* matmulRuntime for one row (mm) or B rows (mmb, out[B][rows]).  With the
 * model's q8_act option a Q8_0 projection runs the Q8_0 x Q8_0 path instead
 * (activations quantized per 32-block, dot_i8 block dots, simd.zig:31-62). */
static int mm(const vtbo_model *m, int q, float *out, const uint8_t *w, const float *x, size_t rows, size_t k) {
    if (m->q8_act && q == VTBO_Q8_0) return vtbo_matmul_q8_0_q8_0(out, w, x, rows, k);
    return vtbo_matmul(q, out, w, x, rows, k);
}
static int mmb(const vtbo_model *m, int q, float *out, const uint8_t *w, const float *acts, size_t rows, size_t k,
               size_t B) {
    if (!(m->q8_act && q == VTBO_Q8_0)) return vtbo_matmul_batched(q, out, w, acts, rows, k, B);
    for (size_t b = 0; b < B; b++)
        if (vtbo_matmul_q8_0_q8_0(out + b * rows, w, acts + b * k, rows, k)) return -1;
    return 0;
}

void vtbo_model_set_q8_activations(vtbo_model *m, int on) { m->q8_act = on != 0; }

vtbo_model *vtbo_model_create(const vtbo_config *c, const vtbo_layer *layers,
                              const uint8_t *token_embd, int q_token_embd,
                              const float *output_norm, const uint8_t *output_w, int q_output) {
    vtbo_model *m = (vtbo_model *)calloc(1, sizeof(*m));
    m->c = *c;
    m->layers = (vtbo_layer *)malloc(sizeof(vtbo_layer) * (size_t)c->n_layers);
    memcpy(m->layers, layers, sizeof(vtbo_layer) * (size_t)c->n_layers);
    m->token_embd = token_embd;
    m->q_embd = q_token_embd;
    m->output_norm = output_norm;
    m->output_w = output_w;
    m->q_out = q_output;
    size_t kvd = (size_t)(c->n_kv_heads * c->head_dim);
    size_t tot = (size_t)c->n_layers * (size_t)c->max_seq * kvd;
    m->k_cache = (float *)calloc(tot, 4);
    m->v_cache = (float *)calloc(tot, 4);
    size_t d = (size_t)c->dim, f = (size_t)c->ffn_dim;
    m->x = (float *)calloc(d, 4);
    m->xb = (float *)calloc(d, 4);
    m->xb2 = (float *)calloc(d, 4);
    m->q = (float *)calloc((size_t)(c->n_heads * c->head_dim), 4);
    m->kc = (float *)calloc(kvd, 4);
    m->vc = (float *)calloc(kvd, 4);
    m->scores = (float *)calloc((size_t)(c->n_heads * c->max_seq), 4);
    m->attn_out = (float *)calloc(d, 4);
    m->gate = (float *)calloc(f, 4);
    m->up = (float *)calloc(f, 4);
    m->ffn_out = (float *)calloc(d, 4);
    return m;
}

void vtbo_model_destroy(vtbo_model *m) {
    if (!m) return;
    free(m->layers); free(m->k_cache); free(m->v_cache);
    free(m->x); free(m->xb); free(m->xb2); free(m->q); free(m->kc); free(m->vc);
    free(m->scores); free(m->attn_out); free(m->gate); free(m->up); free(m->ffn_out);
    free(m);
}

void vtbo_model_reset(vtbo_model *m) { m->pos = 0; }
int64_t vtbo_model_pos(const vtbo_model *m) { return m->pos; }

static size_t kv_dim(const vtbo_config *c) { return (size_t)(c->n_kv_heads * c->head_dim); }
static float *layer_k(const vtbo_model *m, size_t l) { return m->k_cache + l * (size_t)m->c.max_seq * kv_dim(&m->c); }
static float *layer_v(const vtbo_model *m, size_t l) { return m->v_cache + l * (size_t)m->c.max_seq * kv_dim(&m->c); }
const float *vtbo_kv_keys(const vtbo_model *m, size_t l) { return layer_k(m, l); }
const float *vtbo_kv_values(const vtbo_model *m, size_t l) { return layer_v(m, l); }

/* gatherEmbedding, forward.zig:738-845: dequantize row `id` of the table. */
static int gather_embedding(const vtbo_model *m, float *out, uint32_t id) {
    size_t rb = vtbo_row_bytes(m->q_embd, (size_t)m->c.dim);
    return vtbo_dequant(m->q_embd, m->token_embd + (size_t)id * rb, out, (size_t)m->c.dim);
}

/* Causal GQA attention for the query at absolute position cur_pos
 * (cpuAttention forward.zig:187-228 and attentionCausal prefill.zig:237-287
 * share this arithmetic; Llama has no sliding window). */
static void attention_one(const vtbo_model *m, size_t l, const float *q, float *out,
                          float *scores_all, int64_t cur_pos) {
    const vtbo_config *c = &m->c;
    float inv_sqrt_hd = 1.0f / sqrtf((float)c->head_dim);
    size_t seq = (size_t)cur_pos + 1, row = kv_dim(c), hd = (size_t)c->head_dim;
    const float *kb = layer_k(m, l), *vb = layer_v(m, l);
    memset(out, 0, sizeof(float) * (size_t)c->dim);
    for (int64_t h = 0; h < c->n_heads; h++) {
        int64_t kvh = (h * c->n_kv_heads) / c->n_heads;
        const float *qh = q + h * (int64_t)hd;
        float *sc = scores_all + h * c->max_seq;
        for (size_t t = 0; t < seq; t++) {
            const float *kt = kb + t * row + (size_t)kvh * hd;
            float s = 0.f;
            for (size_t d = 0; d < hd; d++) {
                float p = qh[d] * kt[d];
                s += p;
            }
            sc[t] = s * inv_sqrt_hd;
        }
        vtbo_softmax(sc, seq);
        float *oh = out + h * (int64_t)hd;
        for (size_t t = 0; t < seq; t++) {
            const float *vt = vb + t * row + (size_t)kvh * hd;
            float wgt = sc[t];
            for (size_t d = 0; d < hd; d++) {
                float p = wgt * vt[d];
                oh[d] += p;
            }
        }
    }
}

/* cpuLayerStep, forward.zig:230-288 */
static int layer_step(vtbo_model *m, size_t l) {
    const vtbo_config *c = &m->c;
    const vtbo_layer *L = &m->layers[l];
    size_t d = (size_t)c->dim, kvd = kv_dim(c), f = (size_t)c->ffn_dim, hd = (size_t)c->head_dim;
    memcpy(m->xb, m->x, d * 4);
    vtbo_rms_norm(m->xb, L->attn_norm, d, c->rms_eps);
    if (mm(m, L->q_attn_q, m->q, L->attn_q, m->xb, d, d)) return -1;
    if (mm(m, L->q_attn_k, m->kc, L->attn_k, m->xb, kvd, d)) return -1;
    if (mm(m, L->q_attn_v, m->vc, L->attn_v, m->xb, kvd, d)) return -1;
    for (int64_t h = 0; h < c->n_heads; h++) vtbo_rope(m->q + h * (int64_t)hd, hd, (size_t)m->pos, c->rope_base);
    for (int64_t h = 0; h < c->n_kv_heads; h++) vtbo_rope(m->kc + h * (int64_t)hd, hd, (size_t)m->pos, c->rope_base);
    memcpy(layer_k(m, l) + (size_t)m->pos * kvd, m->kc, kvd * 4);
    memcpy(layer_v(m, l) + (size_t)m->pos * kvd, m->vc, kvd * 4);
    attention_one(m, l, m->q, m->attn_out, m->scores, m->pos);
    if (mm(m, L->q_attn_o, m->xb2, L->attn_o, m->attn_out, d, d)) return -1;
    vtbo_add_into(m->x, m->xb2, d);
    memcpy(m->xb, m->x, d * 4);
    vtbo_rms_norm(m->xb, L->ffn_norm, d, c->rms_eps);
    if (mm(m, L->q_ffn_gate, m->gate, L->ffn_gate, m->xb, f, d)) return -1;
    if (mm(m, L->q_ffn_up, m->up, L->ffn_up, m->xb, f, d)) return -1;
    vtbo_swiglu(m->gate, m->up, f);
    if (mm(m, L->q_ffn_down, m->ffn_out, L->ffn_down, m->gate, d, f)) return -1;
    vtbo_add_into(m->x, m->ffn_out, d);
    return 0;
}

/* stepWithBackend, forward.zig:152-172, with CpuBackend finalStep
 * (backend_cpu.zig:88-106). */
int vtbo_step(vtbo_model *m, uint32_t token, float *logits) {
    const vtbo_config *c = &m->c;
    if ((int64_t)token >= c->vocab_size) return -2;
    if (m->pos >= c->max_seq) return -3;
    if (gather_embedding(m, m->x, token)) return -1;
    for (size_t l = 0; l < (size_t)c->n_layers; l++)
        if (layer_step(m, l)) return -1;
    m->pos += 1;
    vtbo_rms_norm(m->x, m->output_norm, (size_t)c->dim, c->rms_eps);
    return mm(m, m->q_out, logits, m->output_w, m->x, (size_t)c->vocab_size, (size_t)c->dim);
}

/* prefillCpu / prefillLayer, prefill.zig:111-232 */
int vtbo_prefill(vtbo_model *m, const uint32_t *tokens, size_t B, float *logits) {
    const vtbo_config *c = &m->c;
    if (B == 0) return 0;
    if (m->pos + (int64_t)B > c->max_seq) return -3;
    for (size_t b = 0; b < B; b++)
        if ((int64_t)tokens[b] >= c->vocab_size) return -2;
    size_t d = (size_t)c->dim, kvd = kv_dim(c), f = (size_t)c->ffn_dim, hd = (size_t)c->head_dim;
    size_t qd = (size_t)(c->n_heads * c->head_dim);
    float *x = (float *)malloc(B * d * 4), *xb = (float *)malloc(B * d * 4), *xb2 = (float *)malloc(B * d * 4);
    float *q = (float *)malloc(B * qd * 4), *kc = (float *)malloc(B * kvd * 4), *vc = (float *)malloc(B * kvd * 4);
    float *ao = (float *)malloc(B * d * 4), *g = (float *)malloc(B * f * 4), *u = (float *)malloc(B * f * 4);
    float *fo = (float *)malloc(B * d * 4);
    float *sc = (float *)malloc((size_t)(c->n_heads * c->max_seq) * 4);
    int rc = 0;
    for (size_t b = 0; b < B; b++)
        if (gather_embedding(m, x + b * d, tokens[b])) { rc = -1; goto done; }
    for (size_t l = 0; l < (size_t)c->n_layers; l++) {
        const vtbo_layer *L = &m->layers[l];
        for (size_t b = 0; b < B; b++) {
            memcpy(xb + b * d, x + b * d, d * 4);
            vtbo_rms_norm(xb + b * d, L->attn_norm, d, c->rms_eps);
        }
        if (mmb(m, L->q_attn_q, q, L->attn_q, xb, d, d, B) ||
            mmb(m, L->q_attn_k, kc, L->attn_k, xb, kvd, d, B) ||
            mmb(m, L->q_attn_v, vc, L->attn_v, xb, kvd, d, B)) { rc = -1; goto done; }
        for (size_t b = 0; b < B; b++) {
            size_t pb = (size_t)m->pos + b;
            for (int64_t h = 0; h < c->n_heads; h++) vtbo_rope(q + b * qd + (size_t)h * hd, hd, pb, c->rope_base);
            for (int64_t h = 0; h < c->n_kv_heads; h++) vtbo_rope(kc + b * kvd + (size_t)h * hd, hd, pb, c->rope_base);
            memcpy(layer_k(m, l) + pb * kvd, kc + b * kvd, kvd * 4);
            memcpy(layer_v(m, l) + pb * kvd, vc + b * kvd, kvd * 4);
        }
        for (size_t b = 0; b < B; b++)
            attention_one(m, l, q + b * qd, ao + b * d, sc, m->pos + (int64_t)b);
        if (mmb(m, L->q_attn_o, xb2, L->attn_o, ao, d, d, B)) { rc = -1; goto done; }
        for (size_t b = 0; b < B; b++) vtbo_add_into(x + b * d, xb2 + b * d, d);
        for (size_t b = 0; b < B; b++) {
            memcpy(xb + b * d, x + b * d, d * 4);
            vtbo_rms_norm(xb + b * d, L->ffn_norm, d, c->rms_eps);
        }
        if (mmb(m, L->q_ffn_gate, g, L->ffn_gate, xb, f, d, B) ||
            mmb(m, L->q_ffn_up, u, L->ffn_up, xb, f, d, B)) { rc = -1; goto done; }
        for (size_t b = 0; b < B; b++) vtbo_swiglu(g + b * f, u + b * f, f);
        if (mmb(m, L->q_ffn_down, fo, L->ffn_down, g, d, f, B)) { rc = -1; goto done; }
        for (size_t b = 0; b < B; b++) vtbo_add_into(x + b * d, fo + b * d, d);
    }
    m->pos += (int64_t)B;
    {
        float *last = x + (B - 1) * d;
        vtbo_rms_norm(last, m->output_norm, d, c->rms_eps);
        rc = mmb(m, m->q_out, logits, m->output_w, last, (size_t)c->vocab_size, d, 1);
    }
done:
    free(x); free(xb); free(xb2); free(q); free(kc); free(vc); free(ao); free(g); free(u); free(fo); free(sc);
    return rc;
}
