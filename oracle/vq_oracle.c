/*
 * CPU oracle for the vq4/v1 hot path, in C -- TEST INFRASTRUCTURE ONLY.
 *
 * A checker and the timed CPU baseline, never the product: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * load it. It restates the same reference algorithms as vq_oracle.py, with
 * a small pthread parallel-for across host cores (VQO_THREADS overrides the
 * count; the default is every CPU this process may run on):
 *
 *   vqo_decode    VQArray.decode            (reference _kit/python/vq.py:117-121)
 *   vqo_encode    encode, float64 argmin    (vq.py:154-179): d += (v-b)*(v-b)
 *                 in component order, lowest index on ties, the partial last
 *                 vector compared on its valid components only (vq.py:171-172)
 *   vqo_dense_nt  decode(W) then X @ W^T    (the CPU path of the north-star
 *                 dense-activation product), float64 accumulation
 *   vqo_adamw     vq4.comp adamw_value      (_kit/kernels/vq4.comp:87-116),
 *                 FP32, every operation rounded on its own (build with
 *                 -ffp-contract=off so nothing is fused)
 *
 * Built by oracle/Makefile into oracle/libvq_oracle.so.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef void (*vqo_body)(int64_t begin, int64_t end, void *ctx);

typedef struct {
    vqo_body body;
    void *ctx;
    int64_t begin, end;
} vqo_slice;

static void *vqo_run(void *arg) {
    vqo_slice *s = (vqo_slice *)arg;
    s->body(s->begin, s->end, s->ctx);
    return NULL;
}

int vqo_threads(void) {
    const char *env = getenv("VQO_THREADS");
    if (env && atoi(env) > 0) return atoi(env);
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof(set), &set) == 0) return CPU_COUNT(&set);
    return 1;
}

/* Split [0, count) into one contiguous slice per thread. */
static void vqo_parallel(int64_t count, vqo_body body, void *ctx) {
    int threads = vqo_threads();
    if (threads > 256) threads = 256;
    if (count < threads) threads = count > 0 ? (int)count : 1;
    pthread_t ids[256];
    vqo_slice slices[256];
    int64_t chunk = (count + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        slices[t].body = body;
        slices[t].ctx = ctx;
        slices[t].begin = t * chunk < count ? t * chunk : count;
        slices[t].end = (t + 1) * chunk < count ? (t + 1) * chunk : count;
        if (t == threads - 1 || pthread_create(&ids[t], NULL, vqo_run, &slices[t]) != 0) {
            vqo_run(&slices[t]);
        } else {
            ++started;
        }
    }
    for (int t = 0; t < started; ++t) pthread_join(ids[t], NULL);
}

static inline uint32_t nibble(const uint32_t *codes, uint64_t vector) {
    return (codes[vector >> 3] >> (4u * (uint32_t)(vector & 7u))) & 15u;
}

typedef struct { const uint32_t *codes; const float *book; uint64_t n; uint32_t g; float *out; } dec_ctx;

static void dec_body(int64_t b, int64_t e, void *p) {
    dec_ctx *c = (dec_ctx *)p;
    for (int64_t v = b; v < e; ++v) {
        const float *row = c->book + (uint64_t)nibble(c->codes, (uint64_t)v) * c->g;
        uint64_t start = (uint64_t)v * c->g;
        uint64_t valid = c->n - start < c->g ? c->n - start : c->g;
        memcpy(c->out + start, row, valid * sizeof(float));
    }
}

void vqo_decode(const uint32_t *codes, const float *book, uint64_t n, uint32_t g, float *out) {
    dec_ctx c = {codes, book, n, g, out};
    vqo_parallel((int64_t)((n + g - 1) / g), dec_body, &c);
}

typedef struct { const float *values; uint64_t n; const float *book; uint32_t g; uint32_t *codes; } enc_ctx;

static void enc_body(int64_t b, int64_t e, void *p) {
    enc_ctx *c = (enc_ctx *)p;
    const uint32_t g = c->g;
    int64_t vectors = (int64_t)((c->n + g - 1) / g);
    for (int64_t w = b; w < e; ++w) {
        uint32_t packed = 0;
        for (int lane = 0; lane < 8; ++lane) {
            int64_t v = w * 8 + lane;
            if (v >= vectors) break;
            uint64_t start = (uint64_t)v * g;
            uint64_t valid = c->n - start < g ? c->n - start : g;
            double best = 0.0;
            uint32_t chosen = 0;
            for (uint32_t k = 0; k < 16; ++k) {
                double d = 0.0;
                for (uint64_t j = 0; j < valid; ++j) {
                    double delta = (double)c->values[start + j] - (double)c->book[k * g + j];
                    double sq = delta * delta;
                    d = d + sq;
                }
                if (k == 0 || d < best) { best = d; chosen = k; }
            }
            packed |= chosen << (4 * lane);
        }
        c->codes[w] = packed;
    }
}

void vqo_encode(const float *values, uint64_t n, const float *book, uint32_t g, uint32_t *codes) {
    enc_ctx c = {values, n, book, g, codes};
    int64_t vectors = (int64_t)((n + g - 1) / g);
    vqo_parallel((vectors + 7) / 8, enc_body, &c);
}

typedef struct {
    const float *x; uint32_t M, K; const uint32_t *codes; const float *book; uint32_t N, g; float *y;
} nt_ctx;

static void nt_body(int64_t b, int64_t e, void *p) {
    nt_ctx *c = (nt_ctx *)p;
    for (int64_t n = b; n < e; ++n) {
        for (uint32_t m = 0; m < c->M; ++m) {
            double acc = 0.0;
            const float *xr = c->x + (uint64_t)m * c->K;
            for (uint32_t k = 0; k < c->K; k += c->g) {
                uint64_t logical = (uint64_t)n * c->K + k;
                const float *row = c->book + (uint64_t)nibble(c->codes, logical / c->g) * c->g;
                for (uint32_t j = 0; j < c->g && k + j < c->K; ++j) acc += (double)xr[k + j] * (double)row[j];
            }
            c->y[(uint64_t)m * c->N + n] = (float)acc;
        }
    }
}

/* y[m, n] = sum_k x[m, k] * decode(W)[n, k], W stored N x K; float64 sums. */
void vqo_dense_nt(const float *x, uint32_t M, uint32_t K, const uint32_t *codes, const float *book,
                  uint32_t N, uint32_t g, float *y) {
    nt_ctx c = {x, M, K, codes, book, N, g, y};
    vqo_parallel((int64_t)N, nt_body, &c);
}

typedef struct {
    const float *w, *m, *v, *g; const float *c; float *wo, *mo, *vo;
} adam_ctx;

static void adam_body(int64_t b, int64_t e, void *p) {
    adam_ctx *a = (adam_ctx *)p;
    const float lr = a->c[0], b1 = a->c[1], b2 = a->c[2], eps = a->c[3], decay = a->c[4];
    const float c1 = a->c[5], c2 = a->c[6];
    for (int64_t i = b; i < e; ++i) {
        float t1 = b1 * a->m[i];
        float ob1 = 1.0f - b1;
        float t2 = ob1 * a->g[i];
        float next_m = t1 + t2;
        float gg = a->g[i] * a->g[i];
        float t3 = b2 * a->v[i];
        float ob2 = 1.0f - b2;
        float t4 = ob2 * gg;
        float next_v = t3 + t4;
        float cm = next_m / c1;
        float cv = next_v / c2;
        float den = sqrtf(cv) + eps;
        float lrd = lr * decay;
        float keep = 1.0f - lrd;
        float decayed = a->w[i] * keep;
        float num = lr * cm;
        float step = num / den;
        a->wo[i] = decayed - step;
        a->mo[i] = next_m;
        a->vo[i] = next_v;
    }
}

/* One FP32 AdamW value per element, vq4.comp:103-109 order. */
void vqo_adamw(const float *w, const float *m, const float *v, const float *g, uint64_t n,
               const float *c, float *w_out, float *m_out, float *v_out) {
    adam_ctx a = {w, m, v, g, c, w_out, m_out, v_out};
    vqo_parallel((int64_t)n, adam_body, &a);
}
