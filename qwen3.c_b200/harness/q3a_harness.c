/*
 * q3a_harness.c -- seeded C harness of the attention block: a C host that
 * links libq3attn.so through include/q3attn.h only (no Python, no CUDA
 * headers), generates the decode shapes of the benchmark configurations and
 * times the full-depth step end to end through the host-pointer API.
 *
 * The per-layer call is the binding a Qwen3.c maintainer adds to forward():
 * attn_init() after the config is known, then one
 * q3a_attn_layer() per layer in place of the inline block of
 * qwen3-8b/cpu-multicore/main.c:1331-1369, on run-state buffers laid out like
 * the reference's State (qwen3-8b/cpu/main.c:646-650).
 *
 * Usage: q3a_harness [--layers N] [--ctx L] [--kv f32|bf16] [--steps K]
 *                    [--warmup W] [--seed S] [--device D] [--dump DIR]
 *   One step = the N layer calls at position L-1 over caches holding rows
 *   0..L-2 (seeded N(0,1) k/v, k normed and rotated: q3a_kv_synth).  Each
 *   call copies q, k, v and the norm gains in from host memory and xb, q, k
 *   out, as the CPU forward() sees them.  Prints one JSON line with the
 *   end-to-end time per layer (CLOCK_MONOTONIC around K steps after W
 *   warm-up steps).  --dump DIR writes, for layer 0, the raw inputs, the
 *   outputs and the cache rows 0..L-2 as raw float32 files, for a checker.
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "q3attn.h"

/* ---- the reference's Config / State fields this block uses
 * (qwen3-8b/cpu/main.c:603-607, 646-650) */
typedef struct {
    int n_layers, n_heads, n_kv_heads, head_dim, max_seq;
    float norm_eps, rope_theta;
} Config;

typedef struct {
    float *q, *k, *v, *xb;
} State;

/* ---- the binding a maintainer adds to forward() */
static q3a_ctx *g_attn;

static void attn_init(const Config *c, int kv_dtype, int device) {
    q3a_cfg cfg;
    q3a_cfg_default(&cfg);
    cfg.n_layers = c->n_layers;  cfg.n_heads = c->n_heads;
    cfg.n_kv_heads = c->n_kv_heads;  cfg.head_dim = c->head_dim;
    cfg.max_seq = c->max_seq;  cfg.norm_eps = c->norm_eps;  cfg.rope_theta = c->rope_theta;
    cfg.ptr_mode = Q3A_PTR_HOST;              /* s->q, s->k, ... are host buffers */
    cfg.kv_dtype = kv_dtype;
    cfg.device = device;
    if (q3a_create(&g_attn, &cfg) != Q3A_OK) {
        fprintf(stderr, "q3a_create: %s\n", q3a_last_error());
        exit(1);                              /* the reference's error convention */
    }
}

static void attn_block(State *s, const float *q_norm_w, const float *k_norm_w, int l, int pos) {
    if (q3a_attn_layer(g_attn, s->xb, s->q, s->k, s->v, q_norm_w, k_norm_w, l, pos) != Q3A_OK) {
        fprintf(stderr, "q3a_attn_layer: %s\n", q3a_last_error());
        exit(1);
    }
}

/* ---- seeded N(0,1) on the host from the integer stream q3a_randn uses:
 * stream key = splitmix64(seed ^ splitmix64(stream + 0x51ED2701)); uniform
 * u(n) = the top 23 bits of one xorshift64* output step (the generator of
 * rng_f32, qwen3-8b/cpu/main.c:1377-1382) seeded by splitmix64(key + n);
 * element i is the Box-Muller transform of u(2j), u(2j+1), j = i/2 (cos for
 * even i, sin for odd), here with the host's libm. */
static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static float u01(uint64_t key, uint64_t n) {
    uint64_t st = splitmix64(key + n);
    st ^= st >> 12;
    st ^= st << 25;
    st ^= st >> 27;
    const uint32_t r = (uint32_t)((st * 0x2545F4914F6CDD1Dull) >> 41);
    return ((float)r + 0.5f) * (1.0f / 8388608.0f);
}

static void randn(float *dst, size_t n, uint64_t seed, uint64_t stream) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream + 0x51ED2701ull));
    for (size_t i = 0; i < n; i++) {
        const uint64_t j = i >> 1;
        const float r = sqrtf(-2.0f * logf(u01(key, 2 * j)));
        const float a = 6.283185307179586f * u01(key, 2 * j + 1);
        dst[i] = (i & 1) ? r * sinf(a) : r * cosf(a);
    }
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

static void *xmalloc(size_t n) {
    void *p = malloc(n);
    if (!p) {
        fprintf(stderr, "out of host memory (%zu bytes)\n", n);
        exit(1);
    }
    return p;
}

static void dump(const char *dir, const char *name, const float *x, size_t n) {
    char path[1024];
    snprintf(path, sizeof(path), "%s/%s.f32", dir, name);
    FILE *f = fopen(path, "wb");
    if (!f || fwrite(x, sizeof(float), n, f) != n) {
        fprintf(stderr, "cannot write %s\n", path);
        exit(1);
    }
    fclose(f);
}

int main(int argc, char **argv) {
    Config c = {36, 32, 8, 128, 8192, 1e-6f, 5e6f};
    int kv_dtype = Q3A_KV_F32, steps = 20, warmup = 5, device = 0;
    uint64_t seed = 1234;
    const char *dump_dir = NULL;
    for (int i = 1; i < argc; i++) {
        const char *a = argv[i];
        const char *v = i + 1 < argc ? argv[i + 1] : NULL;
        if (!v) {
            fprintf(stderr, "%s needs a value\n", a);
            return 2;
        }
        if (!strcmp(a, "--layers")) c.n_layers = atoi(v);
        else if (!strcmp(a, "--ctx")) c.max_seq = atoi(v);
        else if (!strcmp(a, "--kv")) kv_dtype = !strcmp(v, "bf16") ? Q3A_KV_BF16 : Q3A_KV_F32;
        else if (!strcmp(a, "--steps")) steps = atoi(v);
        else if (!strcmp(a, "--warmup")) warmup = atoi(v);
        else if (!strcmp(a, "--seed")) seed = strtoull(v, NULL, 10);
        else if (!strcmp(a, "--device")) device = atoi(v);
        else if (!strcmp(a, "--dump")) dump_dir = v;
        else {
            fprintf(stderr, "unknown option %s\n", a);
            return 2;
        }
        i++;
    }
    if (c.n_layers < 1 || c.max_seq < 2 || steps < 1 || warmup < 0) {
        fprintf(stderr, "bad sizes\n");
        return 2;
    }
    const int pos = c.max_seq - 1;
    const size_t qd = (size_t)c.n_heads * c.head_dim, kd = (size_t)c.n_kv_heads * c.head_dim;
    attn_init(&c, kv_dtype, device);

    /* caches: rows 0..pos-1 of every layer, streams layer*16+1 (k), +2 (v) */
    for (int l = 0; l < c.n_layers; l++) {
        if (q3a_kv_synth(g_attn, 0, l, 0, pos, seed, (uint64_t)l * 16 + 1,
                         (uint64_t)l * 16 + 2) != Q3A_OK) {
            fprintf(stderr, "q3a_kv_synth: %s\n", q3a_last_error());
            return 1;
        }
    }
    /* per-layer new-token projections (streams layer*16+3/4/5), unit gains */
    float *q0 = xmalloc(sizeof(float) * qd * c.n_layers);
    float *k0 = xmalloc(sizeof(float) * kd * c.n_layers);
    float *v0 = xmalloc(sizeof(float) * kd * c.n_layers);
    float *xb = xmalloc(sizeof(float) * qd * c.n_layers);
    float *w = xmalloc(sizeof(float) * c.head_dim);
    for (int l = 0; l < c.n_layers; l++) {
        randn(q0 + l * qd, qd, seed, (uint64_t)l * 16 + 3);
        randn(k0 + l * kd, kd, seed, (uint64_t)l * 16 + 4);
        randn(v0 + l * kd, kd, seed, (uint64_t)l * 16 + 5);
    }
    for (int i = 0; i < c.head_dim; i++) w[i] = 1.0f;
    State s;
    s.q = xmalloc(sizeof(float) * qd);
    s.k = xmalloc(sizeof(float) * kd);

    if (dump_dir) {
        /* layer 0: the cache rows the call attends, its inputs and outputs */
        float *kc = xmalloc(sizeof(float) * kd * pos), *vc = xmalloc(sizeof(float) * kd * pos);
        if (q3a_kv_read(g_attn, 0, 0, 0, pos, kc, vc) != Q3A_OK) {
            fprintf(stderr, "q3a_kv_read: %s\n", q3a_last_error());
            return 1;
        }
        memcpy(s.q, q0, sizeof(float) * qd);
        memcpy(s.k, k0, sizeof(float) * kd);
        s.v = v0;
        s.xb = xb;
        attn_block(&s, w, w, 0, pos);
        dump(dump_dir, "kc", kc, kd * pos);
        dump(dump_dir, "vc", vc, kd * pos);
        dump(dump_dir, "q_in", q0, qd);
        dump(dump_dir, "k_in", k0, kd);
        dump(dump_dir, "v_in", v0, kd);
        dump(dump_dir, "xb", xb, qd);
        dump(dump_dir, "q_out", s.q, qd);
        dump(dump_dir, "k_out", s.k, kd);
        free(kc);
        free(vc);
    }

    uint64_t n0 = 0;
    double t0 = 0.0;
    for (int it = 0; it < warmup + steps; it++) {
        if (it == warmup) {
            n0 = q3a_launch_count(g_attn);
            t0 = now_s();
        }
        for (int l = 0; l < c.n_layers; l++) {
            /* the block normalises and rotates q and k in place: every step
             * starts again from the raw projections */
            memcpy(s.q, q0 + l * qd, sizeof(float) * qd);
            memcpy(s.k, k0 + l * kd, sizeof(float) * kd);
            s.v = v0 + l * kd;
            s.xb = xb + l * qd;
            attn_block(&s, w, w, l, pos);
        }
    }
    const double t = now_s() - t0;
    if (q3a_check_device_error(g_attn) != Q3A_OK) {
        fprintf(stderr, "device error: %s\n", q3a_last_error());
        return 1;
    }
    const uint64_t launches = q3a_launch_count(g_attn) - n0;
    const double us = t * 1e6 / ((double)steps * c.n_layers);
    const size_t h2d = (size_t)c.n_layers * (qd + 2 * kd + 2 * (size_t)c.head_dim) * sizeof(float);
    const size_t d2h = (size_t)c.n_layers * (2 * qd + kd) * sizeof(float);
    double cs = 0.0;
    for (size_t i = 0; i < qd * c.n_layers; i++) cs += fabs((double)xb[i]);
    printf("{\"api\": \"q3a_attn_layer (host pointers, C host)\", \"layers\": %d, \"ctx\": %d, "
           "\"kv\": \"%s\", \"steps\": %d, \"warmup\": %d, \"us_per_layer\": %.4f, "
           "\"t_s\": %.6f, \"h2d_bytes_per_step\": %zu, \"d2h_bytes_per_step\": %zu, "
           "\"launches\": %llu, \"xb_abs_sum\": %.6e}\n",
           c.n_layers, c.max_seq, kv_dtype == Q3A_KV_BF16 ? "bf16" : "f32", steps, warmup, us, t,
           h2d, d2h, (unsigned long long)launches, cs);
    q3a_destroy(g_attn);
    free(q0); free(k0); free(v0); free(xb); free(w); free(s.q); free(s.k);
    return 0;
}
