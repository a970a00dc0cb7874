/*
 * q3a_oracle.c -- CPU restatement of the Qwen3.c GQA attention block.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product): loaded by the
 * tests, by the smoke check and by the bench's CPU-baseline leg.
 *
 * Build: gcc -O3 -std=c11 -fopenmp -fPIC -shared (oracle/Makefile).  The
 * reference builds with gcc -O3 -std=c11 -fopenmp (qwen3-8b/cpu-multicore/
 * Makefile), so in ISO C mode with no fast-math the compiler keeps every
 * float operation in source order and does not contract a*b+c into an FMA;
 * each function below keeps the reference's operation order and is therefore
 * bit-identical to the reference code it cites.
 */
#include "q3a_oracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>

/* qwen3-8b/cpu/main.c:1175-1183; cpu-multicore/main.c:1180-1189 adds the
 * per-head OpenMP loop.  Sequential sum of squares per head, then
 * v *= (1/sqrtf(ss/hd + eps)) * w[i]. */
static void norm_head(float *seg, const float *w, int hd, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < hd; i++) ss += seg[i] * seg[i];
    ss = 1.0f / sqrtf(ss / hd + eps);
    for (int i = 0; i < hd; i++) seg[i] *= ss * w[i];
}

void orc_rmsnorm_head(float *vec, const float *w, int n_heads, int hd, float eps) {
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; h++) norm_head(vec + (size_t)h * hd, w, hd, eps);
}

/* qwen3-8b/cpu/main.c:1282-1295: adjacent pairs (2i, 2i+1) rotated by
 * pos * theta^(-2i/hd), angle and trig in fp32. */
static void rope_head(float *seg, int hd, int pos, float theta) {
    for (int i = 0; i < hd; i += 2) {
        float freq = 1.0f / powf(theta, (float)i / hd);
        float val = pos * freq;
        float cr = cosf(val);
        float ci = sinf(val);
        float v0 = seg[i], v1 = seg[i + 1];
        seg[i] = v0 * cr - v1 * ci;
        seg[i + 1] = v0 * ci + v1 * cr;
    }
}

void orc_rope(float *vec, int n_heads, int hd, int pos, float theta) {
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; h++) rope_head(vec + (size_t)h * hd, hd, pos, theta);
}

/* orc_rmsnorm_head then orc_rope on n consecutive rows [n][n_heads*hd], row t
 * at position pos0 + t: the same per-head arithmetic, parallel over rows
 * (a test-speed helper for building long synthetic caches). */
void orc_prep_rows(float *rows, const float *w, int n, int n_heads, int hd, int pos0,
                   float eps, float theta) {
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < n; t++) {
        for (int h = 0; h < n_heads; h++) {
            float *seg = rows + ((size_t)t * n_heads + h) * hd;
            norm_head(seg, w, hd, eps);
            rope_head(seg, hd, pos0 + t, theta);
        }
    }
}

/* qwen3-8b/cpu/main.c:1185-1195: three passes (max, exp+sum, divide). */
void orc_softmax(float *x, int n) {
    float max_val = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* One q head of qwen3-8b/cpu-multicore/main.c:1346-1369. */
static void attn_head(float *oh, const float *qh, const float *kc, const float *vc,
                      float *att_h, size_t loff, int pos, int kvh, int hd, int kv_dim) {
    float scale = 1.0f / sqrtf((float)hd);
    for (int t = 0; t <= pos; t++) {
        const float *kt = kc + loff + (size_t)t * kv_dim + (size_t)kvh * hd;
        float score = 0.0f;
        for (int i = 0; i < hd; i++) score += qh[i] * kt[i];
        att_h[t] = score * scale;
    }
    orc_softmax(att_h, pos + 1);
    memset(oh, 0, (size_t)hd * sizeof(float));
    for (int t = 0; t <= pos; t++) {
        float a = att_h[t];
        const float *vt = vc + loff + (size_t)t * kv_dim + (size_t)kvh * hd;
        for (int i = 0; i < hd; i++) oh[i] += a * vt[i];
    }
}

void orc_attn_decode(float *xb, const float *q, const float *kc, const float *vc,
                     float *att, size_t loff, int pos, int n_heads, int kv_mul,
                     int hd, int kv_dim, int max_seq) {
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; h++) {
        attn_head(xb + (size_t)h * hd, q + (size_t)h * hd, kc, vc,
                  att + (size_t)h * max_seq, loff, pos, h / kv_mul, hd, kv_dim);
    }
}

/* qwen3-8b/cpu/main.c:1319-1353 for one layer. */
void orc_attn_block(float *xb, float *q, float *k, const float *v,
                    const float *q_norm_w, const float *k_norm_w,
                    float *kc, float *vc, float *att, int layer, int pos,
                    int n_heads, int n_kv, int hd, int max_seq,
                    float eps, float theta) {
    int kv_dim = n_kv * hd;
    int kv_mul = n_heads / n_kv;
    orc_rmsnorm_head(q, q_norm_w, n_heads, hd, eps);   /* :1319 */
    orc_rmsnorm_head(k, k_norm_w, n_kv, hd, eps);      /* :1320 */
    orc_rope(q, n_heads, hd, pos, theta);              /* :1322 */
    orc_rope(k, n_kv, hd, pos, theta);                 /* :1323 */
    size_t loff = (size_t)layer * max_seq * kv_dim;    /* :1325-1329 */
    memcpy(kc + loff + (size_t)pos * kv_dim, k, (size_t)kv_dim * sizeof(float));
    memcpy(vc + loff + (size_t)pos * kv_dim, v, (size_t)kv_dim * sizeof(float));
    orc_attn_decode(xb, q, kc, vc, att, loff, pos, n_heads, kv_mul, hd, kv_dim,
                    max_seq);                          /* :1331-1353 */
}

/* Causal prefill = the decode step looped over prompt positions
 * (qwen3-8b/cpu/main.c:1481-1499 teacher-forces the prompt one token at a
 * time through forward()). */
void orc_prefill_causal(float *out, const float *q, const float *kc, const float *vc,
                        int pos0, int S, int n_heads, int kv_mul, int hd, int kv_dim,
                        int max_seq) {
    size_t qdim = (size_t)n_heads * hd;
    #pragma omp parallel
    {
        float *att = (float *)malloc((size_t)max_seq * sizeof(float));
        #pragma omp for schedule(dynamic, 1) collapse(2)
        for (int s = 0; s < S; s++) {
            for (int h = 0; h < n_heads; h++) {
                attn_head(out + (size_t)s * qdim + (size_t)h * hd,
                          q + (size_t)s * qdim + (size_t)h * hd, kc, vc, att, 0,
                          pos0 + s, h / kv_mul, hd, kv_dim);
            }
        }
        free(att);
    }
}

static float bf16_round1(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {       /* inf / nan: truncate, keep nan quiet */
        if (u & 0x007fffffu) u |= 0x00400000u;
        u &= 0xffff0000u;
    } else {
        uint32_t lsb = (u >> 16) & 1u;
        u += 0x7fffu + lsb;
        u &= 0xffff0000u;
    }
    memcpy(&f, &u, 4);
    return f;
}

void orc_bf16_round(float *x, size_t n) {
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) x[i] = bf16_round1(x[i]);
}

static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

uint64_t orc_stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream + 0x51ED2701ULL));
}

/* Uniform in (0,1) with 23 random bits: splitmix64(key + i) seeds one
 * xorshift64* step (qwen3-8b/cpu/main.c:1377-1382); the top 23 bits of the
 * scrambled output, plus one half, scaled by 2^-23 (exact in fp32). */
float orc_u01(uint64_t key, uint64_t i) {
    uint64_t s = splitmix64(key + i);
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    uint32_t r = (uint32_t)((s * 0x2545F4914F6CDD1DULL) >> 41);
    return ((float)r + 0.5f) * (1.0f / 8388608.0f);
}

/* Box-Muller on pairs of stream elements (2j, 2j+1): element 2j gets the
 * cosine branch, 2j+1 the sine branch. */
void orc_randn(float *dst, size_t n, uint64_t key, uint64_t offset) {
    const float two_pi = 6.283185307179586f;
    #pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
        uint64_t e = offset + i;
        uint64_t j = e >> 1;
        float u1 = orc_u01(key, 2 * j);
        float u2 = orc_u01(key, 2 * j + 1);
        float r = sqrtf(-2.0f * logf(u1));
        float a = two_pi * u2;
        dst[i] = (e & 1) ? r * sinf(a) : r * cosf(a);
    }
}

void orc_lse_merge(float *out, float *lse_out, const float *o_parts,
                   const float *lse_parts, int n_parts, int n_heads, int hd) {
    for (int h = 0; h < n_heads; h++) {
        float m = -INFINITY;
        for (int j = 0; j < n_parts; j++) {
            float l = lse_parts[(size_t)j * n_heads + h];
            if (l > m) m = l;
        }
        double den = 0.0;
        for (int i = 0; i < hd; i++) out[(size_t)h * hd + i] = 0.0f;
        double *acc = (double *)calloc((size_t)hd, sizeof(double));
        for (int j = 0; j < n_parts; j++) {
            float l = lse_parts[(size_t)j * n_heads + h];
            if (l == -INFINITY) continue;
            double w = exp2((double)l - (double)m);
            den += w;
            const float *o = o_parts + ((size_t)j * n_heads + h) * hd;
            for (int i = 0; i < hd; i++) acc[i] += w * (double)o[i];
        }
        for (int i = 0; i < hd; i++) out[(size_t)h * hd + i] = (float)(acc[i] / den);
        if (lse_out) lse_out[h] = (float)((double)m + log2(den));
        free(acc);
    }
}

void orc_attn_partial(float *o, float *lse, const float *q, const float *kc,
                      const float *vc, size_t loff, int t0, int t1, int n_heads,
                      int kv_mul, int hd, int kv_dim) {
    const double log2e = 1.4426950408889634;
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; h++) {
        const float *qh = q + (size_t)h * hd;
        int kvh = h / kv_mul;
        float scale = 1.0f / sqrtf((float)hd);
        int n = t1 - t0;
        double *s = (double *)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
        double m = -INFINITY;
        for (int t = t0; t < t1; t++) {
            const float *kt = kc + loff + (size_t)t * kv_dim + (size_t)kvh * hd;
            double acc = 0.0;
            for (int i = 0; i < hd; i++) acc += (double)qh[i] * (double)kt[i];
            s[t - t0] = acc * scale * log2e;
            if (s[t - t0] > m) m = s[t - t0];
        }
        double den = 0.0;
        double *acc = (double *)calloc((size_t)hd, sizeof(double));
        for (int t = t0; t < t1; t++) {
            double p = exp2(s[t - t0] - m);
            den += p;
            const float *vt = vc + loff + (size_t)t * kv_dim + (size_t)kvh * hd;
            for (int i = 0; i < hd; i++) acc[i] += p * (double)vt[i];
        }
        for (int i = 0; i < hd; i++)
            o[(size_t)h * hd + i] = n > 0 ? (float)(acc[i] / den) : 0.0f;
        lse[h] = n > 0 ? (float)(m + log2(den)) : -INFINITY;
        free(acc);
        free(s);
    }
}

/* fp16 -> fp32 by the IEEE 754 binary16 layout: sign, 5-bit exponent (bias
 * 15), 10-bit mantissa; subnormals normalised, inf/NaN kept (the conversion
 * host_f16f32 performs, qwen3-8b/cpu/main.c:437-458). */
static float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int e = (h >> 10) & 31;
    uint32_t m = h & 1023u, bits;
    if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {  /* subnormal: m * 2^-24, shift the leading one to bit 10 */
        int sh = 0;
        while (!(m & 1024u)) { m <<= 1; sh++; }
        bits = sign | ((uint32_t)(127 - 14 - sh) << 23) | ((m & 1023u) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* mm_f16, qwen3-8b/cpu/main.c:1206-1213 (cpu-multicore/main.c:1213-1221
 * adds the OpenMP loop over rows): o[i] = sequential fp32 sum over j of
 * x[j] * w[i][j], w fp16 row-major [d][n]. */
void orc_mm_f16(float *o, const float *x, const uint16_t *w, int n, int d) {
    #pragma omp parallel for schedule(static)
    for (int i = 0; i < d; i++) {
        const uint16_t *row = w + (size_t)i * n;
        float acc = 0.0f;
        for (int j = 0; j < n; j++) acc += x[j] * f16_to_f32(row[j]);
        o[i] = acc;
    }
}

/* rmsnorm, qwen3-8b/cpu/main.c:1168-1173: sequential sum of squares,
 * ss = 1/sqrtf(ss/n + eps), o[i] = x[i] * ss * w[i] (left to right). */
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / n + eps);
    for (int i = 0; i < n; i++) o[i] = x[i] * ss * w[i];
}
