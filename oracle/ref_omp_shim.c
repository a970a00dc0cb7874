/*
 * ref_omp_shim.c -- exposes the reference's own CPU functions from
 * qwen3-8b/cpu-multicore/main.c (included from the reference tree at build
 * time, never copied) for the oracle pin and the CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/.
 * The reference's main() is renamed so that the file links as a library.
 */
#define main q3ref_omp_program_main
#include "qwen3-8b/cpu-multicore/main.c"
#undef main

/* rmsnorm_head_inplace, qwen3-8b/cpu-multicore/main.c:1180-1189 */
void q3ref_rmsnorm_head(float *vec, const float *w, int n_heads, int hd, float eps) {
    rmsnorm_head_inplace(vec, w, n_heads, hd, eps);
}

/* apply_rope, qwen3-8b/cpu-multicore/main.c:1293-1307 */
void q3ref_rope(float *vec, int n_heads, int hd, int pos, float theta) {
    apply_rope(vec, n_heads, hd, pos, theta);
}

/* softmax, qwen3-8b/cpu-multicore/main.c:1191-1201 */
void q3ref_softmax(float *x, int n) { softmax(x, n); }

/* The attention loop of forward() (qwen3-8b/cpu-multicore/main.c:1346-1369)
 * is inline and cannot be called; this wrapper repeats its three loops
 * around the reference's own compiled softmax() so that golden vectors carry
 * the cpu-multicore normalisation (divide by the sum), which differs from
 * launch_attn's multiply-by-reciprocal (qwen3-8b/xdna2/main.c:2712-2722). */
void q3ref_attn_mc(float *xb, const float *q, const float *kc, const float *vc,
                   float *att, size_t loff, int pos, int n_heads, int kv_mul,
                   int hd, int kv_dim, int max_seq) {
    #pragma omp parallel for schedule(static)
    for (int h = 0; h < n_heads; h++) {
        const float *qh = q + h * hd;
        int kvh = h / kv_mul;
        float *att_h = att + (size_t)h * max_seq;
        float scale = 1.0f / sqrtf((float)hd);
        for (int t = 0; t <= pos; t++) {
            const float *kt = kc + loff + (size_t)t * kv_dim + kvh * hd;
            float score = 0.0f;
            for (int i = 0; i < hd; i++) score += qh[i] * kt[i];
            att_h[t] = score * scale;
        }
        softmax(att_h, pos + 1);
        float *oh = xb + h * hd;
        memset(oh, 0, hd * sizeof(float));
        for (int t = 0; t <= pos; t++) {
            float a = att_h[t];
            const float *vt = vc + loff + (size_t)t * kv_dim + kvh * hd;
            for (int i = 0; i < hd; i++) oh[i] += a * vt[i];
        }
    }
}

/* mm_f16, qwen3-8b/cpu-multicore/main.c:1213-1221: the fp16 GEMV of the
 * q/k/v projections (called through mm() at the forward pass's
 * projections). */
void q3ref_mm_f16(float *o, const float *x, const uint16_t *w, int n, int d) {
    mm_f16(o, x, w, n, d);
}

/* rmsnorm, qwen3-8b/cpu-multicore/main.c:1171-1178, run on one OpenMP
 * thread: its sum-of-squares reduction then adds in index order, the order
 * of the single-core build (qwen3-8b/cpu/main.c:1168-1173). */
void q3ref_rmsnorm(float *o, const float *x, const float *w, int n, float eps) {
    int saved = omp_get_max_threads();
    omp_set_num_threads(1);
    rmsnorm(o, x, w, n, eps);
    omp_set_num_threads(saved);
}
