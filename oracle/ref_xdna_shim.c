/*
 * ref_xdna_shim.c -- exposes launch_attn and its helpers, the one factored
 * attention function of the reference (qwen3-8b/xdna2/main.c:2658-2757,
 * OpenMP over heads), included from the reference tree at build time.
 *
 * TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/.
 */
#define main q3ref_xdna_program_main
#include "qwen3-8b/xdna2/main.c"
#undef main

/* launch_attn, qwen3-8b/xdna2/main.c:2724-2757 */
void q3ref_launch_attn(float *xb, const float *q, const float *kc, const float *vc,
                       float *att, size_t loff, int pos, int n_heads, int kv_mul,
                       int hd, int kv_dim, int max_seq) {
    launch_attn(xb, q, kc, vc, att, loff, pos, n_heads, kv_mul, hd, kv_dim, max_seq);
}

/* launch_rmsnorm_head, qwen3-8b/xdna2/main.c:2658-2669 */
void q3ref_launch_rmsnorm_head(float *vec, const float *w, int n_heads, int hd, float eps) {
    launch_rmsnorm_head(vec, w, n_heads, hd, eps);
}

/* launch_rope, qwen3-8b/xdna2/main.c:2671-2686 */
void q3ref_launch_rope(float *vec, int n_heads, int hd, int pos, float theta) {
    launch_rope(vec, n_heads, hd, pos, theta);
}

/* launch_kv_write, qwen3-8b/xdna2/main.c:2688-2692 */
void q3ref_launch_kv_write(const float *k, const float *v, float *kc_pos, float *vc_pos,
                           int kv_dim) {
    launch_kv_write(k, v, kc_pos, vc_pos, kv_dim);
}
