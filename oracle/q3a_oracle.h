/*
 * q3a_oracle.h -- CPU restatement of the Qwen3.c GQA attention block.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests, the smoke check and the bench's CPU-baseline leg may load it.
 * The product library (libq3attn.so) never links or calls it.
 *
 * Every function restates one piece of the reference (thamada/Qwen3.c) with
 * the same operation order, so that, compiled with the reference's own flags
 * (gcc -O3 -std=c11, no fast-math), its results are bit-identical to the
 * reference's code compiled from its sources (oracle/_ref).  Parity is pinned
 * against golden vectors produced by that compiled reference code
 * (tests/golden/make_golden.py).
 */
#ifndef Q3A_ORACLE_H
#define Q3A_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* qwen3-8b/cpu/main.c:1175-1183 (OpenMP copy cpu-multicore/main.c:1180-1189) */
void orc_rmsnorm_head(float *vec, const float *w, int n_heads, int hd, float eps);

/* qwen3-8b/cpu/main.c:1282-1295 (OpenMP copy cpu-multicore/main.c:1293-1307) */
void orc_rope(float *vec, int n_heads, int hd, int pos, float theta);
void orc_prep_rows(float *rows, const float *w, int n, int n_heads, int hd, int pos0,
                   float eps, float theta);

/* qwen3-8b/cpu/main.c:1185-1195 */
void orc_softmax(float *x, int n);

/* Decode attention over a position-major cache [layers][max_seq][kv_dim];
 * argument list of launch_attn (qwen3-8b/xdna2/main.c:2724-2727), loop body of
 * qwen3-8b/cpu-multicore/main.c:1346-1369 (division by the softmax sum as in
 * cpu/main.c:1194). */
void orc_attn_decode(float *xb, const float *q, const float *kc, const float *vc,
                     float *att, size_t loff, int pos, int n_heads, int kv_mul,
                     int hd, int kv_dim, int max_seq);

/* The whole block of qwen3-8b/cpu/main.c:1319-1353 for one layer:
 * QK-norm (q and k in place), RoPE (in place), KV append at pos, attention.
 * kc/vc are position-major [n_layers][max_seq][n_kv*hd]. */
void orc_attn_block(float *xb, float *q, float *k, const float *v,
                    const float *q_norm_w, const float *k_norm_w,
                    float *kc, float *vc, float *att, int layer, int pos,
                    int n_heads, int n_kv, int hd, int max_seq,
                    float eps, float theta);

/* Causal prefill as the reference defines it (qwen3-8b/cpu/main.c:1481-1499:
 * one decode call per prompt position): q is [S][n_heads*hd] ALREADY normed
 * and rotated, kc/vc position-major [max_seq][kv_dim] holding positions
 * 0..pos0+S-1; out[s] = attention of q[s] over cache[0..pos0+s]. */
void orc_prefill_causal(float *out, const float *q, const float *kc, const float *vc,
                        int pos0, int S, int n_heads, int kv_mul, int hd, int kv_dim,
                        int max_seq);

/* Round-to-nearest-even float -> bf16 -> float, in place (the value the bf16
 * cache holds). */
void orc_bf16_round(float *x, size_t n);

/* Seeded N(0,1) generator.  Uniforms come from the xorshift64* output step of
 * rng_f32 (qwen3-8b/cpu/main.c:1377-1382) applied to a splitmix64-hashed
 * counter, so element i of a stream is computable on its own (the CUDA
 * generator uses the same integer stream); Box-Muller turns pairs into
 * normals.  stream_key() derives one stream per (seed, stream id). */
uint64_t orc_stream_key(uint64_t seed, uint64_t stream);
float orc_u01(uint64_t key, uint64_t i);
void orc_randn(float *dst, size_t n, uint64_t key, uint64_t offset);

/* Log-sum-exp merge of per-chunk partial results (the split-KV and
 * sequence-shard combine):  o[h] = sum_j w_j o_j[h] / sum_j w_j with
 * w_j = 2^(lse_j[h] - max_j lse_j[h]); lse in log2 units.  o_parts is
 * [n_parts][n_heads][hd], lse_parts [n_parts][n_heads]. */
void orc_lse_merge(float *out, float *lse_out, const float *o_parts,
                   const float *lse_parts, int n_parts, int n_heads, int hd);

/* Partial attention of one sequence chunk [t0, t1) of a position-major cache:
 * o = softmax-weighted mean over the chunk (normalised within the chunk) and
 * lse = log2(sum_t 2^(s_t*log2e)) with s_t = q.k_t/sqrt(hd). */
void orc_attn_partial(float *o, float *lse, const float *q, const float *kc,
                      const float *vc, size_t loff, int t0, int t1, int n_heads,
                      int kv_mul, int hd, int kv_dim);

/* mm_f16 (qwen3-8b/cpu/main.c:1206-1213): o[i] = sum_j x[j] * w[i][j], fp16
 * weights [d][n] row-major, one sequential fp32 sum per row. */
void orc_mm_f16(float *o, const float *x, const uint16_t *w, int n, int d);

/* rmsnorm (qwen3-8b/cpu/main.c:1168-1173): the layer input's RMSNorm, one
 * sequential sum of squares. */
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps);

#ifdef __cplusplus
}
#endif
#endif
