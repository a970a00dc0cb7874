// q3a_gemv.cuh -- the streaming fp16 GEMV engine of the projection kernels
// (q3a_proj.cu), parameterised by the number of consumer warps.
//
// The rows of a projection form one list; CTA c of G takes rows
// [c R / G, (c+1) R / G).  A producer thread streams the range with bulk
// copies into a ring of 32 KB shared-memory stages (whole rows); NW consumer
// warps keep their 16-byte pieces of the input vector in registers (pieces
// t, t + 32 NW, ... of a row), take rows in groups of four with independent
// sums and reduce them with a four-row warp butterfly; a row's sum is the
// per-warp sums added in warp order, so results do not depend on timing.
#pragma once

#include <cuda_fp16.h>

#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {
namespace gemv {

// 12 stages of 16 KB (two rows at width 4096) measured slower: the
// consumers' four-row groups run half empty
constexpr int STAGE_BYTES = 32768;
constexpr int STAGES = 6;

__device__ __forceinline__ float2 h2f2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, sizeof(h));
    return __half22float2(h);
}

// acc += the 8 fp16 weights of w times x[0..7] (fp32 products, fp32 sums).
__device__ __forceinline__ void dot8(float2& acc, uint4 w, const float2 (&x)[4]) {
    acc = __ffma2_rn(h2f2(w.x), x[0], acc);
    acc = __ffma2_rn(h2f2(w.y), x[1], acc);
    acc = __ffma2_rn(h2f2(w.z), x[2], acc);
    acc = __ffma2_rn(h2f2(w.w), x[3], acc);
}

// Sums of four rows over the warp: v[r] is this lane's part of row r.  Two
// exchange steps halve the rows a lane carries (xor 16: rows 0,1 or 2,3;
// xor 8: one row), three more add over the remaining lanes; lane l ends with
// the whole sum of row 2*((l>>4)&1) + ((l>>3)&1).  Fixed order: the same
// inputs give the same bits.
__device__ __forceinline__ float warp_sum4(const float (&v)[4], int lane) {
    const bool hi = lane & 16, b3 = lane & 8;
    const float give0 = hi ? v[0] : v[2], give1 = hi ? v[1] : v[3];
    float keep0 = hi ? v[2] : v[0], keep1 = hi ? v[3] : v[1];
    keep0 += __shfl_xor_sync(FULL, give0, 16);
    keep1 += __shfl_xor_sync(FULL, give1, 16);
    const float give = b3 ? keep0 : keep1;
    float keep = b3 ? keep1 : keep0;
    keep += __shfl_xor_sync(FULL, give, 8);
    keep += __shfl_xor_sync(FULL, keep, 4);
    keep += __shfl_xor_sync(FULL, keep, 2);
    keep += __shfl_xor_sync(FULL, keep, 1);
    return keep;
}

// First row of CTA c's range of R rows over G CTAs.
__device__ __forceinline__ int range_row0(int c, int R, int G) {
    return (int)(((long long)c * R) / G);
}

// ---- row sources: copy(row0, n, dst, bar, pol) issues the bulk copies of
// list rows [row0, row0 + n) into dst, row after row, completion on bar.

// q/k/v rows of KV heads [kv0, kv0 + nkv): the held q rows of wq, then the
// held k rows of wk, then the held v rows of wv (whole rows, so rows of one
// matrix are contiguous).
struct QkvRows {
    const __half *wq, *wk, *wv;
    int dim, q_rows, k_rows;  // list rows of q, of k (= of v)
    size_t q_off, k_off;      // element offset of the first held row in wq, in wk / wv
    __device__ void copy(int row0, int n, uint8_t* dst, uint64_t* bar, uint64_t pol) const {
        const int row_bytes = dim * 2;
        for (int a = row0; a < row0 + n;) {
            const __half* src;
            int e;
            if (a < q_rows) {
                src = wq + q_off + (size_t)a * dim;
                e = min(row0 + n, q_rows);
            } else if (a < q_rows + k_rows) {
                src = wk + k_off + (size_t)(a - q_rows) * dim;
                e = min(row0 + n, q_rows + k_rows);
            } else {
                src = wv + k_off + (size_t)(a - q_rows - k_rows) * dim;
                e = row0 + n;
            }
            bulk_load(dst + (a - row0) * row_bytes, src, (uint32_t)((e - a) * row_bytes), bar, pol);
            a = e;
        }
    }
};

__device__ __forceinline__ QkvRows qkv_rows(const QkvParams& P) {
    QkvRows rows;
    rows.wq = P.wq;
    rows.wk = P.wk;
    rows.wv = P.wv;
    rows.dim = P.dim;
    rows.q_rows = P.nq * HD;
    rows.k_rows = P.nkv * HD;
    rows.q_off = (size_t)P.kv0 * GQA * HD * P.dim;
    rows.k_off = (size_t)P.kv0 * HD * P.dim;
    return rows;
}

// Columns [col0, col0 + ncols) of the rows of one matrix with ld columns.
struct SliceRows {
    const __half* w;
    int ld, col0, ncols;
    __device__ void copy(int row0, int n, uint8_t* dst, uint64_t* bar, uint64_t pol) const {
        if (ncols == ld) {
            bulk_load(dst, w + (size_t)row0 * ld, (uint32_t)(n * ld * 2), bar, pol);
            return;
        }
        for (int j = 0; j < n; j++)
            bulk_load(dst + j * ncols * 2, w + (size_t)(row0 + j) * ld + col0, (uint32_t)(ncols * 2),
                      bar, pol);
    }
};

// ---- the ring
// full[s]: one producer arrival plus the stage's bytes; empty[s]: one
// arrival per consumer warp.
template <int NW>
__device__ __forceinline__ void ring_init(uint64_t* full, uint64_t* empty) {
    for (int s = 0; s < STAGES; s++) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
}

// Producer thread: stages of SR rows of [r_begin, r_end) through the ring
// at ring (STAGES x STAGE_BYTES).  Returns the number of stages issued; with
// `drain` it first waits for its copies in flight to land, else for the
// consumers to have released every stage (the ring's memory is then free).
template <class Rows>
__device__ int ring_produce(uint8_t* ring, uint64_t* full, uint64_t* empty, const Rows& rows,
                            int r_begin, int r_end, int row_bytes, int SR, int* err, bool drain) {
    const uint64_t pol = l2_policy_evict_first();
    const int n_stages = (r_end - r_begin + SR - 1) / SR;
    int issued = 0;
    for (int k = 0; k < n_stages; k++) {
        const int st = k % STAGES;
        if (k >= STAGES && !mbar_wait(&empty[st], (uint32_t)((k / STAGES) - 1) & 1u)) {
            atomicExch(err, DEV_ERR_TIMEOUT);
            break;
        }
        const int row0 = r_begin + k * SR;
        const int n = min(SR, r_end - row0);
        mbar_arrive_expect_tx(&full[st], (uint32_t)(n * row_bytes));
        rows.copy(row0, n, ring + st * STAGE_BYTES, &full[st], pol);
        issued = k + 1;
    }
    for (int k = max(0, issued - STAGES); k < issued; k++) {
        const bool ok = drain ? mbar_wait(&full[k % STAGES], (uint32_t)(k / STAGES) & 1u)
                              : mbar_wait(&empty[k % STAGES], (uint32_t)(k / STAGES) & 1u);
        if (!ok) {
            atomicExch(err, DEV_ERR_TIMEOUT);
            break;
        }
    }
    return issued;
}

// The input slice of consumer thread tid (of NW warps) in registers:
// pieces tid, tid + 32 NW, ... of 8 floats (zeros past n_pieces).
template <int NP, int NW>
__device__ __forceinline__ void load_x(float2 (&xv)[NP][4], const float* x, int n_pieces, int tid) {
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const int p = tid + i * NW * 32;
        if (p < n_pieces) {
            const float4* xs = reinterpret_cast<const float4*>(x + (size_t)p * 8);
            const float4 a = xs[0], b = xs[1];
            xv[i][0] = make_float2(a.x, a.y);
            xv[i][1] = make_float2(a.z, a.w);
            xv[i][2] = make_float2(b.x, b.y);
            xv[i][3] = make_float2(b.z, b.w);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) xv[i][j] = make_float2(0.0f, 0.0f);
        }
    }
}

// Consumers (NW warps): per-warp sums of the range's rows into
// red[row][warp].  With stage_done, each warp also counts each stage done
// in that shared counter (after its sums are in red).
template <int NP, int NW>
__device__ void ring_consume(const uint8_t* ring, uint64_t* full, uint64_t* empty, float* red,
                             int n_rows, int row_bytes, int SR, int n_pieces,
                             const float2 (&xv)[NP][4], int tid, int* err,
                             int* stage_done = nullptr) {
    const int warp = tid >> 5, lane = tid & 31;
    const int n_stages = (n_rows + SR - 1) / SR;
    bool ok = true;
    for (int k = 0; k < n_stages; k++) {
        const int st = k % STAGES;
        if (ok && !mbar_wait(&full[st], (uint32_t)(k / STAGES) & 1u)) {
            ok = false;
            atomicExch(err, DEV_ERR_TIMEOUT);
        }
        const int n = min(SR, n_rows - k * SR);
        if (ok) {
            const uint8_t* base = ring + st * STAGE_BYTES;
            for (int j0 = 0; j0 < n; j0 += 4) {
                float v[4];
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    float2 acc = make_float2(0.0f, 0.0f);
                    if (j0 + r < n) {
                        const uint8_t* row = base + (j0 + r) * row_bytes;
#pragma unroll
                        for (int i = 0; i < NP; i++) {
                            const int p = tid + i * NW * 32;
                            if (p < n_pieces)
                                dot8(acc, *reinterpret_cast<const uint4*>(row + p * 16), xv[i]);
                        }
                    }
                    v[r] = acc.x + acc.y;
                }
                const float s = warp_sum4(v, lane);
                const int r = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
                if ((lane & 7) == 0 && j0 + r < n) red[(k * SR + j0 + r) * NW + warp] = s;
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty[st]);
            if (stage_done) {  // this warp's sums of stage k are in red
                __threadfence_block();
                atomicAdd(&stage_done[k], 1);
            }
        }
    }
}

template <int NW>
__device__ __forceinline__ float row_sum(const float* red, int t) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) s += red[t * NW + w];
    return s;
}

// ---- the q/k/v projection's steps around the engine

// The layer's input RMSNorm on the registers, x * (1/sqrtf(mean(x^2) + eps))
// * w (rmsnorm, qwen3-8b/cpu/main.c:1168-1173): every CTA normalises the
// whole input for itself.  wred: NW floats of shared memory; all NW warps
// meet on named barrier bar_id.
template <int NP, int NW>
__device__ __forceinline__ void input_rmsnorm(float2 (&xv)[NP][4], const float* norm_w, int dim,
                                              float eps, int n_pieces, int tid, float* wred,
                                              int bar_id) {
    const int warp = tid >> 5, lane = tid & 31;
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) ss += xv[i][j].x * xv[i][j].x + xv[i][j].y * xv[i][j].y;
    ss = warp_sum(ss);
    if (lane == 0) wred[warp] = ss;
    named_bar_sync(bar_id, NW * 32);
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; w++) tot += wred[w];
    const float sc = 1.0f / sqrtf(tot / (float)dim + eps);
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const int p = tid + i * NW * 32;
        if (p < n_pieces) {
            const float4* ws = reinterpret_cast<const float4*>(norm_w + (size_t)p * 8);
            const float4 a = ws[0], b = ws[1];
            const float wv8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                xv[i][j].x = __fmul_rn(__fmul_rn(xv[i][j].x, sc), wv8[2 * j]);
                xv[i][j].y = __fmul_rn(__fmul_rn(xv[i][j].y, sc), wv8[2 * j + 1]);
            }
        }
    }
}

// One thread: adds this range's rows to the tickets of the heads it touches
// (at most two: a range is shorter than a head) and lists in fin[] the heads
// whose 128 rows are now all summed (this CTA finishes them); returns how
// many.  The acq_rel atomics release this CTA's row sums and acquire the
// other contributors'.
__device__ __forceinline__ int head_tickets(int* ticket, int r_begin, int r_end, volatile int* fin) {
    int nf = 0;
    for (int h = r_begin / HD; h * HD < r_end; h++) {
        const int cnt = min(r_end, (h + 1) * HD) - max(r_begin, h * HD);
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
                     : "=r"(old)
                     : "l"(ticket + h), "r"(cnt)
                     : "memory");
        if (old + cnt == HD) {
            ticket[h] = 0;
            fin[nf++] = h;
        }
    }
    return nf;
}

// One warp finishes list head h (the held q heads, then k, then v) from its
// 128 row sums: q heads normalised and rotated into q_out; k heads
// normalised, rotated, written to k_out and appended at pos; v heads written
// to v_out and appended (rmsnorm_head_inplace, apply_rope and the cache
// write, qwen3-8b/cpu/main.c:1319-1329).
template <typename KV>
__device__ __forceinline__ void finish_head(const QkvParams& P, int h, int lane) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(P.part + (size_t)h * HD) + lane);
    const float2 fr = reinterpret_cast<const float2*>(P.inv_freq)[lane];
    const int pos = P.pos, nq = P.nq, nkv = P.nkv;
    if (h < nq) {
        const float4 w = reinterpret_cast<const float4*>(P.q_norm_w)[lane];
        float* qo = P.q_out + (size_t)(P.kv0 * GQA + h) * HD;
        reinterpret_cast<float4*>(qo)[lane] = norm_rope_lane(v, w, P.eps, pos, fr);
        return;
    }
    const bool is_k = h < nq + nkv;
    const int kvh = is_k ? h - nq : h - nq - nkv;  // local kv head
    float4 out = v;
    if (is_k) {
        const float4 w = reinterpret_cast<const float4*>(P.k_norm_w)[lane];
        out = norm_rope_lane(v, w, P.eps, pos, fr);
        if (P.k_out) reinterpret_cast<float4*>(P.k_out + (size_t)(P.kv0 + kvh) * HD)[lane] = out;
    } else if (P.v_out) {
        reinterpret_cast<float4*>(P.v_out + (size_t)(P.kv0 + kvh) * HD)[lane] = out;
    }
    const long long phys = (long long)P.slot * P.pages_per_seq + pos / P.page_tokens;
    const long long row = (((long long)P.layer * nkv + kvh) * P.n_pages + phys) * P.page_tokens +
                          pos % P.page_tokens;
    KV* cache = reinterpret_cast<KV*>(is_k ? P.kcache : P.vcache);
    store4<KV>(cache + kv_index<KV>(row, 4 * lane), out);
}

}  // namespace gemv
}  // namespace q3a
