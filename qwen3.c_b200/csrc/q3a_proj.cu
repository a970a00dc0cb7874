// q3a_proj.cu -- the fp16 projections on both sides of the attention block:
// the q/k/v projections that produce its inputs (with the layer's input
// RMSNorm before them and the block's QK-RMSNorm, RoPE and KV append after
// them), and the wo projection that consumes its output xb, with the
// residual add (and, over KV-head shards, the sum of the ranks' partial
// projections exchanged over NVLink peer memory inside the same kernel).
//
// Replaces, per layer of forward() (qwen3-8b/cpu/main.c:1313-1356; HIP
// forward_gpu, qwen3-8b/gpu/main.c:2095-2135):
//   rmsnorm(s->xb, s->x, w->norm_att[l], ...)                     main.c:1313
//   mm(s->q/k/v, s->xb, w->wq/wk/wv[l], ...)  (mm_f16)            main.c:1315-1317
//   rmsnorm_head_inplace / apply_rope / kv cache write            main.c:1319-1329
//   mm(s->xb2, s->xb, w->wo[l], ...); x += xb2                    main.c:1355-1356
// with fp16 weights [rows][cols] row-major and fp32 sums (HIP:
// mm_f16_gemv_kernel, qwen3-8b/gpu/main.c:1495-1519; vec_add_kernel :1435).
//
// Both are GEMVs of one token: 50 MB (q/k/v) and 34 MB (wo) of fp16 weights
// per Qwen3-8B layer against 16 KB of input, bound by the HBM stream of the
// weights.  One engine serves both:
//  * the rows of the projection form one list; CTA c of G (one per SM) takes
//    rows [c R / G, (c+1) R / G) -- 41 or 42 q/k/v rows, 28 wo rows;
//  * a producer thread streams the range into a ring of 32 KB shared-memory
//    stages with bulk copies, starting before the dependency wait: weights
//    are not written by the kernel before, only the input vector is;
//  * 512 consumer threads keep their slice of the input in registers (the
//    row's 16-byte pieces go round-robin over the threads, so a warp reads
//    512 contiguous bytes of shared memory per load); rows go in groups of
//    four with independent sums; a row's products are summed per thread,
//    over the warp (a four-row butterfly), then over the 16 warps in warp
//    order, so the result does not depend on timing.
// A context holding KV heads [kv0, kv0 + nkv) projects only their q/k/v rows
// (column-parallel) and multiplies only their xb columns by wo (row-parallel).
#include <cuda_fp16.h>

#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {

namespace proj {
constexpr int STAGE_BYTES = 32768;
constexpr int STAGES = 6;
constexpr int CWARPS = 16;                      // consumer warps
constexpr int NCONS = CWARPS * 32;
constexpr int NTHREADS = NCONS + 32;            // + the producer warp
constexpr int OFF_BAR = STAGES * STAGE_BYTES;   // full[STAGES], empty[STAGES]
constexpr int OFF_MISC = OFF_BAR + 2 * STAGES * 8;  // 16 ints
constexpr int OFF_WRED = OFF_MISC + 64;         // [CWARPS] floats: block reductions
constexpr int MAX_STAGES_T = 64;                // stages of one CTA's range, at most (wo)
constexpr int OFF_CNT = OFF_WRED + 64;          // [MAX_STAGES_T] warps done per stage (wo)
constexpr int OFF_RED = OFF_CNT + MAX_STAGES_T * 4;  // [rows of the range][CWARPS] warp sums
constexpr int WO_THREADS = NTHREADS + 32;       // wo: + a sender warp
}  // namespace proj

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

// ---------------------------------------------------------------- engine
// The rows of a projection as bulk copies: copy(row0, n, dst, bar, pol)
// issues the copies of list rows [row0, row0 + n) into dst, row after row,
// each row_bytes long, completion counted on bar.

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

__device__ __forceinline__ void ring_init(uint64_t* full, uint64_t* empty) {
    for (int s = 0; s < proj::STAGES; s++) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], proj::CWARPS);
    }
    fence_mbar_init();
}

// Producer thread: stages of SR rows of [r_begin, r_end) through the ring;
// waits, before it returns, for its copies in flight to land.
template <class Rows>
__device__ void ring_produce(uint8_t* smem, uint64_t* full, uint64_t* empty, const Rows& rows,
                             int r_begin, int r_end, int row_bytes, int SR, int* err) {
    const uint64_t pol = l2_policy_evict_first();
    const int n_stages = (r_end - r_begin + SR - 1) / SR;
    int issued = 0;
    for (int k = 0; k < n_stages; k++) {
        const int st = k % proj::STAGES;
        if (k >= proj::STAGES && !mbar_wait(&empty[st], (uint32_t)((k / proj::STAGES) - 1) & 1u)) {
            atomicExch(err, DEV_ERR_TIMEOUT);
            break;
        }
        const int row0 = r_begin + k * SR;
        const int n = min(SR, r_end - row0);
        mbar_arrive_expect_tx(&full[st], (uint32_t)(n * row_bytes));
        rows.copy(row0, n, smem + st * proj::STAGE_BYTES, &full[st], pol);
        issued = k + 1;
    }
    for (int k = max(0, issued - proj::STAGES); k < issued; k++)
        if (!mbar_wait(&full[k % proj::STAGES], (uint32_t)(k / proj::STAGES) & 1u)) break;
}

// The input slice of consumer thread tid in registers: pieces tid, tid + 512,
// ... of 8 floats (zeros past n_pieces).
template <int NP>
__device__ __forceinline__ void load_x(float2 (&xv)[NP][4], const float* x, int n_pieces, int tid) {
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const int p = tid + i * proj::NCONS;
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

// Consumers: per-warp sums of the range's rows into red[row][warp]; then
// (after the consumer barrier) row t's sum is red[t][0] + ... + red[t][15].
template <int NP>
__device__ void ring_consume(const uint8_t* smem, uint64_t* full, uint64_t* empty, float* red,
                             int n_rows, int row_bytes, int SR, int n_pieces,
                             const float2 (&xv)[NP][4], int tid, int* err,
                             int* stage_done = nullptr) {
    const int warp = tid >> 5, lane = tid & 31;
    const int n_stages = (n_rows + SR - 1) / SR;
    bool ok = true;
    for (int k = 0; k < n_stages; k++) {
        const int st = k % proj::STAGES;
        if (ok && !mbar_wait(&full[st], (uint32_t)(k / proj::STAGES) & 1u)) {
            ok = false;
            atomicExch(err, DEV_ERR_TIMEOUT);
        }
        const int n = min(SR, n_rows - k * SR);
        if (ok) {
            const uint8_t* base = smem + st * proj::STAGE_BYTES;
            for (int j0 = 0; j0 < n; j0 += 4) {
                float v[4];
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    float2 acc = make_float2(0.0f, 0.0f);
                    if (j0 + r < n) {
                        const uint8_t* row = base + (j0 + r) * row_bytes;
#pragma unroll
                        for (int i = 0; i < NP; i++) {
                            const int p = tid + i * proj::NCONS;
                            if (p < n_pieces)
                                dot8(acc, *reinterpret_cast<const uint4*>(row + p * 16), xv[i]);
                        }
                    }
                    v[r] = acc.x + acc.y;
                }
                const float s = warp_sum4(v, lane);
                const int r = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
                if ((lane & 7) == 0 && j0 + r < n) red[(k * SR + j0 + r) * proj::CWARPS + warp] = s;
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

__device__ __forceinline__ float row_sum(const float* red, int t) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < proj::CWARPS; w++) s += red[t * proj::CWARPS + w];
    return s;
}

// ---------------------------------------------------------------- q/k/v
// NP: 16-byte pieces of a row per consumer thread (dim <= NP * 4096).
template <typename KV, int NP>
__global__ void __launch_bounds__(proj::NTHREADS, 1) qkv_kernel(const __grid_constant__ QkvParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + proj::OFF_BAR);
    uint64_t* empty = full + proj::STAGES;
    volatile int* misc = reinterpret_cast<volatile int*>(smem + proj::OFF_MISC);
    float* wred = reinterpret_cast<float*>(smem + proj::OFF_WRED);
    float* red = reinterpret_cast<float*>(smem + proj::OFF_RED);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int R = P.rows_total;
    const int r_begin = range_row0(c, R, G), r_end = range_row0(c + 1, R, G);
    const int n_rows = r_end - r_begin;
    const int dim = P.dim;
    const int row_bytes = dim * 2;
    const int SR = proj::STAGE_BYTES / row_bytes;  // rows per stage (>= 1)
    const int nq = P.nq, nkv = P.nkv;               // held heads

    if (tid == 0) ring_init(full, empty);
    __syncthreads();

    if (warp == proj::CWARPS) {
        if (lane == 0) {
            QkvRows rows;
            rows.wq = P.wq;
            rows.wk = P.wk;
            rows.wv = P.wv;
            rows.dim = dim;
            rows.q_rows = nq * HD;
            rows.k_rows = nkv * HD;
            rows.q_off = (size_t)P.kv0 * GQA * HD * dim;
            rows.k_off = (size_t)P.kv0 * HD * dim;
            ring_produce(smem, full, empty, rows, r_begin, r_end, row_bytes, SR, P.err);
        }
        return;
    }

    // ================================================ consumers (16 warps)
    griddep_wait();  // x (written by the previous kernel) is visible
    // Dependents (the decode of this layer) may launch once this kernel has
    // passed its own wait: every kernel before it has then completed.
    if (tid == 0) griddep_launch_dependents();
    const int n_pieces = dim >> 3;  // 16-byte pieces per row
    float2 xv[NP][4];
    load_x<NP>(xv, P.x, n_pieces, tid);
    if (P.norm_w) {
        // the layer's input RMSNorm, x * (1/sqrtf(mean(x^2) + eps)) * w
        // (rmsnorm, qwen3-8b/cpu/main.c:1168-1173); every CTA normalises
        // the whole input for itself
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < NP; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) ss += xv[i][j].x * xv[i][j].x + xv[i][j].y * xv[i][j].y;
        ss = warp_sum(ss);
        if (lane == 0) wred[warp] = ss;
        named_bar_sync(1, proj::NCONS);
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < proj::CWARPS; w++) tot += wred[w];
        const float sc = 1.0f / sqrtf(tot / (float)dim + P.eps);
#pragma unroll
        for (int i = 0; i < NP; i++) {
            const int p = tid + i * proj::NCONS;
            if (p < n_pieces) {
                const float4* ws = reinterpret_cast<const float4*>(P.norm_w + (size_t)p * 8);
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
    ring_consume<NP>(smem, full, empty, red, n_rows, row_bytes, SR, n_pieces, xv, tid, P.err);
    named_bar_sync(1, proj::NCONS);
    for (int t = tid; t < n_rows; t += proj::NCONS) P.part[r_begin + t] = row_sum(red, t);
    __threadfence();
    named_bar_sync(1, proj::NCONS);
    // tickets of the heads this range touches (at most two: a range is
    // shorter than a head); the CTA completing a head finishes it
    if (tid == 0) {
        int nf = 0;
        for (int h = r_begin / HD; h * HD < r_end; h++) {
            const int cnt = min(r_end, (h + 1) * HD) - max(r_begin, h * HD);
            int old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
                         : "=r"(old)
                         : "l"(P.ticket + h), "r"(cnt)
                         : "memory");
            if (old + cnt == HD) {
                P.ticket[h] = 0;
                misc[nf++] = h;
            }
        }
        misc[3] = nf;
    }
    named_bar_sync(1, proj::NCONS);
    if (warp >= misc[3]) return;
    const int h = misc[warp];  // list head: held q heads, then k, then v
    // lane: dimensions 4 lane .. 4 lane + 3 of head h
    const float4 v = __ldcg(reinterpret_cast<const float4*>(P.part + (size_t)h * HD) + lane);
    const float2 fr = reinterpret_cast<const float2*>(P.inv_freq)[lane];
    const int pos = P.pos;
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

// ---------------------------------------------------------------- wo
// A sender warp takes each stage's rows as soon as the 16 consumer warps
// have summed them: it adds the warp sums and either adds the row into x
// (one rank) or stores it, tagged with the call number, into its row of
// every rank's exchange buffer (several ranks), so the exchange overlaps the
// weight stream; then it adds the ranks' partials in rank order.
template <int NP>
__global__ void __launch_bounds__(proj::WO_THREADS, 1) wo_kernel(const __grid_constant__ WoParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + proj::OFF_BAR);
    uint64_t* empty = full + proj::STAGES;
    int* cnt = reinterpret_cast<int*>(smem + proj::OFF_CNT);
    float* red = reinterpret_cast<float*>(smem + proj::OFF_RED);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int r_begin = range_row0(c, P.rows, G), r_end = range_row0(c + 1, P.rows, G);
    const int n_rows = r_end - r_begin;
    const int row_bytes = P.ncols * 2;
    const int SR = proj::STAGE_BYTES / row_bytes;
    const int n_stages = (n_rows + SR - 1) / SR;

    if (tid == 0) ring_init(full, empty);
    for (int k = tid; k < proj::MAX_STAGES_T; k += blockDim.x) cnt[k] = 0;
    __syncthreads();

    if (warp == proj::CWARPS) {
        if (lane == 0) {
            SliceRows rows;
            rows.w = P.w;
            rows.ld = P.ld;
            rows.col0 = P.col0;
            rows.ncols = P.ncols;
            ring_produce(smem, full, empty, rows, r_begin, r_end, row_bytes, SR, P.err);
        }
        return;
    }
    if (warp == proj::CWARPS + 1) {
        // ============================================ sender
        griddep_wait();  // x may be read by the kernel before: write it after
        const bool multi = P.world > 1;
        unsigned tag = 0;
        if (multi) tag = __shfl_sync(FULL, lane == 0 ? P.epoch[c] + 1u : 0u, 0);
        const size_t half = (size_t)(tag & 1u) * P.world * WO_MAX_ROWS;
        bool ok = true;
        for (int k = 0; k < n_stages && ok; k++) {
            // the consumers' sums of stage k (bounded wait; they count a
            // stage even when their own wait gave up)
            const long long t0 = clock64();
            while (*reinterpret_cast<volatile int*>(&cnt[k]) < proj::CWARPS) {
                if (clock64() - t0 > P.wait_limit) {
                    ok = false;
                    break;
                }
            }
            if (!ok) break;
            __threadfence_block();
            const int n = min(SR, n_rows - k * SR);
            for (int j = lane; j < n; j += 32) {
                const int t = k * SR + j, r = r_begin + t;
                const float s = row_sum(red, t);
                if (!multi) {
                    P.x[r] = P.x[r] + s;  // x += xb2 (qwen3-8b/cpu/main.c:1356)
                } else {
                    for (int q = 0; q < P.world; q++)
                        st_word_sys(P.recv[q] + half + (size_t)P.rank * WO_MAX_ROWS + r, s, tag);
                }
            }
        }
        if (!ok) {
            if (lane == 0) atomicExch(P.err, DEV_ERR_TIMEOUT);
            return;
        }
        if (!multi) return;
        // every rank's partial of each row, added in rank order
        for (int t = lane; t < n_rows; t += 32) {
            const int r = r_begin + t;
            float tot = 0.0f;
            bool got = true;
            for (int q = 0; q < P.world && got; q++) {
                float v;
                got = wait_word(P.recv[P.rank] + half + (size_t)q * WO_MAX_ROWS + r, tag, v,
                                P.wait_limit);
                tot += v;
            }
            if (got)
                P.x[r] = P.x[r] + tot;
            else
                atomicExch(P.err, DEV_ERR_TIMEOUT);
        }
        __syncwarp();
        if (lane == 0) P.epoch[c] = tag;
        return;
    }

    // ================================================ consumers (16 warps)
    griddep_wait();  // xb (the decode's output) is visible
    if (tid == 0) griddep_launch_dependents();
    const int n_pieces = P.ncols >> 3;
    float2 xv[NP][4];
    load_x<NP>(xv, P.xb + P.col0, n_pieces, tid);
    ring_consume<NP>(smem, full, empty, red, n_rows, row_bytes, SR, n_pieces, xv, tid, P.err, cnt);
}

// ---------------------------------------------------------------- launch
int proj_smem_bytes(int rows, int n_ctas) {
    const int max_rows = (rows + n_ctas - 1) / n_ctas + 1;
    return proj::OFF_RED + max_rows * proj::CWARPS * 4;
}

static cudaError_t launch_pdl(const void* fn, int n_ctas, int threads, int smem, cudaStream_t st,
                              void* arg) {
    cudaError_t e = ensure_smem_attr(fn, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_ctas);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {arg};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_qkv(const QkvParams& p, bool bf16, int n_ctas, cudaStream_t st) {
    // pieces per thread: 512 consumers cover 4096 columns per round
    const bool two = p.dim > 4096;
    const void* fn =
        bf16 ? (two ? reinterpret_cast<const void*>(qkv_kernel<__nv_bfloat16, 2>)
                    : reinterpret_cast<const void*>(qkv_kernel<__nv_bfloat16, 1>))
             : (two ? reinterpret_cast<const void*>(qkv_kernel<float, 2>)
                    : reinterpret_cast<const void*>(qkv_kernel<float, 1>));
    return launch_pdl(fn, n_ctas, proj::NTHREADS, proj_smem_bytes(p.rows_total, n_ctas), st,
                      const_cast<QkvParams*>(&p));
}

cudaError_t launch_wo(const WoParams& p, int n_ctas, cudaStream_t st) {
    const void* fn = p.ncols > 4096 ? reinterpret_cast<const void*>(wo_kernel<2>)
                                    : reinterpret_cast<const void*>(wo_kernel<1>);
    return launch_pdl(fn, n_ctas, proj::WO_THREADS, proj_smem_bytes(p.rows, n_ctas), st,
                      const_cast<WoParams*>(&p));
}

}  // namespace q3a
