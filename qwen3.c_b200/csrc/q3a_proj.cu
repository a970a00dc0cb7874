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
#include "q3a_gemv.cuh"
#include "q3a_internal.h"

namespace q3a {

namespace proj {
constexpr int STAGE_BYTES = gemv::STAGE_BYTES;
constexpr int STAGES = gemv::STAGES;
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

using namespace gemv;
constexpr int NW = proj::CWARPS;

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

    if (tid == 0) ring_init<NW>(full, empty);
    __syncthreads();

    if (warp == proj::CWARPS) {
        if (lane == 0)
            ring_produce(smem, full, empty, qkv_rows(P), r_begin, r_end, row_bytes, SR, P.err, true);
        return;
    }

    // ================================================ consumers (16 warps)
    griddep_wait();  // x (written by the previous kernel) is visible
    // Dependents (the decode of this layer) may launch once this kernel has
    // passed its own wait: every kernel before it has then completed.
    if (tid == 0) griddep_launch_dependents();
    const int n_pieces = dim >> 3;  // 16-byte pieces per row
    float2 xv[NP][4];
    load_x<NP, NW>(xv, P.x, n_pieces, tid);
    if (P.norm_w) input_rmsnorm<NP, NW>(xv, P.norm_w, dim, P.eps, n_pieces, tid, wred, 1);
    ring_consume<NP, NW>(smem, full, empty, red, n_rows, row_bytes, SR, n_pieces, xv, tid, P.err);
    named_bar_sync(1, proj::NCONS);
    for (int t = tid; t < n_rows; t += proj::NCONS) P.part[r_begin + t] = row_sum<NW>(red, t);
    __threadfence();
    named_bar_sync(1, proj::NCONS);
    if (tid == 0) misc[3] = head_tickets(P.ticket, r_begin, r_end, misc);
    named_bar_sync(1, proj::NCONS);
    if (warp < misc[3]) finish_head<KV>(P, misc[warp], lane);
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

    if (tid == 0) ring_init<NW>(full, empty);
    for (int k = tid; k < proj::MAX_STAGES_T; k += blockDim.x) cnt[k] = 0;
    __syncthreads();

    if (warp == proj::CWARPS) {
        if (lane == 0) {
            SliceRows rows;
            rows.w = P.w;
            rows.ld = P.ld;
            rows.col0 = P.col0;
            rows.ncols = P.ncols;
            ring_produce(smem, full, empty, rows, r_begin, r_end, row_bytes, SR, P.err, true);
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
                const float s = row_sum<NW>(red, t);
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
    load_x<NP, NW>(xv, P.xb + P.col0, n_pieces, tid);
    ring_consume<NP, NW>(smem, full, empty, red, n_rows, row_bytes, SR, n_pieces, xv, tid, P.err,
                         cnt);
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
