// q3a_qkv.cu -- the q/k/v projections that produce the attention block's
// inputs, fused with the block's QK-RMSNorm, RoPE and KV append.
//
// Replaces mm(s->q/k/v, s->xb, w->wq/wk/wv[l], ...) (qwen3-8b/cpu/main.c:
// 1315-1317; HIP mm_f16_gemv_kernel, qwen3-8b/gpu/main.c:1495-1519) with fp16
// weights [rows][dim] row-major and fp32 accumulation, followed by
// rmsnorm_head_inplace / apply_rope of q and k and the cache write of k and v
// (qwen3-8b/cpu/main.c:1319-1329): the normalised, rotated q goes to memory
// once, ready for the decode kernel, instead of the projection writing raw q
// and k that the block then reads, rewrites and reads again.
//
// One token is a GEMV: 50 MB of fp16 weights per Qwen3-8B layer against 16 KB
// of input, so the kernel is bound by the HBM stream of the weights.
//  * The q, k and v rows form one list of (nq + 2 nkv) x 128 rows (6144 for
//    Qwen3-8B); CTA c of G (one per SM) takes rows [c R / G, (c+1) R / G):
//    41 or 42 rows, 336 KB of contiguous weights (a range crosses at most one
//    matrix boundary).
//  * A producer thread streams the range into a ring of 32 KB shared-memory
//    stages (whole rows, 4 rows at dim 4096) with bulk copies, starting
//    before the dependency wait: the weights are not written by the kernel
//    before it, only x is.
//  * 512 consumer threads keep their slice of x in registers: the row's
//    16-byte pieces go round-robin over the threads (pieces t, t + 512, ...),
//    so each warp reads 512 contiguous bytes of shared memory per load.  Rows
//    go in groups of four with independent sums (the warps are latency-bound
//    otherwise); a row's products are summed per thread, over the warp (a
//    four-row butterfly), then over the 16 warps in warp order (the result
//    does not depend on timing).
//  * Every row sum goes to a row buffer; per head, a ticket counts the rows
//    summed, and the CTA that completes a head's 128 rows finishes it with
//    one warp: q heads normalised and rotated into q_out; k heads normalised,
//    rotated, written to k_out and appended to the cache at pos; v heads
//    written to v_out and appended.
#include <cuda_fp16.h>

#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {

namespace qkv {
constexpr int STAGE_BYTES = 32768;
constexpr int STAGES = 6;
constexpr int CWARPS = 16;                      // consumer warps
constexpr int NCONS = CWARPS * 32;
constexpr int NTHREADS = NCONS + 32;            // + the producer warp
constexpr int OFF_BAR = STAGES * STAGE_BYTES;   // full[STAGES], empty[STAGES]
constexpr int OFF_MISC = OFF_BAR + 2 * STAGES * 8;  // finisher heads
constexpr int OFF_RED = OFF_MISC + 16;          // [rows of the range][CWARPS] warp sums
}  // namespace qkv

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

// First row of CTA c's range.
__device__ __forceinline__ int qkv_row0(int c, int R, int G) {
    return (int)(((long long)c * R) / G);
}

// NP: 16-byte pieces of a row per consumer thread (dim <= NP * 4096).
template <typename KV, int NP>
__global__ void __launch_bounds__(qkv::NTHREADS, 1) qkv_kernel(const __grid_constant__ QkvParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + qkv::OFF_BAR);
    uint64_t* empty = full + qkv::STAGES;
    volatile int* misc = reinterpret_cast<volatile int*>(smem + qkv::OFF_MISC);
    float* red = reinterpret_cast<float*>(smem + qkv::OFF_RED);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int R = P.rows_total;
    const int r_begin = qkv_row0(c, R, G), r_end = qkv_row0(c + 1, R, G);
    const int n_rows = r_end - r_begin;
    const int dim = P.dim;
    const int row_bytes = dim * 2;
    const int SR = qkv::STAGE_BYTES / row_bytes;  // rows per stage (>= 1)
    const int n_stages = (n_rows + SR - 1) / SR;
    const int q_rows = P.nq * HD, k_rows = P.nkv * HD;

    if (tid == 0) {
        for (int s = 0; s < qkv::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], qkv::CWARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == qkv::CWARPS) {
        // ============================================ producer (one thread)
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            bool dead = false;
            int issued = 0;
            for (int k = 0; k < n_stages && !dead; k++) {
                const int st = k % qkv::STAGES;
                if (k >= qkv::STAGES &&
                    !mbar_wait(&empty[st], (uint32_t)((k / qkv::STAGES) - 1) & 1u)) {
                    dead = true;
                    break;
                }
                const int row0 = r_begin + k * SR;
                const int n = min(SR, r_end - row0);
                mbar_arrive_expect_tx(&full[st], (uint32_t)(n * row_bytes));
                uint8_t* dst = smem + st * qkv::STAGE_BYTES;
                for (int a = row0; a < row0 + n;) {
                    // rows [a, e) lie in one matrix
                    const __half* src;
                    int e;
                    if (a < q_rows) {
                        src = P.wq + (size_t)a * dim;
                        e = min(row0 + n, q_rows);
                    } else if (a < q_rows + k_rows) {
                        src = P.wk + (size_t)(a - q_rows) * dim;
                        e = min(row0 + n, q_rows + k_rows);
                    } else {
                        src = P.wv + (size_t)(a - q_rows - k_rows) * dim;
                        e = row0 + n;
                    }
                    bulk_load(dst + (a - row0) * row_bytes, src, (uint32_t)((e - a) * row_bytes),
                              &full[st], pol);
                    a = e;
                }
                issued = k + 1;
            }
            if (dead) atomicExch(P.err, DEV_ERR_TIMEOUT);
            // the copies in flight land before the CTA may exit
            for (int k = max(0, issued - qkv::STAGES); k < issued; k++)
                if (!mbar_wait(&full[k % qkv::STAGES], (uint32_t)(k / qkv::STAGES) & 1u)) break;
        }
        return;
    }

    // ================================================ consumers (8 warps)
    griddep_wait();  // x (written by the previous kernel) is visible
    // Dependents (the decode of this layer) may launch once this kernel has
    // passed its own wait: every kernel before it has then completed.
    if (tid == 0) griddep_launch_dependents();
    const int n_pieces = dim >> 3;  // 16-byte pieces per row
    float2 xv[NP][4];
#pragma unroll
    for (int i = 0; i < NP; i++) {
        const int p = tid + i * qkv::NCONS;
        if (p < n_pieces) {
            const float4* xs = reinterpret_cast<const float4*>(P.x + (size_t)p * 8);
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
    bool ok = true;
    for (int k = 0; k < n_stages; k++) {
        const int st = k % qkv::STAGES;
        if (ok && !mbar_wait(&full[st], (uint32_t)(k / qkv::STAGES) & 1u)) {
            ok = false;
            atomicExch(P.err, DEV_ERR_TIMEOUT);
        }
        const int n = min(SR, n_rows - k * SR);
        if (ok) {
            const uint8_t* base = smem + st * qkv::STAGE_BYTES;
            // rows in groups of four, each with its own accumulator
            for (int j0 = 0; j0 < n; j0 += 4) {
                float v[4];
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    float2 acc = make_float2(0.0f, 0.0f);
                    if (j0 + r < n) {
                        const uint8_t* row = base + (j0 + r) * row_bytes;
#pragma unroll
                        for (int i = 0; i < NP; i++) {
                            const int p = tid + i * qkv::NCONS;
                            if (p < n_pieces)
                                dot8(acc, *reinterpret_cast<const uint4*>(row + p * 16), xv[i]);
                        }
                    }
                    v[r] = acc.x + acc.y;
                }
                const float s = warp_sum4(v, lane);
                const int r = ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
                if ((lane & 7) == 0 && j0 + r < n) red[(k * SR + j0 + r) * qkv::CWARPS + warp] = s;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    named_bar_sync(1, qkv::NCONS);
    // row sums (warps in order) into the row buffer
    for (int t = tid; t < n_rows; t += qkv::NCONS) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < qkv::CWARPS; w++) s += red[t * qkv::CWARPS + w];
        P.part[r_begin + t] = s;
    }
    __threadfence();
    named_bar_sync(1, qkv::NCONS);
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
    named_bar_sync(1, qkv::NCONS);
    if (warp >= misc[3]) return;
    const int h = misc[warp];
    // lane: dimensions 4 lane .. 4 lane + 3 of head h
    const float4 v = __ldcg(reinterpret_cast<const float4*>(P.part + (size_t)h * HD) + lane);
    const float2 fr = reinterpret_cast<const float2*>(P.inv_freq)[lane];
    const int pos = P.pos;
    const int nq = P.nq, nkv = P.nkv;
    if (h < nq) {
        const float4 w = reinterpret_cast<const float4*>(P.q_norm_w)[lane];
        reinterpret_cast<float4*>(P.q_out + (size_t)h * HD)[lane] = norm_rope_lane(v, w, P.eps, pos, fr);
        return;
    }
    const bool is_k = h < nq + nkv;
    const int kvh = is_k ? h - nq : h - nq - nkv;
    float4 out = v;
    if (is_k) {
        const float4 w = reinterpret_cast<const float4*>(P.k_norm_w)[lane];
        out = norm_rope_lane(v, w, P.eps, pos, fr);
        if (P.k_out) reinterpret_cast<float4*>(P.k_out + (size_t)kvh * HD)[lane] = out;
    } else if (P.v_out) {
        reinterpret_cast<float4*>(P.v_out + (size_t)kvh * HD)[lane] = out;
    }
    const long long phys = (long long)P.slot * P.pages_per_seq + pos / P.page_tokens;
    const long long row = (((long long)P.layer * nkv + kvh) * P.n_pages + phys) * P.page_tokens +
                          pos % P.page_tokens;
    KV* cache = reinterpret_cast<KV*>(is_k ? P.kcache : P.vcache);
    store4<KV>(cache + kv_index<KV>(row, 4 * lane), out);
}

int qkv_smem_bytes(int rows_total, int n_ctas) {
    const int max_rows = (rows_total + n_ctas - 1) / n_ctas + 1;
    return qkv::OFF_RED + max_rows * qkv::CWARPS * 4;
}

cudaError_t launch_qkv(const QkvParams& p, bool bf16, int n_ctas, cudaStream_t st) {
    // pieces per thread: 512 consumers cover 4096 columns per piece round
    const bool two = p.dim > 4096;
    const void* fn =
        bf16 ? (two ? reinterpret_cast<const void*>(qkv_kernel<__nv_bfloat16, 2>)
                    : reinterpret_cast<const void*>(qkv_kernel<__nv_bfloat16, 1>))
             : (two ? reinterpret_cast<const void*>(qkv_kernel<float, 2>)
                    : reinterpret_cast<const void*>(qkv_kernel<float, 1>));
    const int smem = qkv_smem_bytes(p.rows_total, n_ctas);
    cudaError_t e = ensure_smem_attr(fn, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_ctas);
    cfg.blockDim = dim3(qkv::NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<QkvParams*>(&p)};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace q3a
