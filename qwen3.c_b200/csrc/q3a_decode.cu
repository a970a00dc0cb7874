// q3a_decode.cu -- split-KV flash-decode for the Qwen3 GQA block on sm_100a.
//
// Replaces the decode attention of the reference (inline loop of
// qwen3-8b/cpu/main.c:1331-1353, HIP attn_flash_decode_kernel_hd128 at
// qwen3-8b/gpu/main.c:1565-1686) and, in fused mode, also its QK-norm, RoPE
// and KV append of the new token (qwen3-8b/cpu/main.c:1319-1329).
//
// Design (one launch per layer):
//  * Work = 64-token cache tiles of every (sequence, KV head) group, plus one
//    "new token" unit per group in fused mode.  A persistent grid of at most
//    one CTA per SM takes an equal contiguous share of the unit list, so any
//    mix of sequence lengths (the ragged batch included) is balanced to within
//    one tile per SM.
//  * Warp 8 of each CTA is the producer: one lane streams K and V tiles into a
//    ring of shared-memory stages with 2-D TMA loads (cp.async.bulk.tensor)
//    completing on per-stage mbarriers, with an L2 evict-first policy since
//    the cache is read once per step.
//  * Warps 0-7 consume: each takes 8 rows of a tile, so every K/V element
//    leaves shared memory once and feeds all 4 query heads of its KV head (the
//    HIP kernel re-reads K/V once per query head).  q.k uses 8 lanes per row
//    with 16 dims each and a reduce-scatter of 7 shuffles for 8 rows x 4
//    heads; each warp keeps its own online-softmax state (max, sum, o) in
//    registers in log2 units, so no CTA-wide barrier is taken per tile.
//  * At the end of a group's share the 8 warp states merge through shared
//    memory; if several CTAs share a group they write normalised partials
//    (o, lse) to scratch and the last CTA to arrive (atomic counter, reset by
//    that CTA) merges them by log-sum-exp and writes xb.
#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {

template <typename KV>
struct DecCfg {
    static constexpr int TILE = DEC_TILE;
    static constexpr int CWARPS = 8;
    static constexpr int NCONS = CWARPS * 32;
    static constexpr int NTHREADS = NCONS + 32;
    static constexpr int STAGES = sizeof(KV) == 4 ? 3 : 6;
    static constexpr int TILE_BYTES = TILE * HD * (int)sizeof(KV);
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = STAGES * TILE_BYTES;
    static constexpr int OFF_QS = 2 * STAGES * TILE_BYTES;       // float [4][128]
    static constexpr int OFF_NEWK = OFF_QS + GQA * HD * 4;       // KV [8][128] (row 0 used)
    static constexpr int OFF_NEWV = OFF_NEWK + 8 * HD * (int)sizeof(KV);
    static constexpr int OFF_P = OFF_NEWV + 8 * HD * (int)sizeof(KV);  // float [8 warps][32]
    static constexpr int WST = GQA * HD + 8;                     // o[4][128], m[4], l[4]
    static constexpr int OFF_WST = OFF_P + CWARPS * 32 * 4;
    static constexpr int OFF_BAR = OFF_WST + CWARPS * WST * 4;
    static constexpr int OFF_MISC = OFF_BAR + 2 * STAGES * 8;
    static constexpr int SMEM = OFF_MISC + 64;
    static_assert(SMEM <= 232448, "decode shared memory exceeds the sm_100 limit");
};

// Segment of the unit list that one CTA processes for one group.
struct Seg {
    int b;                 // sequence index within the launch
    int kvh;               // local kv head
    long long gstart;      // first unit of the group
    long long gend;        // one past its last unit
    int ncu;               // cache-tile units of the group
    int a0;                // absolute tile index of cache unit 0
};

__device__ __forceinline__ void locate(const DecodeParams& P, long long x, Seg& s) {
    int lo = 0, hi = P.nb;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (P.unit_prefix[mid] <= x) lo = mid; else hi = mid;
    }
    const int b = lo;
    const long long per = (P.unit_prefix[b + 1] - P.unit_prefix[b]) / P.nkv;
    const long long off = x - P.unit_prefix[b];
    s.b = b;
    s.kvh = (int)(off / per);
    s.gstart = P.unit_prefix[b] + (long long)s.kvh * per;
    s.gend = s.gstart + per;
    const int tb = P.t_begin[b], te = P.t_end[b];
    s.a0 = tb / DEC_TILE;
    s.ncu = te > tb ? (te + DEC_TILE - 1) / DEC_TILE - s.a0 : 0;
}

__device__ __forceinline__ int cta_of(const DecodeParams& P, long long x) {
    return (int)(((x + 1) * (long long)P.n_ctas - 1) / P.total_units);
}

// Row of the paged cache holding position `t` of (slot, local kv head).
__device__ __forceinline__ long long paged_row(const DecodeParams& P, int slot, int kvh, int t) {
    const int pt = P.page_tokens;
    const int phys = P.page_table[(long long)slot * P.pages_per_seq + t / pt];
    return (((long long)P.layer * P.nkv + kvh) * P.n_pages + phys) * pt + (t % pt);
}

// q registers of one lane: 4 heads x 16 dims, pre-scaled by log2(e)/sqrt(hd).
// fp32 tiles: lane j=lane&7 holds dims 4j+32s+e (s<4, e<4);
// bf16 tiles: dims 8j+64s+e (s<2, e<8); both give conflict-free 16-byte
// shared loads (8 lanes of a row read 128 consecutive bytes).
template <typename KV>
__device__ __forceinline__ void load_q_regs(const float* sQ, int lane, float sl2e,
                                            float (&qr)[GQA][16]) {
    const int j = lane & 7;
#pragma unroll
    for (int h = 0; h < GQA; h++) {
        if constexpr (sizeof(KV) == 4) {
#pragma unroll
            for (int s = 0; s < 4; s++) {
                const float4 t = *reinterpret_cast<const float4*>(sQ + h * HD + 4 * j + 32 * s);
                qr[h][4 * s + 0] = t.x * sl2e;
                qr[h][4 * s + 1] = t.y * sl2e;
                qr[h][4 * s + 2] = t.z * sl2e;
                qr[h][4 * s + 3] = t.w * sl2e;
            }
        } else {
#pragma unroll
            for (int s = 0; s < 2; s++) {
                const float4 t0 = *reinterpret_cast<const float4*>(sQ + h * HD + 8 * j + 64 * s);
                const float4 t1 =
                    *reinterpret_cast<const float4*>(sQ + h * HD + 8 * j + 64 * s + 4);
                qr[h][8 * s + 0] = t0.x * sl2e;
                qr[h][8 * s + 1] = t0.y * sl2e;
                qr[h][8 * s + 2] = t0.z * sl2e;
                qr[h][8 * s + 3] = t0.w * sl2e;
                qr[h][8 * s + 4] = t1.x * sl2e;
                qr[h][8 * s + 5] = t1.y * sl2e;
                qr[h][8 * s + 6] = t1.z * sl2e;
                qr[h][8 * s + 7] = t1.w * sl2e;
            }
        }
    }
}

__device__ __forceinline__ float sel4(const float (&a)[4], int i) {
    return i == 0 ? a[0] : i == 1 ? a[1] : i == 2 ? a[2] : a[3];
}

// One warp's share (rows 8w..8w+7, restricted to [lo, hi)) of a K/V tile.
template <typename KV>
__device__ __forceinline__ void process_rows(const KV* Kt, const KV* Vt, int lo, int hi, int warp,
                                             int lane, const float (&qr)[GQA][16],
                                             float (&m)[GQA], float& lpart,
                                             float (&O)[GQA][4], float* pw) {
    const int r0 = warp * 8;
    const int rlo = max(lo - r0, 0), rhi = min(hi - r0, 8);
    if (rlo >= rhi) return;
    const int g = lane >> 3, j = lane & 7;

    // ---- scores: acc[tt*4+h] for rows r0+2g+tt
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.0f;
#pragma unroll
    for (int tt = 0; tt < 2; tt++) {
        const int rr = 2 * g + tt;
        if (rr >= rlo && rr < rhi) {
            const KV* kr = Kt + (r0 + rr) * HD;
            if constexpr (sizeof(KV) == 4) {
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    const float4 kv =
                        *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(kr) +
                                                         4 * j + 32 * s);
#pragma unroll
                    for (int h = 0; h < GQA; h++) {
                        float a = acc[tt * 4 + h];
                        a = fmaf(qr[h][4 * s + 0], kv.x, a);
                        a = fmaf(qr[h][4 * s + 1], kv.y, a);
                        a = fmaf(qr[h][4 * s + 2], kv.z, a);
                        a = fmaf(qr[h][4 * s + 3], kv.w, a);
                        acc[tt * 4 + h] = a;
                    }
                }
            } else {
#pragma unroll
                for (int s = 0; s < 2; s++) {
                    const uint4 u = *reinterpret_cast<const uint4*>(
                        reinterpret_cast<const __nv_bfloat16*>(kr) + 8 * j + 64 * s);
                    const float k8[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                                         bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
                    for (int h = 0; h < GQA; h++) {
                        float a = acc[tt * 4 + h];
#pragma unroll
                        for (int e = 0; e < 8; e++) a = fmaf(qr[h][8 * s + e], k8[e], a);
                        acc[tt * 4 + h] = a;
                    }
                }
            }
        }
    }
    // ---- reduce-scatter over the 8 lanes of a row group: lane j ends with
    // the full sum of value index j (row 2g + (j>>2), head j&3).
    float r4[4];
    {
        const bool b2 = (j & 4) != 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float send = b2 ? acc[i] : acc[i + 4];
            const float keep = b2 ? acc[i + 4] : acc[i];
            r4[i] = keep + __shfl_xor_sync(FULL, send, 4);
        }
    }
    float r2[2];
    {
        const bool b1 = (j & 2) != 0;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const float send = b1 ? r4[i] : r4[i + 2];
            const float keep = b1 ? r4[i + 2] : r4[i];
            r2[i] = keep + __shfl_xor_sync(FULL, send, 2);
        }
    }
    float s;
    {
        const bool b0 = (j & 1) != 0;
        const float send = b0 ? r2[0] : r2[1];
        const float keep = b0 ? r2[1] : r2[0];
        s = keep + __shfl_xor_sync(FULL, send, 1);
    }
    const int myrow = 2 * g + (j >> 2);
    if (myrow < rlo || myrow >= rhi) s = -INFINITY;

    // ---- online softmax (per head, lanes with equal lane&3)
    float mx = s;
    mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 16));
    const int hl = lane & 3;
    const float m_old = sel4(m, hl);
    const float m_new = fmaxf(m_old, mx);  // finite: row rlo is valid for every head
    const float alpha = exp2f(m_old - m_new);
    const float p = exp2f(s - m_new);
    lpart = lpart * alpha + p;
    float al[GQA];
#pragma unroll
    for (int h = 0; h < GQA; h++) {
        m[h] = __shfl_sync(FULL, m_new, h);
        al[h] = __shfl_sync(FULL, alpha, h);
    }
    pw[lane] = p;  // index = row*4 + head
    __syncwarp();
#pragma unroll
    for (int h = 0; h < GQA; h++) {
#pragma unroll
        for (int e = 0; e < 4; e++) O[h][e] *= al[h];
    }
    // ---- o += p . v  (lane owns dims 4*lane .. 4*lane+3)
#pragma unroll
    for (int tt = 0; tt < 8; tt++) {
        if (tt >= rlo && tt < rhi) {
            const float4 pv = reinterpret_cast<const float4*>(pw)[tt];
            float v[4];
            if constexpr (sizeof(KV) == 4) {
                const float4 t = *reinterpret_cast<const float4*>(
                    reinterpret_cast<const float*>(Vt) + (r0 + tt) * HD + 4 * lane);
                v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
            } else {
                const uint2 u = *reinterpret_cast<const uint2*>(
                    reinterpret_cast<const __nv_bfloat16*>(Vt) + (r0 + tt) * HD + 4 * lane);
                v[0] = bf16lo(u.x); v[1] = bf16hi(u.x); v[2] = bf16lo(u.y); v[3] = bf16hi(u.y);
            }
#pragma unroll
            for (int e = 0; e < 4; e++) {
                O[0][e] = fmaf(pv.x, v[e], O[0][e]);
                O[1][e] = fmaf(pv.y, v[e], O[1][e]);
                O[2][e] = fmaf(pv.z, v[e], O[2][e]);
                O[3][e] = fmaf(pv.w, v[e], O[3][e]);
            }
        }
    }
    __syncwarp();
}

template <typename KV>
__global__ void __launch_bounds__(DecCfg<KV>::NTHREADS, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ DecodeParams P) {
    using C = DecCfg<KV>;
    extern __shared__ __align__(1024) uint8_t smem[];
    KV* sK = reinterpret_cast<KV*>(smem + C::OFF_K);
    KV* sV = reinterpret_cast<KV*>(smem + C::OFF_V);
    float* sQ = reinterpret_cast<float*>(smem + C::OFF_QS);
    KV* sNewK = reinterpret_cast<KV*>(smem + C::OFF_NEWK);
    KV* sNewV = reinterpret_cast<KV*>(smem + C::OFF_NEWV);
    float* sP = reinterpret_cast<float*>(smem + C::OFF_P);
    float* sW = reinterpret_cast<float*>(smem + C::OFF_WST);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::STAGES;
    volatile int* misc = reinterpret_cast<volatile int*>(smem + C::OFF_MISC);
    float* sScale = reinterpret_cast<float*>(smem + C::OFF_MISC + 16);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x;
    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::CWARPS);
        }
        fence_mbar_init();
    }
    if (warp == C::CWARPS && lane == 0) {
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    __syncthreads();

    const long long u_lo = (long long)c * P.total_units / P.n_ctas;
    const long long u_hi = (long long)(c + 1) * P.total_units / P.n_ctas;

    if (warp == C::CWARPS) {
        // ================================================= producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int it = 0;
            bool dead = false;
            long long x = u_lo;
            while (x < u_hi && !dead) {
                Seg s;
                locate(P, x, s);
                const long long seg_end = min(u_hi, s.gend);
                const int slot = P.slot[s.b];
                for (long long y = x; y < seg_end; y++) {
                    const int u = (int)(y - s.gstart);
                    if (u >= s.ncu) continue;  // the new-token unit needs no load
                    const int stage = it % C::STAGES;
                    const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                    if (it >= C::STAGES && !mbar_wait(&empty[stage], ph ^ 1u)) {
                        atomicExch(P.err, DEV_ERR_TIMEOUT);
                        dead = true;
                        break;
                    }
                    const int t0 = (s.a0 + u) * DEC_TILE;
                    int xc, yc;
                    if (P.cache_mode == CACHE_PAGED) {
                        xc = 0;
                        yc = (int)paged_row(P, slot, s.kvh, t0);
                    } else {
                        xc = (P.kv0 + s.kvh) * HD;
                        yc = t0;
                    }
                    mbar_arrive_expect_tx(&full[stage], 2u * C::TILE_BYTES);
                    tma_load_2d(sK + stage * C::TILE * HD, &tmK, &full[stage], xc, yc, pol);
                    tma_load_2d(sV + stage * C::TILE * HD, &tmV, &full[stage], xc, yc, pol);
                    it++;
                }
                x = seg_end;
            }
            // Drain: the CTA never exits with a bulk copy still writing its
            // shared memory (bounded, like every wait here).
            const int first = it > C::STAGES ? it - C::STAGES : 0;
            for (int k = first; k < it; k++) {
                if (!mbar_wait(&full[k % C::STAGES], (uint32_t)(k / C::STAGES) & 1u)) {
                    atomicExch(P.err, DEV_ERR_TIMEOUT);
                    break;
                }
            }
        }
        return;
    }

    // ===================================================== consumers
    int it = 0;
    long long x = u_lo;
    float* pw = sP + warp * 32;
    while (x < u_hi) {
        Seg s;
        locate(P, x, s);
        const long long seg_end = min(u_hi, s.gend);
        const int b = s.b, kvh = s.kvh;
        const int hq0 = (P.kv0 + kvh) * GQA;
        const int slot = P.slot[b];
        const bool has_new = P.fused && seg_end == s.gend;

        // ---- query of the group: raw -> QK-RMSNorm -> RoPE (fused) or as is
        const float* qsrc = P.q + (size_t)b * P.hq_total * HD + (size_t)hq0 * HD;
        for (int i = tid; i < GQA * HD; i += C::NCONS) sQ[i] = qsrc[i];
        if (has_new) {
            const float* ksrc = P.k_new + (size_t)b * P.nkv_total * HD + (size_t)(P.kv0 + kvh) * HD;
            if (tid < HD) sW[tid] = ksrc[tid];
        }
        named_bar_sync(1, C::NCONS);
        if (P.fused) {
            if (tid < GQA) sScale[tid] = head_rms_scale(sQ + tid * HD, P.eps);
            if (has_new && tid == 32) sScale[4] = head_rms_scale(sW, P.eps);
            named_bar_sync(1, C::NCONS);
            {
                const int h = tid >> 6, pi = tid & 63;
                float* qp = sQ + h * HD + 2 * pi;
                const float sc = sScale[h];
                float v0 = __fmul_rn(qp[0], __fmul_rn(sc, P.q_norm_w[2 * pi]));
                float v1 = __fmul_rn(qp[1], __fmul_rn(sc, P.q_norm_w[2 * pi + 1]));
                rope_pair(v0, v1, P.pos[b], P.inv_freq[pi]);
                qp[0] = v0;
                qp[1] = v1;
            }
            if (has_new) {
                // new token: k normed + rotated, v as is; stored in the cache
                // dtype, appended at pos, and kept in shared memory for use.
                const int pos = P.pos[b];
                const long long row = paged_row(P, slot, kvh, pos);
                KV* kdst = reinterpret_cast<KV*>(P.kcache) + row * HD;
                KV* vdst = reinterpret_cast<KV*>(P.vcache) + row * HD;
                if (tid < 64) {
                    const float sc = sScale[4];
                    float v0 = __fmul_rn(sW[2 * tid], __fmul_rn(sc, P.k_norm_w[2 * tid]));
                    float v1 = __fmul_rn(sW[2 * tid + 1], __fmul_rn(sc, P.k_norm_w[2 * tid + 1]));
                    rope_pair(v0, v1, pos, P.inv_freq[tid]);
                    if (P.k_out) {
                        float* ko = P.k_out + (size_t)b * P.nkv_total * HD +
                                    (size_t)(P.kv0 + kvh) * HD;
                        ko[2 * tid] = v0;
                        ko[2 * tid + 1] = v1;
                    }
                    const KV k0 = from_f32<KV>(v0), k1 = from_f32<KV>(v1);
                    sNewK[2 * tid] = k0;
                    sNewK[2 * tid + 1] = k1;
                    kdst[2 * tid] = k0;
                    kdst[2 * tid + 1] = k1;
                } else if (tid < 64 + HD) {
                    const int i = tid - 64;
                    const float* vsrc = P.v_new + (size_t)b * P.nkv_total * HD +
                                        (size_t)(P.kv0 + kvh) * HD;
                    const KV vv = from_f32<KV>(vsrc[i]);
                    sNewV[i] = vv;
                    vdst[i] = vv;
                }
            }
            named_bar_sync(1, C::NCONS);
        }

        float qr[GQA][16];
        load_q_regs<KV>(sQ, lane, P.scale_log2e, qr);
        float m[GQA] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        float lpart = 0.0f;
        float O[GQA][4];
#pragma unroll
        for (int h = 0; h < GQA; h++) {
#pragma unroll
            for (int e = 0; e < 4; e++) O[h][e] = 0.0f;
        }

        bool dead = false;
        for (long long y = x; y < seg_end; y++) {
            const int u = (int)(y - s.gstart);
            if (u < s.ncu) {
                const int stage = it % C::STAGES;
                const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                if (!mbar_wait(&full[stage], ph)) {
                    atomicExch(P.err, DEV_ERR_TIMEOUT);
                    dead = true;
                    break;
                }
                const int t0 = (s.a0 + u) * DEC_TILE;
                const int lo = max(P.t_begin[b] - t0, 0);
                const int hi = min(P.t_end[b] - t0, DEC_TILE);
                process_rows<KV>(sK + stage * C::TILE * HD, sV + stage * C::TILE * HD, lo, hi,
                                 warp, lane, qr, m, lpart, O, pw);
                if (lane == 0) mbar_arrive(&empty[stage]);
                it++;
            } else {
                process_rows<KV>(sNewK, sNewV, 0, 1, warp, lane, qr, m, lpart, O, pw);
            }
        }
        if (dead) return;

        // ---- merge the 8 warp states of this segment
        float lsum = lpart;
        lsum += __shfl_xor_sync(FULL, lsum, 4);
        lsum += __shfl_xor_sync(FULL, lsum, 8);
        lsum += __shfl_xor_sync(FULL, lsum, 16);
        {
            float* ws = sW + warp * C::WST;
#pragma unroll
            for (int h = 0; h < GQA; h++)
                *reinterpret_cast<float4*>(ws + h * HD + 4 * lane) =
                    make_float4(O[h][0], O[h][1], O[h][2], O[h][3]);
            if (lane < 4) {
                ws[GQA * HD + lane] = sel4(m, lane);
                ws[GQA * HD + 4 + lane] = lsum;
            }
        }
        named_bar_sync(1, C::NCONS);
        const int h = tid >> 6, d = 2 * (tid & 63);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < C::CWARPS; w++) M = fmaxf(M, sW[w * C::WST + GQA * HD + h]);
        float L = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
        for (int w = 0; w < C::CWARPS; w++) {
            const float mw = sW[w * C::WST + GQA * HD + h];
            const float sc = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
            L = fmaf(sW[w * C::WST + GQA * HD + 4 + h], sc, L);
            o0 = fmaf(sW[w * C::WST + h * HD + d], sc, o0);
            o1 = fmaf(sW[w * C::WST + h * HD + d + 1], sc, o1);
        }
        float inv = 1.0f / L;
        o0 *= inv;
        o1 *= inv;
        float lse = M + log2f(L);

        const int cs = cta_of(P, s.gstart), ce = cta_of(P, s.gend - 1);
        const int ncontrib = ce - cs + 1;
        const int grp = b * P.nkv + kvh;
        bool write_out = true;
        if (ncontrib > 1) {
            const long long pslot = (long long)cs + grp + (c - cs);
            float* ps = P.partials + pslot * PART_STRIDE;
            ps[h * HD + d] = o0;
            ps[h * HD + d + 1] = o1;
            if ((tid & 63) == 0) ps[GQA * HD + h] = lse;
            __threadfence();
            named_bar_sync(1, C::NCONS);
            if (tid == 0) {
                const int old = atomicAdd(&P.counters[grp], 1);
                misc[0] = (old == ncontrib - 1) ? 1 : 0;
            }
            named_bar_sync(1, C::NCONS);
            write_out = misc[0] != 0;
            if (write_out) {
                __threadfence();
                const float* pb = P.partials + ((long long)cs + grp) * PART_STRIDE;
                float Mx = -INFINITY;
                for (int jj = 0; jj < ncontrib; jj++)
                    Mx = fmaxf(Mx, __ldcg(pb + (long long)jj * PART_STRIDE + GQA * HD + h));
                float W = 0.0f, a0 = 0.0f, a1 = 0.0f;
                for (int jj = 0; jj < ncontrib; jj++) {
                    const float* pj = pb + (long long)jj * PART_STRIDE;
                    const float lj = __ldcg(pj + GQA * HD + h);
                    const float wj = (lj == -INFINITY) ? 0.0f : exp2f(lj - Mx);
                    W += wj;
                    a0 = fmaf(wj, __ldcg(pj + h * HD + d), a0);
                    a1 = fmaf(wj, __ldcg(pj + h * HD + d + 1), a1);
                }
                const float iw = 1.0f / W;
                o0 = a0 * iw;
                o1 = a1 * iw;
                lse = Mx + log2f(W);
                if (tid == 0) P.counters[grp] = 0;
            }
        }
        if (write_out) {
            float* xo = P.xb + (size_t)b * P.hq_total * HD + (size_t)(hq0 + h) * HD + d;
            *reinterpret_cast<float2*>(xo) = make_float2(o0, o1);
            if (P.lse_out && (tid & 63) == 0) P.lse_out[(size_t)b * P.hq_total + hq0 + h] = lse;
            if (P.fused && P.q_out) {
                float* qo = P.q_out + (size_t)b * P.hq_total * HD + (size_t)hq0 * HD;
                for (int i = tid; i < GQA * HD; i += C::NCONS) qo[i] = sQ[i];
            }
        }
        named_bar_sync(1, C::NCONS);
        x = seg_end;
    }
}

template <typename KV>
static cudaError_t launch_decode_t(const DecodeParams& p, const CUtensorMap& tmK,
                                   const CUtensorMap& tmV, cudaStream_t st) {
    using C = DecCfg<KV>;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<KV>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    decode_kernel<KV><<<p.n_ctas, C::NTHREADS, C::SMEM, st>>>(tmK, tmV, p);
    return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          bool bf16, cudaStream_t st) {
    return bf16 ? launch_decode_t<__nv_bfloat16>(p, tmK, tmV, st)
                : launch_decode_t<float>(p, tmK, tmV, st);
}

int decode_smem_bytes(bool bf16) {
    return bf16 ? DecCfg<__nv_bfloat16>::SMEM : DecCfg<float>::SMEM;
}

}  // namespace q3a
