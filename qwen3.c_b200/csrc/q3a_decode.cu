// q3a_decode.cu -- split-KV flash-decode for the Qwen3 GQA block on sm_100a.
//
// Replaces the decode attention of the reference (inline loop of
// qwen3-8b/cpu/main.c:1331-1353, HIP attn_flash_decode_kernel_hd128 at
// qwen3-8b/gpu/main.c:1565-1686) and, in fused mode, also its QK-norm, RoPE
// and KV append of the new token (qwen3-8b/cpu/main.c:1319-1329).
//
// Design (one launch per layer):
//  * Work is split into contiguous cache-row ranges of (sequence, KV head)
//    groups.  With at most one group per SM (the single-sequence decode of the
//    reference) every CTA gets exactly one range, sized so that ranges are
//    equal to within one 16-row box ("piece mode"); larger batches use a
//    linear list of 64-row tiles cut into equal shares.  Grid size <= SM
//    count, one CTA per SM.
//  * Warp 8 is the producer: one lane streams K and V into a ring of
//    shared-memory stages, each stage of the paged cache as one bulk copy per
//    tensor (cp.async.bulk; two where a stage crosses a page boundary), with
//    an L2 evict-first policy since each cache row is read once per step.
//    The caller-owned position-major cache of q3a_attn_decode is strided and
//    moves in 16-row 2-D TMA boxes (cp.async.bulk.tensor) instead.
//  * fp32 caches are consumed on the CUDA cores by warps 0-7, each taking 8
//    rows of a 64-row stage, so every K/V element leaves shared memory once
//    and feeds all 4 query heads of its KV head; q.k uses 8 lanes per row
//    with 16 dims each (packed fp32x2 FMA), a 7-shuffle reduce-scatter gives
//    one (row, head) score per lane, and each warp keeps its own online
//    softmax (log2 domain), merged through shared memory at the end.
//  * bf16 caches are consumed on the tensor cores (TC instantiation): the
//    cache's 8-row blocks are already the 128B-swizzled operand layout, so a
//    128-row stage is used as is; warp 4 issues S^T = K.Q^T and
//    O^T = V^T.P^T (tcgen05.mma, accumulators in tensor memory) and warps 0-3
//    run the softmax between them.
//  * The prologue issues every global load of the range's inputs at once (q,
//    norm gains, the new token's k and v) and reduces the RMS norms with warp
//    shuffles, overlapping the first stage's load.
//  * Ranges sharing a group merge by log-sum-exp: in piece mode by the
//    spread merge (tagged words in scratch, each range merges one slice of
//    the outputs), in linear mode by a ticket (the last range to arrive
//    merges all partials); sequence shards then exchange (o, lse) with every
//    rank over peer memory the same way.
#include "q3a_common.cuh"
#include "q3a_internal.h"
#include "q3a_tcgen05.cuh"

namespace q3a {

// fp32 caches (CUDA-core consumer): stages of 32 rows (16 KB of K + 16 KB of
// V), six in the ring; the consumer warps form two groups of four that take
// alternate stages, each warp 8 rows of a stage.
template <typename KV, bool TC = false>
struct DecCfg {
    static constexpr int TILE = 32;
    static constexpr int CWARPS = 8;
    static constexpr int NCONS = CWARPS * 32;
    static constexpr int NTHREADS = NCONS + 32;
    static constexpr int STAGES = 6;
    // balanced schedule: units a range streams before claiming (measured at
    // KV 8192: 3 -> 15.32 us/layer, 2 -> 15.41, 4 -> 15.56, 1 -> 15.56)
    static constexpr int STATIC_UNITS = 3;
    static constexpr int TILE_BYTES = TILE * HD * (int)sizeof(KV);
    static constexpr int BOX_BYTES = DEC_BOX * HD * (int)sizeof(KV);
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = STAGES * TILE_BYTES;
    static constexpr int OFF_QS = 2 * STAGES * TILE_BYTES;       // float [4][128]
    static constexpr int OFF_RAW = OFF_QS + GQA * HD * 4;        // float [256] norm gains / raw k,v
    static constexpr int OFF_RAW2 = OFF_RAW + 256 * 4;           // float [256]
    static constexpr int OFF_NEWK = OFF_RAW2 + 256 * 4;          // KV [128]
    static constexpr int OFF_NEWV = OFF_NEWK + HD * (int)sizeof(KV);
    static constexpr int OFF_P = OFF_NEWV + HD * (int)sizeof(KV);  // float2 [8 warps][32]
    static constexpr int WST = GQA * HD + 8;                       // o[4][128], m[4], l[4]
    static constexpr int OFF_WST = OFF_P + CWARPS * 32 * 8;
    static constexpr int OFF_BAR = OFF_WST + CWARPS * WST * 4;
    static constexpr int OFF_META = OFF_BAR + 2 * STAGES * 8;    // int2 [STAGES]: first row, rows
    static constexpr int OFF_MISC = OFF_META + STAGES * 8;
    static constexpr int SMEM = OFF_MISC + 64;
    static_assert(SMEM <= 232448, "decode shared memory exceeds the sm_100 limit");
};

// Tensor-core consumer (bf16 paged caches).  Stages of 128 cache rows, K and
// V each copied as is from the cache, whose 8-row blocks ([2 dim-halves][8
// rows][128 B], 128-byte swizzle) are the MMA operand layout: S^T = K . Q^T
// (A = K, K-major) and O^T = V^T . P^T (A = V read MN-major).  Q^T and P^T
// are [16][128] bf16 operands of two [16 rows][128 B] halves (rows 0-3 the 4
// query heads' high parts, rows 4-7 their low parts, rows 8-15 zero).
template <>
struct DecCfg<__nv_bfloat16, true> {
    static constexpr int TILE = 128;
    static constexpr int CWARPS = 8;
    static constexpr int NCONS = CWARPS * 32;
    static constexpr int NTHREADS = NCONS + 32;
    static constexpr int STAGES = 3;
    // one static unit (measured at KV 8192: 13.44 us/layer against 13.75 with 2)
    static constexpr int STATIC_UNITS = 1;
    static constexpr int TILE_BYTES = TILE * HD * 2;        // one tensor of a stage
    static constexpr int OPB_BYTES = 16 * HD * 2;           // a [16][128] bf16 operand
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = STAGES * TILE_BYTES;
    static constexpr int OFF_QT = 2 * STAGES * TILE_BYTES;  // Q^T
    static constexpr int OFF_PT = OFF_QT + OPB_BYTES;       // P^T, two buffers
    static constexpr int OFF_QS = OFF_PT + 2 * OPB_BYTES;   // float [4][128]
    static constexpr int OFF_RAW = OFF_QS + GQA * HD * 4;
    static constexpr int OFF_RAW2 = OFF_RAW + 256 * 4;
    static constexpr int OFF_NEWK = OFF_RAW2 + 256 * 4;
    static constexpr int OFF_NEWV = OFF_NEWK + HD * 2;
    static constexpr int OFF_P = OFF_NEWV + HD * 2;         // unused here
    static constexpr int WST = 0;
    // o[4][128], lse[4], tile maxima [2][4 warps][4], row sums [4 warps][4]
    static constexpr int OFF_WST = OFF_P + 16;
    static constexpr int W_LSE = GQA * HD, W_RED = W_LSE + GQA, W_LSUM = W_RED + 32;
    static constexpr int OFF_BAR = OFF_WST + (W_LSUM + 16) * 4;
    // full[3] empty[3] sfull[2] pfull[2] ofull[2] newrow drain
    static constexpr int NBAR = 2 * STAGES + 8;
    static constexpr int OFF_META = OFF_BAR + NBAR * 8;       // int2 [STAGES]: first row, rows
    static constexpr int OFF_MISC = OFF_META + STAGES * 8;
    static constexpr int SMEM = OFF_MISC + 64 + 1024;       // + slack for 1024-byte alignment
    static_assert(OFF_QT % 1024 == 0 && OFF_PT % 1024 == 0 && OFF_BAR % 8 == 0, "layout");
    static_assert(SMEM <= 232448, "decode shared memory exceeds the sm_100 limit");
};

// tensor memory columns of the tensor-core consumer: S^T double buffer,
// O^T tile double buffer, 16 columns each
constexpr uint32_t DTC_COLS = 64;
constexpr uint32_t DTC_S_COL = 0, DTC_O_COL = 32;
// instruction descriptors (kind::f16, M=128, N=16): c=F32 (bit 4), a=BF16
// (bits 7-9), b=BF16 (bits 10-12), a_major bit 15, N>>3 at 17, M>>4 at 24
constexpr uint32_t IDESC_DS = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t IDESC_DPV = IDESC_DS | (1u << 15);

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Byte offset of element (row n, k) in a [16][128] bf16 K-major operand with
// 128-byte swizzle: two 64-element halves of [16 rows][128 B], the 16-byte
// chunk index XORed with the row within its 8-row group.
__device__ __forceinline__ uint32_t opb_offset(int n, int k) {
    return (uint32_t)((k >> 6) * 2048 + n * 128 + ((((k & 63) >> 3) ^ (n & 7)) << 4) + (k & 7) * 2);
}

// One contiguous range of cache rows of one group, as processed by a CTA.
struct SegInfo {
    int b;          // sequence index within the launch
    int kvh;        // local kv head
    int r0, r1;     // cache rows [r0, r1) streamed from the cache
    int has_new;    // this range also handles the new token (fused)
    int slot;       // partial slot of this range
    int slot0;      // first partial slot of the group
    int ncontrib;   // ranges of the group
    int grp;        // group index (arrival counter)
};

__device__ __forceinline__ int cta_of(const DecodeParams& P, long long x) {
    return (int)(((x + 1) * (long long)P.n_ctas - 1) / P.total_units);
}

// Next range of CTA c; `cur` is the linear-mode cursor (unit index).
__device__ __forceinline__ bool next_seg(const DecodeParams& P, int c, long long& cur,
                                         SegInfo& s) {
    if (P.n_pieces > 0) {
        if (cur != 0) return false;
        cur = 1;
        const int pi = P.cta_piece[c];
        const Piece pc = P.pieces[pi];
        s.b = pc.g / P.nkv;
        s.kvh = pc.g % P.nkv;
        s.r0 = pc.r0;
        s.r1 = pc.r1;
        s.has_new = P.fused && pc.i == pc.k - 1;
        s.slot = pi;
        s.slot0 = pi - pc.i;
        s.ncontrib = pc.k;
        s.grp = pc.g;
        return true;
    }
    const long long u_hi = (long long)(c + 1) * P.total_units / P.n_ctas;
    if (cur == 0) cur = (long long)c * P.total_units / P.n_ctas + 1;  // stored +1
    const long long x = cur - 1;
    if (x >= u_hi) return false;
    int lo = 0, hi = P.nb;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (P.unit_prefix[mid] <= x) lo = mid; else hi = mid;
    }
    const int b = lo;
    const long long per = (P.unit_prefix[b + 1] - P.unit_prefix[b]) / P.nkv;
    const long long off = x - P.unit_prefix[b];
    const int kvh = (int)(off / per);
    const long long gstart = P.unit_prefix[b] + (long long)kvh * per;
    const long long gend = gstart + per;
    const long long seg_end = min(u_hi, gend);
    const int tb = P.t_begin[b], te = P.t_end[b];
    const int a0 = tb / DEC_TILE;
    const int ncu = te > tb ? (te + DEC_TILE - 1) / DEC_TILE - a0 : 0;
    const int uf = (int)(x - gstart), ul = (int)(seg_end - 1 - gstart);
    if (uf < ncu) {
        s.r0 = max(tb, (a0 + uf) * DEC_TILE);
        s.r1 = min(te, (a0 + min(ul, ncu - 1) + 1) * DEC_TILE);
    } else {
        s.r0 = s.r1 = te;
    }
    s.b = b;
    s.kvh = kvh;
    s.has_new = P.fused && seg_end == gend;
    const int grp = b * P.nkv + kvh;
    const int cs = cta_of(P, gstart), ce = cta_of(P, gend - 1);
    s.slot = c + grp;
    s.slot0 = cs + grp;
    s.ncontrib = ce - cs + 1;
    s.grp = grp;
    cur = seg_end + 1;
    return true;
}

// Row of the paged cache holding position `t` of (slot, local kv head).
// Slot s owns pages [s*pages_per_seq, (s+1)*pages_per_seq) of every
// (layer, kv head) region, so the address is arithmetic only.
__device__ __forceinline__ long long paged_row(const DecodeParams& P, int slot, int kvh, int t) {
    const int pt = P.page_tokens;
    const long long phys = (long long)slot * P.pages_per_seq + t / pt;
    return (((long long)P.layer * P.nkv + kvh) * P.n_pages + phys) * pt + (t % pt);
}

// Balanced schedule (P.dyn, piece mode on the paged cache).  The rows a
// group attends are cut into units of U rows (one stage) aligned at a0;
// units [0, n_claim) are streamed by the group's ranges -- range i first its
// static units [i*S, (i+1)*S), which need nothing from the previous kernel
// and may be streamed before the dependency wait, then units claimed one at
// a time from the group's counter, starting at k*S -- so ranges on slower
// SMs take fewer units.  On the tensor cores with a fused new token the
// range that appends it also streams the tail [tail0, pos+1) last (the unit
// holding pos, after the append).  Rows at or past r_lim are not attended
// (the CUDA-core consumer takes the new token from shared memory).
constexpr int DYN_END = -0x7fffffff;  // stage metadata of an end marker

struct DynPlan {
    int a0, n_claim, tb, r_lim, tail0;
};

template <bool TC>
__device__ __forceinline__ DynPlan dyn_plan(const DecodeParams& P, int b, int U) {
    DynPlan d;
    d.tb = P.t_begin[b];
    const int te = P.t_end[b];
    d.a0 = d.tb & ~(U - 1);
    if (TC && P.fused) {
        const int pos = P.pos[b];  // == te: the new token's row
        d.n_claim = (pos - d.a0) / U;
        d.tail0 = d.a0 + d.n_claim * U;
        d.r_lim = pos + 1;
    } else {
        d.n_claim = te > d.tb ? (te - d.a0 + U - 1) / U : 0;
        d.tail0 = -1;
        d.r_lim = te;
    }
    return d;
}

// acq_rel atomic add at GPU scope: releases this CTA's partial (ordered
// before it by the preceding CTA barrier) and, for the last arrival,
// acquires every other contributor's.
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
                 : "memory");
    return old;
}

// q registers of one lane as fp32 pairs, 4 heads x 16 dims, pre-scaled by
// log2(e)/sqrt(hd): lane j=lane&7 holds dims 4j+32s+e (s<4, e<4), which gives
// conflict-free 16-byte shared loads (the 8 lanes of a row read 128
// consecutive bytes).  The CUDA-core consumer reads fp32 caches only (bf16
// caches go to the tensor cores).
template <typename KV>
__device__ __forceinline__ void load_q_regs(const float* sQ, int lane, float sl2e,
                                            float2 (&qr)[GQA][8]) {
    static_assert(sizeof(KV) == 4, "the CUDA-core consumer reads fp32 caches");
    const int j = lane & 7;
#pragma unroll
    for (int h = 0; h < GQA; h++) {
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const float4 t = *reinterpret_cast<const float4*>(sQ + h * HD + 4 * j + 32 * s);
            qr[h][2 * s] = make_float2(t.x * sl2e, t.y * sl2e);
            qr[h][2 * s + 1] = make_float2(t.z * sl2e, t.w * sl2e);
        }
    }
}

__device__ __forceinline__ float sel4(const float (&a)[4], int i) {
    return i == 0 ? a[0] : i == 1 ? a[1] : i == 2 ? a[2] : a[3];
}

// Scores of rows 2g and 2g+1 (relative to r0) of one warp's 8-row share:
// acc[tt][h] holds fp32 pairs (even/odd dims) for row 2g+tt.  FULL_ROWS
// selects the branch-free body (all 8 rows valid), so every shared-memory
// load can be issued ahead of the math.
template <typename KV, bool FULL_ROWS>
__device__ __forceinline__ void qk_rows(const KV* Kt, int r0, int rlo, int rhi, int g, int j,
                                        const float2 (&qr)[GQA][8], float2 (&acc)[2][GQA]) {
#pragma unroll
    for (int tt = 0; tt < 2; tt++) {
#pragma unroll
        for (int h = 0; h < GQA; h++) acc[tt][h] = make_float2(0.0f, 0.0f);
    }
    static_assert(sizeof(KV) == 4, "the CUDA-core consumer reads fp32 caches");
    {
        float4 kv[2][4];
#pragma unroll
        for (int tt = 0; tt < 2; tt++) {
            const int rr = 2 * g + tt;
            const float* kr = reinterpret_cast<const float*>(Kt) + (r0 + rr) * HD + 4 * j;
#pragma unroll
            for (int s = 0; s < 4; s++) {
                if (FULL_ROWS || (rr >= rlo && rr < rhi))
                    kv[tt][s] = *reinterpret_cast<const float4*>(kr + 32 * s);
                else
                    kv[tt][s] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
        }
#pragma unroll
        for (int tt = 0; tt < 2; tt++) {
#pragma unroll
            for (int s = 0; s < 4; s++) {
                const float2 ka = make_float2(kv[tt][s].x, kv[tt][s].y);
                const float2 kb = make_float2(kv[tt][s].z, kv[tt][s].w);
#pragma unroll
                for (int h = 0; h < GQA; h++) {
                    acc[tt][h] = __ffma2_rn(qr[h][2 * s], ka, acc[tt][h]);
                    acc[tt][h] = __ffma2_rn(qr[h][2 * s + 1], kb, acc[tt][h]);
                }
            }
        }
    }
}

// o += p . v over rows [rlo, rhi) of the warp's share; lane owns dims
// 4*lane .. 4*lane+3; p for (row, head) is duplicated in pw[row*4+head].
template <typename KV, bool FULL_ROWS>
__device__ __forceinline__ void pv_rows(const KV* Vt, int r0, int rlo, int rhi, int lane,
                                        const float2* pw, float2 (&O)[GQA][2]) {
    float2 va[8], vb[8];
#pragma unroll
    for (int tt = 0; tt < 8; tt++) {
        if (FULL_ROWS || (tt >= rlo && tt < rhi)) {
            const float4 t = *reinterpret_cast<const float4*>(
                reinterpret_cast<const float*>(Vt) + (r0 + tt) * HD + 4 * lane);
            va[tt] = make_float2(t.x, t.y);
            vb[tt] = make_float2(t.z, t.w);
        } else {
            va[tt] = vb[tt] = make_float2(0.0f, 0.0f);  // p is 0 there too
        }
    }
#pragma unroll
    for (int tt = 0; tt < 8; tt++) {
        const float4 pa = *reinterpret_cast<const float4*>(pw + 4 * tt);
        const float4 pb = *reinterpret_cast<const float4*>(pw + 4 * tt + 2);
        const float2 p0 = make_float2(pa.x, pa.y), p1 = make_float2(pa.z, pa.w);
        const float2 p2 = make_float2(pb.x, pb.y), p3 = make_float2(pb.z, pb.w);
        O[0][0] = __ffma2_rn(p0, va[tt], O[0][0]);
        O[0][1] = __ffma2_rn(p0, vb[tt], O[0][1]);
        O[1][0] = __ffma2_rn(p1, va[tt], O[1][0]);
        O[1][1] = __ffma2_rn(p1, vb[tt], O[1][1]);
        O[2][0] = __ffma2_rn(p2, va[tt], O[2][0]);
        O[2][1] = __ffma2_rn(p2, vb[tt], O[2][1]);
        O[3][0] = __ffma2_rn(p3, va[tt], O[3][0]);
        O[3][1] = __ffma2_rn(p3, vb[tt], O[3][1]);
    }
}

// One warp's share (rows 8w..8w+7, restricted to [lo, hi)) of a K/V tile.
template <typename KV>
__device__ __forceinline__ void process_rows(const KV* Kt, const KV* Vt, int lo, int hi, int warp,
                                             int lane, const float2 (&qr)[GQA][8],
                                             float (&m)[GQA], float& lpart,
                                             float2 (&O)[GQA][2], float2* pw) {
    const int r0 = warp * 8;
    const int rlo = max(lo - r0, 0), rhi = min(hi - r0, 8);
    if (rlo >= rhi) return;
    const bool full = (rlo == 0 && rhi == 8);
    const int g = lane >> 3, j = lane & 7;

    float2 acc[2][GQA];
    if (full)
        qk_rows<KV, true>(Kt, r0, rlo, rhi, g, j, qr, acc);
    else
        qk_rows<KV, false>(Kt, r0, rlo, rhi, g, j, qr, acc);
    float a8[8];
#pragma unroll
    for (int tt = 0; tt < 2; tt++) {
#pragma unroll
        for (int h = 0; h < GQA; h++) a8[tt * 4 + h] = acc[tt][h].x + acc[tt][h].y;
    }
    // ---- reduce-scatter over the 8 lanes of a row group: lane j ends with
    // the full sum of value index j (row 2g + (j>>2), head j&3).
    float r4[4];
    {
        const bool b2 = (j & 4) != 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float send = b2 ? a8[i] : a8[i + 4];
            const float keep = b2 ? a8[i + 4] : a8[i];
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
    pw[lane] = make_float2(p, p);  // index = row*4 + head, duplicated for fp32x2 math
    __syncwarp();
#pragma unroll
    for (int h = 0; h < GQA; h++) {
        const float2 a2 = make_float2(al[h], al[h]);
        O[h][0] = __fmul2_rn(O[h][0], a2);
        O[h][1] = __fmul2_rn(O[h][1], a2);
    }
    if (full)
        pv_rows<KV, true>(Vt, r0, rlo, rhi, lane, pw, O);
    else
        pv_rows<KV, false>(Vt, r0, rlo, rhi, lane, pw, O);
    __syncwarp();
}

// Same word format inside one GPU (the spread merge of split-KV ranges).
__device__ __forceinline__ void st_word_gpu(unsigned long long* p, float v, unsigned tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
template <bool SYS>
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
    unsigned long long w;
    if constexpr (SYS)
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

constexpr int SPREAD_MAXJ = 8;  // sources per thread in a spread gather

// Log-sum-exp state (max, weight, weighted sum) of one output value; the
// combination of two states is exact in the order it is applied.
__device__ __forceinline__ void lse_fold(float& M, float& W, float& A, float m2, float w2, float a2) {
    const float Mn = fmaxf(M, m2);
    if (Mn == -INFINITY) return;
    const float s1 = exp2f(M - Mn), s2 = exp2f(m2 - Mn);
    W = W * s1 + w2 * s2;
    A = A * s1 + a2 * s2;
    M = Mn;
}

// Spread gather: this thread reads the (o, lse) word pairs of sources
// j = sub, sub + tpv, ... < n at base + j*stride + off_o / off_l, waits
// (bounded) until each carries `tag`, and folds them; then the tpv lanes of
// its value (consecutive lanes of one warp) combine by shuffles.  Returns
// false, in every lane of the warp, when a word did not arrive within
// `limit` SM clocks.  Called by all 32 lanes of the warp.
template <bool SYS>
__device__ __forceinline__ bool spread_gather(const unsigned long long* base, size_t stride, int n,
                                              int sub, int tpv, bool active, size_t off_o,
                                              size_t off_l, unsigned tag, float& M, float& W,
                                              float& A, long long limit) {
    unsigned long long wo[SPREAD_MAXJ], wl[SPREAD_MAXJ];
    unsigned pend = 0;
#pragma unroll
    for (int u = 0; u < SPREAD_MAXJ; u++) {
        const int j = sub + u * tpv;
        wo[u] = wl[u] = 0ull;
        if (active && j < n) {
            wo[u] = ld_word<SYS>(base + (size_t)j * stride + off_o);
            wl[u] = ld_word<SYS>(base + (size_t)j * stride + off_l);
            pend |= 1u << u;
        }
    }
    bool ok = true;
    const long long t0 = clock64();
    while (true) {
#pragma unroll
        for (int u = 0; u < SPREAD_MAXJ; u++)
            if (((pend >> u) & 1u) && (unsigned)(wo[u] >> 32) == tag && (unsigned)(wl[u] >> 32) == tag)
                pend &= ~(1u << u);
        if (pend == 0) break;
        if (clock64() - t0 > limit) {
            ok = false;
            break;
        }
#pragma unroll
        for (int u = 0; u < SPREAD_MAXJ; u++) {
            if ((pend >> u) & 1u) {
                const int j = sub + u * tpv;
                wo[u] = ld_word<SYS>(base + (size_t)j * stride + off_o);
                wl[u] = ld_word<SYS>(base + (size_t)j * stride + off_l);
            }
        }
    }
    M = -INFINITY;
    W = 0.0f;
    A = 0.0f;
#pragma unroll
    for (int u = 0; u < SPREAD_MAXJ; u++) {
        const int j = sub + u * tpv;
        if (ok && active && j < n)
            lse_fold(M, W, A, __uint_as_float((unsigned)wl[u]), 1.0f, __uint_as_float((unsigned)wo[u]));
    }
    for (int o = 1; o < tpv; o <<= 1) {
        const float m2 = __shfl_xor_sync(FULL, M, o);
        const float w2 = __shfl_xor_sync(FULL, W, o);
        const float a2 = __shfl_xor_sync(FULL, A, o);
        lse_fold(M, W, A, m2, w2, a2);
    }
    // a value's sources are spread over tpv lanes of this warp: the value is
    // valid only if every one of them arrived, so one lane's timeout fails
    // the warp (the writer lane must not store a partial merge)
    return __all_sync(FULL, ok);
}

// Bounded wait of one warp until word base + j*stride carries `tag` for
// every j < n (lane l takes j = l, l + 32, ...).  A timeout is left to the
// gather that follows, which waits again and reports it.
template <bool SYS>
__device__ __forceinline__ void wait_sentinels(const unsigned long long* base, size_t stride, int n,
                                               int lane, unsigned tag, long long limit) {
    const long long t0 = clock64();
    for (int j = lane; j < n; j += 32) {
        const unsigned long long* p = base + (size_t)j * stride;
        while ((unsigned)(ld_word<SYS>(p) >> 32) != tag) {
            if (clock64() - t0 > limit) return;
        }
    }
}

// SPREAD: piece-mode launch whose split groups merge by the spread merge
// (a separate instantiation, so the linear-mode kernel keeps its own code).
// TC: bf16 paged cache consumed on the tensor cores (tcgen05): warp 4 issues
// S^T = K.Q^T and O^T = V^T.P^T per 128-row stage, warps 0-3 run the
// softmax (one thread per cache row for S, one per dimension for O).
template <typename KV, bool SPREAD, bool TC>
__global__ void __launch_bounds__(DecCfg<KV, TC>::NTHREADS, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __grid_constant__ DecodeParams P) {
    using C = DecCfg<KV, TC>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw;
    if constexpr (TC) smem += (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    KV* sK = reinterpret_cast<KV*>(smem + C::OFF_K);
    KV* sV = reinterpret_cast<KV*>(smem + C::OFF_V);
    float* sQ = reinterpret_cast<float*>(smem + C::OFF_QS);
    float* sRaw = reinterpret_cast<float*>(smem + C::OFF_RAW);    // q gains | k gains
    float* sRaw2 = reinterpret_cast<float*>(smem + C::OFF_RAW2);  // raw k | raw v
    KV* sNewK = reinterpret_cast<KV*>(smem + C::OFF_NEWK);
    KV* sNewV = reinterpret_cast<KV*>(smem + C::OFF_NEWV);
    float2* sP = reinterpret_cast<float2*>(smem + C::OFF_P);
    float* sW = reinterpret_cast<float*>(smem + C::OFF_WST);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::STAGES;
    // tensor-core path only
    uint64_t* sfull = empty + C::STAGES;  // S^T of a stage in tensor memory
    uint64_t* pfull = sfull + 2;          // P^T of a stage written (128 softmax threads)
    uint64_t* ofull = pfull + 2;          // O^T tile of a stage in tensor memory
    uint64_t* newrow = ofull + 2;         // the new token's row is in the cache
    uint64_t* drain = newrow + 1;         // every issued MMA complete
    volatile int* misc = reinterpret_cast<volatile int*>(smem + C::OFF_MISC);
    // per stage: first cache row and rows loaded (balanced schedule)
    volatile int* meta = reinterpret_cast<volatile int*>(smem + C::OFF_META);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x;

    if (warp == C::CWARPS) {
        // ================================================= producer
        // The producer initialises the stage barriers and starts streaming
        // at once; the consumers wait on named barrier 2 for the init only.
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < C::STAGES; s++) {
                mbar_init(&full[s], 1);
                // a stage is freed by the MMA commit (tensor cores) or by the
                // four warps of the group that consumed it (CUDA cores)
                mbar_init(&empty[s], TC ? 1 : C::CWARPS / 2);
            }
            if constexpr (TC) {
                for (int t = 0; t < 2; t++) {
                    mbar_init(&sfull[t], 1);
                    mbar_init(&pfull[t], 128);
                    mbar_init(&ofull[t], 1);
                }
                mbar_init(newrow, 2);
                mbar_init(drain, 1);
                misc[6] = -1;  // no end marker seen yet (balanced schedule)
            }
            fence_mbar_init();
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        __syncwarp();
        named_bar_arrive(2, C::NTHREADS);
        if (lane == 0) {
            // The producer reads cache rows only.  Unless the host found that
            // the kernel this launch depends on cannot write them (`early`),
            // it first waits for that kernel's writes to be visible; with
            // `early` the stream starts at once, overlapping the previous
            // kernel's tail.
            // A bound on the early rows (`early_rows`) is kept by the
            // balanced schedule only; the static schedules then wait first.
            const bool early = P.early && (P.dyn || P.early_rows == INT_MAX);
            if (!early) griddep_wait();
            const uint64_t pol = l2_policy_evict_first();
            int it = 0;
            bool dead = false;
            long long cur = 0;
            SegInfo s;
            int nnew = 0;  // ranges with a new token so far (phase of `newrow`)
            if (P.dyn) {
                // ---- balanced schedule: one range, units of one stage
                next_seg(P, c, cur, s);
                const int slot = P.slot[s.b];
                const DynPlan d = dyn_plan<TC>(P, s.b, C::TILE);
                const int i = s.slot - s.slot0, k = s.ncontrib;
                int u = i * C::STATIC_UNITS;
                const int u_st_end = min(u + C::STATIC_UNITS, d.n_claim);
                bool waited = !early, held = false;
                constexpr int ESZ = (int)sizeof(KV);
                // the next ring slot, once the consumers have freed it
                auto acquire = [&]() -> bool {
                    const int stage = it % C::STAGES;
                    const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                    return it < C::STAGES || mbar_wait(&empty[stage], ph ^ 1u);
                };
                // fills the acquired slot with rows [row0, row0 + n) of the
                // range's (sequence, kv head); n = 0 is an end marker
                auto fill = [&](int row0, int n, bool with_new) -> bool {
                    const int stage = it % C::STAGES;
                    if (with_new) {  // the consumers have appended the new row
                        if (!mbar_wait(newrow, 0u)) return false;
                        fence_proxy_async_global();
                    }
                    meta[2 * stage] = row0;
                    meta[2 * stage + 1] = n;
                    it++;
                    if (n == 0) {
                        mbar_arrive(&full[stage]);
                        return true;
                    }
                    mbar_arrive_expect_tx(&full[stage], (uint32_t)(2 * n * HD * ESZ));
                    uint8_t* kst = smem + C::OFF_K + stage * C::TILE * HD * ESZ;
                    uint8_t* vst = smem + C::OFF_V + stage * C::TILE * HD * ESZ;
                    for (int a = row0; a < row0 + n;) {
                        // a and the page ends are multiples of 16 rows
                        const int e = min(row0 + n, (a / P.page_tokens + 1) * P.page_tokens);
                        const long long row = paged_row(P, slot, s.kvh, a);
                        const uint32_t nb = (uint32_t)((e - a) * HD * ESZ);
                        const int so = (a - row0) * HD * ESZ;
                        bulk_load(kst + so, reinterpret_cast<const KV*>(P.kcache) + row * HD, nb,
                                  &full[stage], pol);
                        bulk_load(vst + so, reinterpret_cast<const KV*>(P.vcache) + row * HD, nb,
                                  &full[stage], pol);
                        a = e;
                    }
                    return true;
                };
                // rows a unit loads: whole 16-row MMA steps on the tensor cores
                auto unit_rows = [&](int row0) {
                    const int n = min(C::TILE, d.r_lim - row0);
                    return TC ? ((n + DEC_BOX - 1) & ~(DEC_BOX - 1)) : n;
                };
                while (!dead) {
                    int row0;
                    if (u < u_st_end) {
                        // one unit streams before the dependency wait: it fills
                        // the pipeline while the previous kernel finishes,
                        // without flooding the memory queues its merge waits on
                        row0 = d.a0 + u * C::TILE;
                        if (!waited && (u > i * C::STATIC_UNITS ||
                                        row0 + unit_rows(row0) > P.early_rows)) {
                            griddep_wait();
                            waited = true;
                        }
                        u++;
                        if (!acquire()) dead = true;
                    } else {
                        if (!waited) {  // the counters are reset by the kernel before
                            griddep_wait();
                            waited = true;
                        }
                        // claim, then wait for a free slot while the claim returns
                        const int cl = atomicAdd(P.claim + s.grp, 1);
                        if (!acquire()) {
                            dead = true;
                            break;
                        }
                        const int cu = k * C::STATIC_UNITS + cl;
                        if (cu >= d.n_claim) {
                            held = true;  // keep the slot for what follows
                            break;
                        }
                        row0 = d.a0 + cu * C::TILE;
                    }
                    if (dead || !fill(row0, unit_rows(row0), false)) dead = true;
                }
                if (!dead && TC && s.has_new) {  // the tail with the new token
                    if (!held && !acquire()) dead = true;
                    held = false;
                    if (!dead && !fill(d.tail0, (d.r_lim - d.tail0 + DEC_BOX - 1) & ~(DEC_BOX - 1), true))
                        dead = true;
                }
                // end markers: one per consumer sequence (on the CUDA cores
                // two warp groups take alternate stages)
                for (int e = 0; e < (TC ? 1 : 2) && !dead; e++) {
                    if (!held && !acquire()) dead = true;
                    held = false;
                    if (!dead && !fill(DYN_END, 0, false)) dead = true;
                }
                if (dead) atomicExch(P.err, DEV_ERR_TIMEOUT);
            } else if constexpr (TC) {
            while (!dead && next_seg(P, c, cur, s)) {
                // 128-row stages; the cache's 8-row blocks are already in
                // the operand layout, so rows [t0, hi) of a page are one
                // bulk copy per tensor.  The range includes the new token's
                // row, which the consumers append first (the stage holding
                // it is loaded after `newrow`).
                const int slot = P.slot[s.b];
                const int r_end = s.r1 + (s.has_new ? 1 : 0);
                const int lo_all = s.r0 & ~(DEC_BOX - 1);
                const int hi_all = (r_end + DEC_BOX - 1) & ~(DEC_BOX - 1);
                bool need_new = s.has_new != 0;
                for (int t0 = lo_all; t0 < r_end; t0 += C::TILE) {
                    const int stage = it % C::STAGES;
                    const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                    if (it >= C::STAGES && !mbar_wait(&empty[stage], ph ^ 1u)) {
                        atomicExch(P.err, DEV_ERR_TIMEOUT);
                        dead = true;
                        break;
                    }
                    const int hi = min(t0 + C::TILE, hi_all);
                    if (need_new && hi > s.r1) {
                        if (!mbar_wait(newrow, (uint32_t)nnew & 1u)) {
                            atomicExch(P.err, DEV_ERR_TIMEOUT);
                            dead = true;
                            break;
                        }
                        fence_proxy_async_global();
                        need_new = false;
                    }
                    mbar_arrive_expect_tx(&full[stage], (uint32_t)(2 * (hi - t0) * HD * 2));
                    uint8_t* kst = smem + C::OFF_K + stage * C::TILE_BYTES;
                    uint8_t* vst = smem + C::OFF_V + stage * C::TILE_BYTES;
                    for (int a = t0; a < hi;) {
                        // a and the page ends are multiples of 16 rows
                        const int e = min(hi, (a / P.page_tokens + 1) * P.page_tokens);
                        const long long row = paged_row(P, slot, s.kvh, a);
                        const uint32_t nb = (uint32_t)((e - a) * HD * 2);
                        const int so = (a - t0) * HD * 2;
                        bulk_load(kst + so, reinterpret_cast<const KV*>(P.kcache) + row * HD, nb,
                                  &full[stage], pol);
                        bulk_load(vst + so, reinterpret_cast<const KV*>(P.vcache) + row * HD, nb,
                                  &full[stage], pol);
                        a = e;
                    }
                    it++;
                }
                if (s.has_new) nnew++;
            }
            } else {
            while (!dead && next_seg(P, c, cur, s)) {
                const int slot = P.slot[s.b];
                // tiles start at the range's own 16-row-aligned start, so a
                // range of R rows takes ceil(R/64) tiles wherever it begins
                const int lo_all = s.r0 & ~(DEC_BOX - 1);
                const int hi_all = (s.r1 + DEC_BOX - 1) & ~(DEC_BOX - 1);
                for (int t0 = lo_all; t0 < s.r1; t0 += C::TILE) {
                    const int stage = it % C::STAGES;
                    const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
                    if (it >= C::STAGES && !mbar_wait(&empty[stage], ph ^ 1u)) {
                        atomicExch(P.err, DEV_ERR_TIMEOUT);
                        dead = true;
                        break;
                    }
                    const int hi = min(t0 + C::TILE, hi_all);
                    const uint32_t bytes = (uint32_t)((hi - t0) * HD * (int)sizeof(KV));
                    mbar_arrive_expect_tx(&full[stage], 2u * bytes);
                    const int doff = stage * C::TILE * HD;
                    if (P.cache_mode == CACHE_PAGED) {
                        // rows [t0, hi) are contiguous within a page; a tile
                        // that crosses a page boundary moves in two copies
                        const int pb = (t0 / P.page_tokens + 1) * P.page_tokens;
                        const int mid = min(hi, pb);
                        const long long row0 = paged_row(P, slot, s.kvh, t0);
                        const uint32_t b0 = (uint32_t)((mid - t0) * HD * (int)sizeof(KV));
                        bulk_load(sK + doff, reinterpret_cast<const KV*>(P.kcache) + row0 * HD, b0,
                                  &full[stage], pol);
                        bulk_load(sV + doff, reinterpret_cast<const KV*>(P.vcache) + row0 * HD, b0,
                                  &full[stage], pol);
                        if (mid < hi) {
                            const long long row1 = paged_row(P, slot, s.kvh, mid);
                            const int o1 = doff + (mid - t0) * HD;
                            const uint32_t b1 = bytes - b0;
                            bulk_load(sK + o1, reinterpret_cast<const KV*>(P.kcache) + row1 * HD, b1,
                                      &full[stage], pol);
                            bulk_load(sV + o1, reinterpret_cast<const KV*>(P.vcache) + row1 * HD, b1,
                                      &full[stage], pol);
                        }
                    } else {
                        const int xc = (P.kv0 + s.kvh) * HD;
                        for (int t = t0; t < hi; t += DEC_BOX) {
                            const int bo = doff + (t - t0) * HD;
                            tma_load_2d(sK + bo, &tmK, &full[stage], xc, t, pol);
                            tma_load_2d(sV + bo, &tmV, &full[stage], xc, t, pol);
                        }
                    }
                    it++;
                }
            }
            }
            // The next kernel's weights into L2 while this CTA's last stages
            // and the merge run (HBM is otherwise idle then).
            if (P.pf_base) {
                const int r0 = (int)(((long long)c * P.pf_rows) / gridDim.x);
                const int r1 = (int)(((long long)(c + 1) * P.pf_rows) / gridDim.x);
                if ((long long)P.pf_row_bytes == P.pf_ld_bytes) {
                    const uint8_t* a = P.pf_base + (long long)r0 * P.pf_ld_bytes;
                    long long left = (long long)(r1 - r0) * P.pf_row_bytes;
                    for (; left > 0; left -= 32768, a += 32768)
                        l2_prefetch(a, (uint32_t)min(left, 32768LL));
                } else {
                    for (int r = r0; r < r1; r++)
                        l2_prefetch(P.pf_base + (long long)r * P.pf_ld_bytes, (uint32_t)P.pf_row_bytes);
                }
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
    named_bar_sync(2, C::NTHREADS);  // stage barriers initialised
    int it = 0;
    long long cur = 0;
    SegInfo s;
    float2* pw = sP + warp * 32;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(misc + 4);
    if constexpr (TC) {
        if (warp == GQA) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_u32((const void*)tmem_slot)),
                         "r"(DTC_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        // rows 8-15 of Q^T and of both P^T buffers stay zero
        for (int i = tid; i < 3 * 128; i += C::NCONS) {
            const int op = i >> 7, hf = (i >> 6) & 1;
            *reinterpret_cast<uint4*>(smem + C::OFF_QT + op * C::OPB_BYTES + hf * 2048 + 1024 +
                                      (i & 63) * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        tc_fence_before();
    }
    griddep_wait();  // inputs written by the previous kernel are visible
    // Dependents may launch only once this kernel has passed its own wait:
    // then every kernel before the previous one has completed, which is
    // what lets a dependent decode stream cache rows before its wait.
    if (tid == 0) griddep_launch_dependents();
    while (next_seg(P, c, cur, s)) {
        const int b = s.b, kvh = s.kvh;
        const int hq0 = (P.kv0 + kvh) * GQA;
        const int slot = P.slot[b];

        // ---- prologue: one round of global loads, then norm + RoPE
        float2 fr = make_float2(0.0f, 0.0f);
        {
            const float* qsrc = P.q + (size_t)b * P.hq_total * HD + (size_t)hq0 * HD;
            const float2 qv = reinterpret_cast<const float2*>(qsrc)[tid];
            if (P.fused) fr = reinterpret_cast<const float2*>(P.inv_freq)[lane];
            float wv = 0.0f, kv = 0.0f;
            if (P.fused) wv = tid < HD ? P.q_norm_w[tid] : P.k_norm_w[tid - HD];
            if (s.has_new) {
                const size_t o = (size_t)b * P.nkv_total * HD + (size_t)(P.kv0 + kvh) * HD;
                kv = tid < HD ? P.k_new[o + tid] : P.v_new[o + tid - HD];
            }
            reinterpret_cast<float2*>(sQ)[tid] = qv;
            sRaw[tid] = wv;
            sRaw2[tid] = kv;
            // call numbers of the spread merge, read before this range
            // stores any word of the call
            if (tid == 0 && (SPREAD && s.ncontrib > 1)) {
                misc[1] = (int)*reinterpret_cast<volatile const unsigned*>(P.group_epoch + s.grp);
                if (P.peer_world > 0)
                    misc[2] = (int)*reinterpret_cast<volatile const unsigned*>(P.peer_epoch + kvh);
            }
        }
        named_bar_sync(1, C::NCONS);
        if (P.fused) {
            if (warp < GQA) {
                const float4 x = reinterpret_cast<const float4*>(sQ + warp * HD)[lane];
                const float4 w = reinterpret_cast<const float4*>(sRaw)[lane];
                reinterpret_cast<float4*>(sQ + warp * HD)[lane] =
                    norm_rope_lane(x, w, P.eps, P.pos[b], fr);
            } else if (warp == GQA && s.has_new) {
                // new token's k: normalised, rotated, stored in the cache
                // dtype, appended at pos and kept in shared memory for use
                const int pos = P.pos[b];
                const float4 x = reinterpret_cast<const float4*>(sRaw2)[lane];
                const float4 w = reinterpret_cast<const float4*>(sRaw + HD)[lane];
                const float4 kr = norm_rope_lane(x, w, P.eps, pos, fr);
                if (P.k_out) {
                    float* ko = P.k_out + (size_t)b * P.nkv_total * HD + (size_t)(P.kv0 + kvh) * HD;
                    reinterpret_cast<float4*>(ko)[lane] = kr;
                }
                store4<KV>(sNewK + 4 * lane, kr);
                const long long row = paged_row(P, slot, kvh, pos);
                store4<KV>(reinterpret_cast<KV*>(P.kcache) + kv_index<KV>(row, 4 * lane), kr);
                if constexpr (TC) {
                    // the producer loads this row with the range's last stage
                    fence_proxy_async_global();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(newrow);
                }
            } else if (warp == GQA + 1 && s.has_new) {
                const float4 vv = reinterpret_cast<const float4*>(sRaw2 + HD)[lane];
                store4<KV>(sNewV + 4 * lane, vv);
                const long long row = paged_row(P, slot, kvh, P.pos[b]);
                store4<KV>(reinterpret_cast<KV*>(P.vcache) + kv_index<KV>(row, 4 * lane), vv);
                if constexpr (TC) {
                    fence_proxy_async_global();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(newrow);
                }
            }
            named_bar_sync(1, C::NCONS);
        }

        const int h = tid >> 6, d = 2 * (tid & 63);
        float o0, o1, lse;
        if constexpr (TC) {
            // ---- Q^T operand: q in log2 units split into bf16 high and low
            // parts (rows h and h+4), so the scores carry fp32-accurate q
            {
                const int hq = tid >> 6, k = 2 * (tid & 63);
                const float x0 = sQ[hq * HD + k] * P.scale_log2e;
                const float x1 = sQ[hq * HD + k + 1] * P.scale_log2e;
                const __nv_bfloat162 hi2 = __floats2bfloat162_rn(x0, x1);
                const float2 hf = __bfloat1622float2(hi2);
                const __nv_bfloat162 lo2 = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
                *reinterpret_cast<__nv_bfloat162*>(smem + C::OFF_QT + opb_offset(hq, k)) = hi2;
                *reinterpret_cast<__nv_bfloat162*>(smem + C::OFF_QT + opb_offset(hq + GQA, k)) = lo2;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            named_bar_sync(1, C::NCONS);
            tc_fence_after();
            const uint32_t tm = *tmem_slot;
            const uint32_t sb = smem_u32(smem);
            // the range's stages: rows [lo_all, hi_all) in 16-row boxes, of
            // which [r0, r_end) count (r_end includes the new token's row)
            const int r_end = s.r1 + (s.has_new ? 1 : 0);
            const int lo_all = s.r0 & ~(DEC_BOX - 1);
            const int hi_all = (r_end + DEC_BOX - 1) & ~(DEC_BOX - 1);
            const int ntiles = r_end > lo_all ? (r_end - lo_all + C::TILE - 1) / C::TILE : 0;
            const int it0 = it;
            const bool direct = SPREAD && s.ncontrib > 1;
            // balanced schedule: stages carry their rows in `meta` and end
            // with a marker; otherwise ntiles stages from lo_all
            DynPlan dp;
            if (P.dyn) dp = dyn_plan<true>(P, b, C::TILE);
            volatile int* end_stage = misc + 6;  // stage index of the end marker
            if (warp == GQA) {
                // ================================== MMA issuer (one thread)
                if (lane == 0 && (P.dyn || ntiles > 0)) {
                    bool dead = false;
                    auto issue_s = [&](int g) {
                        // S^T (128 rows x 16) = K (128 x 128, K-major) . Q^T
                        const uint32_t kb = sb + C::OFF_K + (g % C::STAGES) * C::TILE_BYTES;
                        const uint32_t qb = sb + C::OFF_QT;
                        const uint32_t dcol = tm + DTC_S_COL + (uint32_t)(g & 1) * 16u;
#pragma unroll
                        for (int kk = 0; kk < HD / 16; kk++) {
                            const uint32_t koff = (kk & 3) * 32;
                            // K: 8-row groups 2048 B apart, dim-halves 1024 B
                            tc_mma_ss(dcol, smem_desc(kb + (kk >> 2) * 1024 + koff, 16, 2048),
                                      smem_desc(qb + (kk >> 2) * 2048 + koff, 16, 1024), IDESC_DS,
                                      kk > 0 ? 1u : 0u);
                        }
                        tc_commit(&sfull[g & 1]);
                    };
                    // stage g (the j-th of the range): is it real, and how many
                    // rows does it hold (balanced: from its metadata, after
                    // its full barrier; static: from the range)
                    auto rows_of = [&](int j, int g) -> int {
                        if (P.dyn) {
                            const int st = g % C::STAGES;
                            return meta[2 * st] == DYN_END ? 0 : meta[2 * st + 1];
                        }
                        const int t0 = lo_all + j * C::TILE;
                        return min(t0 + C::TILE, hi_all) - t0;
                    };
                    // end marker: the softmax threads learn it from end_stage
                    // behind the stage's S barrier
                    auto signal_end = [&](int g) {
                        *end_stage = g;
                        mbar_arrive(&sfull[g & 1]);
                    };
                    int nrows = 0;
                    if (mbar_wait(&full[it0 % C::STAGES], (uint32_t)(it0 / C::STAGES) & 1u)) {
                        tc_fence_after();
                        nrows = rows_of(0, it0);
                        if (nrows > 0)
                            issue_s(it0);
                        else
                            signal_end(it0);
                    } else {
                        dead = true;
                    }
                    for (int j = 0; nrows > 0 && !dead; j++) {
                        const int g = it0 + j;
                        int nrows_next = 0;
                        if (P.dyn || j + 1 < ntiles) {
                            // S of the next stage goes first; its buffer was
                            // freed by the softmax of stage g-1
                            const int gn = g + 1;
                            if (!mbar_wait(&full[gn % C::STAGES], (uint32_t)(gn / C::STAGES) & 1u)) {
                                dead = true;
                                break;
                            }
                            tc_fence_after();
                            nrows_next = rows_of(j + 1, gn);
                            if (nrows_next > 0)
                                issue_s(gn);
                            else if (P.dyn)
                                signal_end(gn);
                        }
                        if (!mbar_wait(&pfull[g & 1], (uint32_t)(g >> 1) & 1u)) {
                            dead = true;
                            break;
                        }
                        tc_fence_after();
                        // O^T tile (128 dims x 16) = V^T (MN-major) . P^T over
                        // the loaded 16-row steps only
                        const int nk = nrows / DEC_BOX;
                        const uint32_t vb = sb + C::OFF_V + (g % C::STAGES) * C::TILE_BYTES;
                        const uint32_t pb = sb + C::OFF_PT + (uint32_t)(g & 1) * C::OPB_BYTES;
                        const uint32_t dcol = tm + DTC_O_COL + (uint32_t)(g & 1) * 16u;
                        // V read MN-major: dim-halves 1024 B apart (LBO), 8-row
                        // groups 2048 B apart (SBO), 16 rows per step
                        for (int kk = 0; kk < nk; kk++)
                            tc_mma_ss(dcol, smem_desc(vb + kk * 4096, 1024, 2048),
                                      smem_desc(pb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024),
                                      IDESC_DPV, kk > 0 ? 1u : 0u);
                        tc_commit(&ofull[g & 1]);
                        tc_commit(&empty[g % C::STAGES]);
                        nrows = nrows_next;
                    }
                    if (dead) atomicExch(P.err, DEV_ERR_TIMEOUT);
                }
                __syncwarp();
            } else if (warp < GQA) {
                // ================================== softmax (128 threads)
                // thread tid: cache row lo_all + 128 j + tid of stage j for
                // the scores, dimension tid for the output
                float mh[GQA], lsum[GQA], Oh[GQA], al_prev[GQA];
#pragma unroll
                for (int q = 0; q < GQA; q++) {
                    mh[q] = -INFINITY;
                    lsum[q] = 0.0f;
                    Oh[q] = 0.0f;
                    al_prev[q] = 1.0f;
                }
                const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
                bool ok = true;
                uint8_t* ptb = smem + C::OFF_PT;
                float* red = sW + C::W_RED;
                // O <- O * alpha(g) + O^T tile of stage g
                auto fold = [&](int g) {
                    bool got = ok && mbar_wait(&ofull[g & 1], (uint32_t)(g >> 1) & 1u);
                    got = __all_sync(FULL, got);
                    if (!got) {
                        ok = false;
                        return;
                    }
                    tc_fence_after();
                    uint32_t r[8];
                    Q3A_TC_LD8(tm + lane_base + DTC_O_COL + (uint32_t)(g & 1) * 16u, r);
                    tc_wait_ld();
#pragma unroll
                    for (int q = 0; q < GQA; q++)
                        Oh[q] = fmaf(Oh[q], al_prev[q], __uint_as_float(r[q]) + __uint_as_float(r[q + GQA]));
                };
                int nt = 0;  // real stages of the range
                for (int j = 0; P.dyn || j < ntiles; j++) {
                    const int g = it0 + j, bf = g & 1;
                    bool got = ok && mbar_wait(&sfull[bf], (uint32_t)(g >> 1) & 1u);
                    got = __all_sync(FULL, got);
                    int row0 = lo_all + j * C::TILE, vlo = s.r0, vhi = r_end, nld = C::TILE;
                    if (P.dyn && got) {
                        if (*end_stage == g) break;  // end marker
                        // the stage's metadata: its full barrier (completed
                        // before its S) orders the producer's stores before
                        // these loads
                        const int st = g % C::STAGES;
                        got = mbar_wait(&full[st], (uint32_t)(g / C::STAGES) & 1u);
                        row0 = meta[2 * st];
                        nld = meta[2 * st + 1];
                        vlo = dp.tb;
                        vhi = dp.r_lim;
                    }
                    got = __all_sync(FULL, got);
                    nt = j + 1;
                    uint32_t r[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
                    if (got) {
                        tc_fence_after();
                        Q3A_TC_LD8(tm + lane_base + DTC_S_COL + (uint32_t)bf * 16u, r);
                        tc_wait_ld();
                    }
                    const int key = row0 + tid;
                    const bool valid = got && tid < nld && key >= vlo && key < vhi;
                    float sc[GQA], mx[GQA];
                    bool grow = false;  // a score above the running maximum + 8
#pragma unroll
                    for (int q = 0; q < GQA; q++) {
                        sc[q] = valid ? __uint_as_float(r[q]) + __uint_as_float(r[q + GQA]) : -INFINITY;
                        mx[q] = sc[q];
                        grow = grow || (sc[q] > mh[q] + 8.0f) || (valid && mh[q] == -INFINITY);
                    }
                    // Lazy rescaling: while every score of the stage stays
                    // within 2^8 of the running maximum (weights <= 256),
                    // the maximum is kept and the stage's cross-warp maximum
                    // is skipped; one vote, which also carries every thread's
                    // wait status, picks the path
                    const bool keep = named_bar_red_and(3, 128, got && !grow);
                    if (!keep) {
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                            for (int q = 0; q < GQA; q++) mx[q] = fmaxf(mx[q], __shfl_xor_sync(FULL, mx[q], o));
                        if (lane == 0)
#pragma unroll
                            for (int q = 0; q < GQA; q++) red[bf * 16 + warp * 4 + q] = mx[q];
                        // the stage's maxima of all 4 warps; a failed wait
                        // anywhere stops all 4 warps together
                        if (!named_bar_red_and(3, 128, got)) {
                            ok = false;
                            break;
                        }
                    }
                    float al[GQA];
#pragma unroll
                    for (int q = 0; q < GQA; q++) {
                        const float tmx = keep ? -INFINITY
                                               : fmaxf(fmaxf(red[bf * 16 + q], red[bf * 16 + 4 + q]),
                                                       fmaxf(red[bf * 16 + 8 + q], red[bf * 16 + 12 + q]));
                        const float mn = fmaxf(mh[q], tmx);
                        const bool none = mn == -INFINITY;
                        al[q] = none ? 1.0f : exp2f(mh[q] - mn);
                        const float pq = none ? 0.0f : exp2f(sc[q] - mn);
                        lsum[q] = fmaf(lsum[q], al[q], pq);
                        mh[q] = mn;
                        // P^T: high and low bf16 parts of p for this row
                        const __nv_bfloat16 ph = __float2bfloat16_rn(pq);
                        const __nv_bfloat16 pl = __float2bfloat16_rn(pq - __bfloat162float(ph));
                        *reinterpret_cast<__nv_bfloat16*>(ptb + bf * C::OPB_BYTES + opb_offset(q, tid)) = ph;
                        *reinterpret_cast<__nv_bfloat16*>(ptb + bf * C::OPB_BYTES + opb_offset(q + GQA, tid)) = pl;
                    }
                    fence_proxy_async_smem();
                    tc_fence_before();
                    mbar_arrive(&pfull[bf]);
                    // the previous stage's O^T tile (its PV ran meanwhile)
                    if (j > 0) fold(g - 1);
#pragma unroll
                    for (int q = 0; q < GQA; q++) al_prev[q] = al[q];
                }
                // row sums over the 128 threads while the last PV runs
                float* lred = sW + C::W_LSUM;
#pragma unroll
                for (int q = 0; q < GQA; q++) {
                    float v = lsum[q];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
                    if (lane == 0) lred[warp * 4 + q] = v;
                }
                named_bar_sync(3, 128);
                if (ok && nt > 0) fold(it0 + nt - 1);
                // a spread-merged range stores its words from here (thread
                // tid holds dimension tid of the 4 heads); otherwise the
                // outputs go through shared memory to the 256-thread layout
                unsigned long long* mine = P.words + (size_t)s.slot * PART_STRIDE;
                const unsigned tag = (((unsigned)misc[1] + 1u) << 8) | ((unsigned)s.grp & 0xFFu);
#pragma unroll
                for (int q = 0; q < GQA; q++) {
                    const float L = lred[q] + lred[4 + q] + lred[8 + q] + lred[12 + q];
                    // a range that attended no row contributes o = 0, lse = -inf
                    const float oq = L > 0.0f ? Oh[q] / L : 0.0f;
                    const float lq = L > 0.0f ? mh[q] + log2f(L) : -INFINITY;
                    if (direct) {
                        st_word_gpu(mine + q * HD + tid, oq, tag);
                        if (tid == q) st_word_gpu(mine + GQA * HD + q, lq, tag);
                    } else {
                        sW[q * HD + tid] = oq;
                        if (tid == q) sW[C::W_LSE + q] = lq;
                    }
                }
                if (!ok) atomicExch(P.err, DEV_ERR_TIMEOUT);
            }
            it += ntiles;
            if (!direct) {
                tc_fence_before();
                named_bar_sync(1, C::NCONS);
                tc_fence_after();
                o0 = sW[h * HD + d];
                o1 = sW[h * HD + d + 1];
                lse = sW[C::W_LSE + h];
            } else {
                o0 = o1 = lse = 0.0f;  // unused: the words are stored
            }
        } else {
            float2 qr[GQA][8];
            load_q_regs<KV>(sQ, lane, P.scale_log2e, qr);
            float m[GQA] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            float lpart = 0.0f;
            float2 O[GQA][2];
#pragma unroll
            for (int hh = 0; hh < GQA; hh++) O[hh][0] = O[hh][1] = make_float2(0.0f, 0.0f);

            // two groups of four warps take alternate stages; warp wl of a
            // group owns rows 8 wl .. 8 wl + 7 of each of its stages
            const int wg = warp >> 2, wl = warp & 3;
            bool dead = false;
            if (P.dyn) {
                const DynPlan dp = dyn_plan<false>(P, b, C::TILE);
                for (int j = wg;; j += 2) {
                    const int g = it + j, stage = g % C::STAGES;
                    if (!mbar_wait(&full[stage], (uint32_t)(g / C::STAGES) & 1u)) {
                        dead = true;
                        break;
                    }
                    const int row0 = meta[2 * stage];
                    if (row0 == DYN_END) break;
                    const int lo = max(dp.tb - row0, 0), hi = min(dp.r_lim - row0, C::TILE);
                    process_rows<KV>(sK + stage * C::TILE * HD, sV + stage * C::TILE * HD, lo, hi, wl,
                                     lane, qr, m, lpart, O, pw);
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
            } else {
                const int lo_all = s.r0 & ~(DEC_BOX - 1);
                const int ntiles = s.r1 > lo_all ? (s.r1 - lo_all + C::TILE - 1) / C::TILE : 0;
                for (int j = wg; j < ntiles; j += 2) {
                    const int g = it + j, stage = g % C::STAGES;
                    if (!mbar_wait(&full[stage], (uint32_t)(g / C::STAGES) & 1u)) {
                        dead = true;
                        break;
                    }
                    const int t0 = lo_all + j * C::TILE;
                    const int lo = max(s.r0 - t0, 0), hi = min(s.r1 - t0, C::TILE);
                    process_rows<KV>(sK + stage * C::TILE * HD, sV + stage * C::TILE * HD, lo, hi, wl,
                                     lane, qr, m, lpart, O, pw);
                    if (lane == 0) mbar_arrive(&empty[stage]);
                }
                it += ntiles;
            }
            // a failed wait voids the result (the error word tells the host);
            // every warp still takes the barriers below
            if (dead) atomicExch(P.err, DEV_ERR_TIMEOUT);
            // the new token from shared memory: warp 0 (rows 8 warp .. of a
            // one-row tile)
            if (s.has_new) process_rows<KV>(sNewK, sNewV, 0, 1, warp, lane, qr, m, lpart, O, pw);

            // ---- merge the 8 warp states of this range
            float lsum = lpart;
            lsum += __shfl_xor_sync(FULL, lsum, 4);
            lsum += __shfl_xor_sync(FULL, lsum, 8);
            lsum += __shfl_xor_sync(FULL, lsum, 16);
            {
                float* ws = sW + warp * C::WST;
#pragma unroll
                for (int hh = 0; hh < GQA; hh++)
                    *reinterpret_cast<float4*>(ws + hh * HD + 4 * lane) =
                        make_float4(O[hh][0].x, O[hh][0].y, O[hh][1].x, O[hh][1].y);
                if (lane < 4) {
                    ws[GQA * HD + lane] = sel4(m, lane);
                    ws[GQA * HD + 4 + lane] = lsum;
                }
            }
            named_bar_sync(1, C::NCONS);
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < C::CWARPS; w++) M = fmaxf(M, sW[w * C::WST + GQA * HD + h]);
            float L = 0.0f;
            o0 = 0.0f;
            o1 = 0.0f;
#pragma unroll
            for (int w = 0; w < C::CWARPS; w++) {
                const float mw = sW[w * C::WST + GQA * HD + h];
                const float sc = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
                L = fmaf(sW[w * C::WST + GQA * HD + 4 + h], sc, L);
                o0 = fmaf(sW[w * C::WST + h * HD + d], sc, o0);
                o1 = fmaf(sW[w * C::WST + h * HD + d + 1], sc, o1);
            }
            // a range that attended no row (possible in the balanced schedule)
            // contributes o = 0, lse = -inf
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            o0 *= inv;
            o1 *= inv;
            lse = L > 0.0f ? M + log2f(L) : -INFINITY;
        }

        bool write_out = true;
        if ((SPREAD && s.ncontrib > 1)) {
            // Spread merge.  Every range of the group stores its (o, lse) as
            // tagged words into its own slot and then merges one slice of
            // the group's 512 outputs from all slots: no ticket round trip,
            // and no single CTA loads every partial.  Ranges wait for one
            // another, which piece mode allows (one CTA per SM, all
            // resident).  The tag is (call number of the group << 8 | group).
            const unsigned gep = (unsigned)misc[1] + 1u;
            const unsigned tag = (gep << 8) | ((unsigned)s.grp & 0xFFu);
            if constexpr (!TC) {  // the tensor-core softmax threads stored them
                unsigned long long* mine = P.words + (size_t)s.slot * PART_STRIDE;
                st_word_gpu(mine + h * HD + d, o0, tag);
                st_word_gpu(mine + h * HD + d + 1, o1, tag);
                if ((tid & 63) == 0) st_word_gpu(mine + GQA * HD + h, lse, tag);
            }
            const int k = s.ncontrib, i = s.slot - s.slot0;
            const int v0 = i * (GQA * HD) / k, nv = (i + 1) * (GQA * HD) / k - v0;
            int tpv = 32;
            while (tpv > 1 && tpv * nv > C::NCONS) tpv >>= 1;
            const int vi = tid / tpv, sub = tid & (tpv - 1);
            const bool act = vi < nv;
            const int v = v0 + (act ? vi : 0), vh = v >> 7, vd = v & (HD - 1);
            // one warp first waits for the last-stored word of every range
            // (head 3's lse), so the full gather below is normally issued
            // once instead of being polled by every thread
            if (warp == 0)
                wait_sentinels<false>(P.words + (size_t)s.slot0 * PART_STRIDE + GQA * HD + GQA - 1,
                                      PART_STRIDE, k, lane, tag, P.wait_limit);
            named_bar_sync(1, C::NCONS);
            float Mv, Wv, Av;
            bool ok = spread_gather<false>(P.words + (size_t)s.slot0 * PART_STRIDE, PART_STRIDE, k,
                                           sub, tpv, act, v, GQA * HD + vh, tag, Mv, Wv, Av,
                                           P.wait_limit);
            float ov = Av / Wv, lv = Mv + log2f(Wv);
            const int gh = hq0 + vh;
            unsigned pep = 0;
            if (P.peer_world > 0) {
                // then the same exchange across ranks, slice by slice: the
                // owner of each value stores it (and the owner of a head's
                // first value that head's lse) into row `rank` of every
                // rank's receive buffer, and every slice merges its values
                // from all ranks' rows
                const int Wr = P.peer_world, R = P.peer_rank;
                const size_t row = (size_t)P.peer_row;
                pep = (unsigned)misc[2] + 1u;
                const int par = (int)(pep & 1u);
                if (ok && act && sub == 0) {
                    for (int r = 0; r < Wr; r++) {
                        unsigned long long* dst = reinterpret_cast<unsigned long long*>(P.peer_recv[r]) +
                                                  ((size_t)par * Wr + R) * row;
                        st_word_sys(dst + (size_t)gh * HD + vd, ov, pep);
                        if (vd == 0) st_word_sys(dst + (size_t)P.hq_total * HD + gh, lv, pep);
                    }
                }
                const unsigned long long* src =
                    reinterpret_cast<const unsigned long long*>(P.peer_recv[R]) + (size_t)par * Wr * row;
                if (warp == 0)
                    wait_sentinels<true>(src + (size_t)P.hq_total * HD + hq0 + (v0 >> 7), row, Wr, lane,
                                         pep, P.wait_limit);
                named_bar_sync(1, C::NCONS);
                ok = spread_gather<true>(src, row, Wr, sub, tpv, act && ok, (size_t)gh * HD + vd,
                                         (size_t)P.hq_total * HD + gh, pep, Mv, Wv, Av,
                                         P.wait_limit) && ok;
                ov = Av / Wv;
                lv = Mv + log2f(Wv);
            }
            if (!ok) atomicExch(P.err, DEV_ERR_TIMEOUT);
            if (ok && act && sub == 0) {
                P.xb[(size_t)b * P.hq_total * HD + (size_t)gh * HD + vd] = ov;
                if (P.lse_out && vd == 0) P.lse_out[(size_t)b * P.hq_total + gh] = lv;
            }
            // the rotated q goes back slice by slice once every range of
            // the group has stored its words (so has read the raw q)
            if (P.fused && P.q_out && P.peer_world == 0 && tid < nv)
                P.q_out[(size_t)b * P.hq_total * HD + (size_t)hq0 * HD + v0 + tid] = sQ[v0 + tid];
            if (i == 0 && tid == 0) {
                // every range of the group has read the call numbers by now,
                // and has stopped claiming units
                *reinterpret_cast<volatile unsigned*>(P.group_epoch + s.grp) = gep;
                if (P.dyn) P.claim[s.grp] = 0;
                if (P.peer_world > 0) *reinterpret_cast<volatile unsigned*>(P.peer_epoch + kvh) = pep;
            }
            write_out = false;
        } else if (s.ncontrib > 1) {
            float* ps = P.partials + (long long)s.slot * PART_STRIDE;
            *reinterpret_cast<float2*>(ps + h * HD + d) = make_float2(o0, o1);
            if ((tid & 63) == 0) ps[GQA * HD + h] = lse;
            named_bar_sync(1, C::NCONS);
            if (tid == 0) {
                const int old = atom_add_acq_rel(&P.counters[s.grp], 1);
                misc[0] = (old == s.ncontrib - 1) ? 1 : 0;
            }
            named_bar_sync(1, C::NCONS);
            write_out = misc[0] != 0;
            if (write_out) {
                // every contributor's (lse, o) in one round of L2 loads per
                // chunk of 32, merged with a running log-sum-exp
                const float* pb = P.partials + (long long)s.slot0 * PART_STRIDE;
                float Mx = -INFINITY, W = 0.0f, a0 = 0.0f, a1 = 0.0f;
                for (int base = 0; base < s.ncontrib; base += 32) {
                    float lj[32];
                    float2 oj[32];
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        lj[jj] = -INFINITY;
                        oj[jj] = make_float2(0.0f, 0.0f);
                        if (base + jj < s.ncontrib) {
                            const float* pj = pb + (long long)(base + jj) * PART_STRIDE;
                            lj[jj] = __ldcg(pj + GQA * HD + h);
                            oj[jj] = __ldcg(reinterpret_cast<const float2*>(pj + h * HD + d));
                        }
                    }
                    float mc = Mx;
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) mc = fmaxf(mc, lj[jj]);
                    const float rs = (Mx == -INFINITY) ? 0.0f : exp2f(Mx - mc);
                    W *= rs;
                    a0 *= rs;
                    a1 *= rs;
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        const float wj = (lj[jj] == -INFINITY) ? 0.0f : exp2f(lj[jj] - mc);
                        W += wj;
                        a0 = fmaf(wj, oj[jj].x, a0);
                        a1 = fmaf(wj, oj[jj].y, a1);
                    }
                    Mx = mc;
                }
                const float iw = 1.0f / W;
                o0 = a0 * iw;
                o1 = a1 * iw;
                lse = Mx + log2f(W);
                if (tid == 0) P.counters[s.grp] = 0;
            }
        }
        if (write_out && P.peer_world > 0) {
            // Sequence-shard exchange over peer memory.  This CTA holds this
            // rank's result for KV head kvh.  Every value of it (o of the 4
            // query heads, their lse) goes as a (value, call) word into row
            // `rank` of every rank's receive buffer (the half of this call's
            // parity; a rank is at most one call ahead); then each thread
            // waits for its own words from every rank and merges them.
            const int W = P.peer_world, R = P.peer_rank, row = P.peer_row;
            const int gh = hq0 + h;
            const unsigned ep = *reinterpret_cast<volatile const unsigned*>(P.peer_epoch + kvh) + 1u;
            const int par = (int)(ep & 1u);
            const size_t my_row = ((size_t)par * W + R) * row;
            for (int r = 0; r < W; r++) {
                unsigned long long* dst = reinterpret_cast<unsigned long long*>(P.peer_recv[r]) + my_row;
                st_word_sys(dst + gh * HD + d, o0, ep);
                st_word_sys(dst + gh * HD + d + 1, o1, ep);
                if ((tid & 63) == 0) st_word_sys(dst + P.hq_total * HD + gh, lse, ep);
            }
            const unsigned long long* src =
                reinterpret_cast<const unsigned long long*>(P.peer_recv[R]) + (size_t)par * W * row;
            // loads for four ranks' words at a time are in flight together;
            // words not there yet are polled (bounded)
            float lr[PEER_MAX], x0[PEER_MAX], x1[PEER_MAX];
            bool ok = true;
            for (int r0 = 0; r0 < W; r0 += 4) {
                unsigned long long wl[4], w0[4], w1[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (r0 + u < W) {
                        const unsigned long long* sr = src + (size_t)(r0 + u) * row;
                        wl[u] = ld_word_sys(sr + P.hq_total * HD + gh);
                        w0[u] = ld_word_sys(sr + gh * HD + d);
                        w1[u] = ld_word_sys(sr + gh * HD + d + 1);
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int r = r0 + u;
                    if (r < W) {
                        const unsigned long long* sr = src + (size_t)r * row;
                        lr[r] = __uint_as_float((unsigned)wl[u]);
                        x0[r] = __uint_as_float((unsigned)w0[u]);
                        x1[r] = __uint_as_float((unsigned)w1[u]);
                        if ((unsigned)(wl[u] >> 32) != ep) ok = ok && wait_word(sr + P.hq_total * HD + gh, ep, lr[r], P.wait_limit);
                        if ((unsigned)(w0[u] >> 32) != ep) ok = ok && wait_word(sr + gh * HD + d, ep, x0[r], P.wait_limit);
                        if ((unsigned)(w1[u] >> 32) != ep) ok = ok && wait_word(sr + gh * HD + d + 1, ep, x1[r], P.wait_limit);
                    }
                }
            }
            if (!ok) atomicExch(P.err, DEV_ERR_TIMEOUT);
            float Mx = -INFINITY;
            for (int r = 0; r < W; r++) Mx = fmaxf(Mx, ok ? lr[r] : -INFINITY);
            float Wt = 0.0f, a0 = 0.0f, a1 = 0.0f;
            for (int r = 0; r < W; r++) {
                const float wr = (!ok || lr[r] == -INFINITY) ? 0.0f : exp2f(lr[r] - Mx);
                Wt += wr;
                a0 = fmaf(wr, x0[r], a0);
                a1 = fmaf(wr, x1[r], a1);
            }
            if (ok) *reinterpret_cast<float2*>(P.xb + (size_t)gh * HD + d) = make_float2(a0 / Wt, a1 / Wt);
            named_bar_sync(1, C::NCONS);
            if (tid == 0) *reinterpret_cast<volatile unsigned*>(P.peer_epoch + kvh) = ep;
            write_out = false;
        }
        // a one-range group of the balanced schedule resets its unit
        // counter (its producer has stopped claiming: the end marker came last)
        if (P.dyn && s.ncontrib == 1 && tid == 0) P.claim[s.grp] = 0;
        if (write_out) {
            float* xo = P.xb + (size_t)b * P.hq_total * HD + (size_t)(hq0 + h) * HD + d;
            *reinterpret_cast<float2*>(xo) = make_float2(o0, o1);
            if (P.lse_out && (tid & 63) == 0) P.lse_out[(size_t)b * P.hq_total + hq0 + h] = lse;
            if (P.fused && P.q_out) {
                float* qo = P.q_out + (size_t)b * P.hq_total * HD + (size_t)hq0 * HD;
                reinterpret_cast<float2*>(qo)[tid] = reinterpret_cast<const float2*>(sQ)[tid];
            }
        }
        named_bar_sync(1, C::NCONS);
    }
    if constexpr (TC) {
        // teardown: every MMA issued has completed (bounded wait) before the
        // allocating warp frees tensor memory
        if (warp == GQA) {
            if (lane == 0) {
                tc_commit(drain);
                if (!mbar_wait(drain, 0u)) atomicExch(P.err, DEV_ERR_TIMEOUT);
            }
            __syncwarp();
        }
        tc_fence_before();
        named_bar_sync(1, C::NCONS);
        tc_fence_after();
        if (warp == GQA) {
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot),
                         "r"(DTC_COLS)
                         : "memory");
        }
    }
}

template <typename KV, bool SPREAD, bool TC>
static cudaError_t launch_decode_t(const DecodeParams& p, const CUtensorMap& tmK,
                                   const CUtensorMap& tmV, cudaStream_t st) {
    using C = DecCfg<KV, TC>;
    cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(decode_kernel<KV, SPREAD, TC>),
                                     C::SMEM);
    if (e != cudaSuccess) return e;
    // programmatic dependent launch: scheduled while the previous kernel of
    // the stream finishes; the kernel waits for it before touching memory
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_ctas);
    cfg.blockDim = dim3(C::NTHREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_kernel<KV, SPREAD, TC>, tmK, tmV, p);
}

cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          bool bf16, cudaStream_t st) {
    // the spread merge needs every range resident at once: piece mode only
    const bool spread = p.spread && p.n_pieces > 0;
    // bf16 caches are the context's paged caches in the operand layout and
    // are consumed on the tensor cores; fp32 caches on the CUDA cores
    if (bf16 != (p.tc != 0) || (p.tc && p.cache_mode != CACHE_PAGED)) return cudaErrorInvalidValue;
    if (p.tc)
        return spread ? launch_decode_t<__nv_bfloat16, true, true>(p, tmK, tmV, st)
                      : launch_decode_t<__nv_bfloat16, false, true>(p, tmK, tmV, st);
    return spread ? launch_decode_t<float, true, false>(p, tmK, tmV, st)
                  : launch_decode_t<float, false, false>(p, tmK, tmV, st);
}

int decode_smem_bytes(bool bf16) {
    return bf16 ? DecCfg<__nv_bfloat16>::SMEM : DecCfg<float>::SMEM;
}

}  // namespace q3a
