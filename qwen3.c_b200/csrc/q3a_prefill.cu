// q3a_prefill.cu -- causal prefill attention on the sm_100a tensor cores.
//
// The reference processes a prompt one token at a time through the decode
// path (qwen3-8b/cpu/main.c:1481-1499), so prompt row s attends to cache
// positions 0..pos0+s.  Here all rows of a prompt run as one causal flash
// attention with tcgen05.mma (kind::f16: bf16 operands, fp32 accumulators in
// tensor memory):
//
//  * Work item = (KV head g, pair of query heads 4g+2p, 4g+2p+1, 128 query
//    rows).  The two query heads of an item share every K/V tile (GQA).
//    Items are dealt to a persistent grid (one CTA per SM) in a snake order
//    of decreasing causal length.
//  * Warp 0 streams Q (3-D TMA, 128B swizzle) and 128-key K/V tiles of the
//    paged bf16 cache through a 2-stage ring.  The cache keeps 8-row blocks
//    in the 128B-swizzled operand layout, so a 64-key run inside a page is
//    one 16 KB bulk copy (cp.async.bulk) per tensor.
//  * Warp 1 issues every MMA from one lane.  Per head t and key tile j:
//    S_t = Q_t.K_j^T (M128 N128 K128, both operands in shared memory) into
//    the head's 128 tensor-memory columns; once the softmax has replaced S_t
//    by P_t (bf16, packed into the first 64 of those columns),
//    O_t += P_t.V_j (M128 N128 K128, A read from tensor memory, B = V from
//    shared memory).  S_t(j+1) overwrites P_t(j), so it is issued once
//    PV_t(j) has completed; the two heads alternate on the tensor core while
//    the other head runs its softmax.
//  * Warps 4-7 / 8-11 are the softmax warpgroups of the two heads: thread r
//    owns query row r, reads its 128 scores with tcgen05.ld, applies the
//    causal mask and an online softmax in log2 units (the reference scale
//    1/sqrt(128) folded with log2 e), writes P back with tcgen05.st, and
//    rescales O in tensor memory only when the running maximum grows by more
//    than 2^8 (the final division uses the same reference maximum, so the
//    result is exact).
//  * The epilogue divides O by the row sum and stores the row (fp32 or bf16).
// Per key tile and head the tensor core reads 64 KB of Q+K and 32 KB of V
// from shared memory for 8.4 MFLOP (N = 128 on both MMAs keeps the
// shared-memory read rate within its bandwidth); P never touches shared
// memory.  Tensor memory: 512 columns (per head 128 S/P + 128 O).
#include "q3a_common.cuh"
#include "q3a_internal.h"
#include "q3a_tcgen05.cuh"

namespace q3a {

namespace pf {

constexpr int QT = 128;        // query rows per head tile
constexpr int KT = 128;        // keys per K/V tile
constexpr int STAGES = 2;
constexpr int NTHREADS = 384;  // 12 warps
constexpr int Q_TILE_BYTES = QT * HD * 2;          // 32 KB: 2 dim-blocks of [128 rows][128 B]
constexpr int KV_TILE_BYTES = KT * HD * 2;         // 32 KB: 16 blocks of [2 dim-halves][8 keys][128 B]
constexpr int OFF_Q = 0;                           // [2 heads][32 KB]
constexpr int OFF_K = OFF_Q + 2 * Q_TILE_BYTES;    // [STAGES][32 KB]
constexpr int OFF_V = OFF_K + STAGES * KV_TILE_BYTES;
constexpr int STG_BYTES = 32 * 128;                 // per softmax warp: 32 rows x 128 B
constexpr int OFF_STG = OFF_V + STAGES * KV_TILE_BYTES;  // [8 warps] epilogue staging
constexpr int OFF_BAR = OFF_STG + 8 * STG_BYTES;
// barriers (8 bytes each)
constexpr int B_QFULL = 0, B_QEMPTY = 1;
constexpr int B_KFULL = 2, B_KEMPTY = B_KFULL + STAGES;
constexpr int B_VFULL = B_KEMPTY + STAGES, B_VEMPTY = B_VFULL + STAGES;
constexpr int B_SFULL = B_VEMPTY + STAGES;  // [head] S in tensor memory
constexpr int B_PLO = B_SFULL + 2;          // [head] P of keys 0-63 written (4 warps)
constexpr int B_PHI = B_PLO + 2;            // [head] P of keys 64-127 written (4 warps)
constexpr int B_PVDONE = B_PHI + 2;         // [head] PV complete, P consumed
constexpr int B_OFULL = B_PVDONE + 2;       // [head] last PV of an item complete
constexpr int B_DRAIN = B_OFULL + 2;        // every issued MMA complete (exit)
constexpr int NBAR = B_DRAIN + 1;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem address, abort flag
constexpr int SMEM = OFF_MISC + 64 + 1024;    // + slack for 1024-byte alignment
static_assert(SMEM <= 232448, "prefill shared memory exceeds the sm_100 limit");

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t HEAD_COLS = 256;  // head t: S/P at t*256, O at t*256 + 128
constexpr uint32_t COL_O = 128;

// instruction descriptors (kind::f16): c=F32 (bit 4), a=BF16 (bits 7-9),
// b=BF16 (bits 10-12), b_major bit 16, N>>3 at bit 17, M>>4 at bit 24
constexpr uint32_t IDESC_S = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(KT >> 3) << 17) |
                             ((uint32_t)(QT >> 4) << 24);
constexpr uint32_t IDESC_PV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) |
                              ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(QT >> 4) << 24);

}  // namespace pf

// 2^x by the hardware approximation (MUFU ex2, flush-to-zero): softmax
// weights p = 2^(s - m) <= 2^8 need no denormal handling.
__device__ __forceinline__ float exp2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr uint32_t NEG_INF_BITS = 0xff800000u;

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// One pair in EXP2_POLY_EVERY of the softmax weights is computed by
// exp2_poly2, which runs on the FMA pipe and so adds throughput next to the
// MUFU unit (16 results per clock per SM).
constexpr int EXP2_POLY_EVERY = 4;

// 2^x for a pair, x <= 9: round x to j = nearest integer by the 1.5 * 2^23
// addition (the integer lands in the low mantissa bits of t), evaluate a
// cubic for 2^f on f = x - j in [-1/2, 1/2], and add j to the exponent
// field.  The cubic is a least-squares fit of 2^f on Chebyshev nodes
// weighted for relative error; its maximum relative error on
// [-1/2, 1/2] is 7.5e-5, far below the bf16 rounding P receives.  x is
// clamped at -126 so the exponent sum cannot wrap (values below 2^-126
// come out as tiny denormals, not zero).
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fmaxf(x.x, -126.0f);
    x.y = fmaxf(x.y, -126.0f);
    const float2 t = __fadd2_rn(x, make_float2(12582912.0f, 12582912.0f));
    const float2 jf = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
    const float2 f = __fadd2_rn(x, make_float2(-jf.x, -jf.y));
    float2 p = __ffma2_rn(make_float2(0.05517168715596199f, 0.05517168715596199f), f,
                          make_float2(0.2426111400127411f, 0.2426111400127411f));
    p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
    p = __ffma2_rn(p, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// Bounded wait that also gives up as soon as another thread of the CTA has
// given up (the shared abort word), so a stalled pipeline unwinds in about
// one wait limit instead of one per remaining wait.
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag || clock64() - t0 > WAIT_LIMIT_CYCLES) {
            if (!*abort_flag) atomicExch(err, DEV_ERR_TIMEOUT);
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

// Work item i (in decreasing-length order) -> (query tile, kv head, pair);
// a chunk is the part of an item over key tiles [j0, j1).
struct PfItem {
    int qt, g, hp, nj;
    int item, part, nparts, j0, j1;
};

__device__ __forceinline__ PfItem pf_item(const PrefillParams& P, int i) {
    const int per_qt = P.nkv * 2;
    const int n_qt = (P.n_tok + pf::QT - 1) / pf::QT;
    PfItem it;
    it.qt = n_qt - 1 - i / per_qt;
    const int rem = i % per_qt;
    it.g = rem / 2;
    it.hp = rem % 2;
    const int last_q = min(P.pos0 + (it.qt + 1) * pf::QT, P.pos0 + P.n_tok) - 1;  // absolute
    it.nj = last_q / pf::KT + 1;
    return it;
}

// Chunk x: part x % nsplit of item x / nsplit (empty, j0 == j1, when the
// item has fewer parts).  Without SPLIT every item is one chunk.
template <bool SPLIT>
__device__ __forceinline__ PfItem pf_chunk(const PrefillParams& P, int x) {
    if constexpr (!SPLIT) {
        PfItem it = pf_item(P, x);
        it.item = x;
        it.part = 0;
        it.nparts = 1;
        it.j0 = 0;
        it.j1 = it.nj;
        return it;
    }
    PfItem it = pf_item(P, x / P.nsplit);
    it.item = x / P.nsplit;
    it.part = x % P.nsplit;
    it.nparts = min(P.nsplit, (it.nj + P.part_tiles - 1) / P.part_tiles);
    it.j0 = it.j1 = 0;
    if (it.part < it.nparts) {
        it.j0 = it.part * it.nj / it.nparts;
        it.j1 = (it.part + 1) * it.nj / it.nparts;
    }
    return it;
}

// The r-th chunk of CTA c in snake order.
__device__ __forceinline__ int pf_item_index(int c, int r, int G) {
    return r * G + ((r & 1) ? (G - 1 - c) : c);
}

// SPLIT: long items are cut into parts merged by the last one to finish (a
// separate instantiation, so the unsplit kernel keeps its own code).
template <bool SPLIT>
__global__ void __launch_bounds__(pf::NTHREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ PrefillParams P) {
    using namespace pf;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128B-swizzle atoms
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);
    const uint32_t s_base = smem_u32(smem);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int n_qt = (P.n_tok + QT - 1) / QT;
    const int n_items = n_qt * P.nkv * 2;
    const int n_chunks = SPLIT ? n_items * P.nsplit : n_items;

    if (tid == 0) {
        mbar_init(&bars[B_QFULL], 1);
        mbar_init(&bars[B_QEMPTY], 1);
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&bars[B_KFULL + s], 1);
            mbar_init(&bars[B_KEMPTY + s], 1);
            mbar_init(&bars[B_VFULL + s], 1);
            mbar_init(&bars[B_VEMPTY + s], 1);
        }
        for (int t = 0; t < 2; t++) {
            mbar_init(&bars[B_SFULL + t], 1);
            mbar_init(&bars[B_PLO + t], 4);
            mbar_init(&bars[B_PHI + t], 4);
            mbar_init(&bars[B_PVDONE + t], 1);
            mbar_init(&bars[B_OFULL + t], 1);
        }
        mbar_init(&bars[B_DRAIN], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void*)tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // the previous kernel's writes (cache, q rows) are visible
    // dependents are released only after this kernel's own wait (so every
    // kernel before the previous one has completed)
    if (tid == 0) griddep_launch_dependents();

    if (warp == 0) {
        // ============================================ TMA producer
        if (lane == 0) {
            const uint64_t pol_q = l2_policy_evict_first();
            const uint64_t pol_kv = l2_policy_evict_last();  // K/V of a head are re-read by 16 items
            int kv_it = 0, item_it = 0, k_issued = 0, v_issued = 0;
            bool dead = false;
            for (int r = 0; !dead; r++) {
                const int i = pf_item_index(c, r, G);
                if (i >= n_chunks) break;
                const PfItem it = pf_chunk<SPLIT>(P, i);
                if (it.j0 == it.j1) continue;
                if (item_it > 0 && !pf_wait(&bars[B_QEMPTY], (item_it - 1) & 1, abort_flag, P.err))
                    break;
                mbar_arrive_expect_tx(&bars[B_QFULL], 2u * Q_TILE_BYTES);
                for (int t = 0; t < 2; t++) {
                    const int h = (P.kv0 + it.g) * GQA + 2 * it.hp + t;
                    uint8_t* dq = smem + OFF_Q + t * Q_TILE_BYTES;
                    tma_load_3d(dq, &tmQ, &bars[B_QFULL], 0, h, it.qt * QT, pol_q);
                    tma_load_3d(dq + QT * 128, &tmQ, &bars[B_QFULL], 64, h, it.qt * QT, pol_q);
                }
                item_it++;
                for (int j = it.j0; j < it.j1; j++, kv_it++) {
                    const int st = kv_it % STAGES;
                    const uint32_t ph = (uint32_t)(kv_it / STAGES) & 1u;
                    // a 128-key tile is two 64-key runs, each inside one page
                    // (pages hold a multiple of 64 tokens); the cache's 8-row
                    // blocks are already in the operand layout, so a run is
                    // one 16 KB bulk copy per tensor
                    long long rows[2];
                    for (int hf = 0; hf < 2; hf++) {
                        const int pt = P.page_tokens;
                        // the last tile may reach past the slot's pages; those
                        // keys are after every query (masked, p = 0), so any
                        // finite rows of the slot serve: its last 64
                        const int t0 = min(j * KT + hf * 64, P.pages_per_seq * pt - 64);
                        const long long phys = (long long)P.slot * P.pages_per_seq + t0 / pt;
                        rows[hf] = (((long long)P.layer * P.nkv + it.g) * P.n_pages + phys) * pt + (t0 % pt);
                    }
                    if (kv_it >= STAGES && !pf_wait(&bars[B_KEMPTY + st], ph ^ 1u, abort_flag, P.err)) {
                        dead = true;
                        break;
                    }
                    uint8_t* dk = smem + OFF_K + st * KV_TILE_BYTES;
                    mbar_arrive_expect_tx(&bars[B_KFULL + st], (uint32_t)KV_TILE_BYTES);
                    for (int hf = 0; hf < 2; hf++)
                        bulk_load(dk + hf * (KV_TILE_BYTES / 2), P.kcache + rows[hf] * HD, KV_TILE_BYTES / 2,
                                  &bars[B_KFULL + st], pol_kv);
                    k_issued = kv_it + 1;
                    if (kv_it >= STAGES && !pf_wait(&bars[B_VEMPTY + st], ph ^ 1u, abort_flag, P.err)) {
                        dead = true;
                        break;
                    }
                    uint8_t* dv = smem + OFF_V + st * KV_TILE_BYTES;
                    mbar_arrive_expect_tx(&bars[B_VFULL + st], (uint32_t)KV_TILE_BYTES);
                    for (int hf = 0; hf < 2; hf++)
                        bulk_load(dv + hf * (KV_TILE_BYTES / 2), P.vcache + rows[hf] * HD, KV_TILE_BYTES / 2,
                                  &bars[B_VFULL + st], pol_kv);
                    v_issued = kv_it + 1;
                }
            }
            // drain: the CTA may not exit with bulk copies still writing its
            // shared memory (only matters after an abort; a no-op otherwise)
            if (item_it > 0) mbar_wait(&bars[B_QFULL], (uint32_t)(item_it - 1) & 1u);
            for (int k = (k_issued > STAGES ? k_issued - STAGES : 0); k < k_issued; k++)
                mbar_wait(&bars[B_KFULL + k % STAGES], (uint32_t)(k / STAGES) & 1u);
            for (int k = (v_issued > STAGES ? v_issued - STAGES : 0); k < v_issued; k++)
                mbar_wait(&bars[B_VFULL + k % STAGES], (uint32_t)(k / STAGES) & 1u);
        }
    } else if (warp == 1) {
        // ============================================ MMA issuer
        if (lane == 0) {
            int kv_base = 0, item_it = 0;
            uint32_t pv_n[2] = {0u, 0u};  // PVs issued per head
            bool dead = false;
            auto issue_s = [&](int t, int st) {
                const uint32_t kb = s_base + OFF_K + st * KV_TILE_BYTES;
                const uint32_t qb = s_base + OFF_Q + t * Q_TILE_BYTES;
                const uint32_t d = tmem + t * HEAD_COLS;
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint32_t koff = (kk & 3) * 32;  // 16 bf16 along K in a 128-byte row
                    const uint64_t da = smem_desc(qb + (kk >> 2) * (QT * 128) + koff, 16, 1024);
                    // K: 8-key groups 2048 B apart, dim-halves 1024 B
                    const uint64_t db = smem_desc(kb + (kk >> 2) * 1024 + koff, 16, 2048);
                    tc_mma_ss(d, da, db, IDESC_S, kk > 0 ? 1u : 0u);
                }
                tc_commit(&bars[B_SFULL + t]);
            };
            for (int r = 0; !dead; r++) {
                const int i = pf_item_index(c, r, G);
                if (i >= n_chunks) break;
                const PfItem it = pf_chunk<SPLIT>(P, i);
                const int nj = it.j1 - it.j0;  // key tiles of this chunk
                if (nj == 0) continue;
                if (!pf_wait(&bars[B_QFULL], item_it & 1, abort_flag, P.err)) break;
                {
                    // S(0) of both heads; head t's columns still hold P of the
                    // previous item until its last PV has completed
                    const int st = kv_base % STAGES;
                    if (!pf_wait(&bars[B_KFULL + st], (uint32_t)(kv_base / STAGES) & 1u, abort_flag, P.err))
                        break;
                    for (int t = 0; t < 2 && !dead; t++) {
                        if (pv_n[t] > 0 &&
                            !pf_wait(&bars[B_PVDONE + t], (pv_n[t] - 1) & 1u, abort_flag, P.err)) {
                            dead = true;
                            break;
                        }
                        tc_fence_after();
                        issue_s(t, st);
                    }
                    if (dead) break;
                    tc_commit(&bars[B_KEMPTY + st]);
                    if (nj == 1) tc_commit(&bars[B_QEMPTY]);
                }
                for (int j = 0; j < nj && !dead; j++) {
                    const int kj = kv_base + j;
                    const int st = kj % STAGES;
                    if (!pf_wait(&bars[B_VFULL + st], (uint32_t)(kj / STAGES) & 1u, abort_flag, P.err)) {
                        dead = true;
                        break;
                    }
                    const int kn = kj + 1;
                    const int stn = kn % STAGES;
                    const uint32_t vb = s_base + OFF_V + st * KV_TILE_BYTES;
                    for (int t = 0; t < 2; t++) {
                        // O_t += P_t . V_j, each half of the keys as soon as the
                        // softmax has written its half of P_t (the first
                        // arrive also orders the epilogue's reads of the
                        // previous item's O before this overwrite)
                        const uint32_t d = tmem + t * HEAD_COLS + COL_O;
                        const uint32_t pa = tmem + t * HEAD_COLS;
                        for (int hf = 0; hf < 2; hf++) {
                            if (!pf_wait(&bars[(hf ? B_PHI : B_PLO) + t], pv_n[t] & 1u, abort_flag, P.err)) {
                                dead = true;
                                break;
                            }
                            tc_fence_after();
#pragma unroll
                            for (int k4 = 0; k4 < KT / 32; k4++) {
                                // A = P columns [8kk, 8kk+8) (16 keys, bf16
                                // pairs); B = V rows [16kk, 16kk+16),
                                // MN-major: dim-halves 1024 B apart, 8-key
                                // groups 2048 B apart
                                const int kk = hf * (KT / 32) + k4;
                                const uint64_t db = smem_desc(vb + kk * 4096, 1024, 2048);
                                tc_mma_ts(d, pa + kk * 8, db, IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
                            }
                        }
                        if (dead) break;
                        tc_commit(&bars[B_PVDONE + t]);
                        pv_n[t]++;
                        if (j == nj - 1) tc_commit(&bars[B_OFULL + t]);
                        if (t == 1) tc_commit(&bars[B_VEMPTY + st]);
                        if (j + 1 < nj) {
                            // S_t(j+1) overwrites P_t(j): wait for that PV
                            if (!pf_wait(&bars[B_PVDONE + t], (pv_n[t] - 1) & 1u, abort_flag, P.err)) {
                                dead = true;
                                break;
                            }
                            if (t == 0 &&
                                !pf_wait(&bars[B_KFULL + stn], (uint32_t)(kn / STAGES) & 1u, abort_flag,
                                         P.err)) {
                                dead = true;
                                break;
                            }
                            tc_fence_after();
                            issue_s(t, stn);
                            if (t == 1) {
                                tc_commit(&bars[B_KEMPTY + stn]);
                                if (j + 2 == nj) tc_commit(&bars[B_QEMPTY]);
                            }
                        }
                    }
                }
                if (dead) break;
                kv_base += nj;
                item_it++;
            }
            // drain: tensor memory is freed only after every issued MMA is done
            tc_commit(&bars[B_DRAIN]);
            mbar_wait(&bars[B_DRAIN], 0u);
        }
    } else if (warp >= 4) {
        // ============================================ softmax warpgroups
        const int t = (warp - 4) >> 2;            // head of the pair
        const int rw = warp & 3;                  // tensor-memory lane quarter
        const int row = rw * 32 + lane;           // query row within the tile
        const uint32_t tl = tmem + ((uint32_t)(rw * 32) << 16) + t * HEAD_COLS;  // this row, head t
        const float2 sc2 = make_float2(P.scale_log2e, P.scale_log2e);
        int s_it = 0, item_it = 0;
        for (int r = 0;; r++) {
            const int i = pf_item_index(c, r, G);
            if (i >= n_chunks) break;
            const PfItem it = pf_chunk<SPLIT>(P, i);
            if (it.j0 == it.j1) continue;
            const int q_abs = P.pos0 + it.qt * QT + row;  // this row's position
            float m_ref = -INFINITY, l_sum = 0.0f;
            bool dead = false;
            for (int j = it.j0; j < it.j1; j++) {
                // the warp leaves together (its lanes later meet in warp
                // barriers and shuffles)
                const bool got = pf_wait(&bars[B_SFULL + t], (uint32_t)s_it & 1u, abort_flag, P.err);
                if (SPLIT ? !__all_sync(FULL, got) : !got) {
                    dead = true;
                    break;
                }
                s_it++;
                tc_fence_after();
                uint32_t sr[128];
                Q3A_TC_LD32(tl, sr, 0);
                Q3A_TC_LD32(tl + 32, sr, 32);
                Q3A_TC_LD32(tl + 64, sr, 64);
                Q3A_TC_LD32(tl + 96, sr, 96);
                tc_wait_ld();
                // causal mask: keys after this row's position, only in tiles
                // the diagonal crosses
                const int lim = q_abs - j * KT;  // last visible key of this tile
                if (lim < KT - 1) {
#pragma unroll
                    for (int cc = 0; cc < 128; cc++)
                        sr[cc] = (cc > lim) ? NEG_INF_BITS : sr[cc];
                }
                // running maximum on raw scores (the scale is positive)
                float mx4[4];
#pragma unroll
                for (int u = 0; u < 4; u++) mx4[u] = max3f(__uint_as_float(sr[u]), __uint_as_float(sr[4 + u]), __uint_as_float(sr[8 + u]));
#pragma unroll
                for (int cc = 12; cc < 124; cc += 8)
#pragma unroll
                    for (int u = 0; u < 4; u++)
                        mx4[u] = max3f(mx4[u], __uint_as_float(sr[cc + u]), __uint_as_float(sr[cc + 4 + u]));
#pragma unroll
                for (int u = 0; u < 4; u++) mx4[u] = fmaxf(mx4[u], __uint_as_float(sr[124 + u]));
                const float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * P.scale_log2e;
                float alpha = 1.0f;
                bool rescale = false;
                if (mt > m_ref + 8.0f) {  // includes the first tile (m_ref = -inf)
                    alpha = (m_ref == -INFINITY) ? 0.0f : exp2_approx(m_ref - mt);
                    rescale = (m_ref != -INFINITY);
                    m_ref = mt;
                }
                // p = 2^(s*scale - m_ref) with packed fp32x2 math, in two
                // halves of 64 keys; each half is packed to bf16 pairs
                // (column c: keys 2c, 2c+1), stored over the first 64 columns
                // of this row's S and signalled on its own barrier, so the
                // first half of PV runs while the second half is computed.
                // One pair in EXP2_POLY_EVERY takes the polynomial 2^x on the
                // FMA pipe instead of the MUFU unit.
                // (a row with no visible key so far -- only in a chunk that
                // starts after the row's position -- gets p = 0, not NaN)
                const float nm = (SPLIT && m_ref == -INFINITY) ? 0.0f : -m_ref;
                const float2 nm2 = make_float2(nm, nm);
                float2 ps2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                 make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    uint32_t pk[32];
#pragma unroll
                    for (int cc = 0; cc < 64; cc += 2) {
                        const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[hf * 64 + cc]),
                                                                __uint_as_float(sr[hf * 64 + cc + 1])),
                                                    sc2, nm2);
                        float2 pp;
                        if (EXP2_POLY_EVERY > 0 && (cc >> 1) % EXP2_POLY_EVERY == EXP2_POLY_EVERY - 1)
                            pp = exp2_poly2(x);
                        else
                            pp = make_float2(exp2_approx(x.x), exp2_approx(x.y));
                        ps2[(cc >> 1) & 3] = __fadd2_rn(ps2[(cc >> 1) & 3], pp);
                        __nv_bfloat162 b2 = __floats2bfloat162_rn(pp.x, pp.y);
                        pk[cc >> 1] = *reinterpret_cast<uint32_t*>(&b2);
                    }
                    Q3A_TC_ST32(tl + hf * 32, pk, 0);
                    if (hf == 0 && rescale) {
                        // O *= alpha before the first half of PV(j) adds to
                        // it.  S_t(j) was issued after PV_t(j-1) completed,
                        // so O holds every tile before j, and no MMA writes
                        // it before P_t(j) is signalled below.
#pragma unroll 1
                        for (int q = 0; q < 4; q++) {
                            uint32_t orr[32];
                            Q3A_TC_LD32(tl + COL_O + 32 * q, orr, 0);
                            tc_wait_ld();
#pragma unroll
                            for (int cc = 0; cc < 32; cc++)
                                orr[cc] = __float_as_uint(__uint_as_float(orr[cc]) * alpha);
                            Q3A_TC_ST32(tl + COL_O + 32 * q, orr, 0);
                        }
                    }
                    tc_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars[(hf ? B_PHI : B_PLO) + t]);
                }
                const float2 s01 = __fadd2_rn(ps2[0], ps2[1]), s23 = __fadd2_rn(ps2[2], ps2[3]);
                const float2 s4 = __fadd2_rn(s01, s23);
                l_sum = l_sum * alpha + (s4.x + s4.y);
            }
            if (dead) break;
            // epilogue: O / l once the item's last PV is done.  Each warp
            // stages 32 rows x 32 columns at a time in its own shared-memory
            // buffer (16-byte chunks XOR-swizzled by row) and writes them
            // back row-contiguous, so every global store fills whole sectors.
            {
                const bool got = pf_wait(&bars[B_OFULL + t], (uint32_t)item_it & 1u, abort_flag, P.err);
                if (SPLIT ? !__all_sync(FULL, got) : !got) break;
            }
            tc_fence_after();
            const int srow0 = it.qt * QT + rw * 32;  // prompt row of lane 0
            const int h = (P.kv0 + it.g) * GQA + 2 * it.hp + t;
            uint8_t* stg = smem + OFF_STG + (warp - 4) * STG_BYTES;
            // columns [32q, 32q+32) of this row, orr (fp32 bits) x sc, to the output
            auto emit = [&](int q, const uint32_t (&orr)[32], float sc) {
                if (P.out_f32) {
                    // row: 32 fp32 = 8 chunks of 16 B
#pragma unroll
                    for (int c4 = 0; c4 < 8; c4++)
                        *reinterpret_cast<float4*>(stg + lane * 128 + ((c4 ^ (lane & 7)) << 4)) =
                            make_float4(__uint_as_float(orr[4 * c4]) * sc, __uint_as_float(orr[4 * c4 + 1]) * sc,
                                        __uint_as_float(orr[4 * c4 + 2]) * sc,
                                        __uint_as_float(orr[4 * c4 + 3]) * sc);
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const int rr = 4 * k + (lane >> 3), c4 = lane & 7;
                        const float4 x =
                            *reinterpret_cast<const float4*>(stg + rr * 128 + ((c4 ^ (rr & 7)) << 4));
                        if (srow0 + rr < P.n_tok)
                            *reinterpret_cast<float4*>(P.out_f32 + ((size_t)(srow0 + rr) * P.hq_total + h) * HD +
                                                       q * 32 + c4 * 4) = x;
                    }
                } else {
                    // row: 32 bf16 = 4 chunks of 16 B
#pragma unroll
                    for (int c8 = 0; c8 < 4; c8++) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(orr[8 * c8 + 2 * e]) * sc,
                                                                      __uint_as_float(orr[8 * c8 + 2 * e + 1]) * sc);
                            w[e] = *reinterpret_cast<uint32_t*>(&b2);
                        }
                        *reinterpret_cast<uint4*>(stg + lane * 128 + ((c8 ^ (lane & 7)) << 4)) =
                            make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int rr = 8 * k + (lane >> 2), c8 = lane & 3;
                        const uint4 x = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((c8 ^ (rr & 7)) << 4));
                        if (srow0 + rr < P.n_tok)
                            *reinterpret_cast<uint4*>(P.out_bf16 + ((size_t)(srow0 + rr) * P.hq_total + h) * HD +
                                                      q * 32 + c8 * 8) = x;
                    }
                }
                __syncwarp();  // the staging buffer is rewritten by the next chunk
            };
            // a row that saw no visible key in this part (only possible in a
            // part after the first) contributes nothing: o = 0, lse = -inf
            const bool none = SPLIT && ((m_ref == -INFINITY) || !(l_sum > 0.0f));
            const float inv = none ? 0.0f : 1.0f / l_sum;
            if (!SPLIT || it.nparts == 1) {
#pragma unroll 1
                for (int q = 0; q < 4; q++) {
                    uint32_t orr[32];
                    Q3A_TC_LD32(tl + COL_O + 32 * q, orr, 0);
                    tc_wait_ld();
                    emit(q, orr, inv);
                }
            } else if constexpr (SPLIT) {
                // split item: store this part's normalised (o, lse) rows for
                // prefill_combine_kernel.  The rows move 32 x 32 at a time
                // through the warp's staging buffer, so the global stores are
                // row-contiguous (a thread-per-row store would touch 32 lines
                // per instruction).
                const size_t pstride = (size_t)2 * PF_PART_FLOATS;  // parts of an item
                float* mine = P.part + ((size_t)it.item * P.nsplit + it.part) * pstride +
                              (size_t)t * PF_PART_FLOATS;
                const int r0w = rw * 32;  // this warp's first row of the tile
#pragma unroll 1
                for (int q = 0; q < 4; q++) {
                    uint32_t orr[32];
                    Q3A_TC_LD32(tl + COL_O + 32 * q, orr, 0);
                    tc_wait_ld();
#pragma unroll
                    for (int c4 = 0; c4 < 8; c4++)
                        *reinterpret_cast<float4*>(stg + lane * 128 + ((c4 ^ (lane & 7)) << 4)) =
                            make_float4(__uint_as_float(orr[4 * c4]) * inv, __uint_as_float(orr[4 * c4 + 1]) * inv,
                                        __uint_as_float(orr[4 * c4 + 2]) * inv,
                                        __uint_as_float(orr[4 * c4 + 3]) * inv);
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        const int rr = 4 * k + (lane >> 3), c4 = lane & 7;
                        *reinterpret_cast<float4*>(mine + (size_t)(r0w + rr) * HD + q * 32 + c4 * 4) =
                            *reinterpret_cast<const float4*>(stg + rr * 128 + ((c4 ^ (rr & 7)) << 4));
                    }
                    __syncwarp();
                }
                mine[128 * HD + row] = none ? -INFINITY : m_ref + log2f(l_sum);
            }
            // the next item's first P arrive (after this code in program
            // order, behind wait::ld and a before_thread_sync fence) is what
            // lets the issuer overwrite O
            tc_fence_before();
            item_it++;
        }
    }
    // teardown: every warp meets here; the allocating warp frees tensor memory
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

// Merge of the parts of split items: one warp per row (CTA = 8 rows of one
// (item, head of its pair)), so every row's loads are in flight at once; a
// row's 128 outputs are one coalesced load per part (lane l: columns
// 4l..4l+3) weighted by 2^(lse_part - max).  CTAs of unsplit items return
// at once.
__global__ void __launch_bounds__(256)
    prefill_combine_kernel(const __grid_constant__ PrefillParams P) {
    const int item = blockIdx.x >> 5, t = (blockIdx.x >> 4) & 1, rg = blockIdx.x & 15;
    griddep_wait();  // the split kernel's partials are complete and visible
    const PfItem it = pf_item(P, item);
    const int nparts = min(P.nsplit, (it.nj + P.part_tiles - 1) / P.part_tiles);
    if (nparts <= 1) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t pstride = (size_t)2 * PF_PART_FLOATS;
    const float* base = P.part + (size_t)item * P.nsplit * pstride + (size_t)t * PF_PART_FLOATS;
    const int h = (P.kv0 + it.g) * GQA + 2 * it.hp + t;
    {
        const int row = rg * 8 + warp;
        const int srow = it.qt * pf::QT + row;
        if (srow >= P.n_tok) return;
        float lp[8], M = -INFINITY;
        float4 x[8];
#pragma unroll
        for (int pp = 0; pp < 8; pp++) {
            lp[pp] = -INFINITY;
            x[pp] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (pp < nparts) {
                const float* src = base + (size_t)pp * pstride;
                lp[pp] = __ldcg(src + 128 * HD + row);
                x[pp] = __ldcg(reinterpret_cast<const float4*>(src + (size_t)row * HD) + lane);
            }
            M = fmaxf(M, lp[pp]);
        }
        float W = 0.0f;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int pp = 0; pp < 8; pp++) {
            const float w = (lp[pp] == -INFINITY) ? 0.0f : exp2f(lp[pp] - M);
            W += w;
            a.x = fmaf(w, x[pp].x, a.x);
            a.y = fmaf(w, x[pp].y, a.y);
            a.z = fmaf(w, x[pp].z, a.z);
            a.w = fmaf(w, x[pp].w, a.w);
        }
        const float iw = W > 0.0f ? 1.0f / W : 0.0f;
        a.x *= iw;
        a.y *= iw;
        a.z *= iw;
        a.w *= iw;
        const size_t o = ((size_t)srow * P.hq_total + h) * HD + 4 * lane;
        if (P.out_f32) {
            *reinterpret_cast<float4*>(P.out_f32 + o) = a;
        } else {
            __nv_bfloat162 b0 = __floats2bfloat162_rn(a.x, a.y), b1 = __floats2bfloat162_rn(a.z, a.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&b0);
            u.y = *reinterpret_cast<uint32_t*>(&b1);
            *reinterpret_cast<uint2*>(P.out_bf16 + o) = u;
        }
    }
}

template <bool SPLIT>
static cudaError_t set_prefill_attr() {
    return ensure_smem_attr(reinterpret_cast<const void*>(prefill_kernel<SPLIT>), pf::SMEM);
}

cudaError_t launch_prefill(const PrefillParams& p, const CUtensorMap& tmQ, cudaStream_t st) {
    const bool split = p.nsplit > 1;
    cudaError_t e = split ? set_prefill_attr<true>() : set_prefill_attr<false>();
    if (e != cudaSuccess) return e;
    const int n_qt = (p.n_tok + pf::QT - 1) / pf::QT;
    const int n_chunks = n_qt * p.nkv * 2 * p.nsplit;
    int nsm = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int grid = n_chunks < nsm ? n_chunks : nsm;
    // programmatic dependent launches: each kernel is scheduled while the
    // previous one of the stream finishes and waits for it before it touches
    // memory
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(pf::NTHREADS);
    cfg.dynamicSmemBytes = pf::SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (split) {
        e = cudaLaunchKernelEx(&cfg, prefill_kernel<true>, tmQ, p);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cc = cfg;
        cc.gridDim = dim3(n_qt * p.nkv * 2 * 2 * 16);
        cc.blockDim = dim3(256);
        cc.dynamicSmemBytes = 0;
        return cudaLaunchKernelEx(&cc, prefill_combine_kernel, p);
    }
    return cudaLaunchKernelEx(&cfg, prefill_kernel<false>, tmQ, p);
}

int prefill_smem_bytes() { return pf::SMEM; }

}  // namespace q3a
