// q3a_common.cuh -- shared device helpers for the sm_100a attention kernels:
// mbarrier and TMA (cp.async.bulk.tensor) wrappers in inline PTX, bounded
// waits, bf16 packing, and the per-head QK-RMSNorm / RoPE arithmetic written
// in the reference's operation order.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q3a {

constexpr int HD = 128;        // head_dim (Qwen3-8B)
constexpr int GQA = 4;         // query heads per KV head (32 / 8)
constexpr unsigned FULL = 0xffffffffu;

// Bounded waits: a spin that has not completed after this many SM clocks
// (about one second at B200 clocks) gives up, records Q3A device error
// ERR_TIMEOUT and lets the kernel return instead of hanging the GPU.
constexpr long long WAIT_LIMIT_CYCLES = 2000000000LL;
constexpr int DEV_ERR_TIMEOUT = 5;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking test of the phase with the given parity.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
    }
    return true;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared (this CTA), completion counted
// on `bar` in bytes.  x is the innermost coordinate (elements).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// 1-D bulk copy global -> shared (this CTA) of `bytes` (multiple of 16, both
// addresses 16-byte aligned), completion counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Bulk prefetch of global memory into L2 (a hint; 16-byte aligned address,
// size a multiple of 16).
__device__ __forceinline__ void l2_prefetch(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
        "l"(policy)
        : "memory");
}

// Named barrier over `nthreads` threads (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrives on a named barrier without waiting (the waiting side uses
// named_bar_sync with the same thread count).
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- bf16
__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) {
    return x;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) {
    return x;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
    return __bfloat162float(x);
}

// ---------------------------------------------------------------- norm / rope
// Sum of squares of one 128-wide head in index order with separately rounded
// multiply and add, the order of rmsnorm_head_inplace
// (qwen3-8b/cpu/main.c:1179): the scale is then bit-identical to the
// reference's 1/sqrtf(ss/hd + eps).
__device__ __forceinline__ float head_rms_scale(const float* x, float eps) {
    float ss = 0.0f;
#pragma unroll 8
    for (int i = 0; i < HD; i++) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
    return 1.0f / sqrtf(__fadd_rn(ss / (float)HD, eps));
}

// One RoPE pair (qwen3-8b/cpu/main.c:1284-1293) at position pos with the
// pair's inverse frequency (host-computed as 1/powf(theta, 2i/hd)); products
// are rounded separately as in the reference (no FMA contraction).
__device__ __forceinline__ void rope_pair(float& v0, float& v1, int pos, float inv_freq) {
    const float ang = __fmul_rn((float)pos, inv_freq);
    float s, c;
    sincosf(ang, &s, &c);
    const float a = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    const float b = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
    v0 = a;
    v1 = b;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

// QK-RMSNorm + RoPE of one 128-wide head held by a warp (lane: dims
// 4*lane..4*lane+3, i.e. RoPE pairs 2*lane and 2*lane+1), as in
// rmsnorm_head_inplace + apply_rope (qwen3-8b/cpu/main.c:1175-1183,
// 1282-1295): v *= (1/sqrtf(mean(v^2)+eps)) * w, then pair rotation.
__device__ __forceinline__ float4 norm_rope_lane(float4 x, float4 w, float eps, int pos,
                                                 float2 inv_freq) {
    float ss = __fadd_rn(__fadd_rn(__fmul_rn(x.x, x.x), __fmul_rn(x.y, x.y)),
                         __fadd_rn(__fmul_rn(x.z, x.z), __fmul_rn(x.w, x.w)));
    ss = warp_sum(ss);
    const float sc = 1.0f / sqrtf(__fadd_rn(ss / (float)HD, eps));
    float v0 = __fmul_rn(x.x, __fmul_rn(sc, w.x));
    float v1 = __fmul_rn(x.y, __fmul_rn(sc, w.y));
    float v2 = __fmul_rn(x.z, __fmul_rn(sc, w.z));
    float v3 = __fmul_rn(x.w, __fmul_rn(sc, w.w));
    rope_pair(v0, v1, pos, inv_freq.x);
    rope_pair(v2, v3, pos, inv_freq.y);
    return make_float4(v0, v1, v2, v3);
}

template <typename KV>
__device__ __forceinline__ void store4(KV* dst, float4 v) {
    if constexpr (sizeof(KV) == 4) {
        *reinterpret_cast<float4*>(dst) = v;
    } else {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
        __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(dst) = u;
    }
}

// Named barrier that also returns the AND of a predicate over its threads.
__device__ __forceinline__ bool named_bar_red_and(int id, int nthreads, bool v) {
    int r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.b32 pi, %1, 0;\n\t"
        "barrier.cta.red.and.pred po, %2, %3, pi;\n\t"
        "selp.b32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((int)v), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Programmatic dependent launch: a kernel launched with the PDL attribute
// may be scheduled while the previous kernel of its stream is still
// running; griddep_wait() returns once that kernel has completed and its
// memory is visible (a no-op without the attribute).  Kernels here wait
// before their first global-memory access, so only launch latency and
// shared-memory set-up overlap the previous kernel.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- peer-memory exchange words: each 8-byte word carries a 32-bit value
// and the call number it belongs to, stored and loaded as one naturally
// aligned 64-bit access, so a reader that sees the call number also sees the
// value -- no flag and no fence are needed on either side.
__device__ __forceinline__ void st_word_sys(unsigned long long* p, float v, unsigned ep) {
    const unsigned long long w = ((unsigned long long)ep << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Bounded wait (`limit` SM clocks) for the word of call `ep`; false on
// timeout.
__device__ __forceinline__ bool wait_word(const unsigned long long* p, unsigned ep, float& v,
                                          long long limit) {
    unsigned long long w = ld_word_sys(p);
    if ((unsigned)(w >> 32) != ep) {
        const long long t0 = clock64();
        do {
            if (clock64() - t0 > limit) return false;
            w = ld_word_sys(p);
        } while ((unsigned)(w >> 32) != ep);
    }
    v = __uint_as_float((unsigned)w);
    return true;
}

// Element index of (row R, dim d) in a context's paged cache.  fp32 rows are
// plain 128-float rows.  bf16 rows are kept in blocks of 8 rows (2 KB, the
// same bytes the 8 rows would occupy row by row): [2 dim-halves][8 rows][64
// dims], the 16-byte chunk c of row r stored at chunk c ^ (r % 8).  That is
// the 128-byte-swizzled K-major operand layout of the tensor cores, so a run
// of whole blocks is one contiguous bulk copy into shared memory, ready for
// tcgen05.mma as K (K-major) and as V (MN-major).
template <typename KV>
__device__ __forceinline__ size_t kv_index(long long R, int d) {
    if constexpr (sizeof(KV) == 2) {
        const int r = (int)(R & 7);
        return (size_t)(R >> 3) * 1024 +
               (size_t)((d >> 6) * 512 + r * 64 + ((((d >> 3) & 7) ^ r) << 3) + (d & 7));
    } else {
        return (size_t)R * HD + d;
    }
}

}  // namespace q3a
