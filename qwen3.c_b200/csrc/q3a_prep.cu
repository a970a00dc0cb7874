// q3a_prep.cu -- the small kernels around the attention core:
//  * KV append of n tokens: per-head QK-RMSNorm + RoPE of k, write of k and v
//    into the paged cache (reference: qwen3-8b/cpu/main.c:1320-1329; HIP
//    rmsnorm_head_kernel / rope_kernel / kv_cache_write_kernel at
//    qwen3-8b/gpu/main.c:1416-1467, 1542-1557, three launches fused here);
//  * cache read-back to the reference's position-major fp32 layout;
//  * row preparation of prompt queries for prefill (norm + RoPE -> bf16);
//  * the seeded N(0,1) generator;
//  * the log-sum-exp combine of sequence-shard partials.
#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {

// One warp per (token, head) row: lanes stage the 128 values in shared
// memory, lane 0 forms the reference's sequential sum of squares, then each
// lane normalises and rotates two adjacent pairs.
constexpr int ROWS_PER_BLOCK = 8;

__device__ __forceinline__ void norm_rope_row(float* row /*smem [128]*/, const float* w, float eps,
                                              int pos, const float* inv_freq, int lane,
                                              float (&out)[4]) {
    __syncwarp();
    float sc = 0.0f;
    if (lane == 0) sc = head_rms_scale(row, eps);
    sc = __shfl_sync(FULL, sc, 0);
#pragma unroll
    for (int pp = 0; pp < 2; pp++) {
        const int i = 4 * lane + 2 * pp;
        float v0 = __fmul_rn(row[i], __fmul_rn(sc, w[i]));
        float v1 = __fmul_rn(row[i + 1], __fmul_rn(sc, w[i + 1]));
        rope_pair(v0, v1, pos, inv_freq[i >> 1]);
        out[2 * pp] = v0;
        out[2 * pp + 1] = v1;
    }
}

template <typename KV>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 32)
    append_kernel(const __grid_constant__ AppendParams P) {
    __shared__ __align__(16) float srow[ROWS_PER_BLOCK][HD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.x * ROWS_PER_BLOCK + warp;
    if (r >= (long long)P.n * P.nkv) return;
    const int tok = (int)(r / P.nkv), kvh = (int)(r % P.nkv);
    const int pos = P.pos0 + tok;
    const size_t src = (size_t)tok * P.nkv_total * HD + (size_t)(P.kv0 + kvh) * HD + 4 * lane;
    float4 kv = *reinterpret_cast<const float4*>(P.k + src);
    const float4 vv = *reinterpret_cast<const float4*>(P.v + src);
    float k4[4] = {kv.x, kv.y, kv.z, kv.w};
    if (P.do_norm_rope) {
        *reinterpret_cast<float4*>(&srow[warp][4 * lane]) = kv;
        norm_rope_row(srow[warp], P.k_norm_w, P.eps, pos, P.inv_freq, lane, k4);
    }
    const int pt = P.page_tokens;
    const long long phys = (long long)P.slot * P.pages_per_seq + pos / pt;
    const long long row = (((long long)P.layer * P.nkv + kvh) * P.n_pages + phys) * pt + pos % pt;
    // dims 4*lane .. 4*lane+3 are contiguous in either layout
    KV* kd = reinterpret_cast<KV*>(P.kcache) + kv_index<KV>(row, 4 * lane);
    KV* vd = reinterpret_cast<KV*>(P.vcache) + kv_index<KV>(row, 4 * lane);
    kd[0] = from_f32<KV>(k4[0]);
    kd[1] = from_f32<KV>(k4[1]);
    kd[2] = from_f32<KV>(k4[2]);
    kd[3] = from_f32<KV>(k4[3]);
    vd[0] = from_f32<KV>(vv.x);
    vd[1] = from_f32<KV>(vv.y);
    vd[2] = from_f32<KV>(vv.z);
    vd[3] = from_f32<KV>(vv.w);
}

template <typename KV>
__global__ void kv_read_kernel(const __grid_constant__ AppendParams P, float* __restrict__ ko,
                               float* __restrict__ vo) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long total = (long long)P.n * P.nkv * HD;
    if (i >= total) return;
    const int d = (int)(i % HD);
    const long long r = i / HD;
    const int tok = (int)(r / P.nkv), kvh = (int)(r % P.nkv);
    const int pos = P.pos0 + tok;
    const int pt = P.page_tokens;
    const long long phys = (long long)P.slot * P.pages_per_seq + pos / pt;
    const long long row = (((long long)P.layer * P.nkv + kvh) * P.n_pages + phys) * pt + pos % pt;
    const size_t dst = (size_t)tok * P.nkv * HD + (size_t)kvh * HD + d;
    ko[dst] = to_f32<KV>(reinterpret_cast<const KV*>(P.kcache)[kv_index<KV>(row, d)]);
    vo[dst] = to_f32<KV>(reinterpret_cast<const KV*>(P.vcache)[kv_index<KV>(row, d)]);
}

__global__ void __launch_bounds__(ROWS_PER_BLOCK * 32)
    prep_rows_kernel(const __grid_constant__ PrepParams P) {
    __shared__ __align__(16) float srow[ROWS_PER_BLOCK][HD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long r = (long long)blockIdx.x * ROWS_PER_BLOCK + warp;
    if (r >= (long long)P.n * P.nheads) return;
    const int tok = (int)(r / P.nheads), h = P.head0 + (int)(r % P.nheads);
    const size_t off = (size_t)tok * P.nheads_total * HD + (size_t)h * HD + 4 * lane;
    const float4 x = *reinterpret_cast<const float4*>(P.src + off);
    float o[4] = {x.x, x.y, x.z, x.w};
    if (P.do_norm_rope) {
        *reinterpret_cast<float4*>(&srow[warp][4 * lane]) = x;
        norm_rope_row(srow[warp], P.w, P.eps, P.pos0 + tok, P.inv_freq, lane, o);
    }
    if (P.dst_f32) *reinterpret_cast<float4*>(P.dst_f32 + off) = make_float4(o[0], o[1], o[2], o[3]);
    if (P.dst_bf16) {
        __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]);
        __nv_bfloat162 b = __floats2bfloat162_rn(o[2], o[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(P.dst_bf16 + off) = u;
    }
}

// ---------------------------------------------------------------- generator
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream + 0x51ED2701ULL));
}

// Uniform in (0,1): splitmix64 of the counter seeds one xorshift64* output
// step (the generator of rng_f32, qwen3-8b/cpu/main.c:1377-1382); 23 bits.
__device__ __forceinline__ float u01(uint64_t key, uint64_t i) {
    uint64_t s = splitmix64(key + i);
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    const uint32_t r = (uint32_t)((s * 0x2545F4914F6CDD1DULL) >> 41);
    return ((float)r + 0.5f) * (1.0f / 8388608.0f);
}

__global__ void randn_kernel(void* dst, int out_bf16, size_t n, uint64_t key, uint64_t offset) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint64_t e = offset + i;
    const uint64_t j = e >> 1;
    const float u1 = u01(key, 2 * j);
    const float u2 = u01(key, 2 * j + 1);
    const float r = sqrtf(-2.0f * logf(u1));
    const float a = 6.283185307179586f * u2;
    const float x = (e & 1) ? r * sinf(a) : r * cosf(a);
    if (out_bf16)
        reinterpret_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(x);
    else
        reinterpret_cast<float*>(dst)[i] = x;
}

// ---------------------------------------------------------------- combine
// One block per head: xb[h] = sum_j 2^(lse_j - M) o_j[h] / sum_j 2^(lse_j - M).
// Part j's output o_j [n_heads][128] starts at o_parts + j * o_stride and its
// log2-sum-exp lse_j [n_heads] at lse_parts + j * lse_stride (dense arrays:
// strides n_heads*128 and n_heads; the one-buffer layout of an all-gather:
// both n_heads*129, lse_parts = o_parts + n_heads*128).
__global__ void lse_combine_kernel(float* __restrict__ xb, const float* __restrict__ o_parts,
                                   size_t o_stride, const float* __restrict__ lse_parts,
                                   size_t lse_stride, int n_parts, int n_heads) {
    const int h = blockIdx.x, d = threadIdx.x;
    float M = -INFINITY;
    for (int j = 0; j < n_parts; j++) M = fmaxf(M, lse_parts[(size_t)j * lse_stride + h]);
    float W = 0.0f, acc = 0.0f;
    for (int j = 0; j < n_parts; j++) {
        const float l = lse_parts[(size_t)j * lse_stride + h];
        const float w = (l == -INFINITY) ? 0.0f : exp2f(l - M);
        W += w;
        acc = fmaf(w, o_parts[(size_t)j * o_stride + (size_t)h * HD + d], acc);
    }
    xb[(size_t)h * HD + d] = acc / W;
}

// ---------------------------------------------------------------- launchers
cudaError_t launch_append(const AppendParams& p, cudaStream_t st) {
    const long long rows = (long long)p.n * p.nkv;
    const unsigned grid = (unsigned)((rows + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK);
    if (grid == 0) return cudaSuccess;
    if (p.bf16)
        append_kernel<__nv_bfloat16><<<grid, ROWS_PER_BLOCK * 32, 0, st>>>(p);
    else
        append_kernel<float><<<grid, ROWS_PER_BLOCK * 32, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_kv_read(const AppendParams& p, float* k_out, float* v_out, cudaStream_t st) {
    const long long total = (long long)p.n * p.nkv * HD;
    const unsigned grid = (unsigned)((total + 255) / 256);
    if (grid == 0) return cudaSuccess;
    if (p.bf16)
        kv_read_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p, k_out, v_out);
    else
        kv_read_kernel<float><<<grid, 256, 0, st>>>(p, k_out, v_out);
    return cudaGetLastError();
}

cudaError_t launch_prep_rows(const PrepParams& p, cudaStream_t st) {
    const long long rows = (long long)p.n * p.nheads;
    const unsigned grid = (unsigned)((rows + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK);
    if (grid == 0) return cudaSuccess;
    prep_rows_kernel<<<grid, ROWS_PER_BLOCK * 32, 0, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_randn(void* dst, int out_bf16, size_t n, uint64_t key, uint64_t offset,
                         cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const size_t grid = (n + 255) / 256;
    randn_kernel<<<(unsigned)grid, 256, 0, st>>>(dst, out_bf16, n, key, offset);
    return cudaGetLastError();
}

cudaError_t launch_lse_combine(float* xb, const float* o_parts, size_t o_stride,
                               const float* lse_parts, size_t lse_stride, int n_parts, int n_heads,
                               cudaStream_t st) {
    lse_combine_kernel<<<n_heads, HD, 0, st>>>(xb, o_parts, o_stride, lse_parts, lse_stride, n_parts,
                                               n_heads);
    return cudaGetLastError();
}

}  // namespace q3a
