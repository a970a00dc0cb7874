// q3a_wire.cu -- the KV-cache wire format: a sequence's cache rows packed
// into one self-checking blob, for handing a prompt's KV pages from a
// prefill GPU to a decode GPU (or to disk) and unpacking them into another
// context.  The reference has no such format (its caches never leave the
// process); this one is defined here.
//
// Blob = 64-byte header (q3a_kv_wire_header, little-endian) + payload.
// Payload: for each layer of [layer0, layer0 + n_layers), each KV head of
// [kv_head_begin, + kv_head_count), K then V: rows of positions
// [pos0, pos0 + n_tok), 128 values each, in the cache dtype (fp32, or bf16
// as rounded on append), row-major -- the head-major pages without the
// cache's internal block swizzle, so any position range can be packed and a
// reader needs no knowledge of the cache layout.
// Checksum: sum over the payload's 64-bit words w_i (i from 0) of
// mix(w_i + i * 0x9E3779B97F4A7C15) modulo 2^64, mix the splitmix64 output
// function; order-independent (so the device adds it in parallel) and
// sensitive to the position of every word.
#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {

__host__ __device__ __forceinline__ uint64_t wire_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

uint64_t wire_checksum_host(const void* payload, size_t bytes) {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(payload);
    uint64_t h = 0;
    for (size_t i = 0; i < bytes / 8; i++) h += wire_mix(w[i] + (uint64_t)i * 0x9E3779B97F4A7C15ULL);
    return h;
}

__global__ void __launch_bounds__(256) wire_checksum_kernel(const uint4* payload, size_t n16,
                                                            unsigned long long* out) {
    uint64_t h = 0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
         i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = payload[i];
        const uint64_t w0 = (uint64_t)v.x | ((uint64_t)v.y << 32);
        const uint64_t w1 = (uint64_t)v.z | ((uint64_t)v.w << 32);
        h += wire_mix(w0 + (uint64_t)(2 * i) * 0x9E3779B97F4A7C15ULL);
        h += wire_mix(w1 + (uint64_t)(2 * i + 1) * 0x9E3779B97F4A7C15ULL);
    }
    for (int o = 16; o > 0; o >>= 1) h += __shfl_xor_sync(FULL, h, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, (unsigned long long)h);
}

// Payload chunk j (16 bytes) <-> its place in the paged cache.  Chunks run
// [layer][head][K|V][token][chunk of the row]; CPR chunks per row (32 fp32,
// 16 bf16).
template <typename KV, bool PACK>
__global__ void __launch_bounds__(256) wire_copy_kernel(const WireParams P) {
    constexpr int EPC = 16 / sizeof(KV);  // elements per chunk
    constexpr int CPR = HD / EPC;
    const size_t per_kv = (size_t)P.n_tok * CPR;      // chunks of one head's K (or V)
    const size_t total = (size_t)P.n_layers * P.nkv * 2 * per_kv;
    const size_t pay_layer = (size_t)P.pay_nkv * 2 * per_kv;  // payload chunks per layer
    uint4* payload = reinterpret_cast<uint4*>(P.payload);
    for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < total;
         j += (size_t)gridDim.x * blockDim.x) {
        const int ch = (int)(j % CPR);
        const size_t r = j / CPR;
        const int t = (int)(r % P.n_tok);
        const size_t r2 = r / P.n_tok;
        const int kv = (int)(r2 & 1);
        const size_t r3 = r2 >> 1;
        const int h = (int)(r3 % P.nkv);            // h-th head copied
        const int li = (int)(r3 / P.nkv);
        const int l = P.layer0 + li;
        const size_t pj = (size_t)li * pay_layer + ((size_t)(P.pay_head0 + h) * 2 + kv) * per_kv +
                          (size_t)t * CPR + ch;
        const int pos = P.pos0 + t;
        const long long phys = (long long)P.slot * P.pages_per_seq + pos / P.page_tokens;
        const long long row =
            (((long long)l * P.ctx_nkv + (P.head_off + h)) * P.n_pages + phys) * P.page_tokens +
            pos % P.page_tokens;
        KV* cache = reinterpret_cast<KV*>(kv ? P.vcache : P.kcache);
        uint4* c = reinterpret_cast<uint4*>(cache + kv_index<KV>(row, ch * EPC));
        if (PACK)
            payload[pj] = *c;
        else
            *c = payload[pj];
    }
}

cudaError_t launch_wire_copy(const WireParams& p, bool bf16, bool pack, cudaStream_t st) {
    const int grid = 148 * 8, block = 256;
    if (bf16) {
        if (pack) wire_copy_kernel<__nv_bfloat16, true><<<grid, block, 0, st>>>(p);
        else wire_copy_kernel<__nv_bfloat16, false><<<grid, block, 0, st>>>(p);
    } else {
        if (pack) wire_copy_kernel<float, true><<<grid, block, 0, st>>>(p);
        else wire_copy_kernel<float, false><<<grid, block, 0, st>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_wire_checksum(const void* payload, size_t bytes, unsigned long long* out,
                                 cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(*out), st);
    if (e != cudaSuccess) return e;
    wire_checksum_kernel<<<148 * 4, 256, 0, st>>>(reinterpret_cast<const uint4*>(payload), bytes / 16,
                                                  out);
    return cudaGetLastError();
}

}  // namespace q3a
