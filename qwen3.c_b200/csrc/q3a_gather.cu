// q3a_gather.cu -- all-gather of column slices over NVLink peer memory.
//
// KV-head sharding leaves rank r with the columns of its query heads (of xb
// or of a prefill output); q3a_gather_cols gives every rank every rank's
// columns in one launch and without a collective library.  The reference
// has no multi-GPU path, so nothing here replaces reference code.
//
// One launch per call, grid <= SM count (all CTAs resident):
//  1. CTA 0 raises its "arrived" flag in every rank's flag block and waits
//     (bounded) until every rank has arrived at this call, so no rank writes
//     into a buffer that another rank may still read from its previous call;
//     it then releases the other CTAs of this grid through a local word;
//  2. every CTA copies its share of the rows' slice, 16 bytes per thread per
//     step, from this rank's matrix into every other rank's matrix (plain
//     stores to the peers' mapped memory), then fences at system scope;
//  3. the last CTA to finish raises its "done" flag in every rank's block and
//     waits (bounded) for every rank's, then advances the call number.
// Flags carry the call number, which only grows, so a rank that is a call
// ahead is seen as having arrived too.
#include "q3a_common.cuh"
#include "q3a_internal.h"

namespace q3a {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until flags[phase][r] >= ep for every rank r; false on timeout.
__device__ __forceinline__ bool wait_all_ranks(const ColGatherParams& P, int phase, unsigned ep) {
    const long long t0 = clock64();
    for (int r = 0; r < P.world; r++) {
        while ((int)(ld_acquire_sys(P.flags + phase * PEER_MAX + r) - ep) < 0) {
            if (clock64() - t0 > P.wait_limit) return false;
        }
    }
    return true;
}

__global__ void __launch_bounds__(256) gather_cols_kernel(const __grid_constant__ ColGatherParams P) {
    __shared__ int ok_s;
    const int tid = threadIdx.x;
    // call number of this launch (the state word advances only after every
    // CTA has arrived at the end, so all CTAs read the same value)
    const unsigned ep = *reinterpret_cast<volatile const unsigned*>(P.state) + 1u;
    if (tid == 0) {
        bool ok = true;
        if (blockIdx.x == 0) {
            for (int r = 0; r < P.world; r++) st_release_sys(P.peer_flags[r] + P.rank, ep);
            ok = wait_all_ranks(P, 0, ep);
            st_release_gpu(P.state + 2, ep);  // go
        } else {
            const long long t0 = clock64();
            while ((int)(ld_acquire_gpu(P.state + 2) - ep) < 0) {
                if (clock64() - t0 > P.wait_limit) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) atomicExch(P.err, DEV_ERR_TIMEOUT);
        ok_s = ok;
    }
    __syncthreads();
    if (ok_s) {
        // GATHER_UNROLL 16-byte vectors per thread per step, loaded together
        // (read-only path) so that many reads are in flight before the
        // stores to the peers; consecutive threads take consecutive vectors
        // of a row's slice, so every store to a peer is a contiguous run
        constexpr int GATHER_UNROLL = 8;
        const long long total = P.rows * P.vecs;
        const long long stride = (long long)gridDim.x * blockDim.x;
        for (long long i0 = (long long)blockIdx.x * blockDim.x + tid; i0 < total;
             i0 += GATHER_UNROLL * stride) {
            int4 v[GATHER_UNROLL];
            long long o[GATHER_UNROLL];
#pragma unroll
            for (int u = 0; u < GATHER_UNROLL; u++) {
                const long long i = i0 + u * stride;
                o[u] = -1;
                if (i < total) {
                    const long long row = i / P.vecs;
                    o[u] = row * P.row_bytes + P.col0 + (i - row * P.vecs) * 16;
                    v[u] = __ldg(reinterpret_cast<const int4*>(P.local + o[u]));
                }
            }
            for (int r = 0; r < P.world; r++) {
                if (r == P.rank) continue;
#pragma unroll
                for (int u = 0; u < GATHER_UNROLL; u++)
                    if (o[u] >= 0) *reinterpret_cast<int4*>(P.peer[r] + o[u]) = v[u];
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(old)
                     : "l"(reinterpret_cast<int*>(P.state + 1))
                     : "memory");
        if (old == (int)gridDim.x - 1) {
            // the last CTA: every copy of this rank is done and fenced
            P.state[1] = 0;
            for (int r = 0; r < P.world; r++) st_release_sys(P.peer_flags[r] + PEER_MAX + P.rank, ep);
            if (!wait_all_ranks(P, 1, ep)) atomicExch(P.err, DEV_ERR_TIMEOUT);
            st_release_gpu(P.state, ep);
        }
    }
}

cudaError_t launch_gather_cols(const ColGatherParams& p, int n_ctas, cudaStream_t st) {
    gather_cols_kernel<<<n_ctas, 256, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace q3a
