// q3a_noalloc.cu -- decode attention for callers that cannot allocate device
// memory.
//
// Some hosts are not allowed to call cudaMalloc at the point where they run
// the attention step: an engine that hands all device memory to its own
// arena allocator up front, a process whose memory budget is fixed at start,
// or code running inside a callback where allocation is forbidden.  Every
// other decode entry point of this library takes its split-KV scratch (the
// per-range partial results and the arrival counters of the cross-CTA
// merge) from a context that q3a_create allocated.  q3a_attn_decode_noalloc
// instead keeps that scratch in one fixed array in this file's device
// memory, which the CUDA runtime reserves once when the library's module is
// loaded on a device and keeps until the process exits.  The caller passes
// the inputs and the output, all in device memory; nothing here calls
// cudaMalloc, cudaFree or any allocating library routine.
//
// Limits: at most NOALLOC_MAX_KV (16) KV heads per call (n_heads <= 64 with
// 4 query heads per KV head), at most MAX_PIECES (160) CTAs, so the array
// holds 160 partial slots of 516 floats, 16 arrival counters and one error
// word: 330,308 bytes.  Every call uses the same array: calls that may run
// at the same time on the GPU (different streams, or several host threads)
// race on it and must be serialised by the caller.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "q3a_common.cuh"
#include "q3a_internal.h"

using namespace q3a;

namespace {

constexpr int NOALLOC_MAX_KV = 16;
constexpr int NOALLOC_SLOTS = MAX_PIECES;
constexpr size_t NOALLOC_PART_BYTES = (size_t)NOALLOC_SLOTS * PART_STRIDE * sizeof(float);
constexpr size_t NOALLOC_CNT_OFF = NOALLOC_PART_BYTES;
constexpr size_t NOALLOC_ERR_OFF = NOALLOC_CNT_OFF + NOALLOC_MAX_KV * sizeof(int);
constexpr size_t NOALLOC_BYTES = NOALLOC_ERR_OFF + sizeof(int);

constexpr int MAX_DEVICES = 64;

struct DeviceScratch {
    bool ready = false;
    unsigned char* base = nullptr;  // device address of q3a_noalloc_scratch
    int num_sms = 0;
};

DeviceScratch g_devices[MAX_DEVICES];
std::mutex g_setup_mutex;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

// The scratch itself: the partial (o, lse) slots of the split-KV merge, the
// per-group arrival counters and the device error word.  Zero at module
// load; the kernel returns each counter to zero after use, and every call
// clears counters and error word again before its launch.
static __device__ __align__(256) unsigned char q3a_noalloc_scratch[NOALLOC_BYTES];

static EncodeTiledFn g_encode = nullptr;  // cuTensorMapEncodeTiled, resolved once per process

// Once per device, with that device current: the device address of the
// scratch array (in host code the symbol names a host-side stand-in, not
// device memory) and the SM count; once per process, the driver's tensor-map
// encoder.  The stored address belongs to the device's current context: a
// cudaDeviceReset destroys that context (and the module holding the array),
// so this entry point must not be used on a device after it was reset.
static int noalloc_setup(int dev, DeviceScratch** out) {
    if (dev < 0 || dev >= MAX_DEVICES)
        return record_error(Q3A_ERR_UNSUPPORTED, "q3a_attn_decode_noalloc: device ordinal too large");
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_encode) {
        void* fnp = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fnp, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return record_error(Q3A_ERR_CUDA,
                                "q3a_attn_decode_noalloc: cuTensorMapEncodeTiled unavailable");
        g_encode = reinterpret_cast<EncodeTiledFn>(fnp);
    }
    DeviceScratch& d = g_devices[dev];
    if (!d.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, q3a_noalloc_scratch);
        if (e != cudaSuccess)
            return record_error(Q3A_ERR_CUDA, "q3a_attn_decode_noalloc: cudaGetSymbolAddress of the "
                                              "scratch array failed");
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || sms <= 0)
            return record_error(Q3A_ERR_CUDA, "q3a_attn_decode_noalloc: SM count query failed");
        d.base = static_cast<unsigned char*>(p);
        d.num_sms = sms;
        d.ready = true;
    }
    *out = &d;
    return Q3A_OK;
}

static int noalloc_map(CUtensorMap* m, const float* base, uint64_t cols, uint64_t rows) {
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * sizeof(float)};
    cuuint32_t box[2] = {HD, DEC_BOX};
    cuuint32_t estr[2] = {1, 1};
    if (g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return record_error(Q3A_ERR_CUDA, "q3a_attn_decode_noalloc: tensor map encoding failed");
    return Q3A_OK;
}

extern "C" int q3a_attn_decode_noalloc(float* xb, const float* q, const float* kc,
                                       const float* vc, size_t loff, int pos, int n_heads,
                                       int kv_mul, int hd, int kv_dim, int max_seq,
                                       void* stream) {
    if (!xb || !q || !kc || !vc)
        return record_error(Q3A_ERR_INVALID, "q3a_attn_decode_noalloc: null argument");
    if (hd != HD || kv_mul != GQA)
        return record_error(Q3A_ERR_UNSUPPORTED,
                            "q3a_attn_decode_noalloc: only head_dim 128 with 4 query heads per KV "
                            "head is implemented");
    if (kv_dim <= 0 || kv_dim % HD != 0 || n_heads != kv_mul * (kv_dim / HD))
        return record_error(Q3A_ERR_INVALID, "q3a_attn_decode_noalloc: n_heads and kv_dim disagree");
    const int nkv = kv_dim / HD;
    if (nkv > NOALLOC_MAX_KV)
        return record_error(Q3A_ERR_INVALID,
                            "q3a_attn_decode_noalloc: more than 16 KV heads exceeds the fixed scratch "
                            "array; use q3a_attn_decode with a context");
    if (pos < 0 || pos >= max_seq)
        return record_error(Q3A_ERR_INVALID, "q3a_attn_decode_noalloc: pos outside [0, max_seq)");
    if (loff % (size_t)kv_dim != 0)
        return record_error(Q3A_ERR_INVALID, "q3a_attn_decode_noalloc: loff is not a row multiple");
    if ((long long)pos + 1 >= (1LL << 31))
        return record_error(Q3A_ERR_INVALID, "q3a_attn_decode_noalloc: too many cache rows");

    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return record_error(Q3A_ERR_CUDA, "q3a_attn_decode_noalloc: no current device");
    DeviceScratch* ds = nullptr;
    int rc = noalloc_setup(dev, &ds);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    const size_t rows = (size_t)pos + 1;
    CUtensorMap tk, tv;
    rc = noalloc_map(&tk, kc + loff, (uint64_t)kv_dim, rows);
    if (rc) return rc;
    rc = noalloc_map(&tv, vc + loff, (uint64_t)kv_dim, rows);
    if (rc) return rc;

    DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.q = q;
    p.xb = xb;
    p.partials = reinterpret_cast<float*>(ds->base);
    p.counters = reinterpret_cast<int*>(ds->base + NOALLOC_CNT_OFF);
    p.err = reinterpret_cast<int*>(ds->base + NOALLOC_ERR_OFF);
    p.scale_log2e = (float)(1.4426950408889634 / sqrt((double)HD));
    p.nb = 1;
    p.nkv = nkv;
    p.kv0 = 0;
    p.hq_total = n_heads;
    p.nkv_total = nkv;
    p.cache_mode = CACHE_POSMAJOR;
    p.fused = 0;
    p.wait_limit = WAIT_LIMIT_CYCLES;
    p.t_begin[0] = 0;
    p.t_end[0] = pos + 1;
    p.unit_prefix[0] = 0;
    p.unit_prefix[1] = (long long)nkv * (((pos + 1) + DEC_TILE - 1) / DEC_TILE);
    p.total_units = p.unit_prefix[1];

    // One sequence: every KV head gets an equal share of the CTAs (the SM
    // count, at most 160), each cutting the rows 0..pos into ranges that meet
    // at multiples of the 16-row TMA box.
    const int G = std::min(ds->num_sms, NOALLOC_SLOTS);
    const int nrows = pos + 1;
    const int cap = 1 + (nrows - 1) / DEC_BOX;
    int np = 0;
    for (int g = 0; g < nkv; g++) {
        int k = G / nkv + (g < G % nkv ? 1 : 0);
        k = std::max(1, std::min(k, cap));
        int bnd[MAX_PIECES + 1];
        int nbd = 0;
        bnd[nbd++] = 0;
        for (int j = 1; j < k; j++) {
            const long long target = (long long)j * nrows / k;
            const int a = (int)(((target + DEC_BOX / 2) / DEC_BOX) * DEC_BOX);
            if (a > bnd[nbd - 1] && a < nrows) bnd[nbd++] = a;
        }
        bnd[nbd++] = nrows;
        for (int j = 0; j < nbd - 1; j++) {
            Piece& pc = p.pieces[np++];
            pc.g = g;
            pc.r0 = bnd[j];
            pc.r1 = bnd[j + 1];
            pc.i = (short)j;
            pc.k = (short)(nbd - 1);
        }
    }
    p.n_pieces = np;
    p.n_ctas = np;
    for (int c = 0; c < np; c++) p.cta_piece[c] = (short)c;

    // counters and the error word must start at zero
    if (cudaMemsetAsync(ds->base + NOALLOC_CNT_OFF, 0, NOALLOC_BYTES - NOALLOC_CNT_OFF, st) !=
        cudaSuccess)
        return record_error(Q3A_ERR_CUDA, "q3a_attn_decode_noalloc: clearing the counters failed");
    if (launch_decode(p, tk, tv, false, st) != cudaSuccess)
        return record_error(Q3A_ERR_CUDA, "q3a_attn_decode_noalloc: kernel launch failed");
    return Q3A_OK;
}

// Reads and clears the error word a bounded wait of the last noalloc launch
// on this device may have set: queued on `stream` behind that launch, then
// the host waits for the stream.  Nothing is allocated: the word is read
// into a host variable and cleared in place.
extern "C" int q3a_noalloc_check_error(void* stream) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return record_error(Q3A_ERR_CUDA, "q3a_noalloc_check_error: no current device");
    DeviceScratch* ds = nullptr;
    int rc = noalloc_setup(dev, &ds);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int h = 0;
    if (cudaMemcpyAsync(&h, ds->base + NOALLOC_ERR_OFF, sizeof(int), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return record_error(Q3A_ERR_CUDA, "q3a_noalloc_check_error: reading the error word failed");
    if (h == 0) return Q3A_OK;
    if (cudaMemsetAsync(ds->base + NOALLOC_ERR_OFF, 0, sizeof(int), st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return record_error(Q3A_ERR_CUDA, "q3a_noalloc_check_error: clearing the error word failed");
    return record_error(Q3A_ERR_TIMEOUT, "q3a_attn_decode_noalloc: a bounded device wait expired");
}
