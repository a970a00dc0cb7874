// q3a_api.cu -- the extern "C" entry points of include/q3attn.h.
//
// Owns the context: the paged head-major KV cache, its TMA tensor maps, the
// decode scratch (partials and arrival counters), host<->device staging for
// host-pointer mode, and the unit schedule the decode kernel consumes.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

#include "q3a_common.cuh"
#include "q3a_internal.h"

using namespace q3a;

// ------------------------------------------------------------------ errors
static thread_local char g_err[512] = "";

static int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

#define CUDA_TRY(expr)                                                                  \
    do {                                                                                \
        cudaError_t _e = (expr);                                                        \
        if (_e != cudaSuccess)                                                          \
            return fail(Q3A_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                        __FILE__, __LINE__);                                            \
    } while (0)

// ------------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D map over a row-major [rows][cols] tensor; box = box_cols x box_rows.
static int make_map_2d(CUtensorMap* m, const void* base, bool bf16, uint64_t cols, uint64_t rows,
                       uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(Q3A_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const size_t es = bf16 ? 2 : 4;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * es};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                    const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(Q3A_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): cols=%llu rows=%llu", (int)r,
                    (unsigned long long)cols, (unsigned long long)rows);
    return Q3A_OK;
}

// ------------------------------------------------------------------ context
struct q3a_ctx {
    q3a_cfg cfg;
    int nkv;              // kv heads held
    int kv0;
    int bf16;
    size_t esize;
    int pages_per_seq;
    int n_pages;          // per (layer, kv head)
    long long total_rows; // cache rows per K (or V) pool
    void* kcache = nullptr;
    void* vcache = nullptr;
    float* partials = nullptr;
    long long part_slots = 0;
    int* counters = nullptr;
    unsigned long long* words = nullptr;  // spread-merge slots (tagged words)
    unsigned* group_epoch = nullptr;      // spread-merge call number per group
    int* claims = nullptr;                // per-group unit counters of the balanced schedule
    float* pf_part = nullptr;             // prefill split partials (growable)
    size_t pf_part_floats = 0;
    int pf_key_tok = -1, pf_key_pos = -1; // prompt shape of the cached split choice
    int pf_nsplit = 1, pf_cap = 1;
    int* err = nullptr;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    long long wait_limit = WAIT_LIMIT_CYCLES;  // SM clocks per wait on another CTA / rank
    int deterministic = 0;         // 1: static row ranges (bitwise-repeatable results)
    CUtensorMap tmK, tmV;          // decode maps of the paged cache
    float inv_freq[64];
    float* d_inv_freq = nullptr;   // the same table in device memory
    // host-mode staging
    float* h_stage = nullptr;      // pinned
    float* d_stage = nullptr;
    size_t stage_floats = 0;
    // growable device scratch (uploads of caller caches, prefill q)
    void* d_scratch = nullptr;
    size_t scratch_bytes = 0;
    uint64_t launches = 0;
    // The last kernel this context queued, for the early cache streaming of
    // the next decode launch: a decode kernel may read cache rows before its
    // programmatic-dependency wait only when the kernel before it on the
    // same stream was this context's decode of another layer (or one that
    // appended nothing), so that no kernel still running can write them.
    cudaStream_t last_stream = nullptr;
    int last_decode_layer = -1;   // layer of the last launch if it was a decode, else -1
    int last_decode_wrote = 0;    // that decode appended a row to its layer
    int last_qkv_layer = -1;      // layer of the last launch if it was the projection kernel
    int last_qkv_pos = -1;        // the row that projection appended (sequence slot 0)
    // projection scratch (q3a_attn_layer_proj): partial sums and tickets
    float* qkv_part = nullptr;
    int* qkv_ticket = nullptr;
    size_t qkv_part_floats = 0;
    unsigned long long* wire_sum = nullptr;  // KV wire format: the payload checksum
    float* sub_q = nullptr;               // q3a_attn_sublayer: prepared q and xb [n_heads*128]
    float* sub_xb = nullptr;
    // peer-memory sequence shards (q3a_peer_export / q3a_peer_open)
    int peer_world = 0;
    int peer_rank = -1;
    float* peer_buf = nullptr;            // this rank's receive buffer
    float* peer_ptrs[PEER_MAX] = {};      // every rank's buffer, mapped here
    unsigned* peer_epoch = nullptr;       // call counter + finisher ticket
    unsigned* wo_epoch = nullptr;         // wo exchange: per-CTA call numbers [WO_MAX_CTAS]
    bool peer_ipc = false;                // peer_ptrs are IPC mappings (closed on destroy)
    // registered caller buffer for column all-gathers (q3a_peer_register)
    uint8_t* reg_buf = nullptr;           // the caller's buffer
    size_t reg_bytes = 0;
    unsigned* reg_flags = nullptr;        // [2 phases][PEER_MAX], written by peers
    unsigned* reg_state = nullptr;        // call number, CTA arrivals, go
    int reg_world = 0, reg_rank = -1;
    uint8_t* reg_peer[PEER_MAX] = {};     // every rank's buffer, mapped here
    unsigned* reg_peer_flags[PEER_MAX] = {};
    void* reg_ipc_bases[PEER_MAX] = {};   // mappings to close
    void* reg_ipc_flags[PEER_MAX] = {};
};

static int ensure_device(const q3a_ctx* c) {
    int cur = -1;
    CUDA_TRY(cudaGetDevice(&cur));
    if (cur != c->cfg.device) CUDA_TRY(cudaSetDevice(c->cfg.device));
    return Q3A_OK;
}

// Records that the last launch was neither a decode nor the projection
// kernel, so the next decode waits for it before reading the cache.
static inline void forget_last(q3a_ctx* c) {
    c->last_decode_layer = -1;
    c->last_qkv_layer = -1;
    c->last_qkv_pos = -1;
}

// Peer receive buffer: words per rank row of the sequence-shard region,
// words of the whole buffer, and the offset of its wo region.
static size_t peer_row(const q3a_ctx* c) { return (size_t)c->cfg.n_heads * HD + c->cfg.n_heads; }
static size_t peer_wo_offset(const q3a_ctx* c, int world) { return (size_t)2 * world * peer_row(c); }
static size_t peer_words(const q3a_ctx* c, int world) {
    return peer_wo_offset(c, world) + (size_t)2 * world * WO_MAX_ROWS;
}

// Host-pointer staging of n tokens: inputs [q | k | v | q gains | k gains]
// then outputs [xb | q out | k out], every part a multiple of 4 floats.
static size_t host_stage_floats(int n_heads, int n_kv, int n) {
    const size_t qd = (size_t)n * n_heads * HD, kd = (size_t)n * n_kv * HD;
    return (qd + 2 * kd + 2 * HD) + (2 * qd + kd);
}

static int grow_stage(q3a_ctx* c, size_t floats) {
    if (floats <= c->stage_floats) return Q3A_OK;
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->d_stage) cudaFree(c->d_stage);
    c->h_stage = nullptr;
    c->d_stage = nullptr;
    c->stage_floats = 0;
    if (cudaMallocHost(&c->h_stage, floats * 4) != cudaSuccess)
        return fail(Q3A_ERR_OOM, "pinned staging of %zu bytes", floats * 4);
    if (cudaMalloc(&c->d_stage, floats * 4) != cudaSuccess)
        return fail(Q3A_ERR_OOM, "device staging of %zu bytes", floats * 4);
    c->stage_floats = floats;
    return Q3A_OK;
}

static int grow_scratch(q3a_ctx* c, size_t bytes) {
    if (bytes <= c->scratch_bytes) return Q3A_OK;
    if (c->d_scratch) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->d_scratch);
    }
    c->d_scratch = nullptr;
    c->scratch_bytes = 0;
    if (cudaMalloc(&c->d_scratch, bytes) != cudaSuccess)
        return fail(Q3A_ERR_OOM, "device scratch of %zu bytes", bytes);
    c->scratch_bytes = bytes;
    return Q3A_OK;
}

extern "C" void q3a_cfg_default(q3a_cfg* cfg) {
    memset(cfg, 0, sizeof(*cfg));
    cfg->n_layers = 36;
    cfg->n_heads = 32;
    cfg->n_kv_heads = 8;
    cfg->head_dim = 128;
    cfg->max_seq = 4096;
    cfg->n_seqs = 1;
    cfg->kv_dtype = Q3A_KV_F32;
    cfg->page_tokens = 64;
    cfg->ptr_mode = Q3A_PTR_HOST;
    cfg->device = 0;
    cfg->norm_eps = 1e-6f;
    cfg->rope_theta = 5e6f;
    cfg->kv_head_begin = 0;
    cfg->kv_head_count = 0;
}

extern "C" const char* q3a_last_error(void) { return g_err; }

// Records a failure message for q3a_last_error() from another translation
// unit of the library and returns `code`.
int q3a::record_error(int code, const char* msg) { return fail(code, "%s", msg); }

cudaError_t q3a::ensure_smem_attr(const void* fn, int bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, int>> done;  // (kernel, device) pairs set
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& d : done)
        if (d.first == fn && d.second == dev) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    // Every kernel of the library asks for the largest shared-memory
    // carveout: an SM runs CTAs of different kernels side by side only in
    // one L1/shared split, so a small kernel that preferred more L1 would
    // keep a decode or prefill CTA off its SM until it exited.
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    done.emplace_back(fn, dev);
    return cudaSuccess;
}

static void destroy_ctx(q3a_ctx* c) {
    if (!c) return;
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (int r = 0; r < PEER_MAX; r++)
        if (c->peer_ipc && c->peer_ptrs[r] && c->peer_ptrs[r] != c->peer_buf)
            cudaIpcCloseMemHandle(c->peer_ptrs[r]);
    cudaFree(c->peer_buf);
    cudaFree(c->peer_epoch);
    for (int r = 0; r < PEER_MAX; r++) {
        if (c->reg_ipc_bases[r]) cudaIpcCloseMemHandle(c->reg_ipc_bases[r]);
        if (c->reg_ipc_flags[r]) cudaIpcCloseMemHandle(c->reg_ipc_flags[r]);
    }
    cudaFree(c->reg_flags);
    cudaFree(c->reg_state);
    cudaFree(c->kcache);
    cudaFree(c->vcache);
    cudaFree(c->partials);
    cudaFree(c->counters);
    cudaFree(c->words);
    cudaFree(c->group_epoch);
    cudaFree(c->claims);
    cudaFree(c->pf_part);
    cudaFree(c->qkv_part);
    cudaFree(c->qkv_ticket);
    cudaFree(c->wire_sum);
    cudaFree(c->sub_q);
    cudaFree(c->sub_xb);
    cudaFree(c->wo_epoch);
    cudaFree(c->err);
    cudaFree(c->d_inv_freq);
    cudaFree(c->d_stage);
    cudaFree(c->d_scratch);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

extern "C" int q3a_create(q3a_ctx** out, const q3a_cfg* cfg_in) {
    g_err[0] = 0;
    if (!out || !cfg_in) return fail(Q3A_ERR_INVALID, "null argument");
    *out = nullptr;
    q3a_cfg cfg = *cfg_in;
    if (cfg.page_tokens == 0) cfg.page_tokens = 64;
    if (cfg.kv_head_count == 0) cfg.kv_head_count = cfg.n_kv_heads - cfg.kv_head_begin;
    if (cfg.head_dim != HD)
        return fail(Q3A_ERR_UNSUPPORTED, "head_dim %d: only 128 is implemented", cfg.head_dim);
    if (cfg.n_kv_heads <= 0 || cfg.n_heads != GQA * cfg.n_kv_heads)
        return fail(Q3A_ERR_UNSUPPORTED, "n_heads %d / n_kv_heads %d: only 4 query heads per KV "
                    "head are implemented", cfg.n_heads, cfg.n_kv_heads);
    if (cfg.n_layers <= 0 || cfg.max_seq <= 0 || cfg.n_seqs <= 0)
        return fail(Q3A_ERR_INVALID, "n_layers, max_seq and n_seqs must be positive");
    if (cfg.page_tokens % DEC_TILE != 0)
        return fail(Q3A_ERR_INVALID, "page_tokens %d is not a multiple of %d", cfg.page_tokens,
                    DEC_TILE);
    if (cfg.kv_dtype != Q3A_KV_F32 && cfg.kv_dtype != Q3A_KV_BF16)
        return fail(Q3A_ERR_INVALID, "kv_dtype %d", cfg.kv_dtype);
    if (cfg.ptr_mode != Q3A_PTR_HOST && cfg.ptr_mode != Q3A_PTR_DEVICE)
        return fail(Q3A_ERR_INVALID, "ptr_mode %d", cfg.ptr_mode);
    if (cfg.kv_head_begin < 0 || cfg.kv_head_count <= 0 ||
        cfg.kv_head_begin + cfg.kv_head_count > cfg.n_kv_heads)
        return fail(Q3A_ERR_INVALID, "kv head range [%d, +%d) outside 0..%d", cfg.kv_head_begin,
                    cfg.kv_head_count, cfg.n_kv_heads);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(Q3A_ERR_CUDA, "no CUDA device available");
    if (cfg.device < 0 || cfg.device >= ndev)
        return fail(Q3A_ERR_INVALID, "device %d of %d", cfg.device, ndev);
    CUDA_TRY(cudaSetDevice(cfg.device));
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, cfg.device));
    if (prop.major != 10)
        return fail(Q3A_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                    cfg.device, prop.major, prop.minor);

    q3a_ctx* c = new q3a_ctx();
    c->cfg = cfg;
    c->nkv = cfg.kv_head_count;
    c->kv0 = cfg.kv_head_begin;
    c->bf16 = cfg.kv_dtype == Q3A_KV_BF16;
    c->esize = c->bf16 ? 2 : 4;
    c->num_sms = prop.multiProcessorCount;
    c->pages_per_seq = (cfg.max_seq + cfg.page_tokens - 1) / cfg.page_tokens;
    c->n_pages = c->pages_per_seq * cfg.n_seqs;
    c->total_rows = (long long)cfg.n_layers * c->nkv * c->n_pages * cfg.page_tokens;
    if (c->total_rows >= (1LL << 31)) {
        destroy_ctx(c);
        return fail(Q3A_ERR_INVALID, "cache of %lld rows exceeds the 2^31 TMA coordinate range",
                    c->total_rows);
    }
    // RoPE inverse frequencies exactly as apply_rope forms them
    // (qwen3-8b/cpu/main.c:1285): 1.0f / powf(theta, (float)i / head_dim).
    for (int i = 0; i < HD; i += 2)
        c->inv_freq[i / 2] = 1.0f / powf(cfg.rope_theta, (float)i / HD);

    const size_t cache_bytes = (size_t)c->total_rows * HD * c->esize;
    int rc = Q3A_OK;
    if (cudaMalloc(&c->kcache, cache_bytes) != cudaSuccess ||
        cudaMalloc(&c->vcache, cache_bytes) != cudaSuccess) {
        destroy_ctx(c);
        return fail(Q3A_ERR_OOM, "KV cache of 2 x %zu bytes", cache_bytes);
    }
    const int max_groups = Q3A_MAX_BATCH * cfg.n_kv_heads;
    c->part_slots = (long long)c->num_sms + max_groups;
    if (cudaMalloc(&c->partials, (size_t)c->part_slots * PART_STRIDE * 4) != cudaSuccess ||
        cudaMalloc(&c->counters, (size_t)max_groups * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&c->words, (size_t)MAX_PIECES * PART_STRIDE * 8) != cudaSuccess ||
        cudaMalloc(&c->group_epoch, (size_t)MAX_PIECES * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&c->claims, (size_t)MAX_PIECES * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&c->err, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&c->d_inv_freq, sizeof(c->inv_freq)) != cudaSuccess) {
        destroy_ctx(c);
        return fail(Q3A_ERR_OOM, "context scratch");
    }
    // a blocking stream: it orders with the legacy default stream, so device
    // buffers that default-stream work wrote before a call are ready for it,
    // and default-stream work queued after a call sees its results
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamDefault) != cudaSuccess) {
        destroy_ctx(c);
        return fail(Q3A_ERR_CUDA, "stream creation");
    }
    c->stream = c->own_stream;
    if (cudaMemsetAsync(c->kcache, 0, cache_bytes, c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->vcache, 0, cache_bytes, c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->counters, 0, (size_t)max_groups * sizeof(int), c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->words, 0, (size_t)MAX_PIECES * PART_STRIDE * 8, c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->group_epoch, 0, (size_t)MAX_PIECES * sizeof(unsigned), c->stream) !=
            cudaSuccess ||
        cudaMemsetAsync(c->claims, 0, (size_t)MAX_PIECES * sizeof(int), c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->err, 0, sizeof(int), c->stream) != cudaSuccess ||
        cudaMemcpyAsync(c->d_inv_freq, c->inv_freq, sizeof(c->inv_freq), cudaMemcpyHostToDevice,
                        c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess) {
        destroy_ctx(c);
        return fail(Q3A_ERR_CUDA, "cache initialisation");
    }
    rc = make_map_2d(&c->tmK, c->kcache, c->bf16, HD, (uint64_t)c->total_rows, HD, DEC_BOX,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc == Q3A_OK)
        rc = make_map_2d(&c->tmV, c->vcache, c->bf16, HD, (uint64_t)c->total_rows, HD, DEC_BOX,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != Q3A_OK) {
        destroy_ctx(c);
        return rc;
    }
    const size_t stage = host_stage_floats(cfg.n_heads, cfg.n_kv_heads, 1);
    rc = grow_stage(c, stage);
    if (rc != Q3A_OK) {
        destroy_ctx(c);
        return rc;
    }
    *out = c;
    return Q3A_OK;
}

extern "C" int q3a_destroy(q3a_ctx* c) {
    if (!c) return Q3A_OK;
    ensure_device(c);
    destroy_ctx(c);
    return Q3A_OK;
}

extern "C" int q3a_set_stream(q3a_ctx* c, void* s) {
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    c->stream = s ? reinterpret_cast<cudaStream_t>(s) : c->own_stream;
    return Q3A_OK;
}

extern "C" int q3a_sync(q3a_ctx* c) {
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    int rc = ensure_device(c);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

// ------------------------------------------------------------------ graphs
struct q3a_graph {
    cudaGraphExec_t exec = nullptr;
    int device = 0;
};

extern "C" int q3a_graph_begin(q3a_ctx* c) {
    g_err[0] = 0;
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    if (c->cfg.ptr_mode != Q3A_PTR_DEVICE)
        return fail(Q3A_ERR_UNSUPPORTED, "graphs record device-pointer calls only");
    int rc = ensure_device(c);
    if (rc) return rc;
    CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    // the first recorded decode must not assume which kernel runs before the
    // graph when it is replayed
    forget_last(c);
    return Q3A_OK;
}

extern "C" int q3a_graph_end(q3a_ctx* c, q3a_graph** out) {
    g_err[0] = 0;
    if (!c || !out) return fail(Q3A_ERR_INVALID, "null argument");
    *out = nullptr;
    int rc = ensure_device(c);
    if (rc) return rc;
    cudaGraph_t g = nullptr;
    CUDA_TRY(cudaStreamEndCapture(c->stream, &g));
    cudaGraphExec_t e = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&e, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) return fail(Q3A_ERR_CUDA, "graph instantiation: %s", cudaGetErrorString(ie));
    q3a_graph* h = new q3a_graph;
    h->exec = e;
    h->device = c->cfg.device;
    *out = h;
    forget_last(c);
    return Q3A_OK;
}

extern "C" int q3a_graph_launch(q3a_ctx* c, q3a_graph* g) {
    g_err[0] = 0;
    if (!c || !g) return fail(Q3A_ERR_INVALID, "null argument");
    if (g->device != c->cfg.device) return fail(Q3A_ERR_INVALID, "graph of device %d", g->device);
    int rc = ensure_device(c);
    if (rc) return rc;
    CUDA_TRY(cudaGraphLaunch(g->exec, c->stream));
    forget_last(c);
    return Q3A_OK;
}

extern "C" int q3a_graph_destroy(q3a_graph* g) {
    if (!g) return Q3A_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != g->device) cudaSetDevice(g->device);
    cudaGraphExecDestroy(g->exec);
    delete g;
    return Q3A_OK;
}

extern "C" int q3a_check_device_error(q3a_ctx* c) {
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    int rc = ensure_device(c);
    if (rc) return rc;
    int h = 0;
    CUDA_TRY(cudaMemcpyAsync(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (h != 0) {
        const int max_groups = Q3A_MAX_BATCH * c->cfg.n_kv_heads;
        CUDA_TRY(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
        // an abandoned launch may have left arrival counters behind, and
        // spread-merge words of a call whose number was never advanced
        CUDA_TRY(cudaMemsetAsync(c->counters, 0, (size_t)max_groups * sizeof(int), c->stream));
        CUDA_TRY(cudaMemsetAsync(c->words, 0, (size_t)MAX_PIECES * PART_STRIDE * 8, c->stream));
        CUDA_TRY(cudaMemsetAsync(c->group_epoch, 0, (size_t)MAX_PIECES * sizeof(unsigned), c->stream));
        CUDA_TRY(cudaMemsetAsync(c->claims, 0, (size_t)MAX_PIECES * sizeof(int), c->stream));
        // and the projection's per-head tickets of an unfinished call
        if (c->qkv_ticket)
            CUDA_TRY(cudaMemsetAsync(c->qkv_ticket, 0,
                                     (size_t)(c->cfg.n_heads + 2 * c->cfg.n_kv_heads) * sizeof(int),
                                     c->stream));
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        return fail(Q3A_ERR_TIMEOUT, "a bounded device wait expired (device error %d)", h);
    }
    return Q3A_OK;
}

extern "C" uint64_t q3a_launch_count(const q3a_ctx* c) { return c ? c->launches : 0; }

extern "C" int q3a_set_deterministic(q3a_ctx* c, int on) {
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    c->deterministic = on ? 1 : 0;
    return Q3A_OK;
}

extern "C" int q3a_set_wait_limit(q3a_ctx* c, double seconds) {
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    if (!(seconds >= 0.0) || seconds > 60.0)
        return fail(Q3A_ERR_INVALID, "wait limit %g s outside [0, 60]", seconds);
    if (seconds == 0.0) {
        c->wait_limit = WAIT_LIMIT_CYCLES;
        return Q3A_OK;
    }
    int rc = ensure_device(c);
    if (rc) return rc;
    // clock64 counts SM clocks: the limit in clocks at the device's highest
    // SM clock (at lower clocks the wait lasts proportionally longer)
    int khz = 0;
    if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, c->cfg.device) != cudaSuccess || khz <= 0)
        khz = 2000000;
    c->wait_limit = std::max(1LL, (long long)(seconds * khz * 1000.0));
    return Q3A_OK;
}

// ------------------------------------------------------------------ decode dispatch
static void base_params(q3a_ctx* c, DecodeParams& p, int layer) {
    memset(&p, 0, sizeof(p));
    p.kcache = c->kcache;
    p.vcache = c->vcache;
    p.partials = c->partials;
    p.counters = c->counters;
    p.words = c->words;
    p.group_epoch = c->group_epoch;
    p.claim = c->claims;
    p.spread = 1;
    p.err = c->err;
    p.eps = c->cfg.norm_eps;
    p.scale_log2e = (float)(1.4426950408889634 / sqrt((double)HD));
    p.nkv = c->nkv;
    p.kv0 = c->kv0;
    p.hq_total = c->cfg.n_heads;
    p.nkv_total = c->cfg.n_kv_heads;
    p.layer = layer;
    p.pages_per_seq = c->pages_per_seq;
    p.page_tokens = c->cfg.page_tokens;
    p.n_pages = c->n_pages;
    p.cache_mode = CACHE_PAGED;
    p.inv_freq = c->d_inv_freq;
    p.wait_limit = c->wait_limit;
}

// Piece-mode schedule: every (sequence, kv head) group gets k_g >= 1 CTAs in
// proportion to its rows (largest-quotient rounding to the SM count), and its
// rows are cut into k_g ranges at multiples of the 16-row TMA box, so one CTA
// handles one range of one group.  Pieces are numbered group-major, which
// makes the pieces (and partial slots) of a group consecutive.
static void schedule_pieces(q3a_ctx* c, DecodeParams& p) {
    const int nkv = p.nkv;
    const int ng = p.nb * nkv;
    const int G = std::min(c->num_sms, MAX_PIECES);
    std::vector<double> work(ng);
    std::vector<int> k(ng), cap(ng);
    double total = 0.0;
    for (int g = 0; g < ng; g++) {
        const int b = g / nkv;
        const int tb = p.t_begin[b], te = p.t_end[b];
        const int rows = te - tb;
        work[g] = rows + (p.fused ? 16.0 : 0.0);  // the new token costs about one box
        total += work[g];
        const int first = (tb / DEC_BOX + 1) * DEC_BOX;
        const int last = te > 0 ? ((te - 1) / DEC_BOX) * DEC_BOX : -1;
        cap[g] = 1 + (last >= first ? (last - first) / DEC_BOX + 1 : 0);
    }
    int sum = 0;
    for (int g = 0; g < ng; g++) {
        int kk = (int)std::floor(G * work[g] / total);
        k[g] = std::max(1, std::min(kk, cap[g]));
        sum += k[g];
    }
    while (sum > G) {  // only when many small groups were lifted to 1
        int best = -1;
        for (int g = 0; g < ng; g++)
            if (k[g] > 1 && (best < 0 || work[g] / (k[g] - 1) < work[best] / (k[best] - 1))) best = g;
        if (best < 0) break;
        k[best]--;
        sum--;
    }
    while (sum < G) {
        int best = -1;
        for (int g = 0; g < ng; g++)
            if (k[g] < cap[g] && (best < 0 || work[g] / k[g] > work[best] / k[best])) best = g;
        if (best < 0) break;
        k[best]++;
        sum++;
    }
    int np = 0;
    for (int g = 0; g < ng; g++) {
        const int b = g / nkv;
        const int tb = p.t_begin[b], te = p.t_end[b];
        const long long rows = te - tb;
        int bnd[MAX_PIECES + 1];
        int nb = 0;
        bnd[nb++] = tb;
        for (int j = 1; j < k[g]; j++) {
            const long long target = tb + j * rows / k[g];
            int a = (int)(((target + DEC_BOX / 2) / DEC_BOX) * DEC_BOX);
            if (a > bnd[nb - 1] && a < te) bnd[nb++] = a;
        }
        bnd[nb++] = te;
        const int kg = nb - 1;
        for (int j = 0; j < kg; j++) {
            Piece& pc = p.pieces[np++];
            pc.g = g;
            pc.r0 = bnd[j];
            pc.r1 = bnd[j + 1];
            pc.i = (short)j;
            pc.k = (short)kg;
        }
    }
    p.n_pieces = np;
    p.n_ctas = np;
    // CTA c takes pieces of the groups in turn (group 0's first piece, group
    // 1's first, ..., group 0's second, ...): SMs with lower memory
    // throughput sit in runs of consecutive ids, so interleaving gives every
    // group a similar mix
    int next[MAX_PIECES], first[MAX_PIECES];
    int q = 0;
    for (int g = 0; g < ng; g++) {
        first[g] = q;
        next[g] = 0;
        while (q < np && p.pieces[q].g == g) q++;
    }
    int cta = 0;
    while (cta < np) {
        for (int g = 0; g < ng && cta < np; g++) {
            const int pi = first[g] + next[g];
            if (pi < np && p.pieces[pi].g == g) {
                p.cta_piece[cta++] = (short)pi;
                next[g]++;
            }
        }
    }
}

// Fills the schedule: piece mode when every group can have its own CTA,
// else the linear unit list (unit_prefix / total_units / n_ctas).
static int schedule(q3a_ctx* c, DecodeParams& p) {
    long long acc = 0;
    p.unit_prefix[0] = 0;
    for (int b = 0; b < p.nb; b++) {
        const int tb = p.t_begin[b], te = p.t_end[b];
        const int a0 = tb / DEC_TILE;
        const long long ncu = te > tb ? (te + DEC_TILE - 1) / DEC_TILE - a0 : 0;
        const long long units = ncu + (p.fused ? 1 : 0);
        if (units == 0) return fail(Q3A_ERR_INVALID, "sequence %d has nothing to attend", b);
        acc += units * p.nkv;
        p.unit_prefix[b + 1] = acc;
    }
    p.total_units = acc;
    p.n_pieces = 0;
    const int n_lin = (int)std::min<long long>(c->num_sms, acc);
    if ((long long)p.nb * p.nkv <= std::min(c->num_sms, MAX_PIECES)) {
        schedule_pieces(c, p);
        // Piece mode gives every group whole CTAs.  With many groups of
        // unequal length (ragged batches, few KV heads per context) the
        // longest ranges can sit far above the even share of the linear
        // list; then the linear list is used instead.
        double piece_max = 0.0;
        for (int i = 0; i < p.n_pieces; i++) {
            const Piece& pc = p.pieces[i];
            const double u = (pc.r1 - pc.r0) / (double)DEC_TILE + (p.fused && pc.i == pc.k - 1 ? 1 : 0);
            piece_max = std::max(piece_max, u);
        }
        const double lin_max = std::ceil((double)acc / n_lin) + 1.0;
        if (piece_max > 1.2 * lin_max) {
            p.n_pieces = 0;
            p.n_ctas = n_lin;
        }
    } else {
        p.n_ctas = n_lin;
    }
    const long long slots = (long long)p.n_ctas + (long long)p.nb * p.nkv;
    if (slots > c->part_slots) return fail(Q3A_ERR_INVALID, "decode scratch too small");
    return Q3A_OK;
}

static int run_decode(q3a_ctx* c, DecodeParams& p, const CUtensorMap& tk, const CUtensorMap& tv,
                      bool bf16) {
    int rc = schedule(c, p);
    if (rc) return rc;
    // the context's bf16 paged cache is consumed on the tensor cores
    p.tc = (bf16 && p.cache_mode == CACHE_PAGED) ? 1 : 0;
    // balanced schedule: piece-mode ranges of the paged cache claim units
    p.dyn = (!c->deterministic && p.n_pieces > 0 && p.spread && p.cache_mode == CACHE_PAGED) ? 1 : 0;
    // early cache streaming: the rows this launch reads from the context's
    // cache cannot be written by the kernel it depends on (the previous
    // launch on this stream was this context's decode of another layer, or
    // a decode that appended nothing), and every kernel of the library
    // releases its dependents only after its own dependency wait, so no
    // earlier kernel is still running either
    p.early = (p.cache_mode == CACHE_PAGED && c->last_decode_layer >= 0 &&
               c->last_stream == c->stream &&
               (c->last_decode_layer != p.layer || !c->last_decode_wrote))
                  ? 1
                  : 0;
    p.early_rows = INT_MAX;
    // after this context's projection kernel, which appends one row: the
    // balanced schedule streams the rows below it early (rows of another
    // layer are all safe)
    if (p.cache_mode == CACHE_PAGED && p.dyn && c->last_qkv_pos >= 0 &&
        c->last_stream == c->stream) {
        p.early = 1;
        p.early_rows = c->last_qkv_layer == p.layer ? c->last_qkv_pos : INT_MAX;
    }
    CUDA_TRY(launch_decode(p, tk, tv, bf16, c->stream));
    c->launches++;
    forget_last(c);
    if (p.cache_mode == CACHE_PAGED) {
        c->last_stream = c->stream;
        c->last_decode_layer = p.layer;
        c->last_decode_wrote = p.fused;
    }
    return Q3A_OK;
}

// Host-pointer form of the fused block for n tokens: the inputs are staged in
// pinned memory and copied to the device in one transfer; the decode kernel
// writes xb and the rotated q and k straight into pinned memory over the bus
// (no device-to-host copy: measured faster than staging them back); one
// stream synchronisation, then the results go to the caller's buffers.  A context holding some KV heads only writes their
// columns of xb: the caller's other columns are staged first and kept.
static int host_block(q3a_ctx* c, DecodeParams& p, float* xb, float* q, float* k, const float* v,
                      const float* qw, const float* kw, int n) {
    const size_t qd = (size_t)n * c->cfg.n_heads * HD, kd = (size_t)n * c->cfg.n_kv_heads * HD;
    int rc = grow_stage(c, host_stage_floats(c->cfg.n_heads, c->cfg.n_kv_heads, n));
    if (rc) return rc;
    const size_t n_in = qd + 2 * kd + 2 * HD;
    float* hs = c->h_stage;
    float* ds = c->d_stage;
    float *h_q = hs, *h_k = h_q + qd, *h_v = h_k + kd, *h_qw = h_v + kd, *h_kw = h_qw + HD;
    float *h_xb = hs + n_in, *h_qo = h_xb + qd, *h_ko = h_qo + qd;
    float *d_q = ds, *d_k = d_q + qd, *d_v = d_k + kd, *d_qw = d_v + kd, *d_kw = d_qw + HD;
    memcpy(h_q, q, qd * 4);
    memcpy(h_k, k, kd * 4);
    memcpy(h_v, v, kd * 4);
    memcpy(h_qw, qw, HD * 4);
    memcpy(h_kw, kw, HD * 4);
    const bool partial_cols = c->nkv != c->cfg.n_kv_heads;
    if (partial_cols) memcpy(h_xb, xb, qd * 4);
    CUDA_TRY(cudaMemcpyAsync(d_q, h_q, n_in * 4, cudaMemcpyHostToDevice, c->stream));
    p.q = d_q; p.k_new = d_k; p.v_new = d_v; p.q_norm_w = d_qw; p.k_norm_w = d_kw;
    p.q_out = h_qo; p.k_out = h_ko; p.xb = h_xb;
    rc = run_decode(c, p, c->tmK, c->tmV, c->bf16);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    memcpy(xb, h_xb, qd * 4);
    // the rotated q and k: whole rows from a context holding every KV head,
    // else the held heads' slices (the caller's rotation of the others is
    // not this context's to give)
    if (!partial_cols) {
        memcpy(q, h_qo, qd * 4);
        memcpy(k, h_ko, kd * 4);
    } else {
        const size_t qh = (size_t)c->nkv * GQA * HD, kh = (size_t)c->nkv * HD;
        for (int b = 0; b < n; b++) {
            const size_t qo = (size_t)b * c->cfg.n_heads * HD + (size_t)c->kv0 * GQA * HD;
            const size_t ko = (size_t)b * c->cfg.n_kv_heads * HD + (size_t)c->kv0 * HD;
            memcpy(q + qo, h_qo + qo, qh * 4);
            memcpy(k + ko, h_ko + ko, kh * 4);
        }
    }
    return Q3A_OK;
}

extern "C" int q3a_attn_layer(q3a_ctx* c, float* xb, float* q, float* k, const float* v,
                              const float* qw, const float* kw, int layer, int pos) {
    g_err[0] = 0;
    if (!c || !xb || !q || !k || !v || !qw || !kw) return fail(Q3A_ERR_INVALID, "null argument");
    if (c->nkv != c->cfg.n_kv_heads)
        return fail(Q3A_ERR_INVALID, "q3a_attn_layer needs a context holding all KV heads");
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    if (pos < 0 || pos >= c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "pos %d outside [0, %d)", pos, c->cfg.max_seq);
    int rc = ensure_device(c);
    if (rc) return rc;
    DecodeParams p;
    base_params(c, p, layer);
    p.nb = 1;
    p.fused = 1;
    p.t_begin[0] = 0;
    p.t_end[0] = pos;
    p.pos[0] = pos;
    p.slot[0] = 0;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        p.q = q; p.k_new = k; p.v_new = v; p.q_norm_w = qw; p.k_norm_w = kw;
        p.q_out = q; p.k_out = k; p.xb = xb;
        return run_decode(c, p, c->tmK, c->tmV, c->bf16);
    }
    return host_block(c, p, xb, q, k, v, qw, kw, 1);
}

// Validates and launches the projection kernel (qkv_kernel) of one token at
// slot 0: the q, k, v fp16 GEMVs of the held KV heads (with the layer's
// input RMSNorm first when norm_w is given) fused with QK-RMSNorm, RoPE and
// the KV append.
static int launch_proj(q3a_ctx* c, float* q, float* k, float* v, const float* x, const float* norm_w,
                       const void* wq, const void* wk, const void* wv, int dim, const float* qw,
                       const float* kw, int layer, int pos) {
    if (!c || !q || !x || !wq || !wk || !wv || !qw || !kw)
        return fail(Q3A_ERR_INVALID, "null argument");
    if (c->cfg.ptr_mode != Q3A_PTR_DEVICE)
        return fail(Q3A_ERR_UNSUPPORTED, "the projection entry points take device pointers only");
    if (dim <= 0 || dim % 8 != 0 || dim > WO_MAX_ROWS)
        return fail(Q3A_ERR_UNSUPPORTED, "dim %d: multiples of 8 up to %d are implemented", dim,
                    WO_MAX_ROWS);
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    if (pos < 0 || pos >= c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "pos %d outside [0, %d)", pos, c->cfg.max_seq);
    const uintptr_t align = (uintptr_t)x | (uintptr_t)norm_w | (uintptr_t)wq | (uintptr_t)wk |
                            (uintptr_t)wv | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v |
                            (uintptr_t)qw | (uintptr_t)kw;
    if (align & 15) return fail(Q3A_ERR_INVALID, "the vectors and weights must be 16-byte aligned");
    int rc = ensure_device(c);
    if (rc) return rc;
    const int nkv = c->nkv, nq = nkv * GQA;
    const int heads_all = c->cfg.n_heads + 2 * c->cfg.n_kv_heads;
    const int rows_total = (nq + 2 * nkv) * HD;
    if (!c->qkv_part) {
        if (cudaMalloc(&c->qkv_ticket, (size_t)heads_all * sizeof(int)) != cudaSuccess ||
            cudaMalloc(&c->qkv_part, (size_t)heads_all * HD * sizeof(float)) != cudaSuccess)
            return fail(Q3A_ERR_OOM, "projection scratch");
        CUDA_TRY(cudaMemsetAsync(c->qkv_ticket, 0, (size_t)heads_all * sizeof(int), c->stream));
        c->qkv_part_floats = (size_t)heads_all * HD;
        forget_last(c);  // the memset above is a launch on the stream
    }
    QkvParams qp;
    memset(&qp, 0, sizeof(qp));
    qp.x = x;
    qp.norm_w = norm_w;
    qp.wq = reinterpret_cast<const __half*>(wq);
    qp.wk = reinterpret_cast<const __half*>(wk);
    qp.wv = reinterpret_cast<const __half*>(wv);
    qp.q_norm_w = qw;
    qp.k_norm_w = kw;
    qp.q_out = q;
    qp.k_out = k;
    qp.v_out = v;
    qp.kcache = c->kcache;
    qp.vcache = c->vcache;
    qp.part = c->qkv_part;
    qp.ticket = c->qkv_ticket;
    qp.err = c->err;
    qp.inv_freq = c->d_inv_freq;
    qp.eps = c->cfg.norm_eps;
    qp.dim = dim;
    qp.nq = nq;
    qp.nkv = nkv;
    qp.kv0 = c->kv0;
    qp.rows_total = rows_total;
    qp.layer = layer;
    qp.pos = pos;
    qp.slot = 0;
    qp.pages_per_seq = c->pages_per_seq;
    qp.page_tokens = c->cfg.page_tokens;
    qp.n_pages = c->n_pages;
    // one CTA per SM; at least one per head, so that a CTA's rows (fewer
    // than 128) touch at most two heads
    const int n_ctas = std::min(rows_total, std::max(c->num_sms, nq + 2 * nkv));
    CUDA_TRY(launch_qkv(qp, c->bf16 != 0, n_ctas, c->stream));
    c->launches++;
    forget_last(c);
    c->last_stream = c->stream;
    c->last_qkv_layer = layer;
    c->last_qkv_pos = pos;
    return Q3A_OK;
}

extern "C" int q3a_qkv_proj(q3a_ctx* c, float* q, float* k, float* v, const float* x,
                            const void* wq, const void* wk, const void* wv, int dim,
                            const float* qw, const float* kw, int layer, int pos) {
    g_err[0] = 0;
    return launch_proj(c, q, k, v, x, nullptr, wq, wk, wv, dim, qw, kw, layer, pos);
}

// The decode of the held heads over rows [0, pos] of slot 0 with the
// prepared q (after launch_proj).
static int decode_after_proj(q3a_ctx* c, float* xb, const float* q, int layer, int pos,
                             const void* wo_next = nullptr, int wo_rows = 0) {
    DecodeParams p;
    base_params(c, p, layer);
    if (wo_next) {  // the wo kernel's rows (held columns) into L2 meanwhile
        p.pf_base = reinterpret_cast<const uint8_t*>(wo_next) + (size_t)c->kv0 * GQA * HD * 2;
        p.pf_rows = wo_rows;
        p.pf_row_bytes = c->nkv * GQA * HD * 2;
        p.pf_ld_bytes = (long long)c->cfg.n_heads * HD * 2;
    }
    p.nb = 1;
    p.fused = 0;
    p.t_begin[0] = 0;
    p.t_end[0] = pos + 1;
    p.slot[0] = 0;
    p.q = q;
    p.xb = xb;
    return run_decode(c, p, c->tmK, c->tmV, c->bf16);
}

// The projections (launch_proj), then the decode of the layer over rows
// [0, pos] with the prepared q.  Device pointers only.
extern "C" int q3a_attn_layer_proj(q3a_ctx* c, float* xb, float* q, float* k, float* v,
                                   const float* x, const void* wq, const void* wk, const void* wv,
                                   int dim, const float* qw, const float* kw, int layer, int pos) {
    g_err[0] = 0;
    if (!xb) return fail(Q3A_ERR_INVALID, "null argument");
    int rc = launch_proj(c, q, k, v, x, nullptr, wq, wk, wv, dim, qw, kw, layer, pos);
    if (rc) return rc;
    return decode_after_proj(c, xb, q, layer, pos);
}

// x += wo[:, held columns] . xb[held columns], summed over the peer set when
// one is open with more than one rank.
static int launch_wo_residual(q3a_ctx* c, float* x, const float* xb, const void* wo, int dim) {
    if (!c || !x || !xb || !wo) return fail(Q3A_ERR_INVALID, "null argument");
    if (c->cfg.ptr_mode != Q3A_PTR_DEVICE)
        return fail(Q3A_ERR_UNSUPPORTED, "the projection entry points take device pointers only");
    if (dim <= 0 || dim > WO_MAX_ROWS)
        return fail(Q3A_ERR_UNSUPPORTED, "dim %d: up to %d rows are implemented", dim, WO_MAX_ROWS);
    if (((uintptr_t)x | (uintptr_t)xb | (uintptr_t)wo) & 15)
        return fail(Q3A_ERR_INVALID, "x, xb and wo must be 16-byte aligned");
    if (c->cfg.n_heads * HD > WO_MAX_ROWS)
        return fail(Q3A_ERR_UNSUPPORTED, "wo with %d columns: up to %d are implemented",
                    c->cfg.n_heads * HD, WO_MAX_ROWS);
    const bool peers = c->peer_rank >= 0 && c->peer_world > 1;
    if (c->nkv != c->cfg.n_kv_heads && !peers)
        return fail(Q3A_ERR_INVALID,
                    "a context holding some KV heads sums the ranks' wo partials over its peer set "
                    "(q3a_peer_export / q3a_peer_open first)");
    int rc = ensure_device(c);
    if (rc) return rc;
    WoParams wp;
    memset(&wp, 0, sizeof(wp));
    wp.w = reinterpret_cast<const __half*>(wo);
    wp.ld = c->cfg.n_heads * HD;
    wp.col0 = c->kv0 * GQA * HD;
    wp.ncols = c->nkv * GQA * HD;
    wp.xb = xb;
    wp.x = x;
    wp.rows = dim;
    wp.world = peers ? c->peer_world : 1;
    wp.rank = peers ? c->peer_rank : 0;
    if (peers) {
        const size_t off = peer_wo_offset(c, c->peer_world);
        for (int r = 0; r < c->peer_world; r++)
            wp.recv[r] = reinterpret_cast<unsigned long long*>(c->peer_ptrs[r]) + off;
        wp.epoch = c->wo_epoch;
    }
    wp.wait_limit = c->wait_limit;
    wp.err = c->err;
    // one CTA per SM; every rank uses the same count (its CTA c exchanges
    // with CTA c of the others)
    const int n_ctas = std::min(std::min(dim, c->num_sms), WO_MAX_CTAS);
    // the sender warp counts at most 64 ring stages per CTA
    const int stage_rows = 32768 / (wp.ncols * 2), cta_rows = (dim + n_ctas - 1) / n_ctas;
    if ((cta_rows + stage_rows - 1) / stage_rows > 64)
        return fail(Q3A_ERR_UNSUPPORTED, "wo of %d rows over %d SMs: too many rows per SM", dim,
                    n_ctas);
    CUDA_TRY(launch_wo(wp, n_ctas, c->stream));
    c->launches++;
    forget_last(c);
    return Q3A_OK;
}

extern "C" int q3a_wo_residual(q3a_ctx* c, float* x, const float* xb, const void* wo, int dim) {
    g_err[0] = 0;
    return launch_wo_residual(c, x, xb, wo, dim);
}

extern "C" int q3a_attn_sublayer(q3a_ctx* c, float* x, const float* att_norm_w, const void* wq,
                                 const void* wk, const void* wv, const float* q_norm_w,
                                 const float* k_norm_w, const void* wo, int dim, int layer, int pos) {
    g_err[0] = 0;
    if (!c || !x || !att_norm_w) return fail(Q3A_ERR_INVALID, "null argument");
    int rc = ensure_device(c);
    if (rc) return rc;
    if (!c->sub_q) {
        const size_t n = (size_t)c->cfg.n_heads * HD;
        if (cudaMalloc(&c->sub_q, n * 4) != cudaSuccess || cudaMalloc(&c->sub_xb, n * 4) != cudaSuccess)
            return fail(Q3A_ERR_OOM, "sublayer scratch");
    }
    rc = launch_proj(c, c->sub_q, nullptr, nullptr, x, att_norm_w, wq, wk, wv, dim, q_norm_w,
                     k_norm_w, layer, pos);
    if (rc) return rc;
    rc = decode_after_proj(c, c->sub_xb, c->sub_q, layer, pos, wo, dim);
    if (rc) return rc;
    return launch_wo_residual(c, x, c->sub_xb, wo, dim);
}

extern "C" int q3a_attn_layer_batched(q3a_ctx* c, float* xb, float* q, float* k, const float* v,
                                      const float* qw, const float* kw, int layer,
                                      const int* seq_ids, const int* pos, int n) {
    g_err[0] = 0;
    if (!c || !xb || !q || !k || !v || !qw || !kw || !seq_ids || !pos)
        return fail(Q3A_ERR_INVALID, "null argument");
    if (n <= 0 || n > Q3A_MAX_BATCH) return fail(Q3A_ERR_INVALID, "batch of %d", n);
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    int rc = ensure_device(c);
    if (rc) return rc;
    DecodeParams p;
    base_params(c, p, layer);
    p.nb = n;
    p.fused = 1;
    std::vector<char> seen(c->cfg.n_seqs, 0);
    for (int b = 0; b < n; b++) {
        if (seq_ids[b] < 0 || seq_ids[b] >= c->cfg.n_seqs || seen[seq_ids[b]])
            return fail(Q3A_ERR_INVALID, "seq_ids[%d] = %d invalid or repeated", b, seq_ids[b]);
        seen[seq_ids[b]] = 1;
        if (pos[b] < 0 || pos[b] >= c->cfg.max_seq)
            return fail(Q3A_ERR_INVALID, "pos[%d] = %d outside [0, %d)", b, pos[b], c->cfg.max_seq);
        p.slot[b] = seq_ids[b];
        p.pos[b] = pos[b];
        p.t_begin[b] = 0;
        p.t_end[b] = pos[b];
    }
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        p.q = q; p.k_new = k; p.v_new = v; p.q_norm_w = qw; p.k_norm_w = kw;
        p.q_out = q; p.k_out = k; p.xb = xb;
        return run_decode(c, p, c->tmK, c->tmV, c->bf16);
    }
    return host_block(c, p, xb, q, k, v, qw, kw, n);
}

extern "C" int q3a_attn_decode(q3a_ctx* c, float* xb, const float* q, const float* kc,
                               const float* vc, float* att, size_t loff, int pos, int n_heads,
                               int kv_mul, int hd, int kv_dim, int max_seq) {
    (void)att;
    g_err[0] = 0;
    if (!c || !xb || !q || !kc || !vc) return fail(Q3A_ERR_INVALID, "null argument");
    if (hd != HD || kv_mul != GQA)
        return fail(Q3A_ERR_UNSUPPORTED, "hd %d kv_mul %d: only 128 / 4 are implemented", hd,
                    kv_mul);
    if (kv_dim <= 0 || kv_dim % HD != 0 || n_heads != kv_mul * (kv_dim / HD))
        return fail(Q3A_ERR_INVALID, "n_heads %d kv_dim %d inconsistent", n_heads, kv_dim);
    if (kv_dim / HD > c->cfg.n_kv_heads)
        return fail(Q3A_ERR_INVALID, "kv_dim %d wider than the context's %d KV heads", kv_dim,
                    c->cfg.n_kv_heads);
    if (pos < 0 || pos >= max_seq) return fail(Q3A_ERR_INVALID, "pos %d of max_seq %d", pos, max_seq);
    if (loff % (size_t)kv_dim != 0) return fail(Q3A_ERR_INVALID, "loff not a row multiple");
    int rc = ensure_device(c);
    if (rc) return rc;
    const int nkv = kv_dim / HD;
    const size_t rows = (size_t)pos + 1;
    const size_t qd = (size_t)n_heads * HD;
    DecodeParams p;
    base_params(c, p, 0);
    p.cache_mode = CACHE_POSMAJOR;
    p.nkv = nkv;
    p.kv0 = 0;
    p.hq_total = n_heads;
    p.nkv_total = nkv;
    p.nb = 1;
    p.fused = 0;
    p.t_begin[0] = 0;
    p.t_end[0] = pos + 1;
    const float *dk, *dv, *dq;
    float* dxb;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        dk = kc + loff;
        dv = vc + loff;
        dq = q;
        dxb = xb;
    } else {
        const size_t cache_bytes = rows * kv_dim * 4;
        rc = grow_scratch(c, 2 * cache_bytes + 2 * qd * 4);
        if (rc) return rc;
        float* s = reinterpret_cast<float*>(c->d_scratch);
        float* sk = s;
        float* sv = s + rows * kv_dim;
        float* sq = sv + rows * kv_dim;
        dxb = sq + qd;
        CUDA_TRY(cudaMemcpyAsync(sk, kc + loff, cache_bytes, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(sv, vc + loff, cache_bytes, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(sq, q, qd * 4, cudaMemcpyHostToDevice, c->stream));
        dk = sk;
        dv = sv;
        dq = sq;
    }
    CUtensorMap tk, tv;
    rc = make_map_2d(&tk, dk, false, (uint64_t)kv_dim, rows, HD, DEC_BOX, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = make_map_2d(&tv, dv, false, (uint64_t)kv_dim, rows, HD, DEC_BOX, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    p.q = dq;
    p.xb = dxb;
    rc = run_decode(c, p, tk, tv, false);
    if (rc) return rc;
    if (c->cfg.ptr_mode == Q3A_PTR_HOST) {
        CUDA_TRY(cudaMemcpyAsync(xb, dxb, qd * 4, cudaMemcpyDeviceToHost, c->stream));
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    }
    return Q3A_OK;
}

extern "C" int q3a_attn_partial(q3a_ctx* c, float* o, float* lse, const float* q, int seq,
                                int layer, int t0, int t1) {
    g_err[0] = 0;
    if (!c || !o || !lse || !q) return fail(Q3A_ERR_INVALID, "null argument");
    if (seq < 0 || seq >= c->cfg.n_seqs) return fail(Q3A_ERR_INVALID, "seq %d", seq);
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    if (t0 < 0 || t1 < t0 || t1 > c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "chunk [%d, %d) outside [0, %d]", t0, t1, c->cfg.max_seq);
    if (c->nkv != c->cfg.n_kv_heads)
        return fail(Q3A_ERR_INVALID, "q3a_attn_partial needs a context holding all KV heads");
    int rc = ensure_device(c);
    if (rc) return rc;
    const size_t qd = (size_t)c->cfg.n_heads * HD;
    const int nh = c->cfg.n_heads;
    if (t0 == t1) {  // empty chunk: o = 0, lse = -inf
        if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
            CUDA_TRY(cudaMemsetAsync(o, 0, qd * 4, c->stream));
            std::vector<float> ninf(nh, -INFINITY);
            CUDA_TRY(cudaMemcpyAsync(lse, ninf.data(), nh * 4, cudaMemcpyHostToDevice, c->stream));
            CUDA_TRY(cudaStreamSynchronize(c->stream));
        } else {
            memset(o, 0, qd * 4);
            for (int h = 0; h < nh; h++) lse[h] = -INFINITY;
        }
        return Q3A_OK;
    }
    DecodeParams p;
    base_params(c, p, layer);
    p.nb = 1;
    p.fused = 0;
    p.partial_out = 1;
    p.slot[0] = seq;
    p.t_begin[0] = t0;
    p.t_end[0] = t1;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        p.q = q;
        p.xb = o;
        p.lse_out = lse;
        return run_decode(c, p, c->tmK, c->tmV, c->bf16);
    }
    float* ds = c->d_stage;
    float *d_o = ds, *d_q = ds + qd, *d_l = d_q + qd;
    CUDA_TRY(cudaMemcpyAsync(d_q, q, qd * 4, cudaMemcpyHostToDevice, c->stream));
    p.q = d_q;
    p.xb = d_o;
    p.lse_out = d_l;
    rc = run_decode(c, p, c->tmK, c->tmV, c->bf16);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(o, d_o, qd * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(lse, d_l, nh * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

extern "C" int q3a_lse_combine(q3a_ctx* c, float* xb, const float* o_parts, const float* lse_parts,
                               int n_parts) {
    g_err[0] = 0;
    if (!c || !xb || !o_parts || !lse_parts || n_parts <= 0)
        return fail(Q3A_ERR_INVALID, "bad argument");
    int rc = ensure_device(c);
    if (rc) return rc;
    const int nh = c->cfg.n_heads;
    const size_t qd = (size_t)nh * HD;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        CUDA_TRY(launch_lse_combine(xb, o_parts, qd, lse_parts, nh, n_parts, nh, c->stream));
        c->launches++;
        forget_last(c);
        return Q3A_OK;
    }
    rc = grow_scratch(c, ((size_t)n_parts * (qd + nh) + qd) * 4);
    if (rc) return rc;
    float* s = reinterpret_cast<float*>(c->d_scratch);
    float *d_o = s, *d_l = s + (size_t)n_parts * qd, *d_x = d_l + (size_t)n_parts * nh;
    CUDA_TRY(cudaMemcpyAsync(d_o, o_parts, (size_t)n_parts * qd * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(d_l, lse_parts, (size_t)n_parts * nh * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(launch_lse_combine(d_x, d_o, qd, d_l, nh, n_parts, nh, c->stream));
    c->launches++;
    forget_last(c);
    CUDA_TRY(cudaMemcpyAsync(xb, d_x, qd * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

// ------------------------------------------------ peer-memory sequence shards

extern "C" int q3a_peer_export(q3a_ctx* c, int world, void* handle) {
    g_err[0] = 0;
    if (!c || !handle) return fail(Q3A_ERR_INVALID, "null argument");
    if (world < 1 || world > PEER_MAX) return fail(Q3A_ERR_INVALID, "world %d outside [1, %d]", world, PEER_MAX);
    if (c->cfg.n_kv_heads > PEER_MAXG)
        return fail(Q3A_ERR_INVALID, "peer shards support at most %d KV heads", PEER_MAXG);
    if (c->cfg.ptr_mode != Q3A_PTR_DEVICE) return fail(Q3A_ERR_UNSUPPORTED, "peer shards run in device-pointer mode");
    if (c->peer_world && c->peer_world != world)
        return fail(Q3A_ERR_INVALID, "already exported for %d ranks", c->peer_world);
    int rc = ensure_device(c);
    if (rc) return rc;
    if (!c->peer_buf) {
        // words of 8 bytes (value, call number): the sequence-shard region
        // [2 parities][world][row], then the wo region [2][world][WO_MAX_ROWS]
        const size_t bytes = peer_words(c, world) * 8;
        if (cudaMalloc(&c->peer_buf, bytes) != cudaSuccess) return fail(Q3A_ERR_OOM, "peer buffer of %zu bytes", bytes);
        if (cudaMalloc(&c->peer_epoch, PEER_MAXG * sizeof(unsigned)) != cudaSuccess ||
            cudaMalloc(&c->wo_epoch, WO_MAX_CTAS * sizeof(unsigned)) != cudaSuccess)
            return fail(Q3A_ERR_OOM, "peer counters");
        CUDA_TRY(cudaMemset(c->peer_buf, 0, bytes));
        CUDA_TRY(cudaMemset(c->peer_epoch, 0, PEER_MAXG * sizeof(unsigned)));
        CUDA_TRY(cudaMemset(c->wo_epoch, 0, WO_MAX_CTAS * sizeof(unsigned)));
        CUDA_TRY(cudaDeviceSynchronize());
        c->peer_world = world;
    }
    cudaIpcMemHandle_t h;
    CUDA_TRY(cudaIpcGetMemHandle(&h, c->peer_buf));
    static_assert(sizeof(h) == Q3A_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return Q3A_OK;
}

extern "C" int q3a_peer_open(q3a_ctx* c, int rank, int world, const void* handles) {
    g_err[0] = 0;
    if (!c || !handles) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->peer_buf || world != c->peer_world)
        return fail(Q3A_ERR_INVALID, "q3a_peer_export(ctx, %d, ...) must come first", world);
    if (rank < 0 || rank >= world) return fail(Q3A_ERR_INVALID, "rank %d of %d", rank, world);
    if (c->peer_rank >= 0) return fail(Q3A_ERR_INVALID, "peers already open");
    int rc = ensure_device(c);
    if (rc) return rc;
    const uint8_t* hs = reinterpret_cast<const uint8_t*>(handles);
    for (int r = 0; r < world; r++) {
        if (r == rank) {
            c->peer_ptrs[r] = c->peer_buf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)r * Q3A_IPC_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return fail(Q3A_ERR_CUDA, "cannot map the buffer of rank %d", r);
        }
        c->peer_ptrs[r] = reinterpret_cast<float*>(p);
        c->peer_ipc = true;
    }
    c->peer_rank = rank;
    return Q3A_OK;
}

extern "C" int q3a_peer_buffer(q3a_ctx* c, void** buf) {
    g_err[0] = 0;
    if (!c || !buf) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->peer_buf) return fail(Q3A_ERR_INVALID, "q3a_peer_export must come first");
    *buf = c->peer_buf;
    return Q3A_OK;
}

extern "C" int q3a_peer_open_ptrs(q3a_ctx* c, int rank, int world, void* const* bufs) {
    g_err[0] = 0;
    if (!c || !bufs) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->peer_buf || world != c->peer_world)
        return fail(Q3A_ERR_INVALID, "q3a_peer_export(ctx, %d, ...) must come first", world);
    if (rank < 0 || rank >= world) return fail(Q3A_ERR_INVALID, "rank %d of %d", rank, world);
    if (c->peer_rank >= 0) return fail(Q3A_ERR_INVALID, "peers already open");
    if (bufs[rank] != c->peer_buf) return fail(Q3A_ERR_INVALID, "bufs[%d] is not this context's buffer", rank);
    for (int r = 0; r < world; r++)
        if (!bufs[r]) return fail(Q3A_ERR_INVALID, "bufs[%d] is null", r);
    for (int r = 0; r < world; r++) c->peer_ptrs[r] = reinterpret_cast<float*>(bufs[r]);
    c->peer_rank = rank;
    return Q3A_OK;
}

// ---------------------------------------------------- column all-gather (peer memory)
typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

extern "C" int q3a_peer_register(q3a_ctx* c, void* buf, size_t bytes, void* handle) {
    g_err[0] = 0;
    if (!c || !buf || !handle || bytes == 0) return fail(Q3A_ERR_INVALID, "bad argument");
    if (c->cfg.ptr_mode != Q3A_PTR_DEVICE) return fail(Q3A_ERR_UNSUPPORTED, "peer gathers run in device-pointer mode");
    if (c->reg_buf) return fail(Q3A_ERR_INVALID, "a buffer is already registered");
    int rc = ensure_device(c);
    if (rc) return rc;
    // the IPC handle names the whole allocation: find its base and our offset
    static AddrRangeFn range = nullptr;
    if (!range) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return fail(Q3A_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
        range = reinterpret_cast<AddrRangeFn>(p);
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(buf)) != CUDA_SUCCESS)
        return fail(Q3A_ERR_INVALID, "buffer is not device memory of this context's device");
    const uint64_t off = reinterpret_cast<CUdeviceptr>(buf) - base;
    if (off + bytes > size) return fail(Q3A_ERR_INVALID, "buffer runs past its allocation");
    if (cudaMalloc(&c->reg_flags, 2 * PEER_MAX * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&c->reg_state, 4 * sizeof(unsigned)) != cudaSuccess)
        return fail(Q3A_ERR_OOM, "gather flags");
    CUDA_TRY(cudaMemset(c->reg_flags, 0, 2 * PEER_MAX * sizeof(unsigned)));
    CUDA_TRY(cudaMemset(c->reg_state, 0, 4 * sizeof(unsigned)));
    CUDA_TRY(cudaDeviceSynchronize());
    cudaIpcMemHandle_t hb, hf;
    CUDA_TRY(cudaIpcGetMemHandle(&hb, reinterpret_cast<void*>(base)));
    CUDA_TRY(cudaIpcGetMemHandle(&hf, c->reg_flags));
    static_assert(2 * sizeof(cudaIpcMemHandle_t) + 8 == Q3A_PEER_REG_BYTES, "handle layout");
    uint8_t* h = reinterpret_cast<uint8_t*>(handle);
    memcpy(h, &hb, sizeof(hb));
    memcpy(h + sizeof(hb), &off, 8);
    memcpy(h + sizeof(hb) + 8, &hf, sizeof(hf));
    c->reg_buf = reinterpret_cast<uint8_t*>(buf);
    c->reg_bytes = bytes;
    return Q3A_OK;
}

extern "C" int q3a_peer_register_open(q3a_ctx* c, int rank, int world, const void* handles) {
    g_err[0] = 0;
    if (!c || !handles) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->reg_buf) return fail(Q3A_ERR_INVALID, "q3a_peer_register must come first");
    if (world < 1 || world > PEER_MAX || rank < 0 || rank >= world)
        return fail(Q3A_ERR_INVALID, "rank %d of %d", rank, world);
    if (c->reg_rank >= 0) return fail(Q3A_ERR_INVALID, "peers already open");
    int rc = ensure_device(c);
    if (rc) return rc;
    const uint8_t* hs = reinterpret_cast<const uint8_t*>(handles);
    for (int r = 0; r < world; r++) {
        if (r == rank) {
            c->reg_peer[r] = c->reg_buf;
            c->reg_peer_flags[r] = c->reg_flags;
            continue;
        }
        const uint8_t* h = hs + (size_t)r * Q3A_PEER_REG_BYTES;
        cudaIpcMemHandle_t hb, hf;
        uint64_t off = 0;
        memcpy(&hb, h, sizeof(hb));
        memcpy(&off, h + sizeof(hb), 8);
        memcpy(&hf, h + sizeof(hb) + 8, sizeof(hf));
        void *pb = nullptr, *pf = nullptr;
        if (cudaIpcOpenMemHandle(&pb, hb, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
            cudaIpcOpenMemHandle(&pf, hf, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return fail(Q3A_ERR_CUDA, "cannot map the registered buffer of rank %d", r);
        }
        c->reg_ipc_bases[r] = pb;
        c->reg_ipc_flags[r] = pf;
        c->reg_peer[r] = reinterpret_cast<uint8_t*>(pb) + off;
        c->reg_peer_flags[r] = reinterpret_cast<unsigned*>(pf);
    }
    c->reg_world = world;
    c->reg_rank = rank;
    return Q3A_OK;
}

extern "C" int q3a_peer_register_flags(q3a_ctx* c, void** flags) {
    g_err[0] = 0;
    if (!c || !flags) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->reg_flags) return fail(Q3A_ERR_INVALID, "q3a_peer_register must come first");
    *flags = c->reg_flags;
    return Q3A_OK;
}

extern "C" int q3a_peer_register_open_ptrs(q3a_ctx* c, int rank, int world, void* const* bufs,
                                           void* const* flags) {
    g_err[0] = 0;
    if (!c || !bufs || !flags) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->reg_buf) return fail(Q3A_ERR_INVALID, "q3a_peer_register must come first");
    if (world < 1 || world > PEER_MAX || rank < 0 || rank >= world)
        return fail(Q3A_ERR_INVALID, "rank %d of %d", rank, world);
    if (c->reg_rank >= 0) return fail(Q3A_ERR_INVALID, "peers already open");
    if (bufs[rank] != c->reg_buf || flags[rank] != c->reg_flags)
        return fail(Q3A_ERR_INVALID, "entry %d is not this context's registration", rank);
    for (int r = 0; r < world; r++)
        if (!bufs[r] || !flags[r]) return fail(Q3A_ERR_INVALID, "entry %d is null", r);
    for (int r = 0; r < world; r++) {
        c->reg_peer[r] = reinterpret_cast<uint8_t*>(bufs[r]);
        c->reg_peer_flags[r] = reinterpret_cast<unsigned*>(flags[r]);
    }
    c->reg_world = world;
    c->reg_rank = rank;
    return Q3A_OK;
}

extern "C" int q3a_gather_cols(q3a_ctx* c, size_t off, long long rows, size_t row_bytes, size_t col0,
                               size_t col_bytes) {
    g_err[0] = 0;
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    if (c->reg_rank < 0) return fail(Q3A_ERR_INVALID, "q3a_peer_register_open must come first");
    if (rows <= 0 || row_bytes % 16 || col0 % 16 || col_bytes % 16 || col_bytes == 0 ||
        col0 + col_bytes > row_bytes || off % 16)
        return fail(Q3A_ERR_INVALID, "rows %lld, row/column bytes must be multiples of 16", rows);
    if (off + (size_t)rows * row_bytes > c->reg_bytes)
        return fail(Q3A_ERR_INVALID, "matrix runs past the registered buffer");
    int rc = ensure_device(c);
    if (rc) return rc;
    ColGatherParams p;
    memset(&p, 0, sizeof(p));
    p.local = c->reg_buf + off;
    for (int r = 0; r < c->reg_world; r++) {
        p.peer[r] = c->reg_peer[r] + off;
        p.peer_flags[r] = c->reg_peer_flags[r];
    }
    p.flags = c->reg_flags;
    p.state = c->reg_state;
    p.world = c->reg_world;
    p.rank = c->reg_rank;
    p.rows = rows;
    p.row_bytes = (long long)row_bytes;
    p.col0 = (long long)col0;
    p.vecs = (int)(col_bytes / 16);
    p.err = c->err;
    p.wait_limit = c->wait_limit;
    const long long work = rows * p.vecs;
    const int n_ctas = (int)std::min<long long>(c->num_sms, std::max<long long>(1, (work + 255) / 256));
    CUDA_TRY(launch_gather_cols(p, n_ctas, c->stream));
    c->launches++;
    forget_last(c);
    return Q3A_OK;
}

extern "C" int q3a_attn_seqshard(q3a_ctx* c, float* xb, const float* q, int seq, int layer,
                                 int n_local) {
    g_err[0] = 0;
    if (!c || !xb || !q) return fail(Q3A_ERR_INVALID, "null argument");
    if (c->peer_rank < 0) return fail(Q3A_ERR_INVALID, "q3a_peer_open must come first");
    if (c->nkv != c->cfg.n_kv_heads)
        return fail(Q3A_ERR_INVALID, "sequence shards need a context holding all KV heads");
    if (seq < 0 || seq >= c->cfg.n_seqs) return fail(Q3A_ERR_INVALID, "seq %d", seq);
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    if (n_local < 1 || n_local > c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "local chunk of %d rows outside [1, %d]", n_local, c->cfg.max_seq);
    int rc = ensure_device(c);
    if (rc) return rc;
    DecodeParams p;
    base_params(c, p, layer);
    p.nb = 1;
    p.fused = 0;
    p.slot[0] = seq;
    p.t_begin[0] = 0;
    p.t_end[0] = n_local;
    p.q = q;
    p.xb = xb;
    // one rank: its own merge is the whole result, nothing to exchange
    p.peer_world = c->peer_world > 1 ? c->peer_world : 0;
    p.peer_rank = c->peer_rank;
    p.peer_row = (int)peer_row(c);
    for (int r = 0; r < c->peer_world; r++) p.peer_recv[r] = c->peer_ptrs[r];
    p.peer_epoch = c->peer_epoch;
    return run_decode(c, p, c->tmK, c->tmV, c->bf16);
}

extern "C" int q3a_lse_combine_packed(q3a_ctx* c, float* xb, const float* parts, int n_parts) {
    g_err[0] = 0;
    if (!c || !xb || !parts || n_parts <= 0) return fail(Q3A_ERR_INVALID, "bad argument");
    int rc = ensure_device(c);
    if (rc) return rc;
    const int nh = c->cfg.n_heads;
    const size_t qd = (size_t)nh * HD, pw = qd + nh;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        CUDA_TRY(launch_lse_combine(xb, parts, pw, parts + qd, pw, n_parts, nh, c->stream));
        c->launches++;
        forget_last(c);
        return Q3A_OK;
    }
    rc = grow_scratch(c, ((size_t)n_parts * pw + qd) * 4);
    if (rc) return rc;
    float* s = reinterpret_cast<float*>(c->d_scratch);
    float *d_p = s, *d_x = s + (size_t)n_parts * pw;
    CUDA_TRY(cudaMemcpyAsync(d_p, parts, (size_t)n_parts * pw * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(launch_lse_combine(d_x, d_p, pw, d_p + qd, pw, n_parts, nh, c->stream));
    c->launches++;
    forget_last(c);
    CUDA_TRY(cudaMemcpyAsync(xb, d_x, qd * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

// ------------------------------------------------------------------ cache I/O
static int cache_io_params(q3a_ctx* c, AppendParams& a, int seq, int layer, int pos0, int n) {
    if (seq < 0 || seq >= c->cfg.n_seqs) return fail(Q3A_ERR_INVALID, "seq %d", seq);
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    if (n < 0 || pos0 < 0 || (long long)pos0 + n > c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "rows [%d, +%d) outside [0, %d)", pos0, n, c->cfg.max_seq);
    memset(&a, 0, sizeof(a));
    a.kcache = c->kcache;
    a.vcache = c->vcache;
    a.eps = c->cfg.norm_eps;
    a.n = n;
    a.nkv = c->nkv;
    a.kv0 = c->kv0;
    a.nkv_total = c->cfg.n_kv_heads;
    a.layer = layer;
    a.slot = seq;
    a.pos0 = pos0;
    a.pages_per_seq = c->pages_per_seq;
    a.page_tokens = c->cfg.page_tokens;
    a.n_pages = c->n_pages;
    a.bf16 = c->bf16;
    a.inv_freq = c->d_inv_freq;
    return Q3A_OK;
}

static int append_common(q3a_ctx* c, int seq, int layer, int pos0, int n, const float* k,
                         const float* v, const float* kw, int norm_rope) {
    g_err[0] = 0;
    if (!c || !k || !v || (norm_rope && !kw)) return fail(Q3A_ERR_INVALID, "null argument");
    int rc = ensure_device(c);
    if (rc) return rc;
    AppendParams a;
    rc = cache_io_params(c, a, seq, layer, pos0, n);
    if (rc) return rc;
    if (n == 0) return Q3A_OK;
    a.do_norm_rope = norm_rope;
    const size_t kd = (size_t)n * c->cfg.n_kv_heads * HD;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        a.k = k; a.v = v; a.k_norm_w = kw;
    } else {
        rc = grow_scratch(c, (2 * kd + HD) * 4);
        if (rc) return rc;
        float* s = reinterpret_cast<float*>(c->d_scratch);
        CUDA_TRY(cudaMemcpyAsync(s, k, kd * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(s + kd, v, kd * 4, cudaMemcpyHostToDevice, c->stream));
        if (norm_rope)
            CUDA_TRY(cudaMemcpyAsync(s + 2 * kd, kw, HD * 4, cudaMemcpyHostToDevice, c->stream));
        a.k = s; a.v = s + kd; a.k_norm_w = s + 2 * kd;
    }
    CUDA_TRY(launch_append(a, c->stream));
    c->launches++;
    forget_last(c);
    if (c->cfg.ptr_mode == Q3A_PTR_HOST) CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

extern "C" int q3a_kv_append(q3a_ctx* c, int seq, int layer, int pos0, int n, const float* k,
                             const float* v, const float* kw) {
    return append_common(c, seq, layer, pos0, n, k, v, kw, 1);
}

extern "C" int q3a_kv_load(q3a_ctx* c, int seq, int layer, int pos0, int n, const float* k,
                           const float* v) {
    return append_common(c, seq, layer, pos0, n, k, v, nullptr, 0);
}

// ------------------------------------------------------------------ KV wire format
static_assert(sizeof(q3a_kv_wire_header) == 64, "the wire header is 64 bytes");

static size_t wire_payload_bytes(int n_layers, int n_heads, int n_tok, size_t esize) {
    return (size_t)n_layers * n_heads * 2 * n_tok * HD * esize;
}

// Header fields that do not depend on a context; reason in `why` when bad.
static bool wire_header_ok(const q3a_kv_wire_header& h, size_t bytes, char* why, size_t why_n) {
    if (h.magic != Q3A_KV_WIRE_MAGIC) return snprintf(why, why_n, "not a KV wire blob (magic %08x)", h.magic), false;
    if (h.version != Q3A_KV_WIRE_VERSION) return snprintf(why, why_n, "wire version %u", h.version), false;
    if (h.dtype != Q3A_KV_F32 && h.dtype != Q3A_KV_BF16) return snprintf(why, why_n, "dtype %u", h.dtype), false;
    if (h.head_dim != HD) return snprintf(why, why_n, "head_dim %u", h.head_dim), false;
    if (h.kv_head_count == 0 || h.kv_head_begin + h.kv_head_count > h.n_kv_heads)
        return snprintf(why, why_n, "heads [%u, +%u) of %u", h.kv_head_begin, h.kv_head_count, h.n_kv_heads), false;
    if (h.n_layers == 0 || h.n_tok == 0) return snprintf(why, why_n, "empty blob"), false;
    const size_t want = wire_payload_bytes(h.n_layers, h.kv_head_count, (int)h.n_tok, h.dtype == Q3A_KV_BF16 ? 2 : 4);
    if (h.payload_bytes != want) return snprintf(why, why_n, "payload of %llu bytes, the fields give %zu", (unsigned long long)h.payload_bytes, want), false;
    if (bytes < sizeof(h) + want) return snprintf(why, why_n, "blob of %zu bytes, needs %zu", bytes, sizeof(h) + want), false;
    return true;
}

extern "C" size_t q3a_kv_wire_bytes(const q3a_ctx* c, int n_layers, int n_tok) {
    if (!c || n_layers <= 0 || n_tok <= 0) return 0;
    return sizeof(q3a_kv_wire_header) + wire_payload_bytes(n_layers, c->nkv, n_tok, c->esize);
}

static int wire_sum_buffer(q3a_ctx* c) {
    if (!c->wire_sum && cudaMalloc(&c->wire_sum, sizeof(unsigned long long)) != cudaSuccess)
        return fail(Q3A_ERR_OOM, "checksum scratch");
    return Q3A_OK;
}

static void wire_params(q3a_ctx* c, WireParams& w, int seq, int layer0, int n_layers, int pos0, int n_tok) {
    memset(&w, 0, sizeof(w));
    w.kcache = c->kcache;
    w.vcache = c->vcache;
    w.layer0 = layer0;
    w.n_layers = n_layers;
    w.nkv = c->nkv;
    w.ctx_nkv = c->nkv;
    w.pos0 = pos0;
    w.n_tok = n_tok;
    w.slot = seq;
    w.pages_per_seq = c->pages_per_seq;
    w.page_tokens = c->cfg.page_tokens;
    w.n_pages = c->n_pages;
}

extern "C" int q3a_kv_pack(q3a_ctx* c, int seq, int layer0, int n_layers, int pos0, int n_tok,
                           void* dst, size_t dst_bytes) {
    g_err[0] = 0;
    if (!c || !dst) return fail(Q3A_ERR_INVALID, "null argument");
    if (seq < 0 || seq >= c->cfg.n_seqs) return fail(Q3A_ERR_INVALID, "seq %d", seq);
    if (layer0 < 0 || n_layers < 1 || layer0 + n_layers > c->cfg.n_layers)
        return fail(Q3A_ERR_INVALID, "layers [%d, +%d) of %d", layer0, n_layers, c->cfg.n_layers);
    if (pos0 < 0 || n_tok < 1 || pos0 + n_tok > c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "positions [%d, +%d) of %d", pos0, n_tok, c->cfg.max_seq);
    const size_t need = q3a_kv_wire_bytes(c, n_layers, n_tok);
    if (dst_bytes < need) return fail(Q3A_ERR_INVALID, "dst of %zu bytes, needs %zu", dst_bytes, need);
    const bool dev = c->cfg.ptr_mode == Q3A_PTR_DEVICE;
    if (dev && ((uintptr_t)dst & 15)) return fail(Q3A_ERR_INVALID, "dst must be 16-byte aligned");
    int rc = ensure_device(c);
    if (rc) return rc;
    if ((rc = wire_sum_buffer(c))) return rc;
    const size_t pay = need - sizeof(q3a_kv_wire_header);
    uint8_t* payload;
    if (dev) {
        payload = reinterpret_cast<uint8_t*>(dst) + sizeof(q3a_kv_wire_header);
    } else {
        if ((rc = grow_scratch(c, pay))) return rc;
        payload = reinterpret_cast<uint8_t*>(c->d_scratch);
    }
    WireParams w;
    wire_params(c, w, seq, layer0, n_layers, pos0, n_tok);
    w.payload = payload;
    w.pay_nkv = c->nkv;
    CUDA_TRY(launch_wire_copy(w, c->bf16 != 0, true, c->stream));
    CUDA_TRY(launch_wire_checksum(payload, pay, c->wire_sum, c->stream));
    c->launches += 2;
    forget_last(c);
    q3a_kv_wire_header h;
    memset(&h, 0, sizeof(h));
    h.magic = Q3A_KV_WIRE_MAGIC;
    h.version = Q3A_KV_WIRE_VERSION;
    h.dtype = (uint16_t)(c->bf16 ? Q3A_KV_BF16 : Q3A_KV_F32);
    h.head_dim = HD;
    h.n_kv_heads = (uint16_t)c->cfg.n_kv_heads;
    h.kv_head_begin = (uint16_t)c->kv0;
    h.kv_head_count = (uint16_t)c->nkv;
    h.layer0 = (uint16_t)layer0;
    h.n_layers = (uint16_t)n_layers;
    h.pos0 = (uint32_t)pos0;
    h.n_tok = (uint32_t)n_tok;
    h.payload_bytes = pay;
    unsigned long long sum = 0;
    CUDA_TRY(cudaMemcpyAsync(&sum, c->wire_sum, sizeof(sum), cudaMemcpyDeviceToHost, c->stream));
    if (!dev)
        CUDA_TRY(cudaMemcpyAsync(reinterpret_cast<uint8_t*>(dst) + sizeof(h), payload, pay,
                                 cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    h.checksum = sum;
    if (dev)
        CUDA_TRY(cudaMemcpy(dst, &h, sizeof(h), cudaMemcpyHostToDevice));
    else
        memcpy(dst, &h, sizeof(h));
    return Q3A_OK;
}

extern "C" int q3a_kv_unpack(q3a_ctx* c, int seq, const void* src, size_t src_bytes) {
    g_err[0] = 0;
    if (!c || !src) return fail(Q3A_ERR_INVALID, "null argument");
    if (seq < 0 || seq >= c->cfg.n_seqs) return fail(Q3A_ERR_INVALID, "seq %d", seq);
    if (src_bytes < sizeof(q3a_kv_wire_header)) return fail(Q3A_ERR_INVALID, "blob of %zu bytes", src_bytes);
    const bool dev = c->cfg.ptr_mode == Q3A_PTR_DEVICE;
    if (dev && ((uintptr_t)src & 15)) return fail(Q3A_ERR_INVALID, "src must be 16-byte aligned");
    int rc = ensure_device(c);
    if (rc) return rc;
    q3a_kv_wire_header h;
    if (dev) {
        CUDA_TRY(cudaMemcpyAsync(&h, src, sizeof(h), cudaMemcpyDeviceToHost, c->stream));
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    } else {
        memcpy(&h, src, sizeof(h));
    }
    char why[160];
    if (!wire_header_ok(h, src_bytes, why, sizeof(why))) return fail(Q3A_ERR_INVALID, "%s", why);
    if (h.dtype != (c->bf16 ? Q3A_KV_BF16 : Q3A_KV_F32))
        return fail(Q3A_ERR_INVALID, "blob dtype %u, context dtype %d", h.dtype, c->cfg.kv_dtype);
    if (h.n_kv_heads != c->cfg.n_kv_heads)
        return fail(Q3A_ERR_INVALID, "blob of a model with %u KV heads", h.n_kv_heads);
    if (c->kv0 < h.kv_head_begin || c->kv0 + c->nkv > h.kv_head_begin + h.kv_head_count)
        return fail(Q3A_ERR_INVALID, "blob holds KV heads [%u, +%u), the context [%d, +%d)",
                    h.kv_head_begin, h.kv_head_count, c->kv0, c->nkv);
    if (h.layer0 + h.n_layers > c->cfg.n_layers)
        return fail(Q3A_ERR_INVALID, "blob layers [%u, +%u) of %d", h.layer0, h.n_layers, c->cfg.n_layers);
    if ((long long)h.pos0 + h.n_tok > c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "blob positions [%u, +%u) beyond %d", h.pos0, h.n_tok, c->cfg.max_seq);
    if ((rc = wire_sum_buffer(c))) return rc;
    const size_t pay = h.payload_bytes;
    const uint8_t* payload;
    if (dev) {
        payload = reinterpret_cast<const uint8_t*>(src) + sizeof(h);
    } else {
        if ((rc = grow_scratch(c, pay))) return rc;
        CUDA_TRY(cudaMemcpyAsync(c->d_scratch, reinterpret_cast<const uint8_t*>(src) + sizeof(h), pay,
                                 cudaMemcpyHostToDevice, c->stream));
        payload = reinterpret_cast<const uint8_t*>(c->d_scratch);
    }
    CUDA_TRY(launch_wire_checksum(payload, pay, c->wire_sum, c->stream));
    c->launches++;
    forget_last(c);
    unsigned long long sum = 0;
    CUDA_TRY(cudaMemcpyAsync(&sum, c->wire_sum, sizeof(sum), cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (sum != h.checksum)
        return fail(Q3A_ERR_INVALID, "checksum mismatch (blob %016llx, payload %016llx)",
                    (unsigned long long)h.checksum, sum);
    WireParams w;
    wire_params(c, w, seq, h.layer0, h.n_layers, (int)h.pos0, (int)h.n_tok);
    w.payload = const_cast<uint8_t*>(payload);
    w.pay_nkv = h.kv_head_count;
    w.pay_head0 = c->kv0 - h.kv_head_begin;
    CUDA_TRY(launch_wire_copy(w, c->bf16 != 0, false, c->stream));
    c->launches++;
    if (!dev) CUDA_TRY(cudaStreamSynchronize(c->stream));  // the scratch is reused by later calls
    return Q3A_OK;
}

extern "C" int q3a_kv_wire_check(const void* blob, size_t bytes) {
    g_err[0] = 0;
    if (!blob || bytes < sizeof(q3a_kv_wire_header)) return fail(Q3A_ERR_INVALID, "blob of %zu bytes", bytes);
    q3a_kv_wire_header h;
    memcpy(&h, blob, sizeof(h));
    char why[160];
    if (!wire_header_ok(h, bytes, why, sizeof(why))) return fail(Q3A_ERR_INVALID, "%s", why);
    const uint64_t sum = wire_checksum_host(reinterpret_cast<const uint8_t*>(blob) + sizeof(h), h.payload_bytes);
    if (sum != h.checksum)
        return fail(Q3A_ERR_INVALID, "checksum mismatch (blob %016llx, payload %016llx)",
                    (unsigned long long)h.checksum, (unsigned long long)sum);
    return Q3A_OK;
}

extern "C" int q3a_kv_synth(q3a_ctx* c, int seq, int layer, int pos0, int n, uint64_t seed,
                            uint64_t stream_k, uint64_t stream_v) {
    g_err[0] = 0;
    if (!c) return fail(Q3A_ERR_INVALID, "null context");
    int rc = ensure_device(c);
    if (rc) return rc;
    AppendParams a;
    rc = cache_io_params(c, a, seq, layer, pos0, n);
    if (rc) return rc;
    if (n == 0) return Q3A_OK;
    // raw rows of all KV heads, as q3a_kv_append takes them; unit gains
    static const float ones[HD] = {
#define Q3A_ONE8 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f
        Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8,
        Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8, Q3A_ONE8};
#undef Q3A_ONE8
    const size_t kd = (size_t)n * c->cfg.n_kv_heads * HD;
    rc = grow_scratch(c, (2 * kd + HD) * 4);
    if (rc) return rc;
    float* s = reinterpret_cast<float*>(c->d_scratch);
    CUDA_TRY(launch_randn(s, 0, kd, stream_key(seed, stream_k), 0, c->stream));
    CUDA_TRY(launch_randn(s + kd, 0, kd, stream_key(seed, stream_v), 0, c->stream));
    CUDA_TRY(cudaMemcpyAsync(s + 2 * kd, ones, sizeof(ones), cudaMemcpyHostToDevice, c->stream));
    a.do_norm_rope = 1;
    a.k = s;
    a.v = s + kd;
    a.k_norm_w = s + 2 * kd;
    CUDA_TRY(launch_append(a, c->stream));
    c->launches += 3;
    forget_last(c);
    if (c->cfg.ptr_mode == Q3A_PTR_HOST) CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

extern "C" int q3a_kv_read(q3a_ctx* c, int seq, int layer, int pos0, int n, float* k, float* v) {
    g_err[0] = 0;
    if (!c || !k || !v) return fail(Q3A_ERR_INVALID, "null argument");
    int rc = ensure_device(c);
    if (rc) return rc;
    AppendParams a;
    rc = cache_io_params(c, a, seq, layer, pos0, n);
    if (rc) return rc;
    if (n == 0) return Q3A_OK;
    const size_t kd = (size_t)n * c->nkv * HD;
    if (c->cfg.ptr_mode == Q3A_PTR_DEVICE) {
        CUDA_TRY(launch_kv_read(a, k, v, c->stream));
        c->launches++;
        forget_last(c);
        return Q3A_OK;
    }
    rc = grow_scratch(c, 2 * kd * 4);
    if (rc) return rc;
    float* s = reinterpret_cast<float*>(c->d_scratch);
    CUDA_TRY(launch_kv_read(a, s, s + kd, c->stream));
    c->launches++;
    forget_last(c);
    CUDA_TRY(cudaMemcpyAsync(k, s, kd * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(v, s + kd, kd * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return Q3A_OK;
}

extern "C" int q3a_randn(q3a_ctx* c, void* dst, int out_dtype, size_t n, uint64_t seed,
                         uint64_t stream_id, uint64_t offset) {
    g_err[0] = 0;
    if (!c || !dst) return fail(Q3A_ERR_INVALID, "null argument");
    if (out_dtype != Q3A_OUT_F32 && out_dtype != Q3A_OUT_BF16)
        return fail(Q3A_ERR_INVALID, "out_dtype %d", out_dtype);
    int rc = ensure_device(c);
    if (rc) return rc;
    CUDA_TRY(launch_randn(dst, out_dtype == Q3A_OUT_BF16, n, stream_key(seed, stream_id), offset,
                          c->stream));
    c->launches++;
    forget_last(c);
    return Q3A_OK;
}

// ------------------------------------------------------------------ prefill
extern "C" int q3a_prefill_attn(q3a_ctx* c, void* out, int out_dtype, const void* q_bf16, int seq,
                                int layer, int pos0, int n_tok);

extern "C" int q3a_prefill(q3a_ctx* c, void* out, int out_dtype, const float* q, const float* k,
                           const float* v, const float* qw, const float* kw, int seq, int layer,
                           int pos0, int n_tok) {
    g_err[0] = 0;
    if (!c || !out || !q || !k || !v || !qw || !kw) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->bf16) return fail(Q3A_ERR_UNSUPPORTED, "prefill needs a bf16 cache");
    if (n_tok <= 0) return fail(Q3A_ERR_INVALID, "n_tok %d", n_tok);
    int rc = ensure_device(c);
    if (rc) return rc;
    AppendParams a;
    rc = cache_io_params(c, a, seq, layer, pos0, n_tok);
    if (rc) return rc;
    const size_t qd = (size_t)n_tok * c->cfg.n_heads * HD;
    const size_t kd = (size_t)n_tok * c->cfg.n_kv_heads * HD;
    const size_t out_bytes = qd * (out_dtype == Q3A_OUT_BF16 ? 2 : 4);
    // scratch: [q bf16 | (host mode) q f32 | k | v | qw | kw | out]
    const bool host = c->cfg.ptr_mode == Q3A_PTR_HOST;
    size_t need = qd * 2 + 256;
    if (host) need += (qd + 2 * kd + 2 * HD) * 4 + out_bytes + 256;
    rc = grow_scratch(c, need);
    if (rc) return rc;
    uint8_t* s = reinterpret_cast<uint8_t*>(c->d_scratch);
    __nv_bfloat16* qb = reinterpret_cast<__nv_bfloat16*>(s);
    const float *dq = q, *dk = k, *dv = v, *dqw = qw, *dkw = kw;
    void* dout = out;
    if (host) {
        float* f = reinterpret_cast<float*>(s + ((qd * 2 + 255) & ~(size_t)255));
        float *fq = f, *fk = fq + qd, *fv = fk + kd, *fqw = fv + kd, *fkw = fqw + HD;
        void* fo = fkw + HD;
        CUDA_TRY(cudaMemcpyAsync(fq, q, qd * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(fk, k, kd * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(fv, v, kd * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(fqw, qw, HD * 4, cudaMemcpyHostToDevice, c->stream));
        CUDA_TRY(cudaMemcpyAsync(fkw, kw, HD * 4, cudaMemcpyHostToDevice, c->stream));
        if (c->nkv != c->cfg.n_kv_heads)  // sharded: keep the caller's other heads' columns
            CUDA_TRY(cudaMemcpyAsync(fo, out, out_bytes, cudaMemcpyHostToDevice, c->stream));
        dq = fq; dk = fk; dv = fv; dqw = fqw; dkw = fkw; dout = fo;
    }
    PrepParams pp;
    memset(&pp, 0, sizeof(pp));
    pp.src = dq;
    pp.dst_bf16 = qb;
    pp.w = dqw;
    pp.eps = c->cfg.norm_eps;
    pp.n = n_tok;
    pp.nheads = c->nkv * GQA;  // this context's query heads
    pp.head0 = c->kv0 * GQA;
    pp.nheads_total = c->cfg.n_heads;
    pp.pos0 = pos0;
    pp.do_norm_rope = 1;
    pp.inv_freq = c->d_inv_freq;
    CUDA_TRY(launch_prep_rows(pp, c->stream));
    c->launches++;
    forget_last(c);
    a.k = dk;
    a.v = dv;
    a.k_norm_w = dkw;
    a.do_norm_rope = 1;
    CUDA_TRY(launch_append(a, c->stream));
    c->launches++;
    forget_last(c);
    // run the attention in device mode on the staged operands
    const int saved_mode = c->cfg.ptr_mode;
    c->cfg.ptr_mode = Q3A_PTR_DEVICE;
    rc = q3a_prefill_attn(c, dout, out_dtype, qb, seq, layer, pos0, n_tok);
    c->cfg.ptr_mode = saved_mode;
    if (rc) return rc;
    if (host) {
        CUDA_TRY(cudaMemcpyAsync(out, dout, out_bytes, cudaMemcpyDeviceToHost, c->stream));
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    }
    return Q3A_OK;
}

extern "C" int q3a_prefill_attn(q3a_ctx* c, void* out, int out_dtype, const void* q_bf16, int seq,
                                int layer, int pos0, int n_tok) {
    if (!c || !out || !q_bf16) return fail(Q3A_ERR_INVALID, "null argument");
    if (!c->bf16) return fail(Q3A_ERR_UNSUPPORTED, "prefill needs a bf16 cache");
    if (out_dtype != Q3A_OUT_F32 && out_dtype != Q3A_OUT_BF16)
        return fail(Q3A_ERR_INVALID, "out_dtype %d", out_dtype);
    if (seq < 0 || seq >= c->cfg.n_seqs) return fail(Q3A_ERR_INVALID, "seq %d", seq);
    if (layer < 0 || layer >= c->cfg.n_layers) return fail(Q3A_ERR_INVALID, "layer %d", layer);
    if (n_tok <= 0 || pos0 < 0 || (long long)pos0 + n_tok > c->cfg.max_seq)
        return fail(Q3A_ERR_INVALID, "rows [%d, +%d) outside [0, %d)", pos0, n_tok, c->cfg.max_seq);
    int rc = ensure_device(c);
    if (rc) return rc;
    const size_t qd = (size_t)n_tok * c->cfg.n_heads * HD;
    const size_t out_bytes = qd * (out_dtype == Q3A_OUT_BF16 ? 2 : 4);
    const void* dq = q_bf16;
    void* dout = out;
    if (c->cfg.ptr_mode == Q3A_PTR_HOST) {
        rc = grow_scratch(c, qd * 2 + 256 + out_bytes);
        if (rc) return rc;
        uint8_t* s = reinterpret_cast<uint8_t*>(c->d_scratch);
        CUDA_TRY(cudaMemcpyAsync(s, q_bf16, qd * 2, cudaMemcpyHostToDevice, c->stream));
        dq = s;
        dout = s + ((qd * 2 + 255) & ~(size_t)255);
        if (c->nkv != c->cfg.n_kv_heads)  // sharded: keep the caller's other heads' columns
            CUDA_TRY(cudaMemcpyAsync(dout, out, out_bytes, cudaMemcpyHostToDevice, c->stream));
    }
    // Q [n_tok][n_heads][128] bf16: 3-D map (d, head, row), box 64 x 1 x 128,
    // 128-byte swizzle -- one head's 128 rows x 64 dims per load
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(Q3A_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    CUtensorMap tq;
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)c->cfg.n_heads, (cuuint64_t)n_tok};
    cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)c->cfg.n_heads * HD * 2};
    cuuint32_t box[3] = {64, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    if (fn(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(dq), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return fail(Q3A_ERR_CUDA, "prefill q tensor map");
    PrefillParams pp;
    memset(&pp, 0, sizeof(pp));
    pp.out_f32 = out_dtype == Q3A_OUT_F32 ? reinterpret_cast<float*>(dout) : nullptr;
    pp.out_bf16 = out_dtype == Q3A_OUT_BF16 ? reinterpret_cast<__nv_bfloat16*>(dout) : nullptr;
    pp.n_tok = n_tok;
    pp.pos0 = pos0;
    pp.hq_total = c->cfg.n_heads;
    pp.nkv = c->nkv;
    pp.kv0 = c->kv0;
    pp.layer = layer;
    pp.slot = seq;
    pp.pages_per_seq = c->pages_per_seq;
    pp.page_tokens = c->cfg.page_tokens;
    pp.n_pages = c->n_pages;
    pp.scale_log2e = (float)(1.4426950408889634 / sqrt((double)HD));
    pp.err = c->err;
    // Long causal items may be split over several CTAs (KV-head-sharded
    // contexts, short prompts leave many SMs idle behind the longest item).
    // The part size is chosen by replaying the kernel's snake deal of chunks
    // on the host with a cost model measured on B200 (per chunk ~2 us of Q
    // load and pipeline start, ~2.3 us per key tile of a head pair, ~3 us to
    // write a split part, ~5 us for the combine launch); the decision is
    // cached per prompt shape.  At most 8 parts, partial scratch <= 1 GiB.
    int pf_launches = 1;
    {
        const int n_qt = (n_tok + 127) / 128;
        const int per_qt = c->nkv * 2;
        const long long n_items = (long long)n_qt * per_qt;
        std::vector<int> nj_of(n_qt);
        int max_nj = 0;
        for (int qt = 0; qt < n_qt; qt++) {
            const int last_q = std::min(pos0 + (qt + 1) * 128, pos0 + n_tok) - 1;
            nj_of[qt] = last_q / 128 + 1;
            max_nj = std::max(max_nj, nj_of[qt]);
        }
        int nsplit = 1, cap = max_nj;
        if (c->pf_key_tok == n_tok && c->pf_key_pos == pos0) {
            nsplit = c->pf_nsplit;
            cap = c->pf_cap;
        } else {
            const int G = std::min<long long>(c->num_sms, n_items * 8);
            auto cost = [&](int ns, int cp) {
                std::vector<double> load(G, 0.0);
                const long long n_chunks = n_items * ns;
                for (int cc = 0; cc < G; cc++) {
                    for (long long r = 0;; r++) {
                        const long long x = r * G + ((r & 1) ? (G - 1 - cc) : cc);
                        if (x >= n_chunks) break;
                        const long long item = x / ns;
                        const int nj = nj_of[n_qt - 1 - (int)(item / per_qt)];
                        const int k = std::min(ns, (nj + cp - 1) / cp);
                        const int part = (int)(x % ns);
                        if (part >= k) continue;
                        const int tiles = (part + 1) * nj / k - part * nj / k;
                        load[cc] += 2.0 + 2.3 * tiles + (k > 1 ? 3.0 : 0.0);
                    }
                }
                return *std::max_element(load.begin(), load.end()) + (ns > 1 ? 5.0 : 0.0);
            };
            double best = cost(1, max_nj);
            for (int cp : {8, 6, 5, 4, 3, 2}) {
                const int ns = (max_nj + cp - 1) / cp;
                if (cp >= max_nj || ns > 8) continue;
                if ((double)n_items * ns * 2 * PF_PART_FLOATS * 4 > (double)(1LL << 30)) continue;
                const double cc = cost(ns, cp);
                if (cc < 0.9 * best) {  // split only for a clear gain
                    best = cc;
                    nsplit = ns;
                    cap = cp;
                }
            }
            c->pf_key_tok = n_tok;
            c->pf_key_pos = pos0;
            c->pf_nsplit = nsplit;
            c->pf_cap = cap;
        }
        if (nsplit > 1) {
            const size_t need = (size_t)n_items * nsplit * 2 * PF_PART_FLOATS;
            if (need > c->pf_part_floats) {
                cudaFree(c->pf_part);
                c->pf_part = nullptr;
                c->pf_part_floats = 0;
                if (cudaMalloc(&c->pf_part, need * 4) != cudaSuccess)
                    return fail(Q3A_ERR_OOM, "prefill split scratch of %zu bytes", need * 4);
                c->pf_part_floats = need;
            }
            pf_launches = 2;  // + prefill_combine_kernel
        }
        pp.nsplit = nsplit;
        pp.part_tiles = std::max(cap, 1);
        pp.part = c->pf_part;
    }
    pp.kcache = reinterpret_cast<const __nv_bfloat16*>(c->kcache);
    pp.vcache = reinterpret_cast<const __nv_bfloat16*>(c->vcache);
    CUDA_TRY(launch_prefill(pp, tq, c->stream));
    c->launches += pf_launches;
    forget_last(c);
    if (c->cfg.ptr_mode == Q3A_PTR_HOST) {
        CUDA_TRY(cudaMemcpyAsync(out, dout, out_bytes, cudaMemcpyDeviceToHost, c->stream));
        CUDA_TRY(cudaStreamSynchronize(c->stream));
    }
    return Q3A_OK;
}
