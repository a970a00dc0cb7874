// q3a_internal.h -- parameter blocks and launchers shared between the C-ABI
// layer (q3a_api.cu) and the kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <limits.h>
#include <stdint.h>

#include "../../include/q3attn.h"

namespace q3a {

constexpr int MAX_B = Q3A_MAX_BATCH;
constexpr int DEC_TILE = 64;        // cache tokens per pipeline stage (decode)
constexpr int DEC_BOX = 16;         // rows per TMA box; split points are multiples of it
constexpr int MAX_PIECES = 160;     // piece-mode schedule capacity (>= SM count)
constexpr int PART_STRIDE = 4 * 128 + 4;  // floats per partial slot: o[4][128], lse[4]
constexpr int PEER_MAX = 8;         // ranks of a peer-memory sequence shard
constexpr int PEER_MAXG = 16;       // KV heads (groups) per flag row

// One contiguous range of cache rows of one (sequence, kv head) group, the
// unit of work of a CTA in piece mode.  Pieces of a group are numbered
// consecutively (piece index = partial slot), i is the index within the
// group and k the group's piece count; the piece with i == k-1 also handles
// the new token in fused mode.
struct Piece {
    int g;       // group = b * nkv + local kv head
    int r0;      // first cache row
    int r1;      // one past the last cache row
    short i;
    short k;
};

// Where the decode kernel finds K/V rows.
enum CacheMode : int {
    CACHE_PAGED = 0,      // context cache [layer][kvh][page][tok][128]
    CACHE_POSMAJOR = 1,   // caller cache [pos][kv_dim] (launch_attn layout)
};

// One decode launch.  Two schedules:
//  * piece mode (n_pieces > 0): CTA c processes pieces[c], one group-aligned
//    row range; used when the groups fit the SMs, so no CTA pays for two
//    groups' prologue and merge;
//  * linear mode: the work is a list of units -- for every (sequence b,
//    local kv head) group, ceil(Lc_b / DEC_TILE) cache tiles plus, when
//    `fused`, one unit for the new token; units are numbered sequence-major,
//    then kv head, then tile, and CTA c owns units
//    [c*total/n_ctas, (c+1)*total/n_ctas).
struct DecodeParams {
    const float* q;          // [nb][hq_total*128]; raw (fused) or prepared
    const float* k_new;      // [nb][nkv_total*128] raw (fused)
    const float* v_new;
    const float* q_norm_w;   // [128]
    const float* k_norm_w;
    float* q_out;            // normalised/rotated q written back (fused), may be null
    float* k_out;            // normalised/rotated k written back (fused), may be null
    float* xb;               // [nb][hq_total*128]; or partial o for attn_partial
    float* lse_out;          // [nb][hq_total] log2-sum-exp output (partial mode), may be null
    void* kcache;            // paged caches (append target in fused mode)
    void* vcache;
    float* partials;         // scratch: slots of PART_STRIDE floats
    int* counters;           // scratch: one per group, zero between launches
    int* err;                // device error flag
    float eps;
    float scale_log2e;       // log2(e)/sqrt(128)
    int nb;                  // sequences in this launch
    int nkv;                 // kv heads processed (local)
    int kv0;                 // global index of local kv head 0
    int hq_total;            // query heads per row of q / xb
    int nkv_total;           // kv heads per row of k_new / v_new
    int layer;
    int pages_per_seq;
    int page_tokens;
    int n_pages;             // pages per (layer, kv head)
    int cache_mode;          // CacheMode
    int fused;               // 1: new token prepared + appended in-kernel
    int partial_out;         // 1: write normalised o + lse instead of xb
    int peer_world;          // > 0: sequence-shard exchange over peer memory
    int peer_rank;
    int peer_row;            // 8-byte words per row: hq_total*128 + hq_total
    float* peer_recv[PEER_MAX];      // every rank's receive buffer (this device's view)
    unsigned* peer_epoch;    // this rank's call counter per KV head (device)
    long long total_units;
    int n_ctas;
    int n_pieces;            // > 0: piece mode with n_ctas == n_pieces
    int spread;              // 1: piece-mode groups merge by the spread merge
    int tc;                  // 1: tensor-core consumer (bf16 paged cache; 16-row swizzled maps)
    int early;               // 1: the producer streams cache rows before the dependency wait
                             //    (the host checked that the kernel depended on cannot write them)
    int early_rows;          // with `early`: only rows below this may stream before the wait
                             //    (the balanced schedule; INT_MAX when every row may)
    int dyn;                 // 1 (piece mode, paged cache, spread merge): each range streams a
                             //    few static units of its group, then claims the group's other
                             //    units from claim[group] (balances ranges on slower SMs)
    int* claim;              // [MAX_PIECES] per-group unit counters, zero between launches
    unsigned long long* words;   // spread merge: MAX_PIECES slots of PART_STRIDE tagged words
    unsigned* group_epoch;   // spread merge: call number per group [MAX_PIECES]
    const float* inv_freq;   // [64] RoPE inverse frequencies (host powf, reference formula)
    long long wait_limit;    // SM clocks a wait on another CTA or rank may take
    // Optional L2 prefetch of the next kernel's weights (the wo rows of the
    // sublayer), issued by each CTA's producer once its cache rows are all
    // requested: rows [c R / G, (c+1) R / G) of pf_rows rows, pf_row_bytes
    // from pf_base + r * pf_ld_bytes (null pf_base: none).
    const uint8_t* pf_base;
    int pf_rows, pf_row_bytes;
    long long pf_ld_bytes;
    Piece pieces[MAX_PIECES];
    short cta_piece[MAX_PIECES];  // piece mode: piece processed by CTA c (groups interleaved)
    int t_begin[MAX_B];      // first cache position attended per sequence
    int t_end[MAX_B];        // one past the last cache position read from the cache
    int pos[MAX_B];          // new-token position (fused)
    int slot[MAX_B];         // cache slot per sequence
    long long unit_prefix[MAX_B + 1];  // prefix of nkv * units_b
};

struct PrepParams {
    const float* src;        // raw rows [n][nheads_total*128]
    float* dst_f32;          // prepared rows (may be null)
    __nv_bfloat16* dst_bf16; // prepared rows (may be null)
    const float* w;          // norm gains [128]
    float eps;
    int n;                   // rows (tokens)
    int nheads;              // heads per row processed
    int head0;               // first head processed
    int nheads_total;        // heads per row in src / dst
    int pos0;                // position of row 0
    int do_norm_rope;
    const float* inv_freq;   // [64] device table
};

struct AppendParams {
    const float* k;          // [n][nkv_total*128]
    const float* v;
    const float* k_norm_w;
    void* kcache;
    void* vcache;
    float eps;
    int n;
    int nkv;                 // local kv heads
    int kv0;
    int nkv_total;
    int layer;
    int slot;
    int pos0;
    int pages_per_seq;
    int page_tokens;
    int n_pages;
    int do_norm_rope;        // 0: rows are already prepared (kv_load)
    int bf16;
    const float* inv_freq;   // [64] device table
};

// The q/k/v projections of one token with fp16 weights for the KV heads a
// context holds, fused with the layer's input RMSNorm (optional) and the
// block's QK-RMSNorm, RoPE and KV append (qkv_kernel, q3a_proj.cu).
struct QkvParams {
    const float* x;          // [dim] input: the layer input (normed in-kernel when norm_w)
    const float* norm_w;     // [dim] input RMSNorm gains, or null (x already normed)
    const __half* wq;        // [n_heads*128][dim] row-major (all heads)
    const __half* wk;        // [n_kv*128][dim]
    const __half* wv;        // [n_kv*128][dim]
    const float* q_norm_w;   // [128]
    const float* k_norm_w;
    float* q_out;            // [n_heads*128] normalised, rotated q (held heads written)
    float* k_out;            // [n_kv*128] normalised, rotated k, may be null
    float* v_out;            // [n_kv*128] v, may be null
    void* kcache;            // the context's paged caches (append at pos)
    void* vcache;
    float* part;             // scratch [rows_total]: the row sums
    int* ticket;             // scratch [nq + 2 nkv] rows summed per head, zero between launches
    int* err;                // device error flag (a wait that expired)
    const float* inv_freq;   // [64] RoPE inverse frequencies
    float eps;
    int dim;                 // columns (multiple of 8, at most 8192)
    int nq, nkv;             // held q heads (nkv * 4) and KV heads
    int kv0;                 // global index of the first held KV head
    int rows_total;          // (nq + 2 nkv) * 128
    int layer, pos, slot, pages_per_seq, page_tokens, n_pages;
};
// n_ctas >= nq + 2 nkv (a CTA's rows then touch at most two heads)
cudaError_t launch_qkv(const QkvParams& p, bool bf16, int n_ctas, cudaStream_t st);

// Rows per rank in the wo exchange region of the peer buffer (the largest
// model width supported).
constexpr int WO_MAX_ROWS = 8192;
constexpr int WO_MAX_CTAS = 256;

// x += wo[:, col0:col0+ncols] . xb[col0:col0+ncols] (wo_kernel, q3a_proj.cu);
// with world > 1 the ranks' partial sums are exchanged and added in rank order.
struct WoParams {
    const __half* w;         // wo [rows][ld] row-major
    int ld, col0, ncols;     // this context's columns (its held heads' xb slice)
    const float* xb;         // [ld] (columns col0.. valid)
    float* x;                // [rows] residual stream, updated in place
    int rows;
    int world, rank;
    unsigned long long* recv[PEER_MAX];  // every rank's wo exchange region, as mapped here
    unsigned* epoch;         // [WO_MAX_CTAS] per-CTA call numbers of this rank
    long long wait_limit;
    int* err;
};
cudaError_t launch_wo(const WoParams& p, int n_ctas, cudaStream_t st);

// Raises the dynamic shared-memory limit of kernel `fn` to `bytes` on the
// current device.  The attribute is per device, so it is set once per
// (kernel, device) pair; safe to call from several host threads.
cudaError_t ensure_smem_attr(const void* fn, int bytes);

// ---------------------------------------------------------------- launchers
// All return a cudaError_t of the launch.
cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap& tmK, const CUtensorMap& tmV,
                          bool bf16, cudaStream_t st);
int decode_smem_bytes(bool bf16);
cudaError_t launch_append(const AppendParams& p, cudaStream_t st);
cudaError_t launch_kv_read(const AppendParams& p, float* k_out, float* v_out, cudaStream_t st);
cudaError_t launch_prep_rows(const PrepParams& p, cudaStream_t st);
cudaError_t launch_randn(void* dst, int out_bf16, size_t n, uint64_t key, uint64_t offset,
                         cudaStream_t st);
cudaError_t launch_lse_combine(float* xb, const float* o_parts, size_t o_stride,
                               const float* lse_parts, size_t lse_stride, int n_parts, int n_heads,
                               cudaStream_t st);

// All-gather of column slices over peer memory (q3a_gather_cols).
struct ColGatherParams {
    const uint8_t* local;          // this rank's matrix (registered buffer + off)
    uint8_t* peer[PEER_MAX];       // every rank's matrix, as mapped here
    unsigned* flags;               // this rank's flag block: [2 phases][PEER_MAX], written by peers
    unsigned* peer_flags[PEER_MAX];// every rank's flag block, as mapped here
    unsigned* state;               // this rank: [0] call number, [1] CTA arrivals, [2] go
    int world, rank;
    long long rows;
    long long row_bytes;
    long long col0;                // bytes
    int vecs;                      // 16-byte vectors per row slice
    int* err;
    long long wait_limit;          // SM clocks a wait on another rank or CTA may take
};
cudaError_t launch_gather_cols(const ColGatherParams& p, int n_ctas, cudaStream_t st);

struct PrefillParams {
    const __nv_bfloat16* kcache;  // the context's paged bf16 caches
    const __nv_bfloat16* vcache;
    float* out_f32;
    __nv_bfloat16* out_bf16;
    int n_tok;
    int pos0;
    int hq_total;            // query heads per row
    int nkv;                 // local kv heads
    int kv0;
    int layer;
    int slot;
    int pages_per_seq;
    int page_tokens;
    int n_pages;
    float scale_log2e;
    int* err;
    // split of long causal items: item i (a 128-row query tile of one head
    // pair) with nj key tiles is cut into min(nsplit, ceil(nj/part_tiles))
    // parts of whole key tiles; every part of a split item writes a
    // normalised partial (o, lse) and prefill_combine_kernel merges them.
    int nsplit;              // most parts of an item (1: nothing is split)
    int part_tiles;          // key tiles per part, at most
    float* part;             // [items][nsplit][2 heads][PF_PART_FLOATS]
};
constexpr int PF_PART_FLOATS = 128 * 128 + 128;  // o [128 rows][128] + lse [128]
cudaError_t launch_prefill(const PrefillParams& p, const CUtensorMap& tmQ, cudaStream_t st);
int prefill_smem_bytes();

// KV-cache wire format (q3a_wire.cu): copies between a blob's payload and
// the paged cache.  Copied heads h < nkv are payload heads pay_head0 + h and
// context-local cache heads head_off + h.
struct WireParams {
    void* payload;           // the blob's payload (device memory)
    void* kcache;
    void* vcache;
    int layer0, n_layers;
    int nkv;                 // heads copied
    int pay_nkv, pay_head0;  // heads per layer in the payload, first one copied
    int ctx_nkv, head_off;   // the context's heads (cache layout), first one copied
    int pos0, n_tok, slot;
    int pages_per_seq, page_tokens, n_pages;
};
cudaError_t launch_wire_copy(const WireParams& p, bool bf16, bool pack, cudaStream_t st);
cudaError_t launch_wire_checksum(const void* payload, size_t bytes, unsigned long long* out,
                                 cudaStream_t st);
uint64_t wire_checksum_host(const void* payload, size_t bytes);

uint64_t stream_key(uint64_t seed, uint64_t stream);

// Sets the message q3a_last_error() returns on this thread; returns code.
int record_error(int code, const char* msg);

}  // namespace q3a
