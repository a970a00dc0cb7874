/*
 * q3attn.h -- C ABI of the B200 (sm_100a) grouped-query attention block of
 * Qwen3.c (Qwen3-VL-8B text decoder: 32 query heads share 8 KV heads,
 * head_dim 128).
 *
 * The reference (thamada/Qwen3.c) has no exported API: the block lives inline
 * in forward() (qwen3-8b/cpu/main.c:1319-1353, qwen3-8b/cpu-multicore/main.c:
 * 1331-1369, qwen3-8b/gpu/main.c:2093-2126) and works on the run-state
 * buffers of `State` (qwen3-8b/cpu/main.c:646-650): q, k, v, att, xb and the
 * caches kc, vc.  The entry points below take those same buffers, so a C host
 * replaces that block by one call.  Conventions:
 *   - every call returns Q3A_OK (0) or an error code; nothing calls exit()
 *     (the reference's HIPCHK exits, qwen3-8b/gpu/main.c:47-53); the message
 *     of the last failure on the calling thread is q3a_last_error();
 *   - one host thread per context; work is ordered on the context's stream;
 *   - pointer mode (q3a_cfg.ptr_mode): Q3A_PTR_HOST takes host pointers, like
 *     the CPU forward(), and returns after the result is in host memory;
 *     Q3A_PTR_DEVICE takes device pointers, like forward_gpu()'s device
 *     `State` (qwen3-8b/gpu/main.c:1287-1323), and returns once the work is
 *     queued on the stream.
 * Only head_dim 128 with 4 query heads per KV head is implemented (the
 * Qwen3-8B shape, qwen3-8b/gpu/main.c:8-10); other shapes return
 * Q3A_ERR_UNSUPPORTED.
 */
#ifndef Q3ATTN_H
#define Q3ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3A_OK 0
#define Q3A_ERR_INVALID 1      /* bad argument, shape or position */
#define Q3A_ERR_CUDA 2         /* CUDA runtime / driver error */
#define Q3A_ERR_OOM 3          /* device or pinned allocation failed */
#define Q3A_ERR_UNSUPPORTED 4  /* shape outside the implemented set */
#define Q3A_ERR_TIMEOUT 5      /* a bounded device-side wait expired */

#define Q3A_KV_F32 0           /* fp32 cache (the reference's layout dtype) */
#define Q3A_KV_BF16 1          /* bf16 cache, round-to-nearest-even on append */

#define Q3A_PTR_HOST 0
#define Q3A_PTR_DEVICE 1

#define Q3A_MAX_PEERS 8         /* ranks of a peer-memory sequence shard */
#define Q3A_IPC_HANDLE_BYTES 64 /* bytes of one exported buffer handle */
#define Q3A_PEER_REG_BYTES 136  /* bytes of one q3a_peer_register handle */

#define Q3A_OUT_F32 0
#define Q3A_OUT_BF16 1

#define Q3A_MAX_BATCH 256      /* sequences per batched call */

/* Shape and placement of one context.  Fields follow Config
 * (qwen3-8b/cpu/main.c:603-607) and the defaults parse_gguf applies
 * (qwen3-8b/cpu/main.c:874-876, 938-941). */
typedef struct q3a_cfg {
    int n_layers;       /* Config.n_layers (36) */
    int n_heads;        /* Config.n_heads (32) */
    int n_kv_heads;     /* Config.n_kv_heads (8) */
    int head_dim;       /* Config.head_dim (128) */
    int max_seq;        /* Config.max_seq: cache positions per sequence */
    int n_seqs;         /* sequences (cache slots) held; 1 for the reference */
    int kv_dtype;       /* Q3A_KV_F32 or Q3A_KV_BF16 */
    int page_tokens;    /* tokens per cache page, multiple of 64 (0: 64) */
    int ptr_mode;       /* Q3A_PTR_HOST or Q3A_PTR_DEVICE */
    int device;         /* CUDA device ordinal */
    float norm_eps;     /* Config.norm_eps (1e-6) */
    float rope_theta;   /* Config.rope_theta (5e6) */
    int kv_head_begin;  /* first KV head held (KV-head sharding); 0 */
    int kv_head_count;  /* KV heads held; 0 means all n_kv_heads */
} q3a_cfg;

typedef struct q3a_ctx q3a_ctx;

/* Fills cfg with the Qwen3-8B shape: 36 layers, 32/8 heads, head_dim 128,
 * max_seq 4096, one sequence, fp32 cache, 64-token pages, host pointers,
 * device 0, eps 1e-6, theta 5e6. */
void q3a_cfg_default(q3a_cfg *cfg);

/* Allocates the device KV cache ([layer][kv head][page][token][128], pages
 * 128-byte aligned, zero-filled; a bf16 cache stores each block of 8 tokens
 * as [2 dim-halves][8 tokens][64 dims] with the 128-byte swizzle of the
 * tensor-core operands, so it is read through q3a_kv_read, not by address)
 * and the context's scratch.  Replaces
 * alloc_state / alloc_state_gpu for the cache (qwen3-8b/cpu/main.c:1134-1148,
 * qwen3-8b/gpu/main.c:1287-1323); sizes are size_t, so 36 layers x 131072
 * positions do not overflow as the reference's int kv_cache_len does. */
int q3a_create(q3a_ctx **ctx, const q3a_cfg *cfg);
int q3a_destroy(q3a_ctx *ctx);

/* Message of the last failed call on this thread ("" if none). */
const char *q3a_last_error(void);

/* Sets the CUDA stream (a cudaStream_t) the context queues work on; NULL
 * selects the context's own stream.  The own stream is a blocking stream: it
 * orders with the legacy default stream (work queued there before a call
 * completes first; work queued there after a call waits for it), not with
 * other non-blocking streams. */
int q3a_set_stream(q3a_ctx *ctx, void *cuda_stream);
int q3a_sync(q3a_ctx *ctx);

/* ---- Recording a token step as one CUDA graph, for C hosts without the
 * CUDA runtime headers (the reference's forward_gpu launches its ~20 kernels
 * per layer one by one, qwen3-8b/gpu/main.c:2069-2161).  q3a_graph_begin
 * starts recording the context's stream (device-pointer mode; a stream set
 * with q3a_set_stream must not be the legacy NULL stream); the library calls
 * made until q3a_graph_end are recorded, not run, and q3a_graph_end returns
 * them as a replayable graph; q3a_graph_launch replays it on the context's
 * stream (same pointers, layers and positions as recorded; the kernels'
 * chaining is kept).  Make one ordinary call of each entry point before
 * recording it (first calls allocate their scratch) and no call that waits
 * for the stream (q3a_sync, host-pointer calls, q3a_kv_pack / unpack) while
 * recording.  The host's own kernels may be recorded in between on the same
 * stream.  q3a_graph_destroy frees a graph. */
typedef struct q3a_graph q3a_graph;
int q3a_graph_begin(q3a_ctx *ctx);
int q3a_graph_end(q3a_ctx *ctx, q3a_graph **graph);
int q3a_graph_launch(q3a_ctx *ctx, q3a_graph *graph);
int q3a_graph_destroy(q3a_graph *graph);

/* Reads and clears the device error flag set by bounded waits in the kernels
 * (Q3A_ERR_TIMEOUT when one expired, else Q3A_OK).  After a timeout the
 * context's own counters are cleared and its next calls run normally; the
 * call numbers of a peer set (sequence shards, column gather, wo exchange)
 * may then disagree between ranks, so a peer set that timed out is
 * re-created on every rank (new contexts, q3a_peer_export / open). */
int q3a_check_device_error(q3a_ctx *ctx);

/* The whole attention block of one layer for one new token at `pos`
 * (qwen3-8b/cpu/main.c:1319-1353; HIP: qwen3-8b/gpu/main.c:2093-2126):
 * per-head QK-RMSNorm of q (n_heads) and k (n_kv_heads) with the layer's
 * q_norm_w / k_norm_w [head_dim], RoPE at pos, append of k and v to the
 * context's cache of sequence 0 at pos, then softmax(q.K^T/sqrt(hd)).V over
 * positions 0..pos into xb.  q and k are normalised and rotated in place as
 * in the reference.  Buffers: xb, q [n_heads*head_dim]; k, v [n_kv*head_dim]. */
int q3a_attn_layer(q3a_ctx *ctx, float *xb, float *q, float *k, const float *v,
                   const float *q_norm_w, const float *k_norm_w, int layer, int pos);

/* Decode attention with the argument list of launch_attn
 * (qwen3-8b/xdna2/main.c:2724-2727) over a caller-owned position-major cache
 * kc/vc [layers][max_seq][kv_dim] (fp32): q already normalised and rotated,
 * position pos already appended.  att is accepted and unused (the reference
 * GPU build allocates it only for head_dim > 256, qwen3-8b/gpu/main.c:1305).
 * In host mode the rows 0..pos of layer offset loff are uploaded per call. */
int q3a_attn_decode(q3a_ctx *ctx, float *xb, const float *q, const float *kc,
                    const float *vc, float *att, size_t loff, int pos, int n_heads,
                    int kv_mul, int hd, int kv_dim, int max_seq);

/* Decode attention with the arguments of q3a_attn_decode, for callers that
 * cannot allocate device memory when they run it.  It has no counterpart in
 * the reference (whose CPU and HIP builds allocate their run state once,
 * qwen3-8b/gpu/main.c:1287-1323, and never need per-call scratch).  All
 * pointers are device memory (q, caches kc/vc at layer offset loff, output
 * xb); no context is needed and nothing is allocated: the split-KV scratch
 * is a fixed array of 330,308 bytes in the library's device memory, reserved
 * when the library's module loads on a device and held until the process
 * exits.  Limit: at most 16 KV heads (kv_dim <= 2048); larger calls return
 * Q3A_ERR_INVALID.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first
 * call before any stream capture.  All calls share the array, so calls that
 * can overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller.  Work is queued on `cuda_stream` (a
 * cudaStream_t, NULL for the legacy default stream) and the call returns
 * without waiting for it.  Each call clears the array's error word before
 * its launch; q3a_noalloc_check_error reports what the last launch left.
 * The stored array address belongs to the device's context: do not use
 * this entry point on a device after cudaDeviceReset. */
int q3a_attn_decode_noalloc(float *xb, const float *q, const float *kc, const float *vc,
                            size_t loff, int pos, int n_heads, int kv_mul, int hd, int kv_dim,
                            int max_seq, void *cuda_stream);

/* Companion of q3a_attn_decode_noalloc, allocating nothing either: waits for
 * `cuda_stream` and reads, then clears, the error word of the current
 * device's fixed array.  Q3A_ERR_TIMEOUT if a bounded wait inside the last
 * noalloc launch expired (its xb is then not valid), else Q3A_OK.  No
 * counterpart in the reference, which has no device-side waits. */
int q3a_noalloc_check_error(void *cuda_stream);

/* The attention block of one token from its layer input: the q/k/v
 * projections mm(s->q/k/v, s->xb, w->wq/wk/wv[l], dim, ...) with fp16
 * weights (mm_f16, qwen3-8b/cpu/main.c:1206-1213 called at 1315-1317; HIP
 * mm_f16_gemv_kernel, qwen3-8b/gpu/main.c:1495-1519), fused with the
 * QK-RMSNorm, RoPE and the KV append of the block (main.c:1319-1329), then
 * the attention of q3a_attn_layer over cache rows 0..pos of slot 0.
 *   x [dim]: the normed layer input (s->xb of the reference);
 *   wq [n_heads*hd][dim], wk, wv [n_kv*hd][dim]: fp16 weights, row-major;
 *   q [n_heads*hd] (out): the normalised, rotated q;
 *   k [n_kv*hd] (out, may be NULL): the normalised, rotated k;
 *   v [n_kv*hd] (out, may be NULL): v;
 *   xb [n_heads*hd] (out): the attention output.
 * Sums are fp32 in a fixed order (per thread, over a warp, then over the
 * consumer warps), not the reference's one sequential sum: q, k and v agree
 * with it to fp32 rounding and repeat bit for bit (xb repeats bit for bit in
 * the deterministic schedule, q3a_set_deterministic).  A context holding KV heads
 * [b, b + n) (kv_head_begin/count) projects only their rows: q heads 4b ..
 * 4(b+n)-1 and KV heads b .. b+n-1, written at their places in the
 * full-width q, k, v (column-parallel), and attends over them (xb: their
 * columns).  Device pointers only (Q3A_PTR_DEVICE); dim a multiple of 8, at
 * most 8192; every vector and weight pointer 16-byte aligned.  The weights
 * are read before the wait on the kernel queued just before the call on the
 * stream (they are streamed while it finishes): that kernel must not write
 * them. */
int q3a_attn_layer_proj(q3a_ctx *ctx, float *xb, float *q, float *k, float *v, const float *x,
                        const void *wq, const void *wk, const void *wv, int dim,
                        const float *q_norm_w, const float *k_norm_w, int layer, int pos);

/* The projection half of q3a_attn_layer_proj alone: q, k, v of one token
 * from the layer input x (fp16 weights, fp32 sums), QK-RMSNorm and RoPE of q
 * and k, and the append of k and v to slot 0 at pos; the attention is left
 * to the caller (qwen3-8b/cpu/main.c:1315-1329, which it replaces).  Same
 * arguments, outputs and limits as q3a_attn_layer_proj. */
int q3a_qkv_proj(q3a_ctx *ctx, float *q, float *k, float *v, const float *x, const void *wq,
                 const void *wk, const void *wv, int dim, const float *q_norm_w,
                 const float *k_norm_w, int layer, int pos);

/* The consumer of xb: x += wo . xb, the o-projection and residual add of
 * the attention sublayer (mm(s->xb2, s->xb, w->wo[l], dim, dim) and
 * x[i] += xb2[i], qwen3-8b/cpu/main.c:1355-1356; HIP mm_f16_gemv_kernel +
 * vec_add_kernel, qwen3-8b/gpu/main.c:2131-2135).  wo is fp16
 * [dim][n_heads*hd] row-major, x [dim] and xb [n_heads*hd] fp32 device
 * buffers; x is updated in place.  A context holding KV heads [b, b + n)
 * multiplies only their query heads' xb columns (row-parallel) and needs a
 * peer set (q3a_peer_export / q3a_peer_open over the ranks that hold the
 * other heads): each rank stores its partial sums into every rank's peer
 * buffer over NVLink inside the kernel and adds all ranks' partials in rank
 * order, so every rank's x gets the same bits; every rank of the set makes
 * the same calls in the same order.  dim at most 8192.  Device pointers only. */
int q3a_wo_residual(q3a_ctx *ctx, float *x, const float *xb, const void *wo, int dim);

/* The attention sublayer of one token at pos (slot 0), from the residual
 * stream x to x + attention: rmsnorm(x, att_norm_w) fused into the q/k/v
 * projections (q3a_qkv_proj), the decode of the held heads over rows 0..pos,
 * then q3a_wo_residual (qwen3-8b/cpu/main.c:1313-1356; HIP forward_gpu
 * qwen3-8b/gpu/main.c:2095-2135).  Three kernels, stream-ordered with
 * programmatic dependent launch (the weights of each stream in while the
 * kernel before finishes).  Weights and limits as q3a_attn_layer_proj and
 * q3a_wo_residual; q and xb live in the context.  Over KV-head shards (a
 * peer set of the ranks holding the other heads) every rank passes the same
 * x and weights and ends with the same x. */
int q3a_attn_sublayer(q3a_ctx *ctx, float *x, const float *att_norm_w, const void *wq,
                      const void *wk, const void *wv, const float *q_norm_w,
                      const float *k_norm_w, const void *wo, int dim, int layer, int pos);

/* Batched ragged decode: n new tokens, token i belongs to cache slot
 * seq_ids[i] (distinct) at position pos[i] (host arrays).  The block of
 * q3a_attn_layer runs for each; q, xb are [n][n_heads*hd], k, v
 * [n][n_kv*hd].  With KV-head sharding (kv_head_count < n_kv_heads) only the
 * held heads' xb slices are written.  The reference has no batch; this is its
 * block applied to n independent sequences. */
int q3a_attn_layer_batched(q3a_ctx *ctx, float *xb, float *q, float *k, const float *v,
                           const float *q_norm_w, const float *k_norm_w, int layer,
                           const int *seq_ids, const int *pos, int n);

/* KV append of n consecutive tokens of slot `seq` at positions pos0..:
 * QK-RMSNorm + RoPE of k (as in the block), then the write of k and v
 * (qwen3-8b/cpu/main.c:1325-1329; HIP kv_cache_write_kernel
 * qwen3-8b/gpu/main.c:1447-1467).  k, v are [n][n_kv*hd] raw projections; k is
 * not modified. */
int q3a_kv_append(q3a_ctx *ctx, int seq, int layer, int pos0, int n, const float *k,
                  const float *v, const float *k_norm_w);

/* Writes already-prepared rows (position-major [n][n_kv*hd], fp32) into the
 * cache at pos0.. without norm or RoPE, converting to the cache dtype. */
int q3a_kv_load(q3a_ctx *ctx, int seq, int layer, int pos0, int n, const float *k,
                const float *v);

/* ---- KV-cache wire format: a sequence's cache rows as one self-checking
 * blob, for handing a prompt's KV pages from a prefill GPU to a decode GPU
 * (or to disk).  No counterpart in the reference, whose caches never leave
 * the process.  Blob = this 64-byte header (little-endian) + payload: for
 * each layer of [layer0, layer0 + n_layers), each KV head of
 * [kv_head_begin, + kv_head_count), K then V, the rows of positions
 * [pos0, pos0 + n_tok), head_dim values each, in the cache dtype (fp32, or
 * bf16 as rounded on append), row-major.  checksum = sum over the payload's
 * 64-bit words w_i of mix(w_i + i * 0x9E3779B97F4A7C15) mod 2^64, mix being
 * the splitmix64 output function. */
#define Q3A_KV_WIRE_MAGIC 0x564B3351u /* "Q3KV" */
#define Q3A_KV_WIRE_VERSION 1
typedef struct q3a_kv_wire_header {
    uint32_t magic;
    uint16_t version;
    uint16_t dtype;          /* Q3A_KV_F32 / Q3A_KV_BF16 */
    uint16_t head_dim;
    uint16_t n_kv_heads;     /* the model's KV heads */
    uint16_t kv_head_begin;  /* heads in this blob */
    uint16_t kv_head_count;
    uint16_t layer0;
    uint16_t n_layers;
    uint32_t pos0;
    uint32_t n_tok;
    uint32_t reserved0;
    uint64_t payload_bytes;
    uint64_t checksum;
    uint8_t reserved[16];
} q3a_kv_wire_header;

/* Bytes of the blob q3a_kv_pack writes for n_layers layers and n_tok
 * positions of the context's held KV heads (0 on bad arguments). */
size_t q3a_kv_wire_bytes(const q3a_ctx *ctx, int n_layers, int n_tok);

/* Packs rows [pos0, pos0 + n_tok) of layers [layer0, layer0 + n_layers) of
 * slot `seq` (the context's held KV heads) into dst (dst_bytes >=
 * q3a_kv_wire_bytes; host or device memory per the pointer mode). */
int q3a_kv_pack(q3a_ctx *ctx, int seq, int layer0, int n_layers, int pos0, int n_tok, void *dst,
                size_t dst_bytes);

/* Unpacks a blob into slot `seq`: the header must match the context (dtype,
 * head_dim, n_kv_heads; the blob's heads must include the context's; layers
 * and positions inside the cache) and the payload's checksum must match;
 * otherwise Q3A_ERR_INVALID and the cache is not touched.  The context's
 * held heads are written at the blob's layers and positions. */
int q3a_kv_unpack(q3a_ctx *ctx, int seq, const void *src, size_t src_bytes);

/* Checks a blob in host memory without a GPU: header fields and the
 * payload's checksum.  Q3A_OK, or Q3A_ERR_INVALID with the reason in
 * q3a_last_error(). */
int q3a_kv_wire_check(const void *blob, size_t bytes);

/* Seeded synthetic cache rows, for harnesses and benchmarks that have no
 * model data: raw k and v rows [n][n_kv*hd] ~ N(0,1) from the generator of
 * q3a_randn (seed; streams stream_k, stream_v), stored at pos0.. exactly as
 * q3a_kv_append stores raw rows with unit norm gains (QK-RMSNorm + RoPE of
 * k at its position).  Generated on the device in the context's scratch, in
 * either pointer mode.  No counterpart in the reference, which fills its
 * cache only from real tokens. */
int q3a_kv_synth(q3a_ctx *ctx, int seq, int layer, int pos0, int n, uint64_t seed,
                 uint64_t stream_k, uint64_t stream_v);

/* Reads cache rows back as fp32 position-major [n][n_kv*hd]. */
int q3a_kv_read(q3a_ctx *ctx, int seq, int layer, int pos0, int n, float *k, float *v);

/* Causal prefill of n_tok prompt tokens of slot `seq` at positions
 * pos0..pos0+n_tok-1: QK-RMSNorm + RoPE of q and k, append of k/v, then for
 * every prompt row s the attention over positions 0..pos0+s.  This is the
 * reference's prompt loop (qwen3-8b/cpu/main.c:1481-1499, one forward() per
 * token) done as one batched causal attention on the tensor cores.
 * q [n_tok][n_heads*hd] raw (left unmodified), k, v [n_tok][n_kv*hd] raw; out
 * [n_tok][n_heads*hd] in out_dtype (Q3A_OUT_F32 / Q3A_OUT_BF16).  Requires a
 * bf16 cache (the tensor-core operands are bf16, softmax and accumulation
 * fp32).  A context created with kv_head_begin/kv_head_count (KV-head
 * sharding) takes the same full-width q, k, v rows, keeps its own KV heads
 * and writes only its query heads' columns of out; the other columns are
 * left as the caller had them. */
int q3a_prefill(q3a_ctx *ctx, void *out, int out_dtype, const float *q, const float *k,
                const float *v, const float *q_norm_w, const float *k_norm_w, int seq,
                int layer, int pos0, int n_tok);

/* Causal attention only, on already-prepared bf16 operands: q_bf16
 * [n_tok][n_heads][hd] (normed, rotated) over the cache of slot seq, rows
 * pos0+s attending to 0..pos0+s.  Same output contract as q3a_prefill. */
int q3a_prefill_attn(q3a_ctx *ctx, void *out, int out_dtype, const void *q_bf16,
                     int seq, int layer, int pos0, int n_tok);

/* Sequence-sharded decode, step 1: attention of one already-prepared query
 * q [n_heads*hd] over cache positions [t0, t1) of slot seq (t0 < t1), giving
 * the chunk's normalised output o [n_heads*hd] and its log-sum-exp lse
 * [n_heads] in log2 units (log2 sum_t 2^(s_t log2 e), s_t = q.k_t/sqrt(hd)).
 * Empty chunks (t0 == t1) give o = 0, lse = -inf. */
int q3a_attn_partial(q3a_ctx *ctx, float *o, float *lse, const float *q, int seq,
                     int layer, int t0, int t1);

/* Sequence-sharded decode, step 2: merges n_parts chunk results
 * (o_parts [n_parts][n_heads*hd], lse_parts [n_parts][n_heads]) into xb by
 * log-sum-exp weights. */
int q3a_lse_combine(q3a_ctx *ctx, float *xb, const float *o_parts,
                    const float *lse_parts, int n_parts);

/* Sequence-sharded decode, step 2 in the layout one all-gather produces:
 * parts [n_parts][n_heads*hd + n_heads], part j = rank j's o followed by its
 * lse (what q3a_attn_partial writes when given o = part, lse = part +
 * n_heads*hd).  Same merge as q3a_lse_combine; the reference has no
 * multi-GPU path, so this replaces nothing in it. */
int q3a_lse_combine_packed(q3a_ctx *ctx, float *xb, const float *parts, int n_parts);

/* Sequence-sharded decode over peer memory (NVLink), one launch per layer
 * and no collective library: the alternative to q3a_attn_partial + an
 * all-gather + q3a_lse_combine_packed.  The reference has no multi-GPU path;
 * these three calls replace nothing in it.
 *
 * Set-up, once per context, in the same order on every rank (one process
 * per GPU, contexts holding all KV heads, device-pointer mode):
 *   q3a_peer_export(ctx, world, handle)  allocates this rank's receive
 *       buffer (two parity halves of world packed (o, lse) rows and their
 *       flags) and writes its IPC handle (Q3A_IPC_HANDLE_BYTES) to `handle`;
 *   the caller exchanges the handles (any transport) and calls
 *   q3a_peer_open(ctx, rank, world, handles)  with all ranks' handles in rank
 *       order, mapping the peers' buffers.
 * Per layer: q3a_attn_seqshard(ctx, xb, q, seq, layer, n_local) attends the
 * prepared q [n_heads*hd] over rows [0, n_local) of this rank's cache; each
 * KV head's result is stored into every rank's buffer, a flag is raised, and
 * once every rank's result for that head has arrived (bounded wait, error
 * Q3A_ERR_TIMEOUT after about a second) the log-sum-exp merge writes that
 * head group of xb on every rank.  All ranks must make the same sequence of
 * calls; a rank may run at most one call ahead of another. */
int q3a_peer_export(q3a_ctx *ctx, int world, void *handle);
int q3a_peer_open(q3a_ctx *ctx, int rank, int world, const void *handles);
int q3a_attn_seqshard(q3a_ctx *ctx, float *xb, const float *q, int seq, int layer,
                      int n_local);

/* Single-process form of the set-up above, for a host that drives every
 * rank's context from one process (one context per GPU with peer access
 * enabled between the devices by the caller, or several on one device):
 * after q3a_peer_export on every context, q3a_peer_buffer gives each
 * context's receive buffer as a device pointer, and
 * q3a_peer_open_ptrs(ctx, rank, world, bufs) takes all ranks' buffers in rank
 * order instead of IPC handles.  No counterpart in the reference. */
int q3a_peer_buffer(q3a_ctx *ctx, void **buf);
int q3a_peer_open_ptrs(q3a_ctx *ctx, int rank, int world, void *const *bufs);

/* All-gather of column slices over peer memory (NVLink), for KV-head shards:
 * rank r computed columns [col0_r, col0_r + col_bytes) of every row of a
 * row-major matrix (its query heads' slice of xb or of a prefill output);
 * afterwards every rank holds every rank's columns.  No collective library
 * is called; the reference has no multi-GPU path and these calls replace
 * nothing in it.
 * Set-up, once per context, in the same order on every rank (one process
 * per GPU, device-pointer mode):
 *   q3a_peer_register(ctx, buf, bytes, handle)  makes the caller's device
 *       buffer [buf, buf+bytes) (cudaMalloc'd, directly or by an allocator)
 *       and a flag block mappable by the other ranks; `handle` receives
 *       Q3A_PEER_REG_BYTES bytes;
 *   the caller exchanges the handles and calls
 *   q3a_peer_register_open(ctx, rank, world, handles)  with all ranks'
 *       handles in rank order.
 * Per call: q3a_gather_cols(ctx, off, rows, row_bytes, col0, col_bytes)
 * gathers the matrix starting `off` bytes into every rank's registered
 * buffer (same layout on every rank; row_bytes, col0 and col_bytes multiples
 * of 16; this rank's columns start at col0).  One launch: the ranks first
 * meet (so no rank writes into a buffer another rank still reads from its
 * previous call), each copies its columns into every other rank's buffer,
 * then they meet again; bounded waits (Q3A_ERR_TIMEOUT after about a
 * second).  Stream-ordered; all ranks make the same sequence of calls. */
int q3a_peer_register(q3a_ctx *ctx, void *buf, size_t bytes, void *handle);
int q3a_peer_register_open(q3a_ctx *ctx, int rank, int world, const void *handles);
int q3a_gather_cols(q3a_ctx *ctx, size_t off, long long rows, size_t row_bytes, size_t col0,
                    size_t col_bytes);

/* Single-process form of q3a_peer_register_open: after q3a_peer_register on
 * every context, q3a_peer_register_flags gives each context's flag block, and
 * q3a_peer_register_open_ptrs takes all ranks' registered buffers (the `buf`
 * each passed to q3a_peer_register) and flag blocks in rank order. */
int q3a_peer_register_flags(q3a_ctx *ctx, void **flags);
int q3a_peer_register_open_ptrs(q3a_ctx *ctx, int rank, int world, void *const *bufs,
                                void *const *flags);

/* Limit of every device-side wait of this context's kernels on another CTA
 * or another rank (the split-KV merge, the sequence-shard exchange, the
 * column all-gather), in seconds at the device's highest SM clock; 0 restores
 * the default of about one second.  A wait that runs out stops the kernel,
 * which leaves its output unwritten and the device error flag set
 * (q3a_check_device_error gives Q3A_ERR_TIMEOUT); the context stays usable.
 * Replaces the reference's HIPCHK exit (qwen3-8b/gpu/main.c:47-53), which has
 * no device-side waits at all. */
int q3a_set_wait_limit(q3a_ctx *ctx, double seconds);

/* Decode work split.  By default (on = 0) the ranges of a (sequence, KV
 * head) group balance their work at run time: each streams a few fixed
 * units of cache rows and then claims the group's remaining units one at a
 * time, so ranges on SMs with lower memory throughput take fewer.  Which
 * range sums which rows then varies from call to call, and results can
 * differ in the last bits between identical calls (within the parity
 * tolerances).  on = 1 gives every range a fixed row range: identical calls
 * give bitwise-identical results, at some cost in speed.  The reference
 * (single-threaded C loops) is deterministic; this switch has no
 * counterpart there. */
int q3a_set_deterministic(q3a_ctx *ctx, int on);

/* Seeded N(0,1) fill of n elements (fp32 or bf16 by out_dtype): element i is
 * the Box-Muller transform of uniforms u(2j), u(2j+1), j = (offset+i)/2, with
 * u from a splitmix64-hashed counter passed through the xorshift64* output
 * step of rng_f32 (qwen3-8b/cpu/main.c:1377-1382).  dst is device memory. */
int q3a_randn(q3a_ctx *ctx, void *dst, int out_dtype, size_t n, uint64_t seed,
              uint64_t stream_id, uint64_t offset);

/* Number of kernels the library launched on this context so far. */
uint64_t q3a_launch_count(const q3a_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif /* Q3ATTN_H */
