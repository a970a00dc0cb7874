"""ctypes binding of lib/libq3attn.so (include/q3attn.h).

This is how the Python harness (tests, bench) reaches the library: the same
extern "C" entry points a C host such as Qwen3.c's forward() links against.
Loading fails loudly if the library was not built; there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libq3attn.so")
IPC_HANDLE_BYTES = 64  # Q3A_IPC_HANDLE_BYTES
PEER_REG_BYTES = 136   # Q3A_PEER_REG_BYTES
MAX_PEERS = 8          # Q3A_MAX_PEERS

OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_UNSUPPORTED, ERR_TIMEOUT = 0, 1, 2, 3, 4, 5
KV_F32, KV_BF16 = 0, 1
PTR_HOST, PTR_DEVICE = 0, 1
OUT_F32, OUT_BF16 = 0, 1
MAX_BATCH = 256

# Every symbol include/q3attn.h declares.
EXPORTS = [
    "q3a_cfg_default", "q3a_create", "q3a_destroy", "q3a_last_error", "q3a_set_stream",
    "q3a_sync", "q3a_check_device_error", "q3a_attn_layer", "q3a_attn_decode",
    "q3a_attn_layer_batched", "q3a_attn_layer_proj", "q3a_qkv_proj",
    "q3a_wo_residual", "q3a_attn_sublayer",
    "q3a_kv_append", "q3a_kv_load", "q3a_kv_read", "q3a_prefill",
    "q3a_prefill_attn", "q3a_attn_partial", "q3a_lse_combine", "q3a_lse_combine_packed",
    "q3a_peer_export", "q3a_peer_open", "q3a_attn_seqshard",
    "q3a_peer_buffer", "q3a_peer_open_ptrs",
    "q3a_peer_register", "q3a_peer_register_open", "q3a_gather_cols",
    "q3a_peer_register_flags", "q3a_peer_register_open_ptrs", "q3a_set_wait_limit",
    "q3a_set_deterministic",
    "q3a_randn", "q3a_kv_synth",
    "q3a_launch_count", "q3a_attn_decode_noalloc", "q3a_noalloc_check_error",
    "q3a_kv_wire_bytes", "q3a_kv_pack", "q3a_kv_unpack", "q3a_kv_wire_check",
    "q3a_graph_begin", "q3a_graph_end", "q3a_graph_launch", "q3a_graph_destroy",
]

KV_WIRE_MAGIC = 0x564B3351
KV_WIRE_VERSION = 1
KV_WIRE_HEADER_BYTES = 64


class Cfg(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("max_seq", ctypes.c_int), ("n_seqs", ctypes.c_int),
        ("kv_dtype", ctypes.c_int), ("page_tokens", ctypes.c_int), ("ptr_mode", ctypes.c_int),
        ("device", ctypes.c_int), ("norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("kv_head_begin", ctypes.c_int), ("kv_head_count", ctypes.c_int),
    ]


class Q3AError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"q3attn error {code}: {msg}")
        self.code = code


_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_U64 = ctypes.c_uint64


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it (make -C qwen3.c_b200)")
        L = ctypes.CDLL(LIB_PATH)
        L.q3a_cfg_default.argtypes = [ctypes.POINTER(Cfg)]
        L.q3a_cfg_default.restype = None
        L.q3a_create.argtypes = [ctypes.POINTER(_P), ctypes.POINTER(Cfg)]
        L.q3a_destroy.argtypes = [_P]
        L.q3a_last_error.restype = ctypes.c_char_p
        L.q3a_set_stream.argtypes = [_P, _P]
        L.q3a_sync.argtypes = [_P]
        L.q3a_check_device_error.argtypes = [_P]
        L.q3a_attn_layer.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I, _I]
        L.q3a_attn_decode.argtypes = [_P, _P, _P, _P, _P, _P, _SZ, _I, _I, _I, _I, _I, _I]
        L.q3a_attn_layer_batched.argtypes = [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I]
        L.q3a_attn_layer_proj.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I, _I]
        L.q3a_qkv_proj.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I, _I]
        L.q3a_wo_residual.argtypes = [_P, _P, _P, _P, _I]
        L.q3a_attn_sublayer.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I]
        L.q3a_kv_append.argtypes = [_P, _I, _I, _I, _I, _P, _P, _P]
        L.q3a_kv_load.argtypes = [_P, _I, _I, _I, _I, _P, _P]
        L.q3a_kv_read.argtypes = [_P, _I, _I, _I, _I, _P, _P]
        L.q3a_prefill.argtypes = [_P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I]
        L.q3a_prefill_attn.argtypes = [_P, _P, _I, _P, _I, _I, _I, _I]
        L.q3a_attn_partial.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I]
        L.q3a_lse_combine.argtypes = [_P, _P, _P, _P, _I]
        L.q3a_lse_combine_packed.argtypes = [_P, _P, _P, _I]
        L.q3a_peer_export.argtypes = [_P, _I, _P]
        L.q3a_peer_open.argtypes = [_P, _I, _I, _P]
        L.q3a_attn_seqshard.argtypes = [_P, _P, _P, _I, _I, _I]
        L.q3a_peer_register.argtypes = [_P, _P, _SZ, _P]
        L.q3a_peer_register_open.argtypes = [_P, _I, _I, _P]
        L.q3a_gather_cols.argtypes = [_P, _SZ, ctypes.c_longlong, _SZ, _SZ, _SZ]
        L.q3a_peer_buffer.argtypes = [_P, ctypes.POINTER(_P)]
        L.q3a_peer_open_ptrs.argtypes = [_P, _I, _I, ctypes.POINTER(_P)]
        L.q3a_peer_register_flags.argtypes = [_P, ctypes.POINTER(_P)]
        L.q3a_peer_register_open_ptrs.argtypes = [_P, _I, _I, ctypes.POINTER(_P),
                                                  ctypes.POINTER(_P)]
        L.q3a_set_wait_limit.argtypes = [_P, ctypes.c_double]
        L.q3a_set_deterministic.argtypes = [_P, _I]
        L.q3a_randn.argtypes = [_P, _P, _I, _SZ, _U64, _U64, _U64]
        L.q3a_kv_synth.argtypes = [_P, _I, _I, _I, _I, _U64, _U64, _U64]
        L.q3a_attn_decode_noalloc.argtypes = [_P, _P, _P, _P, _SZ, _I, _I, _I, _I, _I, _I, _P]
        L.q3a_noalloc_check_error.argtypes = [_P]
        L.q3a_launch_count.argtypes = [_P]
        L.q3a_launch_count.restype = _U64
        L.q3a_kv_wire_bytes.argtypes = [_P, _I, _I]
        L.q3a_kv_wire_bytes.restype = _SZ
        L.q3a_kv_pack.argtypes = [_P, _I, _I, _I, _I, _I, _P, _SZ]
        L.q3a_kv_unpack.argtypes = [_P, _I, _P, _SZ]
        L.q3a_kv_wire_check.argtypes = [_P, _SZ]
        L.q3a_graph_begin.argtypes = [_P]
        L.q3a_graph_end.argtypes = [_P, ctypes.POINTER(_P)]
        L.q3a_graph_launch.argtypes = [_P, _P]
        L.q3a_graph_destroy.argtypes = [_P]
        _lib = L
    return _lib


def check(rc: int):
    if rc != OK:
        raise Q3AError(rc, load().q3a_last_error().decode())


def ptr(x) -> int:
    """Address of a numpy array (host) or a torch tensor (host or device)."""
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        assert x.is_contiguous()
        return x.data_ptr()
    assert x.flags["C_CONTIGUOUS"]
    return x.ctypes.data


def attn_decode_noalloc(xb, q, kc, vc, loff, pos, n_heads, kv_mul, hd, kv_dim, max_seq,
                        stream_handle=None):
    """q3a_attn_decode_noalloc: device pointers only, no context, nothing
    allocated; queued on the given CUDA stream handle."""
    check(load().q3a_attn_decode_noalloc(ptr(xb), ptr(q), ptr(kc), ptr(vc), loff, pos, n_heads,
                                         kv_mul, hd, kv_dim, max_seq, stream_handle))


def kv_wire_check(blob) -> None:
    """q3a_kv_wire_check on a blob in host memory (bytes, bytearray or a
    uint8 numpy array): header fields and payload checksum, no GPU."""
    import numpy as np
    a = np.frombuffer(blob, dtype=np.uint8) if isinstance(blob, (bytes, bytearray)) else blob
    a = np.ascontiguousarray(a)
    check(load().q3a_kv_wire_check(a.ctypes.data, a.nbytes))


def _nbytes(t) -> int:
    if hasattr(t, "element_size"):
        return t.numel() * t.element_size()
    return t.nbytes


def noalloc_check_error(stream_handle=None):
    """q3a_noalloc_check_error: waits for the stream, then reads and clears
    the fixed array's device error word (Q3AError with ERR_TIMEOUT if a
    bounded wait of the last noalloc launch expired)."""
    check(load().q3a_noalloc_check_error(stream_handle))


def default_cfg(**kw) -> Cfg:
    c = Cfg()
    load().q3a_cfg_default(ctypes.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


class Context:
    """Owns one q3a_ctx.  Methods mirror the C entry points one to one."""

    def __init__(self, **cfg):
        self.lib = load()
        self.cfg = default_cfg(**cfg)
        h = _P()
        check(self.lib.q3a_create(ctypes.byref(h), ctypes.byref(self.cfg)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.q3a_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_handle: int | None):
        check(self.lib.q3a_set_stream(self.h, stream_handle))

    def sync(self):
        check(self.lib.q3a_sync(self.h))

    def check_device_error(self):
        check(self.lib.q3a_check_device_error(self.h))

    def launch_count(self) -> int:
        return int(self.lib.q3a_launch_count(self.h))

    def attn_layer(self, xb, q, k, v, qw, kw, layer, pos):
        check(self.lib.q3a_attn_layer(self.h, ptr(xb), ptr(q), ptr(k), ptr(v), ptr(qw), ptr(kw),
                                      layer, pos))

    def attn_layer_proj(self, xb, q, k, v, x, wq, wk, wv, qw, kw, layer, pos):
        """Projections (fp16 weights) + QK-norm + RoPE + append + attention of
        one token from its layer input x; device tensors; k, v may be None."""
        check(self.lib.q3a_attn_layer_proj(self.h, ptr(xb), ptr(q), ptr(k), ptr(v), ptr(x),
                                           ptr(wq), ptr(wk), ptr(wv), int(x.numel()), ptr(qw),
                                           ptr(kw), layer, pos))

    def qkv_proj(self, q, k, v, x, wq, wk, wv, qw, kw, layer, pos):
        """The projection half of attn_layer_proj (no attention)."""
        check(self.lib.q3a_qkv_proj(self.h, ptr(q), ptr(k), ptr(v), ptr(x), ptr(wq), ptr(wk),
                                    ptr(wv), int(x.numel()), ptr(qw), ptr(kw), layer, pos))

    def wo_residual(self, x, xb, wo):
        """x += wo . xb (the held heads' columns; summed over the peer set)."""
        check(self.lib.q3a_wo_residual(self.h, ptr(x), ptr(xb), ptr(wo), int(x.numel())))

    def attn_sublayer(self, x, att_norm_w, wq, wk, wv, qw, kw, wo, layer, pos):
        """x += attention sublayer of one token at pos (device tensors)."""
        check(self.lib.q3a_attn_sublayer(self.h, ptr(x), ptr(att_norm_w), ptr(wq), ptr(wk),
                                         ptr(wv), ptr(qw), ptr(kw), ptr(wo), int(x.numel()),
                                         layer, pos))

    def attn_layer_batched(self, xb, q, k, v, qw, kw, layer, seq_ids, pos):
        import numpy as np
        sid = np.ascontiguousarray(seq_ids, np.int32)
        ps = np.ascontiguousarray(pos, np.int32)
        check(self.lib.q3a_attn_layer_batched(self.h, ptr(xb), ptr(q), ptr(k), ptr(v), ptr(qw),
                                              ptr(kw), layer, ptr(sid), ptr(ps), len(sid)))

    def attn_decode(self, xb, q, kc, vc, att, loff, pos, n_heads, kv_mul, hd, kv_dim, max_seq):
        check(self.lib.q3a_attn_decode(self.h, ptr(xb), ptr(q), ptr(kc), ptr(vc), ptr(att), loff,
                                       pos, n_heads, kv_mul, hd, kv_dim, max_seq))

    def kv_append(self, seq, layer, pos0, n, k, v, kw):
        check(self.lib.q3a_kv_append(self.h, seq, layer, pos0, n, ptr(k), ptr(v), ptr(kw)))

    def kv_load(self, seq, layer, pos0, n, k, v):
        check(self.lib.q3a_kv_load(self.h, seq, layer, pos0, n, ptr(k), ptr(v)))

    def kv_read(self, seq, layer, pos0, n, k, v):
        check(self.lib.q3a_kv_read(self.h, seq, layer, pos0, n, ptr(k), ptr(v)))

    def prefill(self, out, out_dtype, q, k, v, qw, kw, seq, layer, pos0, n_tok):
        check(self.lib.q3a_prefill(self.h, ptr(out), out_dtype, ptr(q), ptr(k), ptr(v), ptr(qw),
                                   ptr(kw), seq, layer, pos0, n_tok))

    def prefill_attn(self, out, out_dtype, q_bf16, seq, layer, pos0, n_tok):
        check(self.lib.q3a_prefill_attn(self.h, ptr(out), out_dtype, ptr(q_bf16), seq, layer, pos0,
                                        n_tok))

    def attn_partial(self, o, lse, q, seq, layer, t0, t1):
        check(self.lib.q3a_attn_partial(self.h, ptr(o), ptr(lse), ptr(q), seq, layer, t0, t1))

    def lse_combine(self, xb, o_parts, lse_parts, n_parts):
        check(self.lib.q3a_lse_combine(self.h, ptr(xb), ptr(o_parts), ptr(lse_parts), n_parts))

    def lse_combine_packed(self, xb, parts, n_parts):
        check(self.lib.q3a_lse_combine_packed(self.h, ptr(xb), ptr(parts), n_parts))

    def peer_export(self, world) -> bytes:
        """This rank's receive-buffer handle (IPC_HANDLE_BYTES bytes)."""
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(self.lib.q3a_peer_export(self.h, world, buf))
        return buf.raw

    def peer_open(self, rank, world, handles):
        """handles: every rank's peer_export() bytes, in rank order."""
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        check(self.lib.q3a_peer_open(self.h, rank, world, buf))

    def peer_buffer(self) -> int:
        """This context's receive buffer (device address), after peer_export."""
        p = _P()
        check(self.lib.q3a_peer_buffer(self.h, ctypes.byref(p)))
        return p.value

    def peer_open_ptrs(self, rank, world, bufs):
        """Single-process set-up: every rank's peer_buffer() in rank order."""
        arr = (_P * world)(*bufs)
        check(self.lib.q3a_peer_open_ptrs(self.h, rank, world, arr))

    def attn_seqshard(self, xb, q, seq, layer, n_local):
        check(self.lib.q3a_attn_seqshard(self.h, ptr(xb), ptr(q), seq, layer, n_local))

    def peer_register(self, buf, nbytes) -> bytes:
        """Registers a device buffer for column all-gathers; returns this
        rank's handle (PEER_REG_BYTES bytes)."""
        out = ctypes.create_string_buffer(PEER_REG_BYTES)
        check(self.lib.q3a_peer_register(self.h, ptr(buf), nbytes, out))
        return out.raw

    def peer_register_open(self, rank, world, handles):
        """handles: every rank's peer_register() bytes, in rank order."""
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        check(self.lib.q3a_peer_register_open(self.h, rank, world, buf))

    def peer_register_flags(self) -> int:
        """This context's gather flag block (device address), after peer_register."""
        p = _P()
        check(self.lib.q3a_peer_register_flags(self.h, ctypes.byref(p)))
        return p.value

    def peer_register_open_ptrs(self, rank, world, bufs, flags):
        """Single-process set-up: every rank's registered buffer and flag
        block, in rank order."""
        b = (_P * world)(*bufs)
        f = (_P * world)(*flags)
        check(self.lib.q3a_peer_register_open_ptrs(self.h, rank, world, b, f))

    def set_deterministic(self, on: bool):
        check(self.lib.q3a_set_deterministic(self.h, 1 if on else 0))

    def set_wait_limit(self, seconds: float):
        check(self.lib.q3a_set_wait_limit(self.h, seconds))

    def gather_cols(self, off, rows, row_bytes, col0, col_bytes):
        check(self.lib.q3a_gather_cols(self.h, off, rows, row_bytes, col0, col_bytes))

    def graph_begin(self):
        check(self.lib.q3a_graph_begin(self.h))

    def graph_end(self):
        """The recorded calls as a graph handle (q3a_graph_destroy frees it)."""
        g = _P()
        check(self.lib.q3a_graph_end(self.h, ctypes.byref(g)))
        return g

    def graph_launch(self, g):
        check(self.lib.q3a_graph_launch(self.h, g))

    def graph_destroy(self, g):
        check(self.lib.q3a_graph_destroy(g))

    def kv_wire_bytes(self, n_layers, n_tok) -> int:
        return int(self.lib.q3a_kv_wire_bytes(self.h, n_layers, n_tok))

    def kv_pack(self, seq, layer0, n_layers, pos0, n_tok, dst):
        """Packs the held heads' rows into dst (a byte buffer: numpy uint8
        in host mode, a torch uint8 device tensor in device mode)."""
        check(self.lib.q3a_kv_pack(self.h, seq, layer0, n_layers, pos0, n_tok, ptr(dst),
                                   _nbytes(dst)))

    def kv_unpack(self, seq, src):
        check(self.lib.q3a_kv_unpack(self.h, seq, ptr(src), _nbytes(src)))

    def kv_synth(self, seq, layer, pos0, n, seed, stream_k, stream_v):
        check(self.lib.q3a_kv_synth(self.h, seq, layer, pos0, n, seed, stream_k, stream_v))

    def randn(self, dst, out_dtype, n, seed, stream_id, offset=0):
        check(self.lib.q3a_randn(self.h, ptr(dst), out_dtype, n, seed, stream_id, offset))
