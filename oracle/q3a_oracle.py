"""ctypes binding of the CPU oracle (oracle/liboracle.so) and, when it was
built, of the reference's own compiled functions (oracle/_ref/libq3ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
the CPU-baseline leg of bench.py, always as the checker, never as the product.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libq3ref.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_U64 = ctypes.c_uint64

_lib = None
_ref = None


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_P)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"oracle library missing: {LIB_PATH} (run make -C oracle)")
        L = ctypes.CDLL(LIB_PATH)
        L.orc_rmsnorm_head.argtypes = [_P, _P, _I, _I, _F]
        L.orc_rope.argtypes = [_P, _I, _I, _I, _F]
        L.orc_prep_rows.argtypes = [_P, _P, _I, _I, _I, _I, _F, _F]
        L.orc_softmax.argtypes = [_P, _I]
        L.orc_attn_decode.argtypes = [_P, _P, _P, _P, _P, _SZ, _I, _I, _I, _I, _I, _I]
        L.orc_attn_block.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I,
                                     _I, _I, _I, _I, _F, _F]
        L.orc_prefill_causal.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I]
        L.orc_bf16_round.argtypes = [_P, _SZ]
        L.orc_stream_key.argtypes = [_U64, _U64]
        L.orc_stream_key.restype = _U64
        L.orc_u01.argtypes = [_U64, _U64]
        L.orc_u01.restype = _F
        L.orc_randn.argtypes = [_P, _SZ, _U64, _U64]
        L.orc_lse_merge.argtypes = [_P, _P, _P, _P, _I, _I, _I]
        L.orc_attn_partial.argtypes = [_P, _P, _P, _P, _P, _SZ, _I, _I, _I, _I, _I, _I]
        L.orc_mm_f16.argtypes = [_P, _P, _P, _I, _I]
        L.orc_rmsnorm.argtypes = [_P, _P, _P, _I, _F]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own functions compiled from its sources."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"reference library not built: {REF_PATH}")
        R = ctypes.CDLL(REF_PATH)
        R.q3ref_rmsnorm_head.argtypes = [_P, _P, _I, _I, _F]
        R.q3ref_rope.argtypes = [_P, _I, _I, _I, _F]
        R.q3ref_softmax.argtypes = [_P, _I]
        R.q3ref_launch_attn.argtypes = [_P, _P, _P, _P, _P, _SZ, _I, _I, _I, _I, _I, _I]
        R.q3ref_launch_rmsnorm_head.argtypes = [_P, _P, _I, _I, _F]
        R.q3ref_launch_rope.argtypes = [_P, _I, _I, _I, _F]
        R.q3ref_launch_kv_write.argtypes = [_P, _P, _P, _P, _I]
        R.q3ref_attn_mc.argtypes = [_P, _P, _P, _P, _P, _SZ, _I, _I, _I, _I, _I, _I]
        R.q3ref_mm_f16.argtypes = [_P, _P, _P, _I, _I]
        R.q3ref_rmsnorm.argtypes = [_P, _P, _P, _I, _F]
        _ref = R
    return _ref


# ---------------------------------------------------------------- generator
def stream_key(seed: int, stream: int) -> int:
    return int(lib().orc_stream_key(seed, stream))


def randn(n: int, seed: int, stream: int, offset: int = 0) -> np.ndarray:
    a = np.empty(n, np.float32)
    lib().orc_randn(_ptr(a), n, stream_key(seed, stream), offset)
    return a


def bf16_round(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32).copy()
    lib().orc_bf16_round(_ptr(a), a.size)
    return a


# ---------------------------------------------------------------- math
def rmsnorm_head(vec: np.ndarray, w: np.ndarray, n_heads: int, hd: int, eps: float):
    lib().orc_rmsnorm_head(_ptr(vec), _ptr(w), n_heads, hd, eps)


def rope(vec: np.ndarray, n_heads: int, hd: int, pos: int, theta: float):
    lib().orc_rope(_ptr(vec), n_heads, hd, pos, theta)


def attn_decode(q, kc, vc, loff, pos, n_heads, kv_mul, hd, kv_dim, max_seq):
    xb = np.zeros(n_heads * hd, np.float32)
    att = np.zeros(n_heads * max_seq, np.float32)
    lib().orc_attn_decode(_ptr(xb), _ptr(q), _ptr(kc), _ptr(vc), _ptr(att), loff, pos,
                          n_heads, kv_mul, hd, kv_dim, max_seq)
    return xb


def attn_block(q, k, v, qw, kw, kc, vc, layer, pos, n_heads, n_kv, hd, max_seq,
               eps=1e-6, theta=5e6):
    """Runs the whole reference block in place on q, k, kc, vc; returns xb."""
    xb = np.zeros(n_heads * hd, np.float32)
    att = np.zeros(n_heads * max_seq, np.float32)
    lib().orc_attn_block(_ptr(xb), _ptr(q), _ptr(k), _ptr(v), _ptr(qw), _ptr(kw),
                         _ptr(kc), _ptr(vc), _ptr(att), layer, pos, n_heads, n_kv, hd,
                         max_seq, eps, theta)
    return xb


def prefill_causal(q, kc, vc, pos0, S, n_heads, kv_mul, hd, kv_dim, max_seq):
    out = np.zeros(S * n_heads * hd, np.float32)
    lib().orc_prefill_causal(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc), pos0, S, n_heads,
                             kv_mul, hd, kv_dim, max_seq)
    return out


def attn_partial(q, kc, vc, loff, t0, t1, n_heads, kv_mul, hd, kv_dim):
    o = np.zeros(n_heads * hd, np.float32)
    lse = np.zeros(n_heads, np.float32)
    lib().orc_attn_partial(_ptr(o), _ptr(lse), _ptr(q), _ptr(kc), _ptr(vc), loff, t0, t1,
                           n_heads, kv_mul, hd, kv_dim)
    return o, lse


def mm_f16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """o = w @ x with fp16 weights w [d][n] (uint16 bits or float16), one
    sequential fp32 sum per row (mm_f16)."""
    w16 = np.ascontiguousarray(w).view(np.uint16)
    d, n = w16.shape
    x = np.ascontiguousarray(x, np.float32)
    o = np.zeros(d, np.float32)
    lib().orc_mm_f16(_ptr(o), _ptr(x), _ptr(w16), n, d)
    return o


def proj_weights(seed: int, d: int, n: int, scale: float = 0.02) -> np.ndarray:
    """Seeded fp16 weights [d][n]: orc_randn (stream 200) * scale, rounded to
    fp16 by numpy (round to nearest even)."""
    return (randn(d * n, seed, 200) * np.float32(scale)).astype(np.float16).reshape(d, n)


def all_f16_patterns() -> np.ndarray:
    """Every fp16 bit pattern once, [64][1024] (zeros, subnormals, normals,
    +-inf, NaNs)."""
    return np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).reshape(64, 1024)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """The layer input's RMSNorm (rmsnorm), a new array."""
    x = np.ascontiguousarray(x, np.float32)
    o = np.zeros_like(x)
    lib().orc_rmsnorm(_ptr(o), _ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), x.size, eps)
    return o


def lse_merge(o_parts: np.ndarray, lse_parts: np.ndarray, n_heads: int, hd: int):
    n_parts = lse_parts.shape[0]
    out = np.zeros(n_heads * hd, np.float32)
    lse = np.zeros(n_heads, np.float32)
    o_parts = np.ascontiguousarray(o_parts, np.float32)
    lse_parts = np.ascontiguousarray(lse_parts, np.float32)
    lib().orc_lse_merge(_ptr(out), _ptr(lse), _ptr(o_parts), _ptr(lse_parts), n_parts,
                        n_heads, hd)
    return out, lse


# ---------------------------------------------------------------- synthetic cache
def make_cache(seed: int, layer: int, n_tok: int, n_kv: int, hd: int, max_seq: int,
               eps: float = 1e-6, theta: float = 5e6, kw: np.ndarray | None = None,
               bf16: bool = False):
    """Position-major K/V cache [max_seq][n_kv*hd] for one layer, rows 0..n_tok-1
    filled: k_t ~ N(0,1) -> QK-RMSNorm (gains kw, unit by default) -> RoPE at t;
    v_t ~ N(0,1).  Streams: layer*16+1 (K), layer*16+2 (V)."""
    kv_dim = n_kv * hd
    kc = np.zeros(max_seq * kv_dim, np.float32)
    vc = np.zeros(max_seq * kv_dim, np.float32)
    if kw is None:
        kw = np.ones(hd, np.float32)
    kraw = randn(n_tok * kv_dim, seed, layer * 16 + 1)
    vraw = randn(n_tok * kv_dim, seed, layer * 16 + 2)
    kc[: n_tok * kv_dim] = kraw
    if n_tok > 0:
        # rmsnorm_head then rope at t, row by row (the same per-head arithmetic)
        lib().orc_prep_rows(_ptr(kc), _ptr(np.ascontiguousarray(kw, np.float32)), n_tok, n_kv,
                            hd, 0, eps, theta)
    vc[: n_tok * kv_dim] = vraw
    if bf16:
        kc = bf16_round(kc)
        vc = bf16_round(vc)
    return kc, vc, kraw, vraw
