"""numpy front end of the C++ CPU oracle — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module,
as the checker.  The product (grout_b200) never imports it.  Arrays of f16
are passed as numpy float16 (bit-identical to the C side's uint16).

Parity status: unpinned against the reference's own outputs (the Rust/cuTile
reference cannot run here and stores no expected outputs); see oracle.cpp.
"""
import ctypes
import os

import numpy as np

from .build import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build()
        _lib = ctypes.CDLL(path)
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a


i32, i64, f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(i32(n))


def pattern(length: int, salt: int) -> np.ndarray:
    """attention_microbench.rs:203-214 pattern, as float16."""
    out = np.empty(length, dtype=np.float16)
    lib().oracle_pattern(i64(length), i64(salt), _p(out))
    return out


def inv_freq(theta: float, head_dim: int) -> np.ndarray:
    out = np.empty(head_dim // 2, dtype=np.float32)
    lib().oracle_inv_freq(f32(theta), i32(head_dim), _p(out))
    return out


def rope_table(inv: np.ndarray, max_seq: int) -> np.ndarray:
    inv = _c(inv, np.float32)
    half = inv.shape[0]
    out = np.empty((max_seq, 2, half), dtype=np.float32)
    lib().oracle_rope_table(_p(inv), i32(half), i32(max_seq), _p(out))
    return out


def qk_norm_rope_kv_prefill(q, k, v, q_w, k_w, table, k_cache, v_cache, pos0, eps):
    """q [S,Hq,128], k/v [S,Hkv,128] float16; caches [Hkv,max_seq,128] updated
    in place; returns q_out [S,Hq,128]."""
    q, k, v = (_c(x, np.float16) for x in (q, k, v))
    S, hq, D = q.shape
    hkv = k.shape[1]
    assert D == 128
    q_out = np.zeros_like(q)
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    lib().oracle_qk_norm_rope_kv_prefill(
        _p(q), _p(k), _p(v), i64(hq * D), i64(hkv * D), _p(_c(q_w, np.float16)),
        _p(_c(k_w, np.float16)), _p(_c(table, np.float32)), _p(q_out), _p(k_cache),
        _p(v_cache), i64(k_cache.shape[1] * D), i32(pos0), i32(S), i32(hq), i32(hkv), f32(eps))
    return q_out


def qk_norm_rope_kv_decode(qkv, q_w, k_w, table, k_cache, v_cache, position, hq, hkv, eps):
    """qkv [B,(Hq+2Hkv)*128]; caches [B,Hkv,max_seq,128] updated in place;
    returns q_out [B,Hq,128]."""
    qkv = _c(qkv, np.float16)
    B = qkv.shape[0]
    position = _c(position, np.uint32)
    q_out = np.zeros((B, hq, 128), dtype=np.float16)
    lib().oracle_qk_norm_rope_kv_decode(
        _p(qkv), _p(_c(q_w, np.float16)), _p(_c(k_w, np.float16)), _p(_c(table, np.float32)),
        _p(q_out), _p(k_cache), _p(v_cache), i64(k_cache[0].size), i64(k_cache.shape[2] * 128),
        _p(position), i32(B), i32(hq), i32(hkv), f32(eps))
    return q_out


def attn_prefill_naive(q, k, v):
    """Reference cpu_reference (attention_microbench.rs:665-702): q [S,Hq,D],
    k/v [Hkv,S,D] float32; returns f32 [S,Hq,D]."""
    q, k, v = (_c(x, np.float32) for x in (q, k, v))
    S, hq, D = q.shape
    out = np.empty_like(q)
    lib().oracle_attn_prefill_naive(_p(q), _p(k), _p(v), _p(out), i32(S), i32(hq),
                                   i32(k.shape[0]), i32(D))
    return out


def attn_prefill(q, k, v, cu_q, pos0, kv_start, hq, hkv, kv_batch_stride, kv_row_stride,
                 kv_head_stride, scale, ideal=False, rows_step=1, out=None):
    """General causal prefill oracle.  q [total_q, Hq, 128] float16 (packed by
    cu_q); k/v flat float16 buffers addressed by the given element strides."""
    q = _c(q, np.float16)
    cu_q = _c(cu_q, np.int32)
    B = cu_q.shape[0] - 1
    pos0 = _c(pos0 if pos0 is not None else np.zeros(B), np.int32)
    kv_start = _c(kv_start if kv_start is not None else np.zeros(B), np.int32)
    if out is None:
        out = np.zeros_like(q)
    lib().oracle_attn_prefill(
        _p(q), _p(k), _p(v), _p(out), _p(cu_q), _p(pos0), _p(kv_start), i32(B), i32(hq),
        i32(hkv), i64(hq * 128), i64(kv_batch_stride), i64(kv_row_stride), i64(kv_head_stride),
        f32(scale), i32(1 if ideal else 0), i32(rows_step))
    return out


def attn_decode(q, k, v, position, hkv, kv_batch_stride, kv_head_stride, qk_scale,
                nks=1, bn=32, ideal=False):
    """Split-K decode oracle.  q [B,Hq,128]; k/v flat float16 buffers."""
    q = _c(q, np.float16)
    B, hq, _ = q.shape
    position = _c(position, np.uint32)
    out = np.zeros_like(q)
    lib().oracle_attn_decode(_p(q), _p(k), _p(v), _p(out), _p(position), i32(B), i32(hq),
                             i32(hkv), i64(kv_batch_stride), i64(kv_head_stride), f32(qk_scale),
                             i32(nks), i32(bn), i32(1 if ideal else 0))
    return out
