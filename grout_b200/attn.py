"""Host-side mirror of the reference's attention ops over the C ABI.

The reference (rtburger/grout, Rust) launches its attention kernels from
three op wrappers; each function here has the same inputs, argument meaning
and error behaviour, and calls libgrout_attn.so (include/grout_attn.h):

    qk_norm_rope_kv_prefill  <- execute_qk_norm_rope_kv_prefill_op_ctx
                                (src/model.rs:4753-4888)
    qk_norm_rope_kv_decode   <- decode-graph record of qk_norm_rope_kv_decode_raw_f16
                                (src/model.rs:2919-2943)
    attention_prefill        <- attend_seq_arc_into_ctx_with_position, Host arm
                                (src/model.rs:6856-7134)
    attention_decode         <- fmha_decode_gqa_split + splitk_reduce_merge records
                                (src/model.rs:3180-3225)

Tensors are torch CUDA tensors (torch is the device-memory and stream
plumbing only); every call is enqueued on torch's current stream.  Shape or
range problems raise GroutError before any launch, like the reference's
`ensure!`s.  There is no CPU fallback: if the library is missing or the
device is not sm_100 the call raises.
"""
import ctypes
import math
import os

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgrout_attn.so")

HEAD_DIM = 128
CLUSTER_MAX_SPLITS = 16
FLAG_DECODE_SCALE_F16 = 0x1

_STATUS = {0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "CUDA", 4: "DEVICE"}


class GroutError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"grout_attn {_STATUS.get(status, status)}: {message}")
        self.status = status


class AttnDims(ctypes.Structure):
    _fields_ = [
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("max_seq", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("qk_scale", ctypes.c_float),
        ("flags", ctypes.c_int32),
    ]


class PrefillVarlenArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("q_row_stride", ctypes.c_int64),
        ("q_rows", ctypes.c_int64),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("kv_batch_stride", ctypes.c_int64),
        ("kv_row_stride", ctypes.c_int64),
        ("kv_head_stride", ctypes.c_int64),
        ("kv_rows", ctypes.c_int64),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("position_start", ctypes.c_void_p),
        ("kv_start", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("max_q_len", ctypes.c_int32),
    ]


class PrefillPagedArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("q_row_stride", ctypes.c_int64),
        ("q_rows", ctypes.c_int64),
        ("k_pages", ctypes.c_void_p),
        ("v_pages", ctypes.c_void_p),
        ("num_pages", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("page_table", ctypes.c_void_p),
        ("table_stride", ctypes.c_int32),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("position_start", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("max_q_len", ctypes.c_int32),
    ]


# Every symbol include/grout_attn.h declares, with its ctypes signature.
_vp, _i32, _i64, _f32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
_DIMS = ctypes.POINTER(AttnDims)
SIGNATURES = {
    "grout_attn_last_error": (ctypes.c_char_p, []),
    "grout_attn_version": (ctypes.c_char_p, []),
    "grout_attn_init": (ctypes.c_int, [_i32]),
    "grout_attn_check_device_error": (ctypes.c_int, [ctypes.POINTER(_i32)]),
    "grout_inv_freq_host": (None, [_f32, _i32, _vp]),
    "grout_rope_table_bytes": (_sz, [_i32, _i32]),
    "grout_rope_table_init": (ctypes.c_int, [_vp, _vp, _i32, _i32, _vp]),
    "grout_qk_norm_rope_kv_prefill": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp,
                                                     _vp, _vp, _i64, _i32, _i32, _DIMS, _vp]),
    "grout_qk_norm_rope_kv_decode": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                                    _vp, _i32, _DIMS, _vp]),
    "grout_attn_prefill": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _DIMS, _vp]),
    "grout_attn_prefill_varlen": (ctypes.c_int, [ctypes.POINTER(PrefillVarlenArgs), _DIMS, _vp]),
    "grout_attn_decode_splits": (_i32, [_i32, _i32, _DIMS]),
    "grout_attn_decode_workspace_bytes": (_sz, [_i32, _i32, _DIMS]),
    "grout_attn_decode": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _i32, _DIMS,
                                         _vp, _sz, _vp]),
    "grout_attn_decode_ex": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _i32, _i32,
                                            _DIMS, _vp, _sz, _vp]),
    "grout_attn_decode_fused": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp,
                                               _vp, _i32, _i32, _DIMS, _vp, _sz, _vp]),
    "grout_add_rms_norm": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "grout_silu_mul": (ctypes.c_int, [_vp, _vp, _i32, _i32, _vp]),
    "grout_tp_comm_create": (ctypes.c_int, [_i32, _i32, ctypes.POINTER(_vp), _vp]),
    "grout_tp_comm_connect": (ctypes.c_int, [_vp, _i32, _vp]),
    "grout_tp_comm_destroy": (None, [_vp]),
    "grout_gemv_allreduce": (ctypes.c_int, [_vp, _vp, _i32, _vp, _vp, _vp, _vp]),
    "grout_allreduce_residual": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "grout_attn_decode_noalloc_max_bytes": (_sz, []),
    "grout_attn_decode_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _i32,
                                                 _DIMS, _vp]),
    "grout_qkv_proj_norm_rope_kv_prefill": (ctypes.c_int, [_vp, _i64, _vp, _i32, _vp, _vp, _vp, _vp,
                                                           _vp, _vp, _i64, _vp, _i32, _i32, _DIMS,
                                                           _vp]),
    "grout_attn_prefill_splits": (_i32, [_i32, _i32, _DIMS]),
    "grout_attn_prefill_splitk_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "grout_attn_prefill_splitk": (ctypes.c_int, [ctypes.POINTER(PrefillVarlenArgs), _i32, _DIMS, _vp,
                                                 _sz, _vp]),
    "grout_attn_prefill_paged": (ctypes.c_int, [ctypes.POINTER(PrefillPagedArgs), _DIMS, _vp]),
    "grout_attn_decode_paged": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _vp, _i32, _vp, _vp, _i32,
                                               _i32, _i32, _DIMS, _vp, _sz, _vp]),
    "grout_qk_norm_rope_kv_decode_paged": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32,
                                                          _i32, _vp, _i32, _vp, _i32, _DIMS, _vp]),
    "grout_qk_norm_rope_kv_prefill_paged": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp,
                                                           _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i32,
                                                           _DIMS, _vp]),
}

_lib = None


def lib():
    """The loaded C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise GroutError(3, f"{LIB_PATH} not found: run `python -m grout_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status):
    if status != 0:
        msg = lib().grout_attn_last_error().decode(errors="replace")
        raise GroutError(status, msg)


def _stream(t=None):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device if t is not None else None).cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def make_dims(num_q_heads, num_kv_heads, max_seq, rms_eps=1e-6, qk_scale=None, flags=0,
              head_dim=HEAD_DIM):
    return AttnDims(num_q_heads, num_kv_heads, head_dim, max_seq, rms_eps,
                    float(qk_scale) if qk_scale else 0.0, flags)


def _need(cond, msg):
    if not cond:
        raise GroutError(1, msg)


def _f16_cuda(t, name):
    _need(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")
    _need(t.dtype == torch.float16, f"{name} must be float16, got {t.dtype}")
    _need(t.is_contiguous(), f"{name} must be contiguous")


def init(device=None):
    """Per-device setup; call before capturing any of these ops in a graph."""
    if device is None:
        device = torch.cuda.current_device()
    _check(lib().grout_attn_init(int(device)))


def check_device_error():
    """Raises GroutError if a kernel recorded a device-side error (and clears it)."""
    code = ctypes.c_int32(0)
    st = lib().grout_attn_check_device_error(ctypes.byref(code))
    if st != 0:
        raise GroutError(st, lib().grout_attn_last_error().decode() + f" (code 0x{code.value:x})")


def inv_freq(theta, head_dim=HEAD_DIM):
    """build_inv_freq (src/model.rs:7295-7306), on the host."""
    out = np.empty(head_dim // 2, dtype=np.float32)
    lib().grout_inv_freq_host(ctypes.c_float(theta), head_dim, out.ctypes.data_as(ctypes.c_void_p))
    return out


def rope_table(theta_or_inv_freq, max_seq, device=None, head_dim=HEAD_DIM):
    """Device RoPE table [max_seq, head_dim] f32 (cos half, sin half per row)."""
    if np.isscalar(theta_or_inv_freq):
        inv = inv_freq(float(theta_or_inv_freq), head_dim)
    else:
        inv = np.ascontiguousarray(theta_or_inv_freq, dtype=np.float32)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    table = torch.empty((max_seq, head_dim), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _check(lib().grout_rope_table_init(_ptr(table), inv.ctypes.data_as(ctypes.c_void_p),
                                           head_dim, max_seq, _stream(table)))
    return table


def qk_norm_rope_kv_prefill(q, k, v, q_norm_w, k_norm_w, rope_table, q_out, k_cache, v_cache,
                            position_start, eps):
    """Fused Q/K RMSNorm + RoPE + KV-cache write for a prefill chunk.

    q, q_out [S, Hq, 128]; k, v [S, Hkv, 128]; caches [Hkv, max_seq, 128]
    (a [B, Hkv, max_seq, 128] cache must be sliced to one sequence)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"),
                 (q_out, "q_out"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _f16_cuda(t, n)
    _need(q.dim() == 3 and q.shape[2] == HEAD_DIM, f"q shape mismatch in fused qk/rope/kv prefill: {tuple(q.shape)}")
    S, hq, _ = q.shape
    _need(k.dim() == 3 and k.shape[0] == S and k.shape[2] == HEAD_DIM, f"k shape mismatch in fused qk/rope/kv prefill: {tuple(k.shape)}")
    _need(v.shape == k.shape, f"v shape mismatch in fused qk/rope/kv prefill: {tuple(v.shape)}")
    _need(q_out.shape == q.shape, f"fused qk/rope/kv output shape mismatch: {tuple(q_out.shape)}")
    hkv = k.shape[1]
    _need(k_cache.dim() == 3 and k_cache.shape[0] == hkv and k_cache.shape[2] == HEAD_DIM,
          f"k_cache shape mismatch in fused qk/rope/kv: {tuple(k_cache.shape)}")
    _need(v_cache.shape == k_cache.shape, f"v_cache shape mismatch in fused qk/rope/kv: {tuple(v_cache.shape)}")
    _need(rope_table.dtype == torch.float32 and rope_table.shape[1] == HEAD_DIM, "rope_table must be [max_seq, 128] f32")
    max_seq = k_cache.shape[1]
    _need(rope_table.shape[0] >= max_seq, "rope_table shorter than max_seq")
    dims = make_dims(hq, hkv, max_seq, eps)
    _check(lib().grout_qk_norm_rope_kv_prefill(
        _ptr(q), _ptr(k), _ptr(v), hq * HEAD_DIM, hkv * HEAD_DIM, _ptr(q_norm_w), _ptr(k_norm_w),
        _ptr(rope_table), _ptr(q_out), _ptr(k_cache), _ptr(v_cache), max_seq * HEAD_DIM,
        int(position_start), S, ctypes.byref(dims), _stream(q)))
    return q_out


def qk_norm_rope_kv_decode(qkv, q_norm_w, k_norm_w, rope_table, q_out, k_cache, v_cache, position,
                           num_q_heads, num_kv_heads, eps):
    """Fused decode step: qkv [B, (Hq+2Hkv)*128], position [B] uint32/int32 on
    the device, q_out [B, Hq, 128], caches [B, Hkv, max_seq, 128] (or
    [Hkv, max_seq, 128] for B = 1)."""
    for t, n in ((qkv, "qkv"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"), (q_out, "q_out"),
                 (k_cache, "k_cache"), (v_cache, "v_cache")):
        _f16_cuda(t, n)
    hq, hkv = num_q_heads, num_kv_heads
    B = qkv.shape[0] if qkv.dim() == 2 else 1
    _need(qkv.numel() == B * (hq + 2 * hkv) * HEAD_DIM, f"qkv shape mismatch: {tuple(qkv.shape)}")
    _need(q_out.numel() == B * hq * HEAD_DIM, f"q_out shape mismatch: {tuple(q_out.shape)}")
    _need(position.is_cuda and position.dtype in (torch.int32, torch.uint32) and position.numel() >= B,
          "position must be a device int32/uint32 tensor with one entry per sequence")
    kc = k_cache if k_cache.dim() == 4 else k_cache.unsqueeze(0)
    _need(kc.shape[1] == hkv and kc.shape[3] == HEAD_DIM and kc.shape[0] >= B, f"k_cache shape mismatch: {tuple(k_cache.shape)}")
    _need(v_cache.shape == k_cache.shape, "v_cache shape mismatch")
    max_seq = kc.shape[2]
    dims = make_dims(hq, hkv, max_seq, eps)
    _check(lib().grout_qk_norm_rope_kv_decode(
        _ptr(qkv), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope_table), _ptr(q_out), _ptr(k_cache),
        _ptr(v_cache), hkv * max_seq * HEAD_DIM, max_seq * HEAD_DIM, _ptr(position), B,
        ctypes.byref(dims), _stream(qkv)))
    return q_out


def attention_prefill(q, k_cache, v_cache, out, position_start=0, qk_scale=None):
    """Causal GQA prefill over the engine's cache: q, out [S, Hq, 128];
    caches [Hkv, max_seq, 128]; row m sees keys 0..position_start+m."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (out, "out")):
        _f16_cuda(t, n)
    _need(q.dim() == 3 and q.shape[2] == HEAD_DIM, f"q shape mismatch in attention: {tuple(q.shape)}")
    _need(out.shape == q.shape, f"attention output shape mismatch: {tuple(out.shape)}")
    _need(k_cache.dim() == 3 and k_cache.shape[2] == HEAD_DIM, f"k_cache shape mismatch: {tuple(k_cache.shape)}")
    _need(v_cache.shape == k_cache.shape, "v_cache shape mismatch")
    S, hq, _ = q.shape
    hkv, max_seq, _ = k_cache.shape
    dims = make_dims(hq, hkv, max_seq, qk_scale=qk_scale)
    _check(lib().grout_attn_prefill(_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out),
                                    max_seq * HEAD_DIM, int(position_start), S,
                                    ctypes.byref(dims), _stream(q)))
    return out


def attention_prefill_varlen(q, k, v, out, cu_seqlens_q, max_q_len, num_kv_heads,
                             kv_row_stride, kv_head_stride, kv_batch_stride=0, kv_rows=None,
                             position_start=None, kv_start=None, qk_scale=None,
                             kv_head_range=None):
    """Packed varlen causal prefill.  q, out [q_rows, Hq, 128]; k/v addressed
    by element strides (see grout_prefill_varlen_args); cu_seqlens_q,
    position_start, kv_start: device int32.

    kv_head_range=(lo, hi) computes only KV heads lo..hi-1 and their query
    heads (the shard one GPU owns when a layer is split by KV head); the
    tensors stay whole, the call addresses the shard in place."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (out, "out")):
        _f16_cuda(t, n)
    _need(cu_seqlens_q.is_cuda and cu_seqlens_q.dtype == torch.int32, "cu_seqlens_q must be device int32")
    _need(out.shape == q.shape, "out shape mismatch")
    B = cu_seqlens_q.numel() - 1
    hq = q.shape[1]
    _need(hq % num_kv_heads == 0, f"{hq} query heads do not group over {num_kv_heads} KV heads")
    G = hq // num_kv_heads
    if kv_rows is None:
        kv_rows = (k.numel() - (B - 1) * kv_batch_stride) // max(1, kv_row_stride) if kv_batch_stride else k.numel() // kv_row_stride
    lo, hi = kv_head_range if kv_head_range is not None else (0, num_kv_heads)
    _need(0 <= lo < hi <= num_kv_heads, f"kv_head_range {kv_head_range} outside 0..{num_kv_heads}")
    qoff = lo * G * HEAD_DIM * 2            # bytes
    kvoff = lo * kv_head_stride * 2
    args = PrefillVarlenArgs(
        q.data_ptr() + qoff, out.data_ptr() + qoff, hq * HEAD_DIM, q.shape[0],
        k.data_ptr() + kvoff, v.data_ptr() + kvoff,
        kv_batch_stride, kv_row_stride, kv_head_stride, int(kv_rows), cu_seqlens_q.data_ptr(),
        position_start.data_ptr() if position_start is not None else None,
        kv_start.data_ptr() if kv_start is not None else None, B, int(max_q_len))
    dims = make_dims((hi - lo) * G, hi - lo, 1 << 30, qk_scale=qk_scale)
    _check(lib().grout_attn_prefill_varlen(ctypes.byref(args), ctypes.byref(dims), _stream(q)))
    return out


def qkv_proj_norm_rope_kv_prefill(x, w_qkv, q_norm_w, k_norm_w, rope_table, q_out, k_cache,
                                  v_cache, position_start, eps, qkv_out=None):
    """QKV projection of a prefill chunk with the fused norm/RoPE/KV write
    as its epilogue: x [S, hidden]; w_qkv [(Hq+2Hkv)*128, hidden] (torch
    Linear layout); q_out [S, Hq, 128]; caches [Hkv, max_seq, 128];
    qkv_out (optional) [S, (Hq+2Hkv)*128] receives the f16 projection."""
    for t, n in ((x, "x"), (w_qkv, "w_qkv"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"),
                 (q_out, "q_out"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _f16_cuda(t, n)
    _need(x.dim() == 2 and x.stride(1) == 1, "x must be [S, hidden] with unit column stride")
    S, hidden = x.shape
    hkv, max_seq = k_cache.shape[0], k_cache.shape[1]
    hq = q_out.shape[1]
    _need(q_out.shape == (S, hq, HEAD_DIM), f"q_out shape mismatch: {tuple(q_out.shape)}")
    _need(w_qkv.shape == ((hq + 2 * hkv) * HEAD_DIM, hidden) and w_qkv.is_contiguous(),
          f"w_qkv must be [{(hq + 2 * hkv) * HEAD_DIM}, {hidden}] contiguous")
    _need(v_cache.shape == k_cache.shape, "v_cache shape mismatch")
    if qkv_out is not None:
        _f16_cuda(qkv_out, "qkv_out")
        _need(qkv_out.shape == (S, (hq + 2 * hkv) * HEAD_DIM) and qkv_out.is_contiguous(), "qkv_out shape mismatch")
    dims = make_dims(hq, hkv, max_seq, eps)
    _check(lib().grout_qkv_proj_norm_rope_kv_prefill(
        _ptr(x), x.stride(0), _ptr(w_qkv), hidden, _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope_table),
        _ptr(q_out), _ptr(k_cache), _ptr(v_cache), max_seq * HEAD_DIM, _ptr(qkv_out),
        int(position_start), S, ctypes.byref(dims), _stream(x)))
    return q_out


def attention_prefill_splitk(q, k, v, out, cu_seqlens_q, max_q_len, num_kv_heads,
                             kv_row_stride, kv_head_stride, kv_batch_stride=0, kv_rows=None,
                             position_start=None, kv_start=None, num_splits=None, workspace=None,
                             qk_scale=None):
    """Split-K form of attention_prefill_varlen for launches with fewer work
    items than SMs (same arguments; cu_seqlens_q may be None for one
    sequence of q.shape[0] rows).  num_splits None = the library's choice."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (out, "out")):
        _f16_cuda(t, n)
    _need(out.shape == q.shape, "out shape mismatch")
    hq = q.shape[1]
    if cu_seqlens_q is not None:
        _need(cu_seqlens_q.is_cuda and cu_seqlens_q.dtype == torch.int32, "cu_seqlens_q must be device int32")
        B = cu_seqlens_q.numel() - 1
    else:
        B = 1
    if kv_rows is None:
        kv_rows = (k.numel() - (B - 1) * kv_batch_stride) // max(1, kv_row_stride) if kv_batch_stride else k.numel() // kv_row_stride
    dims = make_dims(hq, num_kv_heads, 1 << 30, qk_scale=qk_scale)
    if num_splits is None:
        num_splits = lib().grout_attn_prefill_splits(B, int(max_q_len), ctypes.byref(dims))
    need = lib().grout_attn_prefill_splitk_workspace_bytes(B, int(max_q_len), hq, int(num_splits))
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    args = PrefillVarlenArgs(
        q.data_ptr(), out.data_ptr(), hq * HEAD_DIM, q.shape[0], k.data_ptr(), v.data_ptr(),
        kv_batch_stride, kv_row_stride, kv_head_stride, int(kv_rows),
        cu_seqlens_q.data_ptr() if cu_seqlens_q is not None else None,
        position_start.data_ptr() if position_start is not None else None,
        kv_start.data_ptr() if kv_start is not None else None, B, int(max_q_len))
    _check(lib().grout_attn_prefill_splitk(ctypes.byref(args), int(num_splits), ctypes.byref(dims),
                                           _ptr(workspace), ws_bytes, _stream(q)))
    return out


def decode_splits(batch, max_kv_len, num_q_heads, num_kv_heads, max_seq):
    dims = make_dims(num_q_heads, num_kv_heads, max_seq)
    return lib().grout_attn_decode_splits(batch, max_kv_len, ctypes.byref(dims))


def decode_workspace_bytes(batch, max_kv_len, num_q_heads, num_kv_heads, max_seq, num_splits=None):
    if num_splits is None:
        dims = make_dims(num_q_heads, num_kv_heads, max_seq)
        return lib().grout_attn_decode_workspace_bytes(batch, max_kv_len, ctypes.byref(dims))
    # up to CLUSTER_MAX_SPLITS splits merge inside a thread-block cluster
    return 0 if num_splits <= CLUSTER_MAX_SPLITS else batch * num_q_heads * num_splits * 129 * 4


def attention_decode(q, k_cache, v_cache, position, out, max_kv_len, workspace=None,
                     num_splits=None, qk_scale=None, scale_f16=True):
    """Split-K GQA decode + merge.  q, out [B, Hq, 128]; caches
    [B, Hkv, max_seq, 128] (or [Hkv, max_seq, 128] for B = 1); position [B]
    device int32/uint32 (kv_len = position + 1).  scale_f16 reproduces the
    reference's f16 qk_scale (src/model.rs:3177).  A workspace of
    decode_workspace_bytes(...) bytes is allocated if none is given."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (out, "out")):
        _f16_cuda(t, n)
    B = q.shape[0] if q.dim() == 3 else 1
    hq = q.shape[-2]
    kc = k_cache if k_cache.dim() == 4 else k_cache.unsqueeze(0)
    _need(kc.shape[0] >= B and kc.shape[3] == HEAD_DIM, f"k_cache shape mismatch: {tuple(k_cache.shape)}")
    _need(v_cache.shape == k_cache.shape, "v_cache shape mismatch")
    _need(out.shape == q.shape, "out shape mismatch")
    _need(position.is_cuda and position.dtype in (torch.int32, torch.uint32) and position.numel() >= B,
          "position must be a device int32/uint32 tensor with one entry per sequence")
    hkv, max_seq = kc.shape[1], kc.shape[2]
    dims = make_dims(hq, hkv, max_seq, qk_scale=qk_scale,
                     flags=FLAG_DECODE_SCALE_F16 if scale_f16 else 0)
    if num_splits is None:
        num_splits = lib().grout_attn_decode_splits(B, int(max_kv_len), ctypes.byref(dims))
    need = decode_workspace_bytes(B, max_kv_len, hq, hkv, max_seq, num_splits)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _check(lib().grout_attn_decode_ex(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), hkv * max_seq * HEAD_DIM, max_seq * HEAD_DIM,
        _ptr(position), _ptr(out), B, int(max_kv_len), int(num_splits), ctypes.byref(dims),
        _ptr(workspace), ws_bytes, _stream(q)))
    return out


def attention_decode_fused(qkv, q_norm_w, k_norm_w, rope_table, k_cache, v_cache, position, out,
                           max_kv_len, eps, q_out=None, workspace=None, qk_scale=None,
                           scale_f16=True):
    """One decode step of a layer's attention in one kernel: the fused Q/K
    RMSNorm + RoPE + KV-cache write of qk_norm_rope_kv_decode followed by
    attention_decode (same bits as that pair).  qkv [B, (Hq + 2 Hkv) * 128];
    caches [B, Hkv, max_seq, 128] (or [Hkv, max_seq, 128] for B = 1); out
    [B, Hq, 128]; q_out (optional) receives the normalised, rotated query."""
    for t, n in ((qkv, "qkv"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"),
                 (k_cache, "k_cache"), (v_cache, "v_cache"), (out, "out")):
        _f16_cuda(t, n)
    B, hq = out.shape[0], out.shape[1]
    kc = k_cache if k_cache.dim() == 4 else k_cache.unsqueeze(0)
    _need(kc.shape[0] >= B and kc.shape[3] == HEAD_DIM, f"k_cache shape mismatch: {tuple(k_cache.shape)}")
    _need(v_cache.shape == k_cache.shape, "v_cache shape mismatch")
    hkv, max_seq = kc.shape[1], kc.shape[2]
    _need(qkv.numel() == B * (hq + 2 * hkv) * HEAD_DIM, f"qkv shape mismatch: {tuple(qkv.shape)}")
    if q_out is not None:
        _f16_cuda(q_out, "q_out")
        _need(q_out.numel() == B * hq * HEAD_DIM, "q_out shape mismatch")
    _need(position.is_cuda and position.dtype in (torch.int32, torch.uint32) and position.numel() >= B,
          "position must be a device int32/uint32 tensor with one entry per sequence")
    dims = make_dims(hq, hkv, max_seq, rms_eps=eps, qk_scale=qk_scale,
                     flags=FLAG_DECODE_SCALE_F16 if scale_f16 else 0)
    need = lib().grout_attn_decode_workspace_bytes(B, int(max_kv_len), ctypes.byref(dims))
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=qkv.device)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _check(lib().grout_attn_decode_fused(
        _ptr(qkv), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope_table), _ptr(q_out), _ptr(k_cache),
        _ptr(v_cache), hkv * max_seq * HEAD_DIM, max_seq * HEAD_DIM, _ptr(position), _ptr(out), B,
        int(max_kv_len), ctypes.byref(dims), _ptr(workspace), ws_bytes, _stream(qkv)))
    return out


def add_rms_norm(x, weight, out, eps, residual=None, residual_out=None):
    """out = rmsnorm(x + residual) * weight (f32 math, one f16 rounding);
    residual_out (optional) receives f16(x + residual).  x, residual, out,
    residual_out [rows, n]; weight [n]."""
    for t, n in ((x, "x"), (weight, "weight"), (out, "out")):
        _f16_cuda(t, n)
    n = weight.numel()
    rows = x.numel() // n
    _need(x.numel() == rows * n and out.numel() == x.numel(), "add_rms_norm shape mismatch")
    for t, nm in ((residual, "residual"), (residual_out, "residual_out")):
        if t is not None:
            _f16_cuda(t, nm)
            _need(t.numel() == x.numel(), f"{nm} shape mismatch")
    _check(lib().grout_add_rms_norm(_ptr(x), _ptr(residual), _ptr(weight), _ptr(out),
                                    _ptr(residual_out), rows, n, float(eps), _stream(x)))
    return out


def silu_mul(gate_up, out):
    """out [rows, n] = silu(gate) * up for gate_up [rows, 2n] = [gate | up]."""
    _f16_cuda(gate_up, "gate_up")
    _f16_cuda(out, "out")
    n = gate_up.shape[-1] // 2
    rows = gate_up.numel() // (2 * n)
    _need(out.numel() == rows * n, "silu_mul shape mismatch")
    _check(lib().grout_silu_mul(_ptr(gate_up), _ptr(out), rows, n, _stream(gate_up)))
    return out


def _pages(k_pages, v_pages, page_table):
    for t, n in ((k_pages, "k_pages"), (v_pages, "v_pages")):
        _f16_cuda(t, n)
    _need(k_pages.dim() == 4 and k_pages.shape[3] == HEAD_DIM,
          f"k_pages must be [num_pages, Hkv, page_size, 128]: {tuple(k_pages.shape)}")
    _need(v_pages.shape == k_pages.shape, "v_pages shape mismatch")
    _need(page_table.is_cuda and page_table.dtype == torch.int32 and page_table.is_contiguous(),
          "page_table must be a contiguous device int32 tensor")
    return k_pages.shape[0], k_pages.shape[1], k_pages.shape[2]


def attention_prefill_paged(q, k_pages, v_pages, page_table, out, cu_seqlens_q=None,
                            position_start=None, max_q_len=None, max_seq=None, qk_scale=None):
    """Causal prefill over a paged cache.  q, out packed [q_rows, Hq, 128];
    page pools [num_pages, Hkv, page_size, 128]; page_table [B, table_stride]
    device int32; cu_seqlens_q device int32 [B+1] (None: one sequence of all
    q rows); position_start device int32 [B] (None: all 0)."""
    for t, n in ((q, "q"), (out, "out")):
        _f16_cuda(t, n)
    num_pages, hkv, page_size = _pages(k_pages, v_pages, page_table)
    _need(out.shape == q.shape, "out shape mismatch")
    hq = q.shape[1]
    if cu_seqlens_q is not None:
        _need(cu_seqlens_q.is_cuda and cu_seqlens_q.dtype == torch.int32, "cu_seqlens_q must be device int32")
        B = cu_seqlens_q.numel() - 1
        _need(max_q_len is not None, "max_q_len is required with cu_seqlens_q")
    else:
        B = 1
        max_q_len = q.shape[0] if max_q_len is None else max_q_len
    if position_start is not None:
        _need(position_start.is_cuda and position_start.dtype == torch.int32, "position_start must be device int32")
    stride = page_table.shape[-1]
    if max_seq is None:
        max_seq = stride * page_size
    args = PrefillPagedArgs(
        q.data_ptr(), out.data_ptr(), hq * HEAD_DIM, q.shape[0], k_pages.data_ptr(), v_pages.data_ptr(),
        num_pages, page_size, page_table.data_ptr(), stride,
        cu_seqlens_q.data_ptr() if cu_seqlens_q is not None else None,
        position_start.data_ptr() if position_start is not None else None, B, int(max_q_len))
    dims = make_dims(hq, hkv, int(max_seq), qk_scale=qk_scale)
    _check(lib().grout_attn_prefill_paged(ctypes.byref(args), ctypes.byref(dims), _stream(q)))
    return out


def attention_decode_paged(q, k_pages, v_pages, page_table, position, out, max_kv_len,
                           max_seq=None, workspace=None, num_splits=None, qk_scale=None,
                           scale_f16=True):
    """Split-K GQA decode over a paged cache.  q, out [B, Hq, 128]; page pools
    [num_pages, Hkv, page_size, 128]; page_table [B, table_stride] int32
    (position p of sequence b is row p % page_size of page
    page_table[b, p // page_size]); position [B] device int32/uint32.
    max_seq defaults to table_stride * page_size."""
    for t, n in ((q, "q"), (out, "out")):
        _f16_cuda(t, n)
    num_pages, hkv, page_size = _pages(k_pages, v_pages, page_table)
    B, hq = q.shape[0], q.shape[1]
    _need(out.shape == q.shape, "out shape mismatch")
    _need(page_table.dim() == 2 and page_table.shape[0] >= B, "page_table must be [B, table_stride]")
    _need(position.is_cuda and position.dtype in (torch.int32, torch.uint32) and position.numel() >= B,
          "position must be a device int32/uint32 tensor with one entry per sequence")
    stride = page_table.shape[1]
    if max_seq is None:
        max_seq = stride * page_size
    dims = make_dims(hq, hkv, int(max_seq), qk_scale=qk_scale,
                     flags=FLAG_DECODE_SCALE_F16 if scale_f16 else 0)
    if num_splits is None:
        num_splits = lib().grout_attn_decode_splits(B, int(max_kv_len), ctypes.byref(dims))
    need = decode_workspace_bytes(B, max_kv_len, hq, hkv, int(max_seq), num_splits)
    if need and workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _check(lib().grout_attn_decode_paged(
        _ptr(q), _ptr(k_pages), _ptr(v_pages), num_pages, page_size, _ptr(page_table), stride,
        _ptr(position), _ptr(out), B, int(max_kv_len), int(num_splits), ctypes.byref(dims),
        _ptr(workspace), ws_bytes, _stream(q)))
    return out


def qk_norm_rope_kv_decode_paged(qkv, q_norm_w, k_norm_w, rope_table, q_out, k_pages, v_pages,
                                 page_table, position, num_q_heads, num_kv_heads, eps,
                                 max_seq=None):
    """Fused decode step writing K/V into a paged cache (see
    attention_decode_paged for the layout)."""
    for t, n in ((qkv, "qkv"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"), (q_out, "q_out")):
        _f16_cuda(t, n)
    num_pages, hkv, page_size = _pages(k_pages, v_pages, page_table)
    _need(hkv == num_kv_heads, "k_pages head count mismatch")
    hq = num_q_heads
    B = qkv.shape[0] if qkv.dim() == 2 else 1
    _need(qkv.numel() == B * (hq + 2 * hkv) * HEAD_DIM, f"qkv shape mismatch: {tuple(qkv.shape)}")
    _need(q_out.numel() == B * hq * HEAD_DIM, f"q_out shape mismatch: {tuple(q_out.shape)}")
    _need(position.is_cuda and position.dtype in (torch.int32, torch.uint32) and position.numel() >= B,
          "position must be a device int32/uint32 tensor with one entry per sequence")
    stride = page_table.shape[-1]
    if max_seq is None:
        max_seq = stride * page_size
    dims = make_dims(hq, hkv, int(max_seq), eps)
    _check(lib().grout_qk_norm_rope_kv_decode_paged(
        _ptr(qkv), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope_table), _ptr(q_out), _ptr(k_pages),
        _ptr(v_pages), num_pages, page_size, _ptr(page_table), stride, _ptr(position), B,
        ctypes.byref(dims), _stream(qkv)))
    return q_out


def qk_norm_rope_kv_prefill_paged(q, k, v, q_norm_w, k_norm_w, rope_table, q_out, k_pages, v_pages,
                                  page_table_row, position_start, eps, max_seq=None):
    """Fused prefill write of one sequence into a paged cache; page_table_row
    is that sequence's row of the page table (device int32)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"),
                 (q_out, "q_out")):
        _f16_cuda(t, n)
    num_pages, hkv, page_size = _pages(k_pages, v_pages, page_table_row)
    _need(q.dim() == 3 and q.shape[2] == HEAD_DIM, f"q shape mismatch: {tuple(q.shape)}")
    S, hq, _ = q.shape
    _need(k.shape == (S, hkv, HEAD_DIM) and v.shape == k.shape, "k/v shape mismatch")
    _need(q_out.shape == q.shape, "q_out shape mismatch")
    if max_seq is None:
        max_seq = page_table_row.numel() * page_size
    _need(page_table_row.numel() * page_size >= max_seq, "page_table_row shorter than max_seq")
    dims = make_dims(hq, hkv, int(max_seq), eps)
    _check(lib().grout_qk_norm_rope_kv_prefill_paged(
        _ptr(q), _ptr(k), _ptr(v), hq * HEAD_DIM, hkv * HEAD_DIM, _ptr(q_norm_w), _ptr(k_norm_w),
        _ptr(rope_table), _ptr(q_out), _ptr(k_pages), _ptr(v_pages), num_pages, page_size,
        _ptr(page_table_row), int(position_start), S, ctypes.byref(dims), _stream(q)))
    return q_out


def attention_decode_noalloc(q, k_cache, v_cache, position, out, max_kv_len, qk_scale=None,
                             scale_f16=True):
    """attention_decode without a workspace, for callers that cannot allocate
    device memory (a fixed memory plan, an FFI host with no allocator, code
    inside a stream capture).  The split-K scratch is the library's own
    fixed device array (grout_attn_decode_noalloc_max_bytes(), 512 KiB); larger
    shapes raise GroutError.  Calls that can overlap on the GPU share that
    array and race; make the first call on a device before any capture."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (out, "out")):
        _f16_cuda(t, n)
    B = q.shape[0] if q.dim() == 3 else 1
    hq = q.shape[-2]
    kc = k_cache if k_cache.dim() == 4 else k_cache.unsqueeze(0)
    _need(v_cache.shape == k_cache.shape and out.shape == q.shape, "shape mismatch")
    _need(position.is_cuda and position.dtype in (torch.int32, torch.uint32) and position.numel() >= B,
          "position must be a device int32/uint32 tensor with one entry per sequence")
    hkv, max_seq = kc.shape[1], kc.shape[2]
    dims = make_dims(hq, hkv, max_seq, qk_scale=qk_scale,
                     flags=FLAG_DECODE_SCALE_F16 if scale_f16 else 0)
    _check(lib().grout_attn_decode_noalloc(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), hkv * max_seq * HEAD_DIM, max_seq * HEAD_DIM,
        _ptr(position), _ptr(out), B, int(max_kv_len), ctypes.byref(dims), _stream(q)))
    return out


def default_scale(head_dim=HEAD_DIM):
    return 1.0 / math.sqrt(head_dim)
