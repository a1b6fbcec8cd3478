"""The allocation-free decode entry point (grout_attn_decode_noalloc), called
through the C ABI, against the regular grout_attn_decode with a caller
workspace.

It exists for callers that cannot allocate device memory (a fixed memory
plan, an FFI host with no device allocator, code inside a stream capture):
its split-K scratch is a fixed 512 KiB array inside the library.  This file is
named to be collected last, so a run that stops at the first failure has run
every other test before it; it also passes on its own in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from grout_b200 import attn

D = 128
TOL_MAX, TOL_MEAN = 2e-3, 1e-3
pytestmark = pytest.mark.gpu


def _dims(hq, hkv, max_seq):
    return attn.make_dims(hq, hkv, max_seq, flags=attn.FLAG_DECODE_SCALE_F16)


def _case(B, hq, hkv, L, seed):
    g = torch.Generator(device="cuda:0").manual_seed(seed)
    kc = torch.randn(B, hkv, L, D, device="cuda:0", generator=g).half()
    vc = torch.randn(B, hkv, L, D, device="cuda:0", generator=g).half()
    q = torch.randn(B, hq, D, device="cuda:0", generator=g).half()
    pos = torch.randint(0, L, (B,), device="cuda:0", generator=g, dtype=torch.int32)
    pos[0] = L - 1
    return q, kc, vc, pos


def _call_regular(L_, q, kc, vc, pos, L):
    B, hq, _ = q.shape
    hkv = kc.shape[1]
    dims = _dims(hq, hkv, L)
    need = L_.grout_attn_decode_workspace_bytes(B, L, ctypes.byref(dims))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda:0")
    out = torch.empty_like(q)
    st = L_.grout_attn_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), hkv * L * D, L * D,
                              pos.data_ptr(), out.data_ptr(), B, L, ctypes.byref(dims),
                              ws.data_ptr(), ws.numel(), None)
    assert st == 0, L_.grout_attn_last_error()
    return out, need


def _call_noalloc(L_, q, kc, vc, pos, L):
    B, hq, _ = q.shape
    hkv = kc.shape[1]
    dims = _dims(hq, hkv, L)
    out = torch.empty_like(q)
    st = L_.grout_attn_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), hkv * L * D,
                                      L * D, pos.data_ptr(), out.data_ptr(), B, L,
                                      ctypes.byref(dims), None)
    return st, out


def test_noalloc_decode_matches_regular_twice(grout):
    L_ = attn.lib()
    assert L_.grout_attn_decode_noalloc_max_bytes() == 512 << 10
    # Two calls in a row on different shapes and data: the second must not
    # depend on what the first left in the shared scratch array.  One KV head
    # (a tensor-parallel shard) over a long context takes more splits than a
    # cluster merges, so these shapes use the scratch.
    for B, hq, hkv, L, seed in ((1, 8, 1, 8192, 1), (2, 8, 1, 12288, 2)):
        q, kc, vc, pos = _case(B, hq, hkv, L, seed)
        ref, need = _call_regular(L_, q, kc, vc, pos, L)
        assert 0 < need <= L_.grout_attn_decode_noalloc_max_bytes()  # split-K path, scratch used
        st, out = _call_noalloc(L_, q, kc, vc, pos, L)
        assert st == 0, L_.grout_attn_last_error()
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() <= TOL_MAX and err.mean().item() <= TOL_MEAN


def test_noalloc_rejects_oversized_scratch(grout):
    L_ = attn.lib()
    B, hq, hkv, L = 2, 8, 1, 16384  # 64 splits of 2 x 8 heads: 528 KB of scratch
    dims = _dims(hq, hkv, L)
    need = L_.grout_attn_decode_workspace_bytes(B, L, ctypes.byref(dims))
    assert need > L_.grout_attn_decode_noalloc_max_bytes()
    p = torch.empty(16, dtype=torch.float16, device="cuda:0")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda:0")
    st = L_.grout_attn_decode_noalloc(p.data_ptr(), p.data_ptr(), p.data_ptr(), hkv * L * D, L * D,
                                      pos.data_ptr(), p.data_ptr(), B, L, ctypes.byref(dims), None)
    assert st == 1
    assert b"scratch" in L_.grout_attn_last_error()
