"""CPU checks of the C ABI: the library builds, loads, exports every symbol
include/grout_attn.h declares, and its host-only logic (argument validation,
inv_freq, split selection) behaves; no kernel is launched."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle
from grout_b200 import attn, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "grout_attn.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(grout_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    build.build()
    return attn.lib()


def test_every_declared_symbol_is_exported_and_bound(L):
    names = header_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), n
    # the Python mirror binds exactly the declared set
    assert sorted(attn.SIGNATURES) == names


def test_version_and_empty_error(L):
    assert b"sm_100a" in L.grout_attn_version()
    assert L.grout_attn_last_error() is not None


def test_inv_freq_matches_oracle(L):
    for theta in (1.0e4, 1.0e6, 5.0e5):
        a = attn.inv_freq(theta)
        b = oracle.inv_freq(theta, 128)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_rope_table_bytes(L):
    assert L.grout_rope_table_bytes(4096, 128) == 4096 * 128 * 4
    assert L.grout_rope_table_bytes(0, 128) == 0


def _dims(hq=64, hkv=8, hd=128, ms=4096):
    return attn.AttnDims(hq, hkv, hd, ms, 1e-6, 0.0, 0)


def _err(L):
    return L.grout_attn_last_error().decode()


def test_validation_before_launch(L):
    """Shape/range errors are reported as INVALID_ARG / UNSUPPORTED without
    touching a device (this container has none)."""
    p = ctypes.c_void_p(0x10000)  # aligned, never dereferenced
    d = _dims(hd=64)
    st = L.grout_attn_prefill(p, p, p, p, 4096 * 128, 0, 16, ctypes.byref(d), None)
    assert st == 2 and "head_dim" in _err(L)
    d = _dims()
    st = L.grout_attn_prefill(p, p, p, p, 4096 * 128, 4090, 16, ctypes.byref(d), None)
    assert st == 1 and "exceeds max_seq" in _err(L)
    st = L.grout_qk_norm_rope_kv_prefill(p, p, p, 64 * 128, 8 * 128, p, p, p, p, p, p,
                                         4096 * 128, 4095, 2, ctypes.byref(d), None)
    assert st == 1 and "exceeds max_seq" in _err(L)
    st = L.grout_qk_norm_rope_kv_prefill(p, None, p, 64 * 128, 8 * 128, p, p, p, p, p, p,
                                         4096 * 128, 0, 2, ctypes.byref(d), None)
    assert st == 1 and "null" in _err(L)
    bad = ctypes.c_void_p(0x10002)
    st = L.grout_qk_norm_rope_kv_prefill(p, bad, p, 64 * 128, 8 * 128, p, p, p, p, p, p,
                                         4096 * 128, 0, 2, ctypes.byref(d), None)
    assert st == 1 and "aligned" in _err(L)
    d = _dims(hq=64, hkv=4)  # group 16 > 8
    st = L.grout_attn_decode(p, p, p, 0, 4096 * 128, p, p, 1, 100, ctypes.byref(d), None, 0, None)
    assert st == 2 and "group" in _err(L)
    d = _dims()
    st = L.grout_attn_decode_ex(p, p, p, 0, 4096 * 128, p, p, 1, 5000, 4, ctypes.byref(d), None, 0, None)
    assert st == 1 and "max_kv_len" in _err(L)
    # more than 16 splits merge through a workspace, which must be given
    st = L.grout_attn_decode_ex(p, p, p, 0, 4096 * 128, p, p, 1, 4096, 32, ctypes.byref(d), None, 0, None)
    assert st == 1 and "workspace" in _err(L)
    d = _dims(hq=63, hkv=8)
    st = L.grout_attn_prefill(p, p, p, p, 4096 * 128, 0, 16, ctypes.byref(d), None)
    assert st == 1 and "multiple" in _err(L)


def test_paged_validation_before_launch(L):
    """Paged entry points: page size, table stride, pool and table pointers
    are checked on the host before any launch."""
    p = ctypes.c_void_p(0x10000)
    d = _dims()  # max_seq 4096
    args = lambda ps, stride, pages=p, table=p: (p, pages, pages, 64, ps, table, stride, p, p, 2,
                                                 100, 0, ctypes.byref(d), None, 0, None)
    assert L.grout_attn_decode_paged(*args(96, 64)) == 1 and "page_size" in _err(L)
    assert L.grout_attn_decode_paged(*args(32, 128)) == 1 and "page_size" in _err(L)
    assert L.grout_attn_decode_paged(*args(64, 63)) == 1 and "table_stride" in _err(L)
    assert L.grout_attn_decode_paged(*args(64, 64, table=None)) == 1 and "null" in _err(L)
    assert L.grout_attn_decode_paged(*args(64, 64, pages=ctypes.c_void_p(0x10008))) == 1
    assert "aligned" in _err(L)
    st = L.grout_qk_norm_rope_kv_decode_paged(p, p, p, p, p, p, p, 0, 64, p, 64, p, 1,
                                              ctypes.byref(d), None)
    assert st == 1 and "num_pages" in _err(L)
    st = L.grout_qk_norm_rope_kv_prefill_paged(p, p, p, 64 * 128, 8 * 128, p, p, p, p, p, p, 8,
                                               128, p, 4000, 200, ctypes.byref(d), None)
    assert st == 1 and "exceeds max_seq" in _err(L)
    # empty batch: a no-op before any pointer check
    assert L.grout_attn_decode_paged(None, None, None, 0, 0, None, 0, None, None, 0, 1, 0,
                                     ctypes.byref(d), None, 0, None) == 0


def test_prefill_split_heuristic(L):
    """Split-K prefill only for launches with fewer work items than SMs."""
    d = _dims(hq=64, hkv=8)
    assert L.grout_attn_prefill_splits(1, 4096, ctypes.byref(d)) == 1   # 1024 items
    d = _dims(hq=8, hkv=1)
    n = L.grout_attn_prefill_splits(1, 2048, ctypes.byref(d))         # 64 items
    assert 2 <= n <= 8
    assert L.grout_attn_prefill_splitk_workspace_bytes(1, 2048, 8, 1) == 0
    assert L.grout_attn_prefill_splitk_workspace_bytes(1, 2048, 8, 3) == 8 * 8 * 3 * 2 * 128 * 130 * 4


def test_splitk_and_qkv_validation_before_launch(L):
    p = ctypes.c_void_p(0x10000)
    d = _dims()
    st = L.grout_attn_prefill_splitk(None, 2, ctypes.byref(d), None, 0, None)
    assert st == 1 and "args" in _err(L)
    args = attn.PrefillVarlenArgs(0x10000, 0x10000, 64 * 128, 100, 0x10000, 0x10000, 0, 128,
                                  4096 * 128, 4096, None, None, None, 2, 100)
    st = L.grout_attn_prefill_splitk(ctypes.byref(args), 3, ctypes.byref(d), None, 0, None)
    assert st == 1 and "cu_seqlens_q" in _err(L)
    args.batch = 1
    st = L.grout_attn_prefill_splitk(ctypes.byref(args), 9, ctypes.byref(d), None, 0, None)
    assert st == 1 and "num_splits" in _err(L)
    st = L.grout_qkv_proj_norm_rope_kv_prefill(p, 5120, p, 5100, p, p, p, p, p, p, 4096 * 128, None,
                                               0, 16, ctypes.byref(d), None)
    assert st == 1 and "hidden" in _err(L)
    st = L.grout_qkv_proj_norm_rope_kv_prefill(p, 5120, p, 5120, p, p, p, p, p, p, 4096 * 128, None,
                                               4090, 16, ctypes.byref(d), None)
    assert st == 1 and "exceeds max_seq" in _err(L)


def test_init_without_gpu_fails_cleanly(L):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    st = L.grout_attn_init(0)
    assert st == 3 and _err(L)


def test_decode_split_heuristic(L):
    """Split count: about one CTA per SM in total, at least 256 keys per
    split, one split once the batch alone fills the GPU."""
    for B in (1, 8, 32, 64):
        for Lk in (1024, 2048, 8192, 16384, 32768):
            n = attn.decode_splits(B, Lk, 64, 8, 32768)
            tiles = Lk // 64
            assert 1 <= n <= max(1, tiles // 4)
            assert B * 8 * (n - 1) < 148
            if B * 8 >= 148:
                assert n == 1
    # 19 splits would cover 152 SMs; 16 still cover 128 and merge in a cluster
    assert attn.decode_splits(1, 32768, 64, 8, 32768) == 16
    assert attn.decode_splits(8, 8192, 64, 8, 32768) == 3
    # up to 16 splits need no workspace (cluster merge)
    for B in (1, 8, 32):
        assert attn.decode_workspace_bytes(B, 8192, 64, 8, 32768) == 0
    # one KV head (tensor-parallel degree 8): more splits than a cluster holds
    n = attn.decode_splits(1, 8448, 8, 1, 8448)
    assert n == 33
    assert attn.decode_workspace_bytes(1, 8448, 8, 1, 8448) == 8 * n * 129 * 4


def test_python_mirror_rejects_cpu_tensors():
    import torch
    q = torch.zeros(4, 8, 128, dtype=torch.float16)
    with pytest.raises(attn.GroutError):
        attn.attention_prefill(q, torch.zeros(2, 16, 128, dtype=torch.float16),
                               torch.zeros(2, 16, 128, dtype=torch.float16), q.clone())
