"""GPU parity: split-K GQA decode + merge against the oracle (reference
rounding points, and the f64 ideal), within 2e-3 max-abs / 1e-3 mean-abs."""
import math

import numpy as np
import pytest
import torch

import oracle
from grout_b200 import synth

D = 128
TOL_MAX, TOL_MEAN = 2e-3, 1e-3
pytestmark = pytest.mark.gpu
SCALE_F16 = float(np.float16(1.0 / math.sqrt(D)))


def _inputs(B, hq, hkv, ms, seed=0):
    q = synth.normal(100 + seed, B * hq * D).reshape(B, hq, D)
    k = synth.normal(200 + seed, B * hkv * ms * D).reshape(B, hkv, ms, D)
    v = synth.normal(300 + seed, B * hkv * ms * D).reshape(B, hkv, ms, D)
    return q, k, v


def _run(grout, q, k, v, pos, max_kv_len, num_splits=None):
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq = T(q)
    out = torch.empty_like(dq)
    grout.attention_decode(dq, T(k), T(v), T(pos.astype(np.int32)), out, max_kv_len,
                           num_splits=num_splits)
    torch.cuda.synchronize()
    grout.check_device_error()
    return out.cpu().numpy()


def _check(out, ref):
    err = np.abs(out.astype(np.float64) - ref.astype(np.float64))
    assert err.max() <= TOL_MAX and err.mean() <= TOL_MEAN, (err.max(), err.mean())


@pytest.mark.parametrize("B,hq,hkv,ms,positions", [
    (1, 32, 8, 1024, [1023]),              # config 1 (Qwen3-4B layer, L = 1024)
    (1, 64, 8, 2048, [2047]),              # config 3 smallest cell
    (3, 64, 8, 700, [0, 63, 699]),         # L = 1, one tile, ragged tail
    (4, 32, 8, 4096, [4095, 1000, 2049, 130]),
    (2, 16, 16, 512, [511, 300]),          # G = 1
    (2, 16, 8, 512, [200, 511]),           # G = 2
])
def test_decode_matches_oracle(grout, B, hq, hkv, ms, positions):
    q, k, v = _inputs(B, hq, hkv, ms)
    pos = np.array(positions, np.uint32)
    out = _run(grout, q, k, v, pos, ms)
    ref = oracle.attn_decode(q, k, v, pos, hkv, hkv * ms * D, ms * D, SCALE_F16, nks=1, bn=64)
    _check(out, ref)
    ideal = oracle.attn_decode(q, k, v, pos, hkv, hkv * ms * D, ms * D, 1.0 / math.sqrt(D), ideal=True)
    _check(out, ideal)


@pytest.mark.parametrize("nks", [1, 2, 7, 16, 64])
def test_split_count_invariance(grout, nks):
    B, hq, hkv, ms = 2, 64, 8, 4096
    q, k, v = _inputs(B, hq, hkv, ms, seed=1)
    pos = np.array([4095, 2500], np.uint32)
    out = _run(grout, q, k, v, pos, ms, num_splits=nks)
    ref = oracle.attn_decode(q, k, v, pos, hkv, hkv * ms * D, ms * D, SCALE_F16, nks=nks, bn=64)
    _check(out, ref)


def test_decode_equal_rows_and_zero_query(grout):
    """KATs: identical V rows give that row; q = 0 gives the mean of V."""
    B, hq, hkv, ms = 1, 8, 1, 256
    q, k, v = _inputs(B, hq, hkv, ms, seed=2)
    v_same = np.broadcast_to(v[:, :, 7:8], v.shape).copy()
    out = _run(grout, q, k, v_same, np.array([200], np.uint32), ms)
    assert np.abs(out.astype(np.float32) - v_same[0, 0, 7].astype(np.float32)).max() <= TOL_MAX
    out = _run(grout, np.zeros_like(q), k, v, np.array([99], np.uint32), ms)
    mean = v[0, 0, :100].astype(np.float64).mean(0)
    assert np.abs(out[0].astype(np.float64) - mean).max() <= TOL_MAX


def test_decode_graph_replay_with_device_position(grout):
    """Captured once, replayed as the device position grows (decode-graph use)."""
    B, hq, hkv, ms = 1, 64, 8, 2048
    q, k, v = _inputs(B, hq, hkv, ms, seed=3)
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dk, dv = T(q), T(k), T(v)
    pos = torch.tensor([10], dtype=torch.int32, device=dev)
    out = torch.empty_like(dq)
    ws = torch.empty(grout.decode_workspace_bytes(B, ms, hq, hkv, ms) or 16, dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        grout.attention_decode(dq, dk, dv, pos, out, ms, workspace=ws)  # warm
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            grout.attention_decode(dq, dk, dv, pos, out, ms, workspace=ws)
    for p in (10, 777, 2047):
        pos.fill_(p)
        g.replay()
        torch.cuda.synchronize()
        ref = oracle.attn_decode(q, k, v, np.array([p], np.uint32), hkv, hkv * ms * D, ms * D,
                                 SCALE_F16, nks=1, bn=64)
        _check(out.cpu().numpy(), ref)
    grout.check_device_error()


def test_decode_golden(grout):
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    B, hkv, ms, _ = g["dc_k"].shape
    out = _run(grout, g["dc_q"], g["dc_k"], g["dc_v"], g["dc_pos"], ms)
    _check(out, g["dc_out"])


def test_decode_position_beyond_split_hint(grout):
    """max_kv_len only fixes the split count; a position past it (below
    max_seq) is still attended over all its keys."""
    B, hq, hkv, ms = 2, 64, 8, 2048
    q, k, v = _inputs(B, hq, hkv, ms, seed=4)
    pos = np.array([1500, 2047], np.uint32)
    out = _run(grout, q, k, v, pos, 256)
    ref = oracle.attn_decode(q, k, v, pos, hkv, hkv * ms * D, ms * D, SCALE_F16, nks=1, bn=64)
    _check(out, ref)


def test_decode_empty_batch_is_a_no_op(grout):
    q = torch.zeros(0, 8, D, dtype=torch.float16, device="cuda:0")
    kc = torch.zeros(1, 1, 64, D, dtype=torch.float16, device="cuda:0")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    grout.attention_decode(q, kc, kc.clone(), pos, q.clone(), 64)
    torch.cuda.synchronize()
