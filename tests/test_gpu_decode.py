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


def test_decode_position_out_of_range_gives_zero_row(grout):
    """A position >= max_seq is caught on the device: device error 0x200, that
    sequence's output row is zero, the other sequences are unaffected."""
    B, hq, hkv, ms = 2, 64, 8, 512
    q, k, v = _inputs(B, hq, hkv, ms, seed=5)
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    for nks in (1, 4, 32):  # direct write, cluster merge, workspace merge
        pos = torch.tensor([300, ms + 5], dtype=torch.int32, device=dev)
        out = torch.full((B, hq, D), 7.0, dtype=torch.float16, device=dev)
        grout.attention_decode(T(q), T(k), T(v), pos, out, ms, num_splits=nks)
        torch.cuda.synchronize()
        with pytest.raises(grout.GroutError, match="0x200"):
            grout.check_device_error()
        o = out.cpu().numpy()
        assert not o[1].any()
        ref = oracle.attn_decode(q[:1], k[:1], v[:1], np.array([300], np.uint32), hkv,
                                 hkv * ms * D, ms * D, SCALE_F16, nks=1, bn=64)
        _check(o[:1], ref)


def _fused_case(B, hq, hkv, ms, positions, seed):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    qkv = torch.randn(B, (hq + 2 * hkv) * D, device=dev, generator=g).half()
    qw = (1 + 0.02 * torch.randn(D, device=dev, generator=g)).half()
    kw = (1 + 0.02 * torch.randn(D, device=dev, generator=g)).half()
    kc = torch.randn(B, hkv, ms, D, device=dev, generator=g).half()
    vc = torch.randn(B, hkv, ms, D, device=dev, generator=g).half()
    pos = torch.tensor(positions, dtype=torch.int32, device=dev)
    return qkv, qw, kw, kc, vc, pos


@pytest.mark.parametrize("B,hq,hkv,ms,positions", [
    (1, 64, 8, 8448, [8447]),           # config 5 at TP = 1 (16 splits, cluster merge)
    (1, 8, 1, 8448, [8300]),            # config 5 at TP = 8 (33 splits, workspace merge)
    (3, 32, 8, 1024, [0, 63, 64]),      # first key, tile edges
    (2, 64, 8, 4096, [4095, 2047]),
    (2, 16, 16, 512, [511, 128]),       # G = 1
])
def test_fused_decode_equals_separate_ops(grout, B, hq, hkv, ms, positions):
    """grout_attn_decode_fused = qk_norm_rope_kv_decode then attention_decode,
    bit for bit: caches, q_out and the attention output."""
    qkv, qw, kw, kc, vc, pos = _fused_case(B, hq, hkv, ms, positions, seed=B * 7 + hq)
    eps = 1e-6
    table = grout.rope_table(1.0e6, ms, torch.device("cuda", 0))
    kc1, vc1 = kc.clone(), vc.clone()
    q1 = torch.empty(B, hq, D, dtype=torch.float16, device="cuda:0")
    o1 = torch.empty_like(q1)
    grout.qk_norm_rope_kv_decode(qkv, qw, kw, table, q1, kc1, vc1, pos, hq, hkv, eps)
    grout.attention_decode(q1, kc1, vc1, pos, o1, ms)
    kc2, vc2 = kc.clone(), vc.clone()
    q2 = torch.empty_like(q1)
    o2 = torch.empty_like(q1)
    grout.attention_decode_fused(qkv, qw, kw, table, kc2, vc2, pos, o2, ms, eps, q_out=q2)
    torch.cuda.synchronize()
    grout.check_device_error()
    for a, b in ((kc1, kc2), (vc1, vc2), (q1, q2), (o1, o2)):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    # and against the oracle: fused write + split-free decode
    kc3, vc3 = kc.cpu().numpy(), vc.cpu().numpy()
    qo = oracle.qk_norm_rope_kv_decode(qkv.cpu().numpy(), qw.cpu().numpy(), kw.cpu().numpy(),
                                       table.cpu().numpy(), kc3, vc3,
                                       pos.cpu().numpy().astype(np.uint32), hq, hkv, eps)
    ref = oracle.attn_decode(qo, kc3, vc3, pos.cpu().numpy().astype(np.uint32), hkv,
                             hkv * ms * D, ms * D, SCALE_F16, nks=1, bn=64)
    _check(o2.cpu().numpy(), ref)


def test_fused_decode_graph_replay(grout):
    """The fused step recorded once and replayed while the position grows,
    across a tile boundary, as in the decode graph."""
    B, hq, hkv, ms = 1, 64, 8, 1024
    qkv, qw, kw, kc, vc, pos = _fused_case(B, hq, hkv, ms, [60], seed=11)
    table = grout.rope_table(1.0e6, ms, torch.device("cuda", 0))
    out = torch.empty(B, hq, D, dtype=torch.float16, device="cuda:0")
    ref_k, ref_v = kc.clone(), vc.clone()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        grout.attention_decode_fused(qkv, qw, kw, table, kc, vc, pos, out, ms, 1e-6)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            grout.attention_decode_fused(qkv, qw, kw, table, kc, vc, pos, out, ms, 1e-6)
    q1 = torch.empty_like(out)
    o1 = torch.empty_like(out)
    for p in (60, 63, 64, 65, 700):
        pos.fill_(p)
        qkv.copy_(torch.randn_like(qkv.float()).half())
        g.replay()
        grout.qk_norm_rope_kv_decode(qkv, qw, kw, table, q1, ref_k, ref_v, pos, hq, hkv, 1e-6)
        grout.attention_decode(q1, ref_k, ref_v, pos, o1, ms)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), o1.view(torch.int16))
        assert torch.equal(kc[:, :, p].view(torch.int16), ref_k[:, :, p].view(torch.int16))
    grout.check_device_error()
