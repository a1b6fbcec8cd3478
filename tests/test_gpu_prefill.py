"""GPU parity: tcgen05 causal GQA prefill against the oracle (reference
rounding points and f64 ideal), within 2e-3 max-abs / 1e-3 mean-abs."""
import math
import os

import numpy as np
import pytest
import torch

import oracle
from grout_b200 import synth

D = 128
TOL_MAX, TOL_MEAN = 2e-3, 1e-3
SCALE = 1.0 / math.sqrt(D)
pytestmark = pytest.mark.gpu


def _check(out, ref, rows=None):
    o = out.astype(np.float64)
    r = ref.astype(np.float64)
    if rows is not None:
        o, r = o[rows], r[rows]
    err = np.abs(o - r)
    assert np.isfinite(o).all()
    assert err.max() <= TOL_MAX and err.mean() <= TOL_MEAN, (err.max(), err.mean())


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.device("cuda", 0))


def _engine_case(grout, S, hq, hkv, P, ms, seed=0, rows_step=1):
    q = synth.normal(10 + seed, S * hq * D).reshape(S, hq, D)
    k = synth.normal(20 + seed, hkv * ms * D).reshape(hkv, ms, D)
    v = synth.normal(30 + seed, hkv * ms * D).reshape(hkv, ms, D)
    out = torch.empty(S, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill(_dev(q), _dev(k), _dev(v), out, P)
    torch.cuda.synchronize()
    grout.check_device_error()
    ref = oracle.attn_prefill(q, k, v, np.array([0, S]), np.array([P]), None, hq, hkv, 0, D,
                              ms * D, SCALE, rows_step=rows_step)
    return out.cpu().numpy(), ref


@pytest.mark.parametrize("S,hq,hkv,P,ms", [
    (1, 8, 2, 0, 128),
    (128, 8, 2, 0, 128),
    (256, 8, 8, 0, 256),       # G = 1
    (300, 16, 2, 17, 512),     # ragged tail, position offset
    (640, 32, 8, 0, 640),      # G = 4 (Qwen3-4B/8B heads), 2.5 tile pairs
    (1000, 64, 8, 100, 1200),  # G = 8 (Qwen3-32B heads)
])
def test_prefill_matches_oracle(grout, S, hq, hkv, P, ms):
    out, ref = _engine_case(grout, S, hq, hkv, P, ms)
    _check(out, ref)


def test_prefill_reference_pattern_kat(grout):
    """attention_microbench --check inputs (pattern salts 1/2/3, K/V laid out
    [H_kv, S, D]) against the reference's own f32 cpu_reference."""
    S, hq, hkv = 384, 16, 4
    q = oracle.pattern(S * hq * D, 1).reshape(S, hq, D)
    k = oracle.pattern(hkv * S * D, 2).reshape(hkv, S, D)
    v = oracle.pattern(hkv * S * D, 3).reshape(hkv, S, D)
    out = torch.empty(S, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill(_dev(q), _dev(k), _dev(v), out, 0)
    torch.cuda.synchronize()
    ref = oracle.attn_prefill_naive(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    _check(out.cpu().numpy(), ref)


def test_prefill_golden(grout):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    q, k, v, P = g["pf_q"], g["pf_k"], g["pf_v"], int(g["pf_pos0"])
    out = torch.empty(q.shape, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill(_dev(q), _dev(k), _dev(v), out, P)
    torch.cuda.synchronize()
    _check(out.cpu().numpy(), g["pf_out"])


def test_prefill_varlen_packed(grout):
    """Packed varlen (config 4 layout): K/V [total, Hkv, D] addressed through
    cu_seqlens, sequences of ragged lengths, one launch."""
    hq, hkv = 32, 8
    lens = np.array([1, 130, 257, 511, 64], np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    q = synth.normal(41, tot * hq * D).reshape(tot, hq, D)
    k = synth.normal(42, tot * hkv * D).reshape(tot, hkv, D)
    v = synth.normal(43, tot * hkv * D).reshape(tot, hkv, D)
    out = torch.zeros(tot, hq, D, dtype=torch.float16, device="cuda:0")
    dcu = _dev(cu)
    grout.attention_prefill_varlen(_dev(q), _dev(k), _dev(v), out, dcu, int(lens.max()), hkv,
                                   kv_row_stride=hkv * D, kv_head_stride=D, kv_rows=tot,
                                   kv_start=dcu[:-1].contiguous())
    torch.cuda.synchronize()
    grout.check_device_error()
    ref = oracle.attn_prefill(q, k, v, cu, None, cu[:-1], hq, hkv, 0, hkv * D, D, SCALE)
    _check(out.cpu().numpy(), ref)


def test_prefill_varlen_batched_cache_with_positions(grout):
    """Batched per-sequence caches [B, Hkv, max_seq, D] with a chunk at a
    position offset per sequence (chunked prefill)."""
    hq, hkv, ms = 16, 4, 1024
    lens = np.array([200, 77, 513], np.int32)
    pos0 = np.array([0, 300, 500], np.int32)
    B = len(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    q = synth.normal(51, tot * hq * D).reshape(tot, hq, D)
    k = synth.normal(52, B * hkv * ms * D).reshape(B, hkv, ms, D)
    v = synth.normal(53, B * hkv * ms * D).reshape(B, hkv, ms, D)
    out = torch.zeros(tot, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill_varlen(_dev(q), _dev(k), _dev(v), out, _dev(cu), int(lens.max()), hkv,
                                   kv_row_stride=D, kv_head_stride=ms * D,
                                   kv_batch_stride=hkv * ms * D, kv_rows=ms,
                                   position_start=_dev(pos0))
    torch.cuda.synchronize()
    grout.check_device_error()
    ref = oracle.attn_prefill(q, k, v, cu, pos0, None, hq, hkv, hkv * ms * D, D, ms * D, SCALE)
    _check(out.cpu().numpy(), ref)


def test_prefill_config2_full_size_sampled_rows(grout):
    """Config 2 shape (S = 4096, 64/8 heads) at full size, checked on every
    61st query row (the oracle's bounded sample) including the last row."""
    S, hq, hkv = 4096, 64, 8
    out, ref = _engine_case(grout, S, hq, hkv, 0, S, seed=5, rows_step=61)
    rows = np.arange(0, S, 61)
    _check(out, ref, rows=rows)


def test_prefill_kv_head_shards_are_bitwise_identical(grout):
    """Config 4 sharding: each KV-head shard (what one GPU of 2/4/8 computes)
    reproduces its rows of the unsharded launch bit for bit."""
    hq, hkv = 32, 8
    lens = synth.ragged_lengths(5, 5, 128, 700)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    q = _dev(synth.normal(61, tot * hq * D).reshape(tot, hq, D))
    k = _dev(synth.normal(62, tot * hkv * D).reshape(tot, hkv, D))
    v = _dev(synth.normal(63, tot * hkv * D).reshape(tot, hkv, D))
    dcu = _dev(cu)
    kw = dict(kv_row_stride=hkv * D, kv_head_stride=D, kv_rows=tot, kv_start=dcu[:-1].contiguous())
    full = torch.zeros(tot, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill_varlen(q, k, v, full, dcu, int(lens.max()), hkv, **kw)
    for world in (2, 4, 8):
        shard = torch.zeros_like(full)
        per = hkv // world
        for r in range(world):
            grout.attention_prefill_varlen(q, k, v, shard, dcu, int(lens.max()), hkv,
                                           kv_head_range=(r * per, (r + 1) * per), **kw)
        torch.cuda.synchronize()
        assert torch.equal(shard.view(torch.int16), full.view(torch.int16)), world
    grout.check_device_error()


@pytest.mark.parametrize("S,P", [(127, 0), (129, 0), (255, 1), (256, 0), (257, 0), (384, 128), (513, 383)])
def test_prefill_tile_boundaries(grout, S, P):
    """Lengths and offsets around the 128-row / 256-row / 128-key tile edges."""
    out, ref = _engine_case(grout, S, 16, 4, P, S + P + 7, seed=S + P)
    _check(out, ref)


def test_prefill_empty_is_a_no_op(grout):
    q = torch.zeros(0, 8, D, dtype=torch.float16, device="cuda:0")
    kc = torch.zeros(2, 16, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill(q, kc, kc.clone(), q.clone(), 0)
    torch.cuda.synchronize()
    grout.check_device_error()
