"""GPU parity of the split-K prefill (the reference's microbench-only
fmha_prefill_gqa_lpt_split + prefill_splitk_reduce_merge): low-parallelism
launches split along the KV range, merged in the log2 domain, against the
oracle within 2e-3 max-abs / 1e-3 mean-abs (and close to the unsplit kernel)."""
import math

import numpy as np
import pytest
import torch

import oracle
from grout_b200 import synth

D = 128
TOL_MAX, TOL_MEAN = 2e-3, 1e-3
SCALE = 1.0 / math.sqrt(D)
pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.device("cuda", 0))


def _check(out, ref, rows=None):
    o, r = out.astype(np.float64), ref.astype(np.float64)
    if rows is not None:
        o, r = o[rows], r[rows]
    assert np.isfinite(o).all()
    err = np.abs(o - r)
    assert err.max() <= TOL_MAX and err.mean() <= TOL_MEAN, (err.max(), err.mean())


@pytest.mark.parametrize("nks", [2, 3, 8])
def test_splitk_single_sequence_low_parallelism(grout, nks):
    S, hq, hkv, ms = 2048, 8, 1, 2048  # 8 pairs x 8 heads = 64 items for 148 SMs
    q = synth.normal(110, S * hq * D).reshape(S, hq, D)
    k = synth.normal(111, hkv * ms * D).reshape(hkv, ms, D)
    v = synth.normal(112, hkv * ms * D).reshape(hkv, ms, D)
    out = torch.empty(S, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill_splitk(_dev(q), _dev(k), _dev(v), out, None, S, hkv, kv_row_stride=D,
                                   kv_head_stride=ms * D, kv_rows=ms, num_splits=nks)
    base = torch.empty_like(out)
    grout.attention_prefill(_dev(q), _dev(k), _dev(v), base, 0)
    torch.cuda.synchronize()
    grout.check_device_error()
    rows = np.arange(0, S, 7)
    ref = oracle.attn_prefill(q, k, v, np.array([0, S]), np.array([0]), None, hq, hkv, 0, D,
                              ms * D, SCALE, rows_step=7)
    _check(out.cpu().numpy(), ref, rows=rows)
    assert (out.float() - base.float()).abs().max().item() <= TOL_MAX


def test_splitk_position_offset_uneven_chunks(grout):
    """A chunk at a position offset; 4 splits over 5-tile ranges leave one
    split empty (its slot is skipped by the merge)."""
    S, hq, hkv, P, ms = 600, 16, 2, 500, 1200
    q = synth.normal(120, S * hq * D).reshape(S, hq, D)
    k = synth.normal(121, hkv * ms * D).reshape(hkv, ms, D)
    v = synth.normal(122, hkv * ms * D).reshape(hkv, ms, D)
    out = torch.empty(S, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill_splitk(_dev(q), _dev(k), _dev(v), out, None, S, hkv, kv_row_stride=D,
                                   kv_head_stride=ms * D, kv_rows=ms,
                                   position_start=_dev(np.array([P], np.int32)), num_splits=4)
    torch.cuda.synchronize()
    grout.check_device_error()
    ref = oracle.attn_prefill(q, k, v, np.array([0, S]), np.array([P]), None, hq, hkv, 0, D,
                              ms * D, SCALE)
    _check(out.cpu().numpy(), ref)


def test_splitk_varlen_batched_cache(grout):
    hq, hkv, ms = 16, 4, 1024
    lens = np.array([200, 77, 513], np.int32)
    pos0 = np.array([0, 300, 500], np.int32)
    B = len(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    q = synth.normal(131, tot * hq * D).reshape(tot, hq, D)
    k = synth.normal(132, B * hkv * ms * D).reshape(B, hkv, ms, D)
    v = synth.normal(133, B * hkv * ms * D).reshape(B, hkv, ms, D)
    out = torch.zeros(tot, hq, D, dtype=torch.float16, device="cuda:0")
    grout.attention_prefill_splitk(_dev(q), _dev(k), _dev(v), out, _dev(cu), int(lens.max()), hkv,
                                   kv_row_stride=D, kv_head_stride=ms * D,
                                   kv_batch_stride=hkv * ms * D, kv_rows=ms,
                                   position_start=_dev(pos0), num_splits=3)
    torch.cuda.synchronize()
    grout.check_device_error()
    ref = oracle.attn_prefill(q, k, v, cu, pos0, None, hq, hkv, hkv * ms * D, D, ms * D, SCALE)
    _check(out.cpu().numpy(), ref)
