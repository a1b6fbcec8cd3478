"""Parity at the sizes bench.py measures, not only at small test shapes.

- Config 3 decode cells B = 8, L = 32768 and B = 64, L = 8192 (Qwen3-32B
  heads 64/8) at the split count the bench uses (grout_attn_decode_splits),
  checked against the decode oracle (src/kernels.rs:4016-4304 rounding
  points) on sampled sequences; every sequence at the last position.
- Config 4's actual batch: 16 ragged sequences, L ~ U[128, 8192] (seed 5),
  62 505 tokens at Qwen3-8B heads 32/8, checked against the causal prefill
  oracle (src/kernels.rs:2943-3298) on every 97th query row.
- Config 4's KV-head shards computed on two real GPUs (one process each)
  equal the one-GPU launch bit for bit.
The oracle samples keep each check to seconds of CPU time."""
import math
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from grout_b200 import synth

D = 128
TOL_MAX, TOL_MEAN = 2e-3, 1e-3
SCALE_F16 = float(np.float16(1.0 / math.sqrt(D)))
pytestmark = pytest.mark.gpu


def _check(out, ref):
    err = np.abs(out.astype(np.float64) - ref.astype(np.float64))
    assert np.isfinite(out.astype(np.float32)).all()
    assert err.max() <= TOL_MAX and err.mean() <= TOL_MEAN, (err.max(), err.mean())


@pytest.mark.parametrize("B,L,sampled", [(8, 32768, (0, 5)), (64, 8192, (0, 31, 63))])
def test_config3_cell_matches_oracle(grout, B, L, sampled):
    hq, hkv = 64, 8
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(B * 1000 + L)
    kc = torch.randn(B, hkv, L, D, device=dev, generator=g).half()
    vc = torch.randn(B, hkv, L, D, device=dev, generator=g).half()
    q = torch.randn(B, hq, D, device=dev, generator=g).half()
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    nks = grout.decode_splits(B, L, hq, hkv, L)
    grout.attention_decode(q, kc, vc, pos, out, L)
    torch.cuda.synchronize()
    grout.check_device_error()
    for b in sampled:
        qb = q[b:b + 1].cpu().numpy()
        kb = kc[b:b + 1].cpu().numpy()
        vb = vc[b:b + 1].cpu().numpy()
        p = np.array([L - 1], np.uint32)
        ref = oracle.attn_decode(qb, kb, vb, p, hkv, hkv * L * D, L * D, SCALE_F16, nks=nks, bn=64)
        _check(out[b:b + 1].cpu().numpy(), ref)


def _c4_inputs(dev):
    hq, hkv = 32, 8
    lens = synth.ragged_lengths(5, 16, 128, 8192)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(tot, hq, D, device=dev, generator=g).half()
    k = torch.randn(tot, hkv, D, device=dev, generator=g).half()
    v = torch.randn(tot, hkv, D, device=dev, generator=g).half()
    return hq, hkv, lens, cu, tot, q, k, v


def _c4_run(grout, dev, hq, hkv, lens, cu, tot, q, k, v, kv_head_range=None):
    dcu = torch.from_numpy(cu).to(dev)
    out = torch.zeros_like(q)
    grout.attention_prefill_varlen(q, k, v, out, dcu, int(lens.max()), hkv,
                                   kv_row_stride=hkv * D, kv_head_stride=D, kv_rows=tot,
                                   kv_start=dcu[:-1].contiguous(), kv_head_range=kv_head_range)
    torch.cuda.synchronize()
    grout.check_device_error()
    return out


def test_config4_batch_matches_oracle(grout):
    dev = torch.device("cuda", 0)
    hq, hkv, lens, cu, tot, q, k, v = _c4_inputs(dev)
    assert tot == 62505
    out = _c4_run(grout, dev, hq, hkv, lens, cu, tot, q, k, v).cpu().numpy()
    step = 97
    ref = oracle.attn_prefill(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), cu, None, cu[:-1],
                              hq, hkv, 0, hkv * D, D, 1.0 / math.sqrt(D), rows_step=step)
    # rows_step samples rows m % step == 0 within each sequence
    rows = np.concatenate([np.arange(cu[i], cu[i + 1])[::step] for i in range(len(lens))])
    _check(out[rows], ref[rows])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, q_):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import grout_b200 as g
        g.init(rank)
        dev = torch.device("cuda", rank)
        hq, hkv, lens, cu, tot, q, k, v = _c4_inputs(dev)
        per = hkv // world
        out = _c4_run(g, dev, hq, hkv, lens, cu, tot, q, k, v,
                      kv_head_range=(rank * per, (rank + 1) * per))
        G = hq // hkv
        # numpy (f16 bits as int16) travels by value through the queue
        mine = out[:, rank * per * G:(rank + 1) * per * G].contiguous().cpu().view(torch.int16).numpy()
        full = (_c4_run(g, dev, hq, hkv, lens, cu, tot, q, k, v).cpu().view(torch.int16).numpy()
                if rank == 0 else None)
        q_.put((rank, (mine, full)))
        dist.barrier()
        dist.destroy_process_group()
    finally:
        q_.close()
        q_.join_thread()
    os._exit(0)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_config4_kv_head_shards_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_ = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q_)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q_.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = res[0][1]
    joined = np.concatenate([res[0][0], res[1][0]], 1)
    assert np.array_equal(joined, full)
