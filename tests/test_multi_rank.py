"""Host logic of the multi-GPU path on CPU: two gloo ranks exchange their
timings exactly as bench.py's NCCL ranks do (max over ranks), and the
KV-head partition covers every head once."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = [10.0 + rank, 5.0 * (world - rank), 1.0 + rank, 2.0]
        mx = bench.reduce_max(local, dist, "cpu")
        lo, hi = bench.shard_kv_heads(8, world, rank)
        q.put((rank, mx, (lo, hi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_max_over_ranks_and_head_partition(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    expect = [10.0 + world - 1, 5.0 * world, 1.0 + world - 1, 2.0]
    for _, mx, _ in res:
        assert mx == expect
    heads = sorted(h for _, _, (lo, hi) in res for h in range(lo, hi))
    assert heads == list(range(8))


def test_job_value_counts_all_ranks():
    f = bench.prefill_flops(4096)
    assert abs(f - 2.749e11) / 2.749e11 < 1e-3
    assert bench.job_tflops(f, 10, 4, 10.0) == pytest.approx(4 * f * 10 / 0.01 / 1e12)
    with pytest.raises(ValueError):
        bench.shard_kv_heads(8, 3, 0)
