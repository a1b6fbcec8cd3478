"""GPU checks of the tensor-parallel GEMV + all-reduce (grout_gemv_allreduce).

Numerics against a torch fp32 reference (the kernel accumulates in f32 and
rounds the final sum to f16 once): max-abs <= 2e-3 relative to the output
scale.  Multi-rank cases run one child process per GPU (skipped with fewer
than two GPUs); the host side of the handle exchange uses gloo."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
HIDDEN = 5120


def _ref(ws, xs, residual):
    y = sum(w.float() @ x.float() for w, x in zip(ws, xs))
    return y + residual.float()


def _inputs(rank, k, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed * 100 + rank)
    w = (torch.randn(HIDDEN, k, device="cuda", generator=g) * 0.02).half()
    x = torch.randn(k, device="cuda", generator=g).half()
    return w, x


def _tol(ref):
    return 2e-3 * max(1.0, ref.abs().max().item())


def test_gemv_allreduce_single_rank(grout):
    from grout_b200 import tp
    comm = tp.TPComm(0, 1, HIDDEN)
    for k in (256, 1024, 3200, 4096, 12800):
        w, x = _inputs(0, k, seed=k)
        res = torch.randn(HIDDEN, device="cuda").half()
        out = torch.empty(HIDDEN, device="cuda", dtype=torch.float16)
        for _ in range(3):  # successive calls alternate receive slots
            comm.gemv_allreduce(w, x, out, residual=res)
            torch.cuda.synchronize()
            ref = _ref([w], [x], res)
            assert (out.float() - ref).abs().max().item() <= _tol(ref)
    # recorded once in a CUDA graph, replayed with new inputs
    w, x = _inputs(0, 4096, seed=7)
    out = torch.empty(HIDDEN, device="cuda", dtype=torch.float16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        comm.gemv_allreduce(w, x, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        comm.gemv_allreduce(w, x, out)
    for i in range(3):
        x.copy_(torch.randn(4096, device="cuda").half())
        g.replay()
        torch.cuda.synchronize()
        ref = _ref([w], [x], torch.zeros(HIDDEN, device="cuda"))
        assert (out.float() - ref).abs().max().item() <= _tol(ref)
    grout.check_device_error()
    comm.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, k, mode, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import grout_b200 as g
        from grout_b200 import tp
        g.init(rank)
        # allocations before the comm, as in an engine: the exchange buffer
        # must still be mapped at exactly its own address in the peer
        junk = [torch.empty(12345 + 777 * i, device="cuda") for i in range(5)]
        comm = tp.TPComm(rank, world, HIDDEN)
        res = torch.full((HIDDEN,), 0.5, device="cuda").half()
        out = torch.empty(HIDDEN, device="cuda", dtype=torch.float16)
        if mode == "timeout":
            # rank 1 leaves between steps: it never makes the call, so rank 0's
            # bounded wait must expire and report a device error.
            if rank == 0:
                w, x = _inputs(rank, k)
                comm.gemv_allreduce(w, x, out, residual=res)
                torch.cuda.synchronize()
                msgs = []
                try:
                    g.check_device_error()
                    msgs.append("no-error")
                except g.GroutError as e:
                    msgs.append("error:" + str(e))
                # the comm is now out of step: the next call fails at once
                import time
                t0 = time.time()
                comm.gemv_allreduce(w, x, out, residual=res)
                torch.cuda.synchronize()
                dt = time.time() - t0
                try:
                    g.check_device_error()
                    msgs.append("no-error")
                except g.GroutError as e:
                    msgs.append("error:" + str(e))
                q.put((rank, (msgs, dt)))
            else:
                q.put((rank, "skipped"))
            dist.barrier()
            return
        if mode == "backtoback":
            # Eight calls with no host synchronisation between them, each
            # rank delayed by a different amount before each call, so a fast
            # rank finishes call n and raises its call n+1 flags while a slow
            # one is still waiting on call n.
            steps = 8
            ins = [_inputs(rank, k, seed=100 + s_) for s_ in range(steps)]
            outs_d = [torch.empty(HIDDEN, device="cuda", dtype=torch.float16) for _ in range(steps)]
            parts = [(w.float() @ x.float()).half() for w, x in ins]
            torch.cuda.synchronize()
            dist.barrier()
            for s_ in range(steps):
                torch.cuda._sleep(int(20000 * ((rank * 3 + s_ * 5) % 7)))
                w, x = ins[s_]
                if s_ % 2:
                    comm.allreduce(parts[s_], outs_d[s_], residual=res)
                else:
                    comm.gemv_allreduce(w, x, outs_d[s_], residual=res)
            torch.cuda.synchronize()
            outs = []
            for s_ in range(steps):
                allx = [_inputs(r, k, seed=100 + s_) for r in range(world)]
                ref = _ref([a for a, _ in allx], [b for _, b in allx], res)
                err = (outs_d[s_].float() - ref).abs().max().item()
                outs.append((err, _tol(ref), outs_d[s_].cpu().view(torch.int16).numpy()))
            g.check_device_error()
            comm.close()
            q.put((rank, outs))
            dist.barrier()
            return
        outs = []
        for step in range(4):
            w, x = _inputs(rank, k, seed=step)
            if step % 2:  # alternate with the exchange-only entry on the same comm
                comm.allreduce((w.float() @ x.float()).half(), out, residual=res)
            else:
                comm.gemv_allreduce(w, x, out, residual=res)
            torch.cuda.synchronize()
            allx = [_inputs(r, k, seed=step) for r in range(world)]
            ref = _ref([a for a, _ in allx], [b for _, b in allx], res)
            err = (out.float() - ref).abs().max().item()
            outs.append((err, _tol(ref), out.cpu().view(torch.int16).numpy()))
        g.check_device_error()
        comm.close()
        q.put((rank, outs))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _spawn(world, k, mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, k, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _need(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


def _check_ranks(res, world, steps):
    for step in range(steps):
        tol = res[0][step][1] * (2 if step % 2 else 1)  # exchange-only sums f16-rounded partials
        for r in range(world):
            assert res[r][step][0] <= tol
            assert np.array_equal(res[r][step][2], res[0][step][2])  # identical bits on every rank


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("k", [4096, 12800])
def test_gemv_allreduce_ranks(world, k):
    _need(world)
    k = k // (world // 2)  # the row-parallel shard shrinks with the TP degree
    _check_ranks(_spawn(world, k, "sum"), world, 4)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemv_allreduce_back_to_back_without_sync(world):
    _need(world)
    _check_ranks(_spawn(world, 1024, "backtoback"), world, 8)


@pytest.mark.parametrize("world", [2, 4])
def test_gemv_allreduce_missing_peer_times_out(world):
    _need(world)
    res = _spawn(world, 4096, "timeout")
    assert all(res[r] == "skipped" for r in range(1, world))
    (first, second), dt = res[0]
    assert first.startswith("error:") and "0x13c" in first
    assert second.startswith("error:") and "0x13d" in second and dt < 1.0
