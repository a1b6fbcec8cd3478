"""Config 5's tensor-parallel decoder is one network at every TP degree.

A reduced Qwen3 (2 layers, hidden 1024, 16 query / 8 KV heads, head_dim 128,
intermediate 2048, vocab 4096) is built at TP = 1 and at TP = N from the same
block-seeded weights (grout_b200/qwen3_tp.py), then runs a prompt and 16
greedy tokens under CUDA-graph replay, the path of the reference engine's
prefill + decode_greedy (src/api.rs:118-130, graph decode src/model.rs:
2631-4007).  TP = N must give the TP = 1 tokens; the final-norm hidden state
of every step agrees within an f16 tolerance (the all-reduce sums the same
partials in another order).  A token may only differ where the TP = 1 top-2
logit margin is below what that tolerance allows, and then the sequences
are compared no further.

The layer-0 check runs the oracle (tests only) on the layer-0 QKV activations
the model produced in prefill and in one eager decode step: the caches must
equal the oracle's fused write bit for bit, the prefill attention rows must
match the oracle's causal prefill, and the decode row (position S) must match
the oracle's decode at that position (prefill/decode consistency)."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PROMPT, GEN = 100, 16
HID_TOL = 2e-2      # max-abs on the final-norm hidden state (values ~ 1)
MARGIN_OK = 0.05    # a top-2 logit margin this small may flip under TOL


def _shape():
    from grout_b200.qwen3_tp import Qwen3Shape
    return Qwen3Shape(layers=2, hidden=1024, heads=16, kv_heads=8, head_dim=128, inter=2048,
                      vocab=4096)


def _prompt(dev):
    g = torch.Generator(device=dev).manual_seed(6)
    return torch.randint(0, _shape().vocab, (PROMPT,), device=dev, generator=g)


def _run(m, tokens):
    """Prefill + GEN graph-replayed greedy steps: (tokens, hidden states)."""
    toks = [int(m.prefill(tokens).item())]
    hs = [m.h_last.float().cpu().clone()]
    m.capture()
    for _ in range(GEN):
        m.graph.replay()
        toks.append(int(m.tok.item()))
        hs.append(m.h_last.float().cpu().clone())
    return toks, hs


def _compare(ref_m, ref, got):
    """Tokens equal, hidden states within HID_TOL, up to the first near-tie."""
    (t1, h1), (tn, hn) = ref, got
    lm = ref_m.lm_head.float().cpu()
    for i in range(len(t1)):
        err = (h1[i] - hn[i]).abs().max().item()
        assert err <= HID_TOL, f"step {i}: hidden max-abs {err}"
        if t1[i] != tn[i]:
            logits = (h1[i] @ lm.t()).view(-1)
            top = torch.topk(logits, 2).values
            margin = (top[0] - top[1]).item()
            assert margin < MARGIN_OK, f"step {i}: token {tn[i]} != {t1[i]} at margin {margin}"
            return i
    return len(t1)


def test_graph_decode_matches_eager(grout):
    """The replayed decode graph computes what the eager step computes (the
    GEMMs may pick other cuBLAS kernels under capture, so within HID_TOL)."""
    from grout_b200.qwen3_tp import Qwen3TP
    dev = torch.device("cuda", 0)
    tokens = _prompt(dev)
    a = Qwen3TP(_shape(), PROMPT + GEN + 4, device=dev)
    b = Qwen3TP(_shape(), PROMPT + GEN + 4, device=dev)
    ta, ha = _run(a, tokens)
    tb = [int(b.prefill(tokens).item())]
    hb = [b.h_last.float().cpu().clone()]
    for _ in range(GEN):
        tb.append(b.step_eager())
        hb.append(b.h_last.float().cpu().clone())
    assert _compare(b, (tb, hb), (ta, ha)) == len(ta)
    grout.check_device_error()


def test_layer0_prefill_decode_consistency(grout, oracle):
    from grout_b200.qwen3_tp import Qwen3TP
    dev = torch.device("cuda", 0)
    c = _shape()
    max_seq = PROMPT + 8
    m = Qwen3TP(c, max_seq, device=dev)
    m.trace = {}
    m.prefill(_prompt(dev))
    m.step_eager()
    qkv_p, o_p = (t.cpu() for t in m.trace["prefill"])
    qkv_d, o_d = (t.cpu() for t in m.trace["decode"])
    L0 = m.layers[0]
    hq, hkv, D, S = c.heads, c.kv_heads, c.head_dim, PROMPT
    qkv = torch.cat([qkv_p, qkv_d.view(1, -1)], 0).numpy()           # [S+1, (hq+2hkv)*D]
    q = qkv[:, :hq * D].reshape(S + 1, hq, D)
    k = qkv[:, hq * D:(hq + hkv) * D].reshape(S + 1, hkv, D)
    v = qkv[:, (hq + hkv) * D:].reshape(S + 1, hkv, D)
    table = oracle.rope_table(oracle.inv_freq(c.theta, D), max_seq)
    kc = np.zeros((hkv, max_seq, D), np.float16)
    vc = np.zeros_like(kc)
    q_out = oracle.qk_norm_rope_kv_prefill(q, k, v, L0["q_norm"].cpu().numpy(),
                                           L0["k_norm"].cpu().numpy(), table, kc, vc, 0, c.eps)
    # the fused writes of prefill (rows 0..S-1) and decode (row S): bit for bit
    assert np.array_equal(L0["k_cache"][:, :S + 1].cpu().numpy().view(np.uint16),
                          kc[:, :S + 1].view(np.uint16))
    assert np.array_equal(L0["v_cache"][:, :S + 1].cpu().numpy().view(np.uint16),
                          vc[:, :S + 1].view(np.uint16))
    # prefill rows against the causal prefill oracle (f32 scale)
    ref = oracle.attn_prefill(q_out[:S], kc, vc, np.array([0, S]), None, None, hq, hkv, 0, D,
                              max_seq * D, 1.0 / np.sqrt(D))
    err = np.abs(o_p.numpy().astype(np.float32) - ref.astype(np.float32))
    assert err.max() <= 2e-3 and err.mean() <= 1e-3
    # the decode row at position S against the decode oracle (f16 scale)
    ref_d = oracle.attn_decode(q_out[S:S + 1], kc, vc, np.array([S]), hkv, 0, max_seq * D,
                               float(np.float16(1.0 / np.sqrt(D))))
    err = np.abs(o_d.numpy().astype(np.float32).reshape(1, hq, D) - ref_d.astype(np.float32))
    assert err.max() <= 2e-3 and err.mean() <= 1e-3
    # and against the prefill oracle's row for the same position
    ref_full = oracle.attn_prefill(q_out, kc, vc, np.array([0, S + 1]), None, None, hq, hkv, 0,
                                   D, max_seq * D, 1.0 / np.sqrt(D))
    err = np.abs(o_d.numpy().astype(np.float32).reshape(hq, D) - ref_full[S].astype(np.float32))
    assert err.max() <= 2e-3 and err.mean() <= 1e-3
    grout.check_device_error()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fused, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    code = 1
    try:
        import grout_b200 as g
        from grout_b200.qwen3_tp import Qwen3TP
        g.init(rank)
        dev = torch.device("cuda", rank)
        tokens = _prompt(dev)
        m = Qwen3TP(_shape(), PROMPT + GEN + 4, rank, world, dist.group.WORLD, dev,
                    fused_allreduce=fused)
        got = _run(m, tokens)
        g.check_device_error()
        if rank == 0:
            m1 = Qwen3TP(_shape(), PROMPT + GEN + 4, 0, 1, None, dev)
            ref = _run(m1, tokens)
            # numpy travels by value: the queue then needs nothing of this process
            np_ = lambda r: (r[0], [h.numpy() for h in r[1]])
            q.put((rank, (np_(ref), np_(got), m1.lm_head.float().cpu().numpy())))
        else:
            q.put((rank, None))
        dist.barrier()
        code = 0
    finally:
        q.close()
        q.join_thread()
        # No process-group teardown: NCCL communicators captured in the decode
        # graphs can block it; the process ends here (code 1 on an exception).
        os._exit(code)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fused", [True, False], ids=["grout_allreduce", "nccl"])
def test_tp_degree_is_the_same_model(world, fused):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fused, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref, got, lm = res[0]
    tt = lambda r: (r[0], [torch.from_numpy(h) for h in r[1]])
    ref, got = tt(ref), tt(got)

    class _M:
        lm_head = torch.from_numpy(lm)
    n = _compare(_M, ref, got)
    assert n >= 4, f"sequences diverged at step {n}"
