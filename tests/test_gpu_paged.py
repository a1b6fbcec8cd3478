"""GPU checks of the paged KV cache: the same data scattered into shuffled
pages gives bit-identical results to the contiguous cache (decode attention,
fused decode write, fused prefill write), the paged decode matches the oracle,
and a bad page-table entry is reported without a fault or a stray write."""
import math

import numpy as np
import pytest
import torch

import oracle
from grout_b200 import synth

D = 128
pytestmark = pytest.mark.gpu
SCALE_F16 = float(np.float16(1.0 / math.sqrt(D)))


def _paged(kc, page_size, seed):
    """Scatter [B, Hkv, max_seq, D] caches into a shuffled page pool
    [num_pages, Hkv, page_size, D] plus two spare pages; returns (pool, table)."""
    B, hkv, ms, _ = kc.shape
    per = ms // page_size
    n = B * per + 2
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n, generator=g)[: B * per].view(B, per).to(torch.int32)
    pool = torch.zeros(n, hkv, page_size, D, dtype=kc.dtype, device=kc.device)
    for b in range(B):
        for pg in range(per):
            pool[int(perm[b, pg])] = kc[b, :, pg * page_size:(pg + 1) * page_size]
    return pool, perm.to(kc.device)


def _gather(pool, table, ms):
    B, per = table.shape
    ps = pool.shape[2]
    out = torch.empty(B, pool.shape[1], ms, D, dtype=pool.dtype, device=pool.device)
    for b in range(B):
        for pg in range(per):
            out[b, :, pg * ps:(pg + 1) * ps] = pool[int(table[b, pg])]
    return out


@pytest.mark.parametrize("page_size", [64, 128, 256])
@pytest.mark.parametrize("nks", [None, 1, 7])
def test_paged_decode_bitwise_equals_contiguous(grout, page_size, nks):
    B, hq, hkv, ms = 3, 64, 8, 2048
    dev = torch.device("cuda", 0)
    q = torch.from_numpy(synth.normal(40, B * hq * D).reshape(B, hq, D)).to(dev)
    kc = torch.from_numpy(synth.normal(41, B * hkv * ms * D).reshape(B, hkv, ms, D)).to(dev)
    vc = torch.from_numpy(synth.normal(42, B * hkv * ms * D).reshape(B, hkv, ms, D)).to(dev)
    pos = torch.tensor([ms - 1, 700, 64], dtype=torch.int32, device=dev)
    ref = torch.empty_like(q)
    grout.attention_decode(q, kc, vc, pos, ref, ms, num_splits=nks)
    kp, table = _paged(kc, page_size, 1)
    vp, _ = _paged(vc, page_size, 1)
    out = torch.empty_like(q)
    grout.attention_decode_paged(q, kp, vp, table, pos, out, ms, num_splits=nks)
    torch.cuda.synchronize()
    grout.check_device_error()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_paged_decode_matches_oracle(grout):
    B, hq, hkv, ms, ps = 2, 32, 8, 1024, 64
    dev = torch.device("cuda", 0)
    q = synth.normal(50, B * hq * D).reshape(B, hq, D)
    k = synth.normal(51, B * hkv * ms * D).reshape(B, hkv, ms, D)
    v = synth.normal(52, B * hkv * ms * D).reshape(B, hkv, ms, D)
    pos = np.array([1023, 333], np.uint32)
    kp, table = _paged(torch.from_numpy(k).to(dev), ps, 2)
    vp, _ = _paged(torch.from_numpy(v).to(dev), ps, 2)
    out = torch.empty(B, hq, D, dtype=torch.float16, device=dev)
    grout.attention_decode_paged(torch.from_numpy(q).to(dev), kp, vp, table,
                                 torch.from_numpy(pos.astype(np.int32)).to(dev), out, ms, num_splits=1)
    torch.cuda.synchronize()
    grout.check_device_error()
    ref = oracle.attn_decode(q, k, v, pos, hkv, hkv * ms * D, ms * D, SCALE_F16, nks=1, bn=64)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref.astype(np.float64))
    assert err.max() <= 2e-3 and err.mean() <= 1e-3, (err.max(), err.mean())


def test_paged_decode_write_bitwise_equals_contiguous(grout):
    B, hq, hkv, ms, ps = 4, 32, 8, 512, 128
    eps, theta = 1e-6, 1.0e6
    dev = torch.device("cuda", 0)
    qkv = torch.from_numpy(synth.normal(60, B * (hq + 2 * hkv) * D).reshape(B, -1)).to(dev)
    qw = torch.from_numpy(synth.norm_weight(4, D)).to(dev)
    kw = torch.from_numpy(synth.norm_weight(5, D)).to(dev)
    table = grout.rope_table(theta, ms, dev)
    pos = torch.tensor([0, 127, 128, 511], dtype=torch.int32, device=dev)
    base_k = torch.from_numpy(synth.normal(61, B * hkv * ms * D).reshape(B, hkv, ms, D)).to(dev)
    base_v = torch.from_numpy(synth.normal(62, B * hkv * ms * D).reshape(B, hkv, ms, D)).to(dev)
    kc, vc = base_k.clone(), base_v.clone()
    q_ref = torch.empty(B, hq, D, dtype=torch.float16, device=dev)
    grout.qk_norm_rope_kv_decode(qkv, qw, kw, table, q_ref, kc, vc, pos, hq, hkv, eps)
    kp, ptab = _paged(base_k, ps, 3)
    vp, _ = _paged(base_v, ps, 3)
    q_out = torch.empty_like(q_ref)
    grout.qk_norm_rope_kv_decode_paged(qkv, qw, kw, table, q_out, kp, vp, ptab, pos, hq, hkv, eps)
    torch.cuda.synchronize()
    grout.check_device_error()
    assert torch.equal(q_out.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(_gather(kp, ptab, ms).view(torch.int16), kc.view(torch.int16))
    assert torch.equal(_gather(vp, ptab, ms).view(torch.int16), vc.view(torch.int16))


def test_paged_prefill_write_bitwise_equals_contiguous(grout):
    S, hq, hkv, ms, ps, pos0 = 300, 64, 8, 1024, 64, 100
    eps, theta = 1e-6, 1.0e6
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = T(synth.normal(70, S * hq * D).reshape(S, hq, D))
    k = T(synth.normal(71, S * hkv * D).reshape(S, hkv, D))
    v = T(synth.normal(72, S * hkv * D).reshape(S, hkv, D))
    qw, kw = T(synth.norm_weight(4, D)), T(synth.norm_weight(5, D))
    table = grout.rope_table(theta, ms, dev)
    kc = torch.zeros(hkv, ms, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    q_ref = torch.empty_like(q)
    grout.qk_norm_rope_kv_prefill(q, k, v, qw, kw, table, q_ref, kc, vc, pos0, eps)
    kp, ptab = _paged(torch.zeros(1, hkv, ms, D, dtype=torch.float16, device=dev), ps, 4)
    vp = torch.zeros_like(kp)
    q_out = torch.empty_like(q)
    grout.qk_norm_rope_kv_prefill_paged(q, k, v, qw, kw, table, q_out, kp, vp, ptab[0], pos0, eps)
    torch.cuda.synchronize()
    grout.check_device_error()
    assert torch.equal(q_out.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(_gather(kp, ptab, ms)[0].view(torch.int16), kc.view(torch.int16))
    assert torch.equal(_gather(vp, ptab, ms)[0].view(torch.int16), vc.view(torch.int16))


def test_bad_page_entry_is_reported_without_a_write(grout):
    hq, hkv, ms, ps = 8, 2, 256, 64
    dev = torch.device("cuda", 0)
    qkv = torch.randn(1, (hq + 2 * hkv) * D, device=dev).half()
    w = torch.ones(D, dtype=torch.float16, device=dev)
    table = grout.rope_table(1.0e6, ms, dev)
    kp = torch.zeros(4, hkv, ps, D, dtype=torch.float16, device=dev)
    vp = torch.zeros_like(kp)
    ptab = torch.tensor([[0, 1, 99, 3]], dtype=torch.int32, device=dev)  # page 99 does not exist
    pos = torch.tensor([150], dtype=torch.int32, device=dev)            # lands in table entry 2
    q_out = torch.empty(1, hq, D, dtype=torch.float16, device=dev)
    grout.qk_norm_rope_kv_decode_paged(qkv, w, w, table, q_out, kp, vp, ptab, pos, hq, hkv, 1e-6)
    with pytest.raises(grout.GroutError, match="0x201"):
        grout.check_device_error()
    assert kp.abs().sum().item() == 0 and vp.abs().sum().item() == 0
    # decode attention over the same table: the tile of the bad entry is
    # masked out (its keys get no weight) and reported, so the result equals
    # attention over the valid tiles alone (keys 0..127) bit for bit
    kp.copy_(torch.randn_like(kp.float()).half())
    vp.copy_(torch.randn_like(vp.float()).half())
    for nks in (1, 2):
        out = torch.empty(1, hq, D, dtype=torch.float16, device=dev)
        grout.attention_decode_paged(q_out, kp, vp, ptab, pos, out, ms, num_splits=nks)
        with pytest.raises(grout.GroutError, match="0x201"):
            grout.check_device_error()
        kc = torch.cat([kp[0], kp[1]], 1).unsqueeze(0).contiguous()   # pages 0, 1 = keys 0..127
        vc = torch.cat([vp[0], vp[1]], 1).unsqueeze(0).contiguous()
        ref = torch.empty_like(out)
        grout.attention_decode(q_out, kc, vc, torch.tensor([127], dtype=torch.int32, device=dev),
                               ref, 128, num_splits=1)
        torch.cuda.synchronize()
        if nks == 1:
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        else:
            assert (out.float() - ref.float()).abs().max().item() <= 2e-3
    grout.check_device_error()  # cleared


@pytest.mark.parametrize("page_size", [64, 128, 192])
def test_paged_prefill_single_sequence_bitwise_equals_contiguous(grout, page_size):
    """Chunked prefill at a position offset: the same cache in shuffled pages
    gives the contiguous kernel's bits (tiles straddling pages included)."""
    S, hq, hkv, pos0 = 500, 64, 8, 300
    ms = 1152  # a multiple of 64, 128 and 192
    dev = torch.device("cuda", 0)
    q = torch.from_numpy(synth.normal(80, S * hq * D).reshape(S, hq, D)).to(dev)
    kc = torch.from_numpy(synth.normal(81, hkv * ms * D).reshape(hkv, ms, D)).to(dev)
    vc = torch.from_numpy(synth.normal(82, hkv * ms * D).reshape(hkv, ms, D)).to(dev)
    ref = torch.empty_like(q)
    grout.attention_prefill(q, kc, vc, ref, pos0)
    kp, table = _paged(kc[None], page_size, 5)
    vp, _ = _paged(vc[None], page_size, 5)
    out = torch.empty_like(q)
    grout.attention_prefill_paged(q, kp, vp, table, out,
                                  position_start=torch.tensor([pos0], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    grout.check_device_error()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_paged_prefill_varlen_bitwise_equals_batched_cache(grout):
    """Ragged batch with per-sequence position offsets over one shared pool."""
    hq, hkv, ms, ps = 16, 4, 1024, 128
    lens = np.array([200, 77, 513], np.int32)
    pos0 = np.array([0, 300, 500], np.int32)
    B = len(lens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = T(synth.normal(91, tot * hq * D).reshape(tot, hq, D))
    kc = T(synth.normal(92, B * hkv * ms * D).reshape(B, hkv, ms, D))
    vc = T(synth.normal(93, B * hkv * ms * D).reshape(B, hkv, ms, D))
    ref = torch.zeros(tot, hq, D, dtype=torch.float16, device=dev)
    grout.attention_prefill_varlen(q, kc, vc, ref, T(cu), int(lens.max()), hkv, kv_row_stride=D,
                                   kv_head_stride=ms * D, kv_batch_stride=hkv * ms * D, kv_rows=ms,
                                   position_start=T(pos0))
    kp, table = _paged(kc, ps, 6)
    vp, _ = _paged(vc, ps, 6)
    out = torch.zeros_like(ref)
    grout.attention_prefill_paged(q, kp, vp, table, out, cu_seqlens_q=T(cu), position_start=T(pos0),
                                  max_q_len=int(lens.max()))
    torch.cuda.synchronize()
    grout.check_device_error()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_paged_decode_graph_replay_across_pages(grout):
    """A decode step (fused paged write + paged attention) recorded once in a
    CUDA graph and replayed while positions grow across a page boundary; the
    next page is appended to the table between steps (outside the graph).
    Every step equals the contiguous-cache path bit for bit."""
    B, hq, hkv, ms, ps = 2, 32, 8, 512, 64
    eps, theta = 1e-6, 1.0e6
    dev = torch.device("cuda", 0)
    qw = torch.from_numpy(synth.norm_weight(4, D)).to(dev)
    kw = torch.from_numpy(synth.norm_weight(5, D)).to(dev)
    table = grout.rope_table(theta, ms, dev)
    # contiguous reference caches and a paged pool holding the same rows
    kc = torch.from_numpy(synth.normal(141, B * hkv * ms * D).reshape(B, hkv, ms, D)).to(dev)
    vc = torch.from_numpy(synth.normal(142, B * hkv * ms * D).reshape(B, hkv, ms, D)).to(dev)
    kp, ptab = _paged(kc, ps, 9)
    vp, _ = _paged(vc, ps, 9)
    live = ptab.clone()
    ptab[:, 1:] = -1  # pages past the first are appended as positions grow
    qkv = torch.empty(B, (hq + 2 * hkv) * D, dtype=torch.float16, device=dev)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    q_out = torch.empty(B, hq, D, dtype=torch.float16, device=dev)
    out = torch.empty_like(q_out)
    ws = torch.empty(max(16, grout.decode_workspace_bytes(B, ms, hq, hkv, ms)), dtype=torch.uint8, device=dev)

    def step():
        grout.qk_norm_rope_kv_decode_paged(qkv, qw, kw, table, q_out, kp, vp, ptab, pos, hq, hkv, eps)
        grout.attention_decode_paged(q_out, kp, vp, ptab, pos, out, ms, workspace=ws)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        qkv.copy_(torch.randn_like(qkv))
        pos.fill_(0)
        step()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    grout.check_device_error()
    q_ref = torch.empty_like(q_out)
    o_ref = torch.empty_like(out)
    # the warm-up step wrote position 0 into the pool: mirror it
    grout.qk_norm_rope_kv_decode(qkv, qw, kw, table, q_ref, kc, vc, pos, hq, hkv, eps)
    for p in (60, 62, 63, 64, 65, 127, 128):
        pg = p // ps
        ptab[:, pg] = live[:, pg]  # the page this position lands in
        qkv.copy_(torch.from_numpy(synth.normal(150 + p, qkv.numel()).reshape(qkv.shape)).to(dev))
        pos.fill_(p)
        g.replay()
        grout.qk_norm_rope_kv_decode(qkv, qw, kw, table, q_ref, kc, vc, pos, hq, hkv, eps)
        grout.attention_decode(q_ref, kc, vc, pos, o_ref, ms)
        torch.cuda.synchronize()
        grout.check_device_error()
        assert torch.equal(q_out.view(torch.int16), q_ref.view(torch.int16)), p
        assert torch.equal(out.view(torch.int16), o_ref.view(torch.int16)), p
