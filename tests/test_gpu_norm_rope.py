"""GPU parity: fused Q/K RMSNorm + RoPE + KV write, bit-exact against the
oracle (q_out and K cache byte for byte, V copied bitwise)."""
import numpy as np
import pytest
import torch

import oracle
from grout_b200 import synth

D = 128
pytestmark = pytest.mark.gpu


def _u16(t):
    return t.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("S,hq,hkv,pos0,ms", [
    (1, 8, 2, 0, 16),
    (37, 32, 8, 5, 64),
    (256, 64, 8, 0, 256),
    (513, 64, 8, 1000, 2048),
])
def test_prefill_bit_exact(grout, S, hq, hkv, pos0, ms):
    eps, theta = 1e-6, 1.0e6
    q = synth.normal(1, S * hq * D).reshape(S, hq, D)
    k = synth.normal(2, S * hkv * D).reshape(S, hkv, D)
    v = synth.normal(3, S * hkv * D).reshape(S, hkv, D)
    qw, kw = synth.norm_weight(4, D), synth.norm_weight(5, D)
    inv = oracle.inv_freq(theta, D)
    tab = oracle.rope_table(inv, ms)
    kc = synth.normal(8, hkv * ms * D).reshape(hkv, ms, D)  # stale contents must survive
    vc = synth.normal(9, hkv * ms * D).reshape(hkv, ms, D)
    kc_ref, vc_ref = kc.copy(), vc.copy()
    q_ref = oracle.qk_norm_rope_kv_prefill(q, k, v, qw, kw, tab, kc_ref, vc_ref, pos0, eps)

    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    table = grout.rope_table(theta, ms, dev)
    assert np.array_equal(table.cpu().numpy().reshape(ms, 2, D // 2).view(np.uint32), tab.view(np.uint32))
    dq, dk, dv, dkc, dvc = T(q), T(k), T(v), T(kc), T(vc)
    q_out = torch.empty_like(dq)
    grout.qk_norm_rope_kv_prefill(dq, dk, dv, T(qw), T(kw), table, q_out, dkc, dvc, pos0, eps)
    torch.cuda.synchronize()
    grout.check_device_error()
    assert np.array_equal(_u16(q_out), q_ref.view(np.uint16))
    assert np.array_equal(_u16(dkc), kc_ref.view(np.uint16))
    assert np.array_equal(_u16(dvc), vc_ref.view(np.uint16))


@pytest.mark.parametrize("B,hq,hkv,ms", [(1, 32, 8, 1024), (5, 64, 8, 300)])
def test_decode_bit_exact(grout, B, hq, hkv, ms):
    eps, theta = 1e-6, 1.0e6
    qkv = synth.normal(11, B * (hq + 2 * hkv) * D).reshape(B, -1)
    qw, kw = synth.norm_weight(4, D), synth.norm_weight(5, D)
    tab = oracle.rope_table(oracle.inv_freq(theta, D), ms)
    pos = (np.arange(B, dtype=np.uint32) * 97 + 3) % ms
    pos[-1] = ms - 1
    kc = np.zeros((B, hkv, ms, D), np.float16)
    vc = np.zeros_like(kc)
    q_ref = oracle.qk_norm_rope_kv_decode(qkv, qw, kw, tab, kc, vc, pos, hq, hkv, eps)

    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    table = grout.rope_table(theta, ms, dev)
    dkc, dvc = torch.zeros(B, hkv, ms, D, dtype=torch.float16, device=dev), torch.zeros(B, hkv, ms, D, dtype=torch.float16, device=dev)
    q_out = torch.empty(B, hq, D, dtype=torch.float16, device=dev)
    dpos = T(pos.astype(np.int32))
    grout.qk_norm_rope_kv_decode(T(qkv), T(qw), T(kw), table, q_out, dkc, dvc, dpos, hq, hkv, eps)
    torch.cuda.synchronize()
    grout.check_device_error()
    assert np.array_equal(_u16(q_out), q_ref.view(np.uint16))
    assert np.array_equal(_u16(dkc), kc.view(np.uint16))
    assert np.array_equal(_u16(dvc), vc.view(np.uint16))


def test_decode_position_out_of_range_sets_device_error(grout):
    """A device position >= max_seq skips the write and is reported; no fault."""
    hq, hkv, ms = 8, 2, 16
    dev = torch.device("cuda", 0)
    qkv = torch.randn(1, (hq + 2 * hkv) * D, device=dev).half()
    w = torch.ones(D, dtype=torch.float16, device=dev)
    table = grout.rope_table(1.0e6, ms, dev)
    kc = torch.zeros(1, hkv, ms, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(1, hq, D, dtype=torch.float16, device=dev)
    pos = torch.tensor([ms], dtype=torch.int32, device=dev)
    grout.qk_norm_rope_kv_decode(qkv, w, w, table, q_out, kc, vc, pos, hq, hkv, 1e-6)
    with pytest.raises(grout.GroutError, match="0x200"):
        grout.check_device_error()
    assert kc.abs().sum().item() == 0
    grout.check_device_error()  # cleared


def test_v_copied_bitwise_including_nan_and_inf(grout):
    """V is copied bit for bit: arbitrary f16 bit patterns (NaN payloads,
    infinities, subnormals) survive; the write lands at the last cache row."""
    S, hq, hkv, ms = 3, 8, 2, 16
    rng = np.random.default_rng(7)
    q = synth.normal(1, S * hq * D).reshape(S, hq, D)
    k = synth.normal(2, S * hkv * D).reshape(S, hkv, D)
    vbits = rng.integers(0, 1 << 16, size=(S, hkv, D), dtype=np.uint16)
    vbits[0, 0, :4] = [0x7C00, 0xFC00, 0x7E01, 0x0001]
    v = vbits.view(np.float16)
    w = np.ones(D, np.float16)
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    table = grout.rope_table(1.0e6, ms, dev)
    kc = torch.zeros(hkv, ms, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(S, hq, D, dtype=torch.float16, device=dev)
    grout.qk_norm_rope_kv_prefill(T(q), T(k), T(v), T(w), T(w), table, q_out, kc, vc, ms - S, 1e-6)
    torch.cuda.synchronize()
    got = vc.cpu().numpy().view(np.uint16)
    assert np.array_equal(got[:, ms - S:].transpose(1, 0, 2), vbits)
    assert not got[:, : ms - S].any()
    with pytest.raises(grout.GroutError, match="exceeds max_seq"):
        grout.qk_norm_rope_kv_prefill(T(q), T(k), T(v), T(w), T(w), table, q_out, kc, vc,
                                      ms - S + 1, 1e-6)
