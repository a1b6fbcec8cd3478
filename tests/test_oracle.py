"""CPU checks of the oracle against the golden vectors, the reference's own
f32 cpu_reference (attention_microbench.rs:665-702) and analytic KATs."""
import math
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
D = 128


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def test_f16_conversion_matches_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * 10,
        np.array([0.0, -0.0, 65504.0, 65520.0, 70000.0, 1e-8, 6e-8, 3e-5, np.inf, -np.inf], np.float32),
        (rng.standard_normal(10000) * 1e-6).astype(np.float32),
    ])
    out = np.empty(x.shape, np.uint16)
    oracle.lib().oracle_f32_to_f16(oracle._p(x), oracle._p(out), oracle.i64(x.size))
    assert np.array_equal(out, x.astype(np.float16).view(np.uint16))
    back = np.empty(x.shape, np.float32)
    oracle.lib().oracle_f16_to_f32(oracle._p(out), oracle._p(back), oracle.i64(x.size))
    assert np.array_equal(back, out.view(np.float16).astype(np.float32))


def test_pattern_kat_matches_reference_generator(g):
    for salt in (1, 2, 3):
        assert np.array_equal(oracle.pattern(4096, salt).view(np.uint16),
                              g[f"pattern_{salt}"].view(np.uint16))


def test_inv_freq_and_rope_table(g):
    inv = oracle.inv_freq(1.0e6, D)
    assert np.array_equal(inv.view(np.uint32), g["inv_freq"].view(np.uint32))
    tab = oracle.rope_table(inv, 16)
    assert np.array_equal(tab.view(np.uint32), g["rope_table"].view(np.uint32))


def test_fused_norm_rope_bit_exact_vs_golden(g):
    q, k, v = g["nr_q"], g["nr_k"], g["nr_v"]
    kc = np.zeros((2, 16, D), np.float16)
    vc = np.zeros_like(kc)
    tab = oracle.rope_table(oracle.inv_freq(1.0e6, D), 16)
    q_out = oracle.qk_norm_rope_kv_prefill(q, k, v, g["nr_qw"], g["nr_kw"], tab, kc, vc, 3, 1e-6)
    assert np.array_equal(q_out.view(np.uint16), g["nr_q_out"].view(np.uint16))
    assert np.array_equal(kc.view(np.uint16), g["nr_k_cache"].view(np.uint16))
    assert np.array_equal(vc.view(np.uint16), g["nr_v_cache"].view(np.uint16))


def test_fused_decode_equals_prefill_row():
    """Decode at position p writes what prefill writes for the token at p."""
    from grout_b200 import synth
    hq, hkv, ms = 8, 2, 32
    tab = oracle.rope_table(oracle.inv_freq(1.0e6, D), ms)
    qw, kw = synth.norm_weight(4, D), synth.norm_weight(5, D)
    qkv = synth.normal(9, 2 * (hq + 2 * hkv) * D).reshape(2, -1)
    pos = np.array([5, 17], np.uint32)
    kc = np.zeros((2, hkv, ms, D), np.float16)
    vc = np.zeros_like(kc)
    q_out = oracle.qk_norm_rope_kv_decode(qkv, qw, kw, tab, kc, vc, pos, hq, hkv, 1e-6)
    for b in range(2):
        row = qkv[b]
        q = row[: hq * D].reshape(1, hq, D)
        k = row[hq * D:(hq + hkv) * D].reshape(1, hkv, D)
        v = row[(hq + hkv) * D:].reshape(1, hkv, D)
        kc2 = np.zeros((hkv, ms, D), np.float16)
        vc2 = np.zeros_like(kc2)
        q2 = oracle.qk_norm_rope_kv_prefill(q, k, v, qw, kw, tab, kc2, vc2, int(pos[b]), 1e-6)
        assert np.array_equal(q_out[b].view(np.uint16), q2[0].view(np.uint16))
        assert np.array_equal(kc[b].view(np.uint16), kc2.view(np.uint16))
        assert np.array_equal(vc[b].view(np.uint16), vc2.view(np.uint16))


def test_norm_kat_constant_row():
    """x = c, w = 1, pos = 0 (cos 1, sin 0): y = c / sqrt(c^2 + eps)."""
    c = np.float16(0.5)
    q = np.full((1, 1, D), c, np.float16)
    k = np.full((1, 1, D), c, np.float16)
    v = np.zeros((1, 1, D), np.float16)
    w = np.ones(D, np.float16)
    tab = oracle.rope_table(oracle.inv_freq(1.0e6, D), 4)
    kc = np.zeros((1, 4, D), np.float16)
    vc = np.zeros_like(kc)
    q_out = oracle.qk_norm_rope_kv_prefill(q, k, v, w, w, tab, kc, vc, 0, 1e-6)
    expect = np.float16(0.5 / math.sqrt(0.25 + 1e-6))
    assert np.all(q_out == expect) and np.all(kc[0, 0] == expect)


def test_prefill_exact_vs_golden_f64(g):
    P = int(g["pf_pos0"])
    q = g["pf_q"]
    S, hq, _ = q.shape
    hkv, ms, _ = g["pf_k"].shape
    out = oracle.attn_prefill(q, g["pf_k"], g["pf_v"], np.array([0, S]), np.array([P]), None, hq,
                              hkv, 0, D, ms * D, 1.0 / math.sqrt(D))
    err = np.abs(out.astype(np.float64) - g["pf_out"])
    assert err.max() < 2e-3 and err.mean() < 1e-3
    ideal = oracle.attn_prefill(q, g["pf_k"], g["pf_v"], np.array([0, S]), np.array([P]), None, hq,
                                hkv, 0, D, ms * D, 1.0 / math.sqrt(D), ideal=True)
    assert np.abs(ideal.astype(np.float64) - g["pf_out"]).max() <= 2 ** -10


def test_prefill_matches_reference_cpu_reference_on_pattern():
    """The reference's own f32 check path (attention_microbench.rs:617-702) on
    its own pattern inputs, S=96, 8/2 heads."""
    S, hq, hkv = 96, 8, 2
    q = oracle.pattern(S * hq * D, 1).reshape(S, hq, D)
    k = oracle.pattern(hkv * S * D, 2).reshape(hkv, S, D)
    v = oracle.pattern(hkv * S * D, 3).reshape(hkv, S, D)
    ref = oracle.attn_prefill_naive(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    out = oracle.attn_prefill(q, k, v, np.array([0, S]), None, None, hq, hkv, 0, D, S * D,
                              1.0 / math.sqrt(D))
    err = np.abs(out.astype(np.float32) - ref)
    assert err.max() < 2e-3 and err.mean() < 1e-3


def test_decode_exact_vs_golden_f64(g):
    q, k, v, pos = g["dc_q"], g["dc_k"], g["dc_v"], g["dc_pos"]
    B, hkv, ms, _ = k.shape
    for nks, bn in ((1, 32), (4, 32), (16, 16)):
        out = oracle.attn_decode(q, k, v, pos, hkv, hkv * ms * D, ms * D,
                                 float(np.float16(1.0 / math.sqrt(D))), nks=nks, bn=bn)
        err = np.abs(out.astype(np.float64) - g["dc_out"])
        assert err.max() < 2e-3 and err.mean() < 1e-3, (nks, bn, err.max())


def test_decode_kats():
    """L = 1 gives V[0]; equal V rows give that row; Q = 0 gives the mean."""
    from grout_b200 import synth
    hq, hkv, ms = 4, 1, 64
    k = synth.normal(1, hkv * ms * D).reshape(1, hkv, ms, D)
    v = synth.normal(2, hkv * ms * D).reshape(1, hkv, ms, D)
    q = synth.normal(3, hq * D).reshape(1, hq, D)
    out = oracle.attn_decode(q, k, v, np.array([0], np.uint32), hkv, k.size, ms * D, 0.0883789)
    assert np.array_equal(out[0], np.broadcast_to(v[0, 0, 0], (hq, D)))
    v2 = np.broadcast_to(v[0, 0, 5], v.shape).copy()
    out = oracle.attn_decode(q, k, v2, np.array([40], np.uint32), hkv, k.size, ms * D, 0.0883789, nks=3)
    assert np.abs(out.astype(np.float32) - v2[0, 0, 5].astype(np.float32)).max() < 2e-3
    q0 = np.zeros_like(q)
    out = oracle.attn_decode(q0, k, v, np.array([19], np.uint32), hkv, k.size, ms * D, 0.0883789)
    mean = v[0, 0, :20].astype(np.float64).mean(axis=0)
    assert np.abs(out[0].astype(np.float64) - mean).max() < 2e-3


def test_decode_equals_last_prefill_row():
    """Decode at position p equals row p of a causal prefill over the same cache."""
    from grout_b200 import synth
    hq, hkv, L = 8, 2, 77
    q = synth.normal(5, L * hq * D).reshape(L, hq, D)
    k = synth.normal(6, hkv * L * D).reshape(1, hkv, L, D)
    v = synth.normal(7, hkv * L * D).reshape(1, hkv, L, D)
    pf = oracle.attn_prefill(q, k, v, np.array([0, L]), None, None, hq, hkv, 0, D, L * D,
                             1.0 / math.sqrt(D), ideal=True)
    dc = oracle.attn_decode(q[L - 1:L], k, v, np.array([L - 1], np.uint32), hkv, k.size, L * D,
                            1.0 / math.sqrt(D), ideal=True)
    assert np.abs(pf[L - 1].astype(np.float32) - dc[0].astype(np.float32)).max() <= 2 ** -10
