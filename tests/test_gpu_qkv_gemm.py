"""GPU checks of the QKV projection with the fused norm/RoPE/KV write as its
epilogue: the epilogue equals the fused kernel applied to the kernel's own
f16 projection bit for bit, and the projection matches an f32 GEMM within
f16 rounding (max-abs <= 4e-3 at these magnitudes)."""
import numpy as np
import pytest
import torch

from grout_b200 import synth

D = 128
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S,hidden,hq,hkv,pos0,ms", [
    (300, 512, 16, 4, 37, 512),       # partial token tile, position offset
    (1024, 5120, 64, 8, 0, 1024),     # Qwen3-32B projection
])
def test_qkv_proj_epilogue_bit_exact_and_gemm_accuracy(grout, S, hidden, hq, hkv, pos0, ms):
    dev = torch.device("cuda", 0)
    eps, theta = 1e-6, 1.0e6
    N = (hq + 2 * hkv) * D
    x = torch.from_numpy(synth.normal(160, S * hidden).reshape(S, hidden)).to(dev)
    w = (torch.from_numpy(synth.normal(161, N * hidden).reshape(N, hidden)).to(dev).float() * 0.02).half()
    qw = torch.from_numpy(synth.norm_weight(4, D)).to(dev)
    kw = torch.from_numpy(synth.norm_weight(5, D)).to(dev)
    table = grout.rope_table(theta, ms, dev)
    q_out = torch.empty(S, hq, D, dtype=torch.float16, device=dev)
    kc = torch.zeros(hkv, ms, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    qkv = torch.empty(S, N, dtype=torch.float16, device=dev)
    grout.qkv_proj_norm_rope_kv_prefill(x, w, qw, kw, table, q_out, kc, vc, pos0, eps, qkv_out=qkv)
    torch.cuda.synchronize()
    grout.check_device_error()
    # the projection against an f32 GEMM
    ref = x.float() @ w.float().t()
    err = (qkv.float() - ref).abs()
    assert err.max().item() <= 4e-3 * max(1.0, ref.abs().max().item() / 4), err.max().item()
    # the epilogue against the fused kernel on the same f16 projection
    q_in = qkv[:, :hq * D].contiguous().view(S, hq, D)
    k_in = qkv[:, hq * D:(hq + hkv) * D].contiguous().view(S, hkv, D)
    v_in = qkv[:, (hq + hkv) * D:].contiguous().view(S, hkv, D)
    q_ref = torch.empty_like(q_out)
    kc_ref = torch.zeros_like(kc)
    vc_ref = torch.zeros_like(vc)
    grout.qk_norm_rope_kv_prefill(q_in, k_in, v_in, qw, kw, table, q_ref, kc_ref, vc_ref, pos0, eps)
    torch.cuda.synchronize()
    assert torch.equal(q_out.view(torch.int16), q_ref.view(torch.int16))
    assert torch.equal(kc.view(torch.int16), kc_ref.view(torch.int16))
    assert torch.equal(vc.view(torch.int16), vc_ref.view(torch.int16))


def test_qkv_proj_without_activation_output(grout):
    """qkv_out is optional: the caches and q_out alone are written."""
    dev = torch.device("cuda", 0)
    S, hidden, hq, hkv, ms = 130, 256, 8, 2, 256
    N = (hq + 2 * hkv) * D
    x = torch.randn(S, hidden, device=dev).half()
    w = (torch.randn(N, hidden, device=dev) * 0.05).half()
    ones = torch.ones(D, dtype=torch.float16, device=dev)
    table = grout.rope_table(1.0e6, ms, dev)
    q_a = torch.empty(S, hq, D, dtype=torch.float16, device=dev)
    kc_a, vc_a = torch.zeros(hkv, ms, D, dtype=torch.float16, device=dev), torch.zeros(hkv, ms, D, dtype=torch.float16, device=dev)
    grout.qkv_proj_norm_rope_kv_prefill(x, w, ones, ones, table, q_a, kc_a, vc_a, 0, 1e-6)
    q_b = torch.empty_like(q_a)
    kc_b, vc_b = torch.zeros_like(kc_a), torch.zeros_like(vc_a)
    qkv = torch.empty(S, N, dtype=torch.float16, device=dev)
    grout.qkv_proj_norm_rope_kv_prefill(x, w, ones, ones, table, q_b, kc_b, vc_b, 0, 1e-6, qkv_out=qkv)
    torch.cuda.synchronize()
    grout.check_device_error()
    assert torch.equal(q_a, q_b) and torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
