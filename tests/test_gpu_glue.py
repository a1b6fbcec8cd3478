"""GPU checks of the decode-graph glue kernels (grout_add_rms_norm,
grout_silu_mul) against a plain torch fp32 reference of the same op.  The
kernels compute in f32 and round once to f16, so the bar is the f16 rounding
of the result: |err| <= 2^-10 * |ref| + 1e-3."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(out, ref):
    err = (out.float() - ref).abs()
    bound = ref.abs() * 2.0 ** -10 + 1e-3
    assert bool((err <= bound).all()), float((err - bound).max())


@pytest.mark.parametrize("rows,n", [(1, 5120), (3, 1024), (17, 8192), (2, 16384), (5, 8)])
def test_add_rms_norm(grout, rows, n):
    g = torch.Generator(device="cuda").manual_seed(rows * n)
    x = torch.randn(rows, n, device="cuda", generator=g).half()
    r = torch.randn(rows, n, device="cuda", generator=g).half()
    w = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).half()
    eps = 1e-6
    out = torch.empty_like(x)
    rout = torch.empty_like(x)
    grout.add_rms_norm(x, w, out, eps, residual=r, residual_out=rout)
    c = x.float() + r.float()
    ref = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    torch.cuda.synchronize()
    _close(out, ref)
    assert torch.equal(rout, c.half())
    # without a residual
    grout.add_rms_norm(x, w, out, eps)
    xf = x.float()
    _close(out, xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float())


@pytest.mark.parametrize("rows,n", [(1, 25600), (1, 3200), (4, 1024), (3, 8)])
def test_silu_mul(grout, rows, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    gu = (3 * torch.randn(rows, 2 * n, device="cuda", generator=g)).half()
    out = torch.empty(rows, n, device="cuda", dtype=torch.float16)
    grout.silu_mul(gu, out)
    gf, uf = gu[:, :n].float(), gu[:, n:].float()
    ref = torch.sigmoid(gf) * gf * uf
    torch.cuda.synchronize()
    _close(out, ref)


def test_glue_validation(grout):
    x = torch.zeros(2, 12, device="cuda", dtype=torch.float16)
    with pytest.raises(grout.GroutError):  # n not a multiple of 8
        grout.add_rms_norm(x, torch.ones(12, device="cuda", dtype=torch.float16), x.clone(), 1e-6)

