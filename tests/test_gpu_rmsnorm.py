"""Native RMSNorm of the decoder block against a float64 restatement of the
reference module (cuda/continuum_attention.py:815-821)."""
import pytest
import torch

from continuum_attention_b200.rmsnorm import rms_norm

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference(x, w, eps):
    x = x.double()
    return w.double() * x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


@pytest.mark.parametrize("D", [128, 256, 512, 1024])
@pytest.mark.parametrize("x_dtype,out_dtype", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                               (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32)])
def test_forward_backward_match_float64(D, x_dtype, out_dtype):
    g = torch.Generator().manual_seed(D)
    rows = 777
    x = (torch.randn(3, rows // 3 + 1, D, generator=g) * 2.5).to(DEV, x_dtype)
    w = (1 + 0.3 * torch.randn(D, generator=g)).to(DEV)
    dy = torch.randn(x.shape, generator=g).to(DEV, out_dtype)
    eps = 1e-6
    xr = x.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    y = rms_norm(xr, wr, eps, out_dtype)
    assert y.dtype == out_dtype and y.shape == x.shape
    dx, dw = torch.autograd.grad(y, (xr, wr), dy)
    assert dx.dtype == x_dtype and dw.dtype == torch.float32

    x64 = x.double().requires_grad_(True)
    w64 = w.double().requires_grad_(True)
    ref = _reference(x64, w64, eps)
    rdx, rdw = torch.autograd.grad(ref, (x64, w64), dy.double())
    # output: fp32 to 1e-5 relative of the row scale, bf16 to one rounding
    tol_y = 2e-5 if out_dtype == torch.float32 else 2 ** -7
    err_y = ((y.double() - ref.detach()).abs() / ref.detach().abs().clamp_min(1e-3)).max().item()
    assert err_y < tol_y, err_y
    tol_g = 1e-4 if x_dtype == torch.float32 else 1e-2
    err_dx = ((dx.double() - rdx).abs().max() / rdx.abs().max()).item()
    err_dw = ((dw.double() - rdw).abs().max() / rdw.abs().max()).item()
    assert err_dx < tol_g, err_dx
    assert err_dw < 1e-4, err_dw


def test_deterministic_and_errors():
    g = torch.Generator().manual_seed(7)
    x = torch.randn(4096, 1024, generator=g).to(DEV)
    w = torch.randn(1024, generator=g).to(DEV).requires_grad_(True)
    dy = torch.randn(4096, 1024, generator=g).to(DEV, torch.bfloat16)
    grads = []
    for _ in range(2):
        xr = x.clone().requires_grad_(True)
        y = rms_norm(xr, w, 1e-6, torch.bfloat16)
        grads.append(torch.autograd.grad(y, (xr, w), dy))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])
    with pytest.raises(ValueError):
        rms_norm(torch.randn(8, 768, device=DEV), torch.ones(768, device=DEV), 1e-6)
    with pytest.raises(ValueError):
        rms_norm(torch.randn(8, 128, device=DEV, dtype=torch.float16), torch.ones(128, device=DEV), 1e-6)


def test_decoder_block_norm_matches_torch_rms_norm():
    from continuum_attention_b200.decoder import RMSNorm
    g = torch.Generator().manual_seed(3)
    norm = RMSNorm(1024).to(DEV)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.2 * torch.randn(1024, generator=g))
    x = torch.randn(2, 64, 1024, generator=g).to(DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = norm(x)
    assert y.dtype == torch.bfloat16
    ref = torch.nn.functional.rms_norm(x, (1024,), norm.weight, norm.eps).to(torch.bfloat16)
    assert (y.float() - ref.float()).abs().max().item() <= 2 ** -7 * ref.float().abs().max().item()


@pytest.mark.parametrize("D", [128, 1024])
@pytest.mark.parametrize("use_xnew", [True, False])
def test_add_rms_norm_matches_float64(D, use_xnew):
    from continuum_attention_b200.rmsnorm import add_rms_norm
    g = torch.Generator().manual_seed(100 + D)
    x = torch.randn(2, 300, D, generator=g).to(DEV)
    r = (torch.randn(2, 300, D, generator=g) * 0.5).to(DEV, torch.bfloat16)
    w = (1 + 0.3 * torch.randn(D, generator=g)).to(DEV)
    gy = torch.randn(x.shape, generator=g).to(DEV, torch.bfloat16)
    gx = torch.randn(x.shape, generator=g).to(DEV)
    eps = 1e-6
    xs, rs, ws = (t.detach().clone().requires_grad_(True) for t in (x, r, w))
    xn, y = add_rms_norm(xs, rs, ws, eps)
    assert xn.dtype == torch.float32 and y.dtype == torch.bfloat16
    loss = (y.float() * gy.float()).sum() + ((xn * gx).sum() if use_xnew else 0.0)
    dx, dr, dw = torch.autograd.grad(loss, (xs, rs, ws))

    x64, r64, w64 = (t.double().requires_grad_(True) for t in (x, r, w))
    xn64 = x64 + r64
    y64 = _reference(xn64, w64, eps)
    loss64 = (y64 * gy.double()).sum() + ((xn64 * gx.double()).sum() if use_xnew else 0.0)
    rdx, rdr, rdw = torch.autograd.grad(loss64, (x64, r64, w64))
    assert (xn.double() - xn64.detach()).abs().max().item() < 1e-5
    err_y = ((y.double() - y64.detach()).abs() / y64.detach().abs().clamp_min(1e-3)).max().item()
    assert err_y < 2 ** -7, err_y
    for name, a, b, tol in (("dx", dx, rdx, 1e-4), ("dr", dr, rdr, 1e-2), ("dw", dw, rdw, 1e-4)):
        err = ((a.double() - b).abs().max() / b.abs().max()).item()
        assert err < tol, (name, err)
