"""The [B,T,H,D] output layout (ca_forward_ex / ca_backward_ex, out_layout="bthd")
computes exactly what the [B,H,T,D] layout computes: the same kernels, only the
rows of o and dO are placed differently."""
import pytest
import torch

import continuum_attention_b200 as ca

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(q, k, v, lg, dy, layout, impl, grad_as_projection):
    qs, ks, vs = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    lgs = lg.detach().clone().requires_grad_(True)
    with ca.use_impl(impl):
        y = ca.continuum_attention(qs, ks, vs, lgs, 64, out_layout=layout)
        B, H, T, D = y.shape
        if grad_as_projection:
            # as in a decoder: the output projection reads y as [B,T,H*D]
            z = y.transpose(1, 2).reshape(B, T, H * D)
            loss = (z.float() * dy.transpose(1, 2).reshape(B, T, H * D).float()).sum()
        else:
            loss = (y.float() * dy.float()).sum()
        grads = torch.autograd.grad(loss, (qs, ks, vs, lgs))
    torch.cuda.synchronize()
    return y.detach(), grads


@pytest.mark.parametrize("dtype,impl", [(torch.bfloat16, "auto"), (torch.float16, "tcgen05"),
                                        (torch.bfloat16, "simt"), (torch.float32, "auto")])
@pytest.mark.parametrize("grad_as_projection", [True, False])
@pytest.mark.parametrize("T", [333, 400])   # natural key order; permuted (T % 16 == 0) with a partial tile
def test_bthd_layout_matches_bhtd(dtype, impl, grad_as_projection, T):
    g = torch.Generator().manual_seed(11)
    shape = (2, 3, T, 64)
    q, k, v, dy = (torch.randn(shape, generator=g).to(DEV, dtype) for _ in range(4))
    lg = torch.tensor([0.0, 0.3, -0.2], device=DEV)
    y0, g0 = _run(q, k, v, lg, dy, "bhtd", impl, grad_as_projection)
    y1, g1 = _run(q, k, v, lg, dy, "bthd", impl, grad_as_projection)
    assert y1.shape == y0.shape and y1.transpose(1, 2).is_contiguous()
    assert torch.equal(y0, y1)
    for name, a, b in zip(("dq", "dk", "dv", "dlog_gain"), g1, g0):
        if name == "dq":   # fp32 accumulation order across key tiles is not fixed
            err = ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()
            assert err < (1e-5 if dtype == torch.float32 else 1e-2), (name, err)
        else:
            assert torch.equal(a, b), name


def test_bthd_inference_and_errors():
    g = torch.Generator().manual_seed(12)
    q, k, v = (torch.randn(1, 2, 130, 64, generator=g).to(DEV, torch.bfloat16) for _ in range(3))
    lg = torch.zeros(2, device=DEV)
    with torch.no_grad():
        y0 = ca.continuum_attention(q, k, v, lg, 64)
        y1 = ca.continuum_attention(q, k, v, lg, 64, out_layout="bthd")
    assert torch.equal(y0, y1)
    with pytest.raises(ValueError):
        ca.continuum_attention(q, k, v, lg, 64, out_layout="tbhd")
