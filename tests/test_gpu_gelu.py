"""Native tanh-approximate GELU (ca_gelu_tanh_forward / _backward) against float64.

The reference MLP's activation is F.gelu(fc1(x), approximate='tanh')
(cuda/continuum_attention.py:866-867).  The kernels compute it in fp32 and store
in the input dtype, so the bar is fp32 rounding for fp32 and one rounding of the
storage type for bf16 / fp16 (checked against the float64 value and against
torch's own kernel in the same dtype).
"""
import math

import pytest
import torch
import torch.nn.functional as F

from continuum_attention_b200 import _native
from continuum_attention_b200.gelu import gelu_tanh, supported

pytestmark = pytest.mark.gpu

_C = math.sqrt(2.0 / math.pi)
_K = 0.044715


def _ref(x):
    # 0.5 (1 + tanh u) = sigmoid(2u), written so that float64 keeps its precision
    # where 1 + tanh u cancels (x below about -5)
    x = x.double()
    u = _C * (x + _K * x ** 3)
    s = torch.sigmoid(2 * u)
    y = x * s
    d = s + 2 * x * s * (1 - s) * _C * (1 + 3 * _K * x * x)
    return y, d


def _inputs(dtype, n=1 << 16, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g) * 3
    special = torch.tensor([-100.0, -30.0, -10.0, -5.0, -1.0, -1e-3, -1e-20, 0.0, 1e-20, 1e-3, 1.0, 5.0,
                            10.0, 30.0, 100.0, 0.5])
    x[:special.numel()] = special
    dy = torch.randn(n, generator=g)
    return x.to("cuda", dtype), dy.to("cuda", dtype)


# |out - ref| <= rel * |ref| + floor (+ 1e-6 |dy| for the gradient, whose two terms
# cancel near gelu's minimum).  fp32: the exponent argument z = 2u carries fp32
# rounding, which exp amplifies by |z|, so rel = 2e-6 + 2 eps |z|; 16-bit types:
# one rounding of the storage type.
def _bound(dtype, x, ref, dy=None):
    z = 2 * _C * (x.double() + _K * x.double() ** 3)
    if dtype == torch.float32:
        rel, floor = 2e-6 + 2.4e-7 * z.abs(), 1e-30
    elif dtype == torch.bfloat16:
        rel, floor = 2.0 ** -8 + 0 * z, 1e-30
    else:
        rel, floor = 2.0 ** -10 + 0 * z, 6e-8
    bound = rel * ref.abs() + floor
    if dy is not None:
        bound = bound + 1e-6 * dy.double().abs()
    return bound


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_forward_backward_against_float64(dtype):
    x, dy = _inputs(dtype)
    xr = x.detach().clone().requires_grad_(True)
    y = gelu_tanh(xr)
    (dx,) = torch.autograd.grad(y, xr, dy)
    torch.cuda.synchronize()
    yr, dr = _ref(x)
    gr = dr * dy.double()
    for name, out, ref, bound in (("y", y, yr, _bound(dtype, x, yr)), ("dx", dx, gr, _bound(dtype, x, gr, dy))):
        assert torch.isfinite(out).all()
        excess = (out.double() - ref).abs() - bound
        worst = excess.max().item()
        i = int(excess.argmax())
        assert worst <= 0, (f"{dtype} {name}: at x={x[i].item():.6g} got {out[i].item():.9g}, "
                            f"float64 {ref[i].item():.9g}, bound {bound[i].item():.3e}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_matches_torch_kernel_within_one_rounding(dtype):
    x, dy = _inputs(dtype, seed=1)
    xr = x.detach().clone().requires_grad_(True)
    xt = x.detach().clone().requires_grad_(True)
    y = gelu_tanh(xr)
    yt = F.gelu(xt, approximate="tanh")
    (dx,) = torch.autograd.grad(y, xr, dy)
    (dxt,) = torch.autograd.grad(yt, xt, dy)
    # torch evaluates 0.5 x (1 + tanh u) and 1 - tanh^2 u in fp32, which cancel for
    # x below about -3 (absolute errors up to ~1e-5 in the gradient there): an
    # absolute allowance of 2e-5 |dy| covers them; elsewhere one storage rounding
    eps = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    for a, b, slack in ((y, yt, 1e-6), (dx, dxt, 2e-5)):
        diff = (a.float() - b.float()).abs()
        assert (diff <= eps * b.float().abs() + slack * (1 + dy.float().abs())).all()


def test_rejects_unsupported_and_counts_one_launch():
    x = torch.randn(12, device="cuda", dtype=torch.bfloat16)
    assert not supported(x)
    with pytest.raises(ValueError):
        gelu_tanh(x)
    x = torch.randn(64, device="cuda", dtype=torch.bfloat16)
    gelu_tanh(x)
    assert _native.lib().ca_last_launch_count() == 1
