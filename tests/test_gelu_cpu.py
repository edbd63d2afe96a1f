"""CPU checks of the math the native GELU kernels compute (csrc/ca_gelu.cu).

The kernels evaluate the reference MLP's tanh-approximate GELU
(cuda/continuum_attention.py:866-867) in the sigmoid form
x * sigmoid(2u), u = sqrt(2/pi) (x + 0.044715 x^3), and its derivative
s + 2 x s (1 - s) du/dx.  Here, in float64, both forms are checked against
torch's own tanh-form GELU and its autograd derivative where those do not cancel.
"""
import math

import torch
import torch.nn.functional as F

from continuum_attention_b200.gelu import supported

_C = math.sqrt(2.0 / math.pi)
_K = 0.044715


def test_sigmoid_form_equals_tanh_form_and_its_derivative():
    x = torch.linspace(-4.0, 6.0, 2001, dtype=torch.float64, requires_grad=True)
    y_t = F.gelu(x, approximate="tanh")
    (d_t,) = torch.autograd.grad(y_t.sum(), x)
    xd = x.detach()
    u = _C * (xd + _K * xd ** 3)
    s = torch.sigmoid(2 * u)
    y_s = xd * s
    d_s = s + 2 * xd * s * (1 - s) * _C * (1 + 3 * _K * xd * xd)
    assert torch.allclose(y_s, y_t.detach(), rtol=1e-12, atol=1e-13)
    assert torch.allclose(d_s, d_t, rtol=1e-10, atol=1e-12)


def test_native_gelu_is_cuda_only():
    assert not supported(torch.zeros(16, dtype=torch.bfloat16))
