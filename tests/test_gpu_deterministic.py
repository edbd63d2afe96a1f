"""The deterministic backward (CA_BWD_DETERMINISTIC): dQ's key-tile contributions
are summed in one fixed order, so every gradient is bitwise reproducible run to
run, as the reference's per-query-tile accumulation is
(cuda/continuum_attention.py:754-764)."""
import warnings

import pytest
import torch

import continuum_attention_b200 as ca
from ca_testlib import cosine, gen_inputs

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _grads(q, k, v, lg, dy, det, layout="bhtd", runs=2):
    o, stats, o32 = ca.forward_raw(q, k, v, lg, want_f32=True, out_layout=layout)
    do = dy.transpose(1, 2).contiguous() if layout == "bthd" else dy
    return [ca.backward_raw(q, k, v, None, do, lg, stats, o_f32=o32, layout=layout, deterministic=det)
            for _ in range(runs)]


@pytest.mark.parametrize("shape,layout", [((2, 4, 600, 64), "bhtd"), ((2, 16, 2048, 64), "bhtd"),
                                          ((1, 3, 1000, 64), "bthd")])
def test_deterministic_backward_is_bitwise_reproducible(shape, layout):
    q, k, v, dy = (t.to(DEV, torch.bfloat16) for t in gen_inputs(shape, 91, qk_mag=1.5))
    lg = torch.linspace(-0.3, 0.4, shape[1], device=DEV)
    a, b = _grads(q, k, v, lg, dy, True, layout)
    for name, x, y in zip(("dq", "dk", "dv", "dlog_gain"), a, b):
        assert torch.equal(x, y), f"{name} differs between two deterministic runs"
    # the ordinary mode differs only in dQ's summation order
    c = _grads(q, k, v, lg, dy, False, layout, runs=1)[0]
    for name, x, y in zip(("dk", "dv", "dlog_gain"), a[1:], c[1:]):
        assert torch.equal(x, y), f"{name} differs between the modes"
    assert cosine(a[0], c[0]) >= 0.99999


def test_deterministic_backward_against_oracle():
    from oracle.ca_oracle import ca_forward_backward
    shape = (1, 2, 384, 64)
    q, k, v, dy = (t.to(DEV, torch.bfloat16) for t in gen_inputs(shape, 92, qk_mag=2.0, dup_frac=0.1))
    lg = torch.tensor([0.0, 0.5], device=DEV)
    got = _grads(q, k, v, lg, dy, True, runs=1)[0]
    ref = ca_forward_backward(*(t.double().cpu() for t in (q, k, v)), lg.double().cpu(), dy.double().cpu())
    for name, x, y in zip(("dq", "dk", "dv"), got[:3], ref[1:4]):
        assert cosine(x, y) >= 0.9999, name


def test_op_honours_deterministic_modes():
    q, k, v, dy = (t.to(DEV, torch.bfloat16) for t in gen_inputs((1, 2, 512, 64), 93))
    lg = torch.zeros(2, device=DEV, requires_grad=True)

    def grads():
        qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
        y = ca.continuum_attention(qq, kk, vv, lg)
        return torch.autograd.grad(y, (qq, kk, vv, lg), dy)

    with ca.deterministic_backward():
        g1, g2 = grads(), grads()
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))
    prev = torch.are_deterministic_algorithms_enabled()
    try:
        torch.use_deterministic_algorithms(True)
        g3 = grads()
        assert all(torch.equal(a, b) for a, b in zip(g1, g3))
        # fp32 inputs run the CUDA-core kernels, which have no deterministic dQ
        q32, k32, v32 = (t.float().detach().requires_grad_(True) for t in (q, k, v))
        with pytest.raises(RuntimeError, match="deterministic"):
            torch.autograd.grad(ca.continuum_attention(q32, k32, v32, lg), (q32,), dy.float())
        torch.use_deterministic_algorithms(True, warn_only=True)
        with warnings.catch_warnings(record=True) as w:
            warnings.simplefilter("always")
            y = ca.continuum_attention(q32, k32, v32, lg)
            torch.autograd.grad(y, (q32,), dy.float())
        assert any("not deterministic" in str(x.message) for x in w)
    finally:
        torch.use_deterministic_algorithms(prev)
