"""Fused rotary embedding + QKV unpacking (ca_rope_qkv_forward / _backward) against the
torch formulation of apply_rope (cuda/continuum_attention.py:825-835) in float64."""
import pytest
import torch

from continuum_attention_b200 import _native
from continuum_attention_b200.rope import apply_rope_torch, cos_sin_table, rope_qkv

pytestmark = pytest.mark.gpu

THETA = 10000.0


def reference(qkv64, heads):
    """float64 q, k, v [B,H,T,D] from the projection output [B,T,3C]."""
    B, T, C3 = qkv64.shape
    D = C3 // (3 * heads)
    q, k, v = qkv64.reshape(B, T, 3, heads, D).permute(2, 0, 3, 1, 4).unbind(0)
    q, k = apply_rope_torch(q, k, THETA)
    return q, k, v


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 37, 3, 64), (1, 128, 16, 64), (2, 5, 2, 8), (1, 33, 2, 128)])
def test_rope_qkv_forward_backward(dtype, shape):
    B, T, H, D = shape
    g = torch.Generator().manual_seed(B * 1000 + T * 10 + H)
    qkv = torch.randn(B, T, 3 * H * D, generator=g).to("cuda", dtype)
    qkv64 = qkv.double().cpu().requires_grad_(True)
    ref = reference(qkv64, H)
    x = qkv.detach().requires_grad_(True)
    out = rope_qkv(x, H, THETA)
    # tables are computed in float32 like the reference's; one rounding per output element
    ulp = {torch.float32: 2.0 ** -22, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -10}[dtype]
    for name, o, r in zip("qkv", out, ref):
        assert o.shape == (B, H, T, D) and o.is_contiguous()
        err = (o.double().cpu() - r.detach()).abs()
        bound = ulp * r.detach().abs() + 4e-6 * r.detach().abs().max() + 1e-7
        assert bool((err <= bound).all()), f"{name}: max err {err.max().item():.3e}"
    grads = [torch.randn(B, H, T, D, generator=g).to("cuda", dtype) for _ in range(3)]
    dx, = torch.autograd.grad(out, x, grads)
    dref, = torch.autograd.grad(ref, qkv64, [t.double().cpu() for t in grads])
    err = (dx.double().cpu() - dref).abs()
    bound = 2 * ulp * dref.abs() + 4e-6 * dref.abs().max() + 1e-7
    assert bool((err <= bound).all()), f"dqkv max err {err.max().item():.3e}"


def test_rope_qkv_table_and_errors():
    tab = cos_sin_table(16, 64, THETA, torch.device("cuda"))
    assert tab.shape == (16, 32, 2) and tab.dtype == torch.float32
    assert torch.equal(tab[0, :, 0].cpu(), torch.ones(32)) and torch.equal(tab[0, :, 1].cpu(), torch.zeros(32))
    lib = _native.lib()
    x = torch.zeros(1, 4, 3 * 2 * 12, device="cuda", dtype=torch.bfloat16)
    q = torch.empty(1, 2, 4, 12, device="cuda", dtype=torch.bfloat16)
    t12 = torch.zeros(4, 6, 2, device="cuda")
    st = lib.ca_rope_qkv_forward(x.data_ptr(), t12.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                 1, 4, 2, 12, 1, None)
    assert st == 2 and b"multiple of 8" in lib.ca_last_error()          # D = 12 unsupported
    st = lib.ca_rope_qkv_forward(x.data_ptr() + 2, t12.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                 1, 4, 2, 8, 1, None)
    assert st == 1 and b"aligned" in lib.ca_last_error()
    st = lib.ca_rope_qkv_forward(None, None, None, None, None, 0, 4, 2, 64, 1, None)
    assert st == 0                                                       # empty problem: no-op
