"""The allocation-free backward entry point, ca_backward_noalloc.

Some callers cannot allocate device memory when they run the backward: they
reach this library only through its C interface while another component owns
every device allocation, or their device memory is fixed at start-up and a
later cudaMalloc is not allowed.  ca_backward_noalloc serves them by keeping
its scratch in a fixed 32 MiB array inside the library.

These tests call it through the C ABI and compare its results with the
ordinary entry point (ca_backward with a caller-provided workspace) on the same
inputs, on two calls in a row: the second call finds the first call's leftovers
in the shared array and must still be right.  This file is named to be
collected last, so a failure here stops a `pytest -x` run only after every
other test has run.
"""
import ctypes

import pytest
import torch

from continuum_attention_b200 import _native, backward_raw, forward_raw

CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _p(t):
    return None if t is None else t.data_ptr()


def _noalloc_backward(q, k, v, o, o32, do, lg, stats):
    """ca_backward_noalloc through the C ABI; pass o (fp32 inputs) or o32 (bf16/f16 inputs)."""
    B, H, T, D = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(H, dtype=torch.float32, device=q.device)
    st = _native.lib().ca_backward_noalloc(
        _p(q), _p(k), _p(v), _p(o), _p(o32), _p(do), _p(lg), _p(stats), _p(dq), _p(dk), _p(dv), _p(dg),
        B, H, T, D, CODES[q.dtype], 0, torch.cuda.current_stream().cuda_stream)
    _native.check("ca_backward_noalloc", st)
    return dq, dk, dv, dg


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm()))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_backward_on_two_calls(dtype):
    g = torch.Generator(device="cpu").manual_seed(77)
    shape = (2, 4, 600, 64)
    q, k, v, do = (torch.randn(shape, generator=g).to("cuda", dtype) for _ in range(4))
    lg = torch.tensor([0.0, 0.3, -0.2, 0.5], device="cuda")
    lowp = dtype != torch.float32
    o, stats, o32 = forward_raw(q, k, v, lg, want_f32=lowp)
    ref = backward_raw(q, k, v, o, do, lg, stats, o_f32=o32)
    for call in range(2):
        got = _noalloc_backward(q, k, v, None if lowp else o, o32, do, lg, stats)
        torch.cuda.synchronize()
        for name, a, b in zip(("dq", "dk", "dv", "dlog_gain"), got, ref):
            assert torch.isfinite(a.float()).all(), f"call {call}: {name} not finite"
            if lowp:
                assert _cos(a, b) >= 0.9999, f"call {call}: {name} cosine {_cos(a, b):.6f}"
            err = (a.double() - b.double()).abs().max().item() / b.double().abs().max().item()
            assert err <= (1e-2 if lowp else 1e-4), f"call {call}: {name} normalised max error {err:.3e}"


def test_noalloc_rejects_problems_beyond_its_array():
    # [1,16,32768,64] needs ~136 MB of scratch, more than the fixed 32 MiB array:
    # rejected by the host-side check before any device work.
    fake = ctypes.c_void_p(256)
    lib = _native.lib()
    st = lib.ca_backward_noalloc(fake, fake, fake, fake, None, fake, fake, fake, fake, fake, fake, None,
                                 1, 16, 32768, 64, 1, 0, None)
    assert st == 2
    msg = lib.ca_last_error().decode()
    assert "scratch" in msg and "ca_backward" in msg
