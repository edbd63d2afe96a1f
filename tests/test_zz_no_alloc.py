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


def _noalloc_backward(q, k, v, o, o32, do, lg, stats, impl=0):
    """ca_backward_noalloc through the C ABI; pass o (fp32 inputs) or o32 (bf16/f16 inputs)."""
    B, H, T, D = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(H, dtype=torch.float32, device=q.device)
    st = _native.lib().ca_backward_noalloc(
        _p(q), _p(k), _p(v), _p(o), _p(o32), _p(do), _p(lg), _p(stats), _p(dq), _p(dk), _p(dv), _p(dg),
        B, H, T, D, CODES[q.dtype], impl, torch.cuda.current_stream().cuda_stream)
    _native.check("ca_backward_noalloc", st)
    return dq, dk, dv, dg


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm()))


IMPLS = {"auto": 0, "simt": 1}


def _check_two_calls(shape, dtype, impl, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q, k, v, do = (torch.randn(shape, generator=g).to("cuda", dtype) for _ in range(4))
    lg = (torch.rand(shape[1], generator=g) - 0.5).to("cuda")
    lowp = dtype != torch.float32
    o, stats, o32 = forward_raw(q, k, v, lg, want_f32=lowp, impl=impl)
    ref = backward_raw(q, k, v, o, do, lg, stats, o_f32=o32, impl=impl)
    for call in range(2):
        got = _noalloc_backward(q, k, v, None if lowp else o, o32, do, lg, stats, impl=IMPLS[impl])
        torch.cuda.synchronize()
        # dk, dv and d log_gain come out of fixed-order reductions: bit-identical to the
        # workspace entry point.  dq is summed by reduce-adds in whatever order the key
        # tiles finish, so it may differ in the last bits: cosine / normalised error.
        for name, a, b in zip(("dk", "dv", "dlog_gain"), got[1:], ref[1:]):
            assert torch.equal(a, b), f"call {call}: {name} differs from ca_backward"
        a, b = got[0], ref[0]
        assert torch.isfinite(a.float()).all(), f"call {call}: dq not finite"
        if lowp:
            assert _cos(a, b) >= 0.9999, f"call {call}: dq cosine {_cos(a, b):.6f}"
        err = (a.double() - b.double()).abs().max().item() / b.double().abs().max().item()
        assert err <= (1e-2 if lowp else 1e-4), f"call {call}: dq normalised max error {err:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_backward_on_two_calls(dtype):
    _check_two_calls((2, 4, 600, 64), dtype, "auto", 77)


@pytest.mark.gpu
def test_noalloc_cuda_core_kernels_on_two_calls():
    _check_two_calls((1, 3, 333, 64), torch.bfloat16, "simt", 78)


@pytest.mark.gpu
def test_noalloc_near_its_limit():
    # a problem whose scratch fills most of the fixed array
    shape = (1, 8, 15000, 64)
    need = _native.lib().ca_backward_workspace_size(*shape, 1)
    assert 28 << 20 < need <= 32 << 20
    _check_two_calls(shape, torch.bfloat16, "auto", 79)


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
