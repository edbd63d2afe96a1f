"""RMSNorm of the CA-S decoder block as native kernels.

``rms_norm(x, weight, eps, out_dtype)`` computes ``weight * x * rsqrt(mean(x^2)
+ eps)`` over the last axis (the reference module RMSNorm,
cuda/continuum_attention.py:815-821) with one native kernel forward and two
backward (``ca_rmsnorm_forward`` / ``ca_rmsnorm_backward``).  The output may be
written directly in the dtype the following projection consumes (bfloat16 under
autocast), which saves the separate cast; the gradient of ``weight`` is summed
over rows in a fixed order.
"""
from __future__ import annotations

import torch

from . import _native
from .attention import ctypes_ptr

_CODE = {torch.float32: _native.CA_DTYPE_F32, torch.bfloat16: _native.CA_DTYPE_BF16}
_DIMS = (128, 256, 512, 1024)


def supported(x: torch.Tensor, out_dtype: torch.dtype) -> bool:
    """True when the native kernels cover this call (CUDA, D in 128/256/512/1024,
    float32 or bfloat16 input and output)."""
    return x.is_cuda and x.shape[-1] in _DIMS and x.dtype in _CODE and out_dtype in _CODE


class RMSNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps: float, out_dtype):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        rows = x2.shape[0]
        w = weight.detach().to(torch.float32).contiguous()
        y = torch.empty(x2.shape, dtype=out_dtype, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        lib = _native.lib()
        with torch.cuda.device(x.device):
            st = lib.ca_rmsnorm_forward(ctypes_ptr(x2), ctypes_ptr(w), ctypes_ptr(y), ctypes_ptr(rstd), rows, D,
                                        float(eps), _CODE[x.dtype], _CODE[out_dtype],
                                        torch.cuda.current_stream(x.device).cuda_stream)
        _native.check("ca_rmsnorm_forward", st)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        ctx.out_dtype = out_dtype
        ctx.weight_dtype = weight.dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        rows, D = x2.shape
        dy2 = dy.reshape(-1, D).to(ctx.out_dtype).contiguous()
        dx = torch.empty_like(x2)
        dw = torch.empty(D, dtype=torch.float32, device=x2.device)
        lib = _native.lib()
        ws = torch.empty(max(int(lib.ca_rmsnorm_workspace_size(rows, D)), 16), dtype=torch.uint8, device=x2.device)
        with torch.cuda.device(x2.device):
            st = lib.ca_rmsnorm_backward(ctypes_ptr(x2), ctypes_ptr(w), ctypes_ptr(dy2), ctypes_ptr(rstd),
                                         ctypes_ptr(dx), ctypes_ptr(dw), ws.data_ptr(), ws.numel(), rows, D,
                                         _CODE[x2.dtype], _CODE[ctx.out_dtype],
                                         torch.cuda.current_stream(x2.device).cuda_stream)
        _native.check("ca_rmsnorm_backward", st)
        return dx.view(ctx.shape), dw.to(ctx.weight_dtype), None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out_dtype=None) -> torch.Tensor:
    """Native RMSNorm; ``out_dtype`` defaults to the input dtype.  Raises when the
    native kernels do not cover the call (see ``supported``)."""
    out_dtype = out_dtype or x.dtype
    if not supported(x, out_dtype):
        raise ValueError(f"native rms_norm covers CUDA float32/bfloat16 tensors with last dim in {_DIMS}; "
                         f"got {x.device} {x.dtype} -> {out_dtype}, last dim {x.shape[-1]}")
    return RMSNormFunction.apply(x, weight, eps, out_dtype)


class AddRMSNormFunction(torch.autograd.Function):
    """(x_new, y) = (x + r, rms_norm(x + r)) with x float32 and r, y bfloat16."""

    @staticmethod
    def forward(ctx, x, r, weight, eps: float):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        r2 = r.reshape(-1, D).contiguous()
        rows = x2.shape[0]
        w = weight.detach().to(torch.float32).contiguous()
        xn = torch.empty_like(x2)
        y = torch.empty(x2.shape, dtype=torch.bfloat16, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        lib = _native.lib()
        with torch.cuda.device(x.device):
            st = lib.ca_add_rmsnorm_forward(ctypes_ptr(x2), ctypes_ptr(r2), ctypes_ptr(w), ctypes_ptr(xn),
                                            ctypes_ptr(y), ctypes_ptr(rstd), rows, D, float(eps),
                                            torch.cuda.current_stream(x.device).cuda_stream)
        _native.check("ca_add_rmsnorm_forward", st)
        ctx.save_for_backward(xn, w, rstd)
        ctx.shape = x.shape
        ctx.weight_dtype = weight.dtype
        return xn.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, g_xn, g_y):
        xn, w, rstd = ctx.saved_tensors
        rows, D = xn.shape
        dy = (torch.zeros_like(xn, dtype=torch.bfloat16) if g_y is None
              else g_y.reshape(-1, D).to(torch.bfloat16).contiguous())
        gx = None if g_xn is None else g_xn.reshape(-1, D).to(torch.float32).contiguous()
        dx = torch.empty_like(xn)
        dr = torch.empty(xn.shape, dtype=torch.bfloat16, device=xn.device)
        dw = torch.empty(D, dtype=torch.float32, device=xn.device)
        lib = _native.lib()
        ws = torch.empty(max(int(lib.ca_rmsnorm_workspace_size(rows, D)), 16), dtype=torch.uint8, device=xn.device)
        with torch.cuda.device(xn.device):
            st = lib.ca_add_rmsnorm_backward(ctypes_ptr(xn), ctypes_ptr(w), ctypes_ptr(dy), ctypes_ptr(rstd),
                                             None if gx is None else ctypes_ptr(gx), ctypes_ptr(dx), ctypes_ptr(dr),
                                             ctypes_ptr(dw), ws.data_ptr(), ws.numel(), rows, D,
                                             torch.cuda.current_stream(xn.device).cuda_stream)
        _native.check("ca_add_rmsnorm_backward", st)
        return dx.view(ctx.shape), dr.view(ctx.shape), dw.to(ctx.weight_dtype), None


def add_supported(x: torch.Tensor, r: torch.Tensor) -> bool:
    """True when the fused residual add + norm covers the call: CUDA, x float32,
    r bfloat16 of the same shape, last dim in 128/256/512/1024."""
    return (x.is_cuda and r.is_cuda and x.dtype == torch.float32 and r.dtype == torch.bfloat16
            and x.shape == r.shape and x.shape[-1] in _DIMS)


def add_rms_norm(x: torch.Tensor, r: torch.Tensor, weight: torch.Tensor, eps: float):
    """(x + r, rms_norm(x + r)) in one native kernel; the normalised output is
    bfloat16.  Raises when ``add_supported`` is false."""
    if not add_supported(x, r):
        raise ValueError("native add_rms_norm covers CUDA float32 x with bfloat16 r of the same shape and last "
                         f"dim in {_DIMS}; got {x.dtype}/{r.dtype} {tuple(x.shape)}/{tuple(r.shape)}")
    return AddRMSNormFunction.apply(x, r, weight, eps)
