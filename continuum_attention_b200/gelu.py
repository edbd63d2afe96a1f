"""Tanh-approximate GELU of the CA-S decoder MLP as native kernels.

``gelu_tanh(x)`` is ``F.gelu(x, approximate='tanh')`` (the reference MLP,
cuda/continuum_attention.py:866-867) with one native kernel forward and one
backward (``ca_gelu_tanh_forward`` / ``ca_gelu_tanh_backward``): fp32 arithmetic,
the result in x's dtype, 16-byte vector access over the contiguous tensor.
"""
from __future__ import annotations

import torch

from . import _native
from .attention import ctypes_ptr

_CODE = {torch.float32: _native.CA_DTYPE_F32, torch.bfloat16: _native.CA_DTYPE_BF16,
         torch.float16: _native.CA_DTYPE_F16}


def supported(x: torch.Tensor) -> bool:
    """True when the native kernels cover x: CUDA, f32/bf16/f16, contiguous, 16-byte
    aligned, and a whole number of 16-byte vectors."""
    if not (x.is_cuda and x.dtype in _CODE and x.is_contiguous()):
        return False
    return x.data_ptr() % 16 == 0 and (x.numel() * x.element_size()) % 16 == 0


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


class GeluTanhFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = torch.empty_like(x)
        with torch.cuda.device(x.device):
            st = _native.lib().ca_gelu_tanh_forward(ctypes_ptr(x), ctypes_ptr(y), x.numel(), _CODE[x.dtype],
                                                    _stream(x))
        _native.check("ca_gelu_tanh_forward", st)
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dy = dy.to(x.dtype).contiguous()
        if not supported(dy):
            dy = dy.clone()
        dx = torch.empty_like(x)
        with torch.cuda.device(x.device):
            st = _native.lib().ca_gelu_tanh_backward(ctypes_ptr(x), ctypes_ptr(dy), ctypes_ptr(dx), x.numel(),
                                                     _CODE[x.dtype], _stream(x))
        _native.check("ca_gelu_tanh_backward", st)
        return dx


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """F.gelu(x, approximate='tanh') on the native kernels; x must satisfy ``supported``."""
    if not supported(x):
        raise ValueError("gelu_tanh: needs a contiguous, 16-byte aligned CUDA tensor of f32/bf16/f16 "
                         "holding a whole number of 16-byte vectors")
    return GeluTanhFunction.apply(x)
