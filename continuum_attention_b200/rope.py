"""Rotary embedding fused with the QKV unpacking of the CA-S attention block.

``rope_qkv(qkv, heads, theta)`` takes the projection output ``[B, T, 3*C]``
(C = heads * D) and returns contiguous ``q, k, v`` of shape ``[B, H, T, D]``
with the rotary embedding of ``apply_rope`` (cuda/continuum_attention.py:825-835)
applied to q and k.  On CUDA tensors it is one native kernel each way
(``ca_rope_qkv_forward`` / ``ca_rope_qkv_backward``), replacing the reshape /
permute / unbind (:850-852), the dozen elementwise kernels of apply_rope and
the operand copies of the attention op.  CPU tensors take the plain torch
formulation (used by the CPU tests of the decoder).
"""
from __future__ import annotations

import threading

import torch

from . import _native
from .attention import _DTYPE_CODE, _stream, ctypes_ptr

_tables = {}
_tables_lock = threading.Lock()


def rope_phase(T: int, D: int, theta: float, device) -> torch.Tensor:
    """Phase table [T, D/2] in float32, computed as the reference computes it."""
    freq = 1.0 / (theta ** (torch.arange(0, D, 2, device=device, dtype=torch.float32) / D))
    pos = torch.arange(T, device=device, dtype=torch.float32)
    return torch.outer(pos, freq)


def cos_sin_table(T: int, D: int, theta: float, device) -> torch.Tensor:
    """float32 [T, D/2, 2] = (cos, sin) of the phase table, cached per device."""
    key = (T, D, float(theta), str(device))
    tab = _tables.get(key)
    if tab is None:
        with _tables_lock:
            tab = _tables.get(key)
            if tab is None:
                ph = rope_phase(T, D, theta, device)
                tab = torch.stack((ph.cos(), ph.sin()), -1).contiguous()
                _tables[key] = tab
    return tab


def apply_rope_torch(q, k, theta: float):
    """The torch formulation of the rotary embedding on interleaved pairs."""
    ph = rope_phase(q.shape[-2], q.shape[-1], theta, q.device)
    cos = torch.repeat_interleave(ph.cos(), 2, -1).to(q.dtype)[None, None]
    sin = torch.repeat_interleave(ph.sin(), 2, -1).to(q.dtype)[None, None]

    def rotate(t):
        return torch.stack((-t[..., 1::2], t[..., 0::2]), -1).flatten(-2)

    return q * cos + rotate(q) * sin, k * cos + rotate(k) * sin


class RopeQKVFunction(torch.autograd.Function):
    """qkv [B,T,3,H,D] -> (q, k, v) [B,H,T,D] with q, k rotated; native both ways."""

    @staticmethod
    def forward(ctx, qkv5, cos_sin):
        B, T, three, H, D = qkv5.shape
        qkv5 = qkv5.contiguous()
        q = torch.empty(B, H, T, D, dtype=qkv5.dtype, device=qkv5.device)
        k, v = torch.empty_like(q), torch.empty_like(q)
        with torch.cuda.device(qkv5.device):
            st = _native.lib().ca_rope_qkv_forward(
                ctypes_ptr(qkv5), ctypes_ptr(cos_sin), ctypes_ptr(q), ctypes_ptr(k), ctypes_ptr(v),
                B, T, H, D, _DTYPE_CODE[qkv5.dtype], _stream(qkv5.device))
        _native.check("ca_rope_qkv_forward", st)
        ctx.save_for_backward(cos_sin)
        ctx.shape = (B, T, H, D)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        (cos_sin,) = ctx.saved_tensors
        B, T, H, D = ctx.shape
        ref = next(g for g in (dq, dk, dv) if g is not None)
        grads = [torch.zeros_like(ref) if g is None else g.contiguous() for g in (dq, dk, dv)]
        dqkv = torch.empty(B, T, 3, H, D, dtype=ref.dtype, device=ref.device)
        with torch.cuda.device(ref.device):
            st = _native.lib().ca_rope_qkv_backward(
                ctypes_ptr(grads[0]), ctypes_ptr(grads[1]), ctypes_ptr(grads[2]), ctypes_ptr(cos_sin),
                ctypes_ptr(dqkv), B, T, H, D, _DTYPE_CODE[ref.dtype], _stream(ref.device))
        _native.check("ca_rope_qkv_backward", st)
        return dqkv, None


def rope_qkv(qkv: torch.Tensor, heads: int, theta: float):
    """Split the projection output [B, T, 3*C] into rotated q, k and v, each [B, H, T, D]."""
    B, T, C3 = qkv.shape
    D = C3 // (3 * heads)
    qkv5 = qkv.reshape(B, T, 3, heads, D)
    if not qkv.is_cuda:
        q, k, v = qkv5.permute(2, 0, 3, 1, 4).unbind(0)
        q, k = apply_rope_torch(q, k, theta)
        return q, k, v
    return RopeQKVFunction.apply(qkv5, cos_sin_table(T, D, theta, qkv.device))
