"""The Continuum Attention operator: the drop-in for the reference's autograd op.

``continuum_attention(q, k, v, log_gain, query_tile=64)`` keeps the signature,
layout, dtype rules and error behaviour of the reference's public op
(cuda/continuum_attention.py:768-783, autograd class :650-766): q, k, v are
[B,H,T,D] of one dtype, ``log_gain`` is the per-head log score gain [H], the
result is [B,H,T,D] in the input dtype, gradients come back in the input
dtypes, and only first-order gradients exist.  ``query_tile`` is accepted for
signature compatibility; the reference documents it as a memory-only knob
(cuda/continuum_attention.py:958) and the fused kernels here need no query
tiling in HBM.

The work happens in the native library (include/continuum_attention_b200.h)
on the current CUDA stream; there is no CPU path.
"""
from __future__ import annotations

import math

import torch

from . import _native

_DTYPE_CODE = {torch.float32: _native.CA_DTYPE_F32, torch.bfloat16: _native.CA_DTYPE_BF16,
               torch.float16: _native.CA_DTYPE_F16}

_IMPL_CODE = {"auto": _native.CA_IMPL_AUTO, "simt": _native.CA_IMPL_SIMT,
              "tcgen05": _native.CA_IMPL_TCGEN05}

# storage order of the output o and of its gradient (q, k, v and their gradients are [B,H,T,D])
_LAYOUT_CODE = {"bhtd": _native.CA_LAYOUT_BHTD, "bthd": _native.CA_LAYOUT_BTHD}


def ctypes_ptr(t: torch.Tensor):
    return t.data_ptr() if t.numel() > 0 else None


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _validate(q, k, v, log_gain):
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("CA Q,K,V must share dtype")
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"CA expects q, k, v of one shape [B,H,T,D]; got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    if q.dtype not in _DTYPE_CODE:
        raise TypeError(f"CA supports float32, bfloat16 and float16 inputs, not {q.dtype}")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("continuum_attention_b200 runs on CUDA tensors only (no CPU fallback)")
    if k.device != q.device or v.device != q.device:
        raise RuntimeError("q, k, v must be on the same CUDA device")
    H = q.shape[1]
    if log_gain.dim() != 1 or log_gain.shape[0] != H:
        raise ValueError(f"log_gain must have shape [H]=[{H}], got {tuple(log_gain.shape)}")


def forward_raw(q, k, v, log_gain_f32, impl="auto", want_f32=False, want_stats=True, out_layout="bhtd"):
    """Run the native forward; returns (o, row_stats or None, o_f32 or None).

    q, k, v contiguous CUDA [B,H,T,D]; log_gain_f32 contiguous float32 [H] on the
    same device.  ``want_stats=False`` is the inference form (no backward follows,
    the per-row statistics are not written).  ``out_layout="bthd"`` returns o as a
    contiguous [B,T,H,D] tensor (the attention output projection's input order);
    o_f32 stays [B,H,T,D].  Used by the autograd op, the tests and the benchmark.
    """
    B, H, T, D = q.shape
    lib = _native.lib()
    o = torch.empty((B, T, H, D), dtype=q.dtype, device=q.device) if out_layout == "bthd" else torch.empty_like(q)
    stats = (torch.empty(B * H * T * lib.ca_row_stats_floats(), dtype=torch.float32, device=q.device)
             if want_stats else None)
    o32 = torch.empty(q.shape, dtype=torch.float32, device=q.device) if want_f32 else None
    with torch.cuda.device(q.device):
        st = lib.ca_forward_ex(ctypes_ptr(q), ctypes_ptr(k), ctypes_ptr(v), ctypes_ptr(log_gain_f32),
                               ctypes_ptr(o), None if o32 is None else ctypes_ptr(o32),
                               None if stats is None else ctypes_ptr(stats),
                               B, H, T, D, _DTYPE_CODE[q.dtype], _IMPL_CODE[impl], _LAYOUT_CODE[out_layout],
                               _stream(q.device))
    _native.check("ca_forward", st)
    return o, stats, o32


def workspace_bytes(B, H, T, D, dtype) -> int:
    return int(_native.lib().ca_backward_workspace_size(B, H, T, D, _DTYPE_CODE[dtype]))


def backward_raw(q, k, v, o, do, log_gain_f32, stats, want_dgain=True, impl="auto", workspace=None,
                 o_f32=None, layout="bhtd", deterministic=False):
    """Run the native backward; returns (dq, dk, dv, dlog_gain float32 [H] or None).

    ``o_f32`` (optional) is the forward's fp32 accumulator; it makes the row
    terms D_i = dO_i . O_i exact to fp32 for bf16/f16 inputs.  ``layout="bthd"``:
    o and do are contiguous [B,T,H,D] tensors.  ``deterministic``: dQ is summed in
    one fixed order, so all four gradients are bitwise reproducible (tcgen05
    kernels only; RuntimeError where the CUDA-core kernels would run).
    """
    B, H, T, D = q.shape
    lib = _native.lib()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(H, dtype=torch.float32, device=q.device) if want_dgain else None
    nbytes = workspace_bytes(B, H, T, D, q.dtype)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        st = lib.ca_backward_ex2(ctypes_ptr(q), ctypes_ptr(k), ctypes_ptr(v),
                                 None if o is None else ctypes_ptr(o), None if o_f32 is None else ctypes_ptr(o_f32),
                                 ctypes_ptr(do), ctypes_ptr(log_gain_f32), ctypes_ptr(stats), ctypes_ptr(dq),
                                 ctypes_ptr(dk), ctypes_ptr(dv), None if dg is None else ctypes_ptr(dg),
                                 workspace.data_ptr(), workspace.numel(), B, H, T, D,
                                 _DTYPE_CODE[q.dtype], _IMPL_CODE[impl], _LAYOUT_CODE[layout],
                                 _native.CA_BWD_DETERMINISTIC if deterministic else 0, _stream(q.device))
    _native.check("ca_backward", st)
    return dq, dk, dv, dg


class ContinuumAttentionFunction(torch.autograd.Function):
    """Autograd op with the reference's contract (cuda/continuum_attention.py:650-766).

    Saves q, k, v, the output and the per-row statistics (row max and
    normaliser) instead of recomputing the forward in the backward.  For
    bf16/f16 inputs the saved output is the fp32 accumulator, so the backward's
    row terms D_i = dO_i . O_i carry no output rounding.
    """

    @staticmethod
    def forward(ctx, q, k, v, log_gain, query_tile, out_layout="bhtd"):
        _validate(q, k, v, log_gain)
        if out_layout not in _LAYOUT_CODE:
            raise ValueError(f"out_layout must be one of {sorted(_LAYOUT_CODE)}")
        lg = log_gain.detach().to(device=q.device, dtype=torch.float32).contiguous()
        lowp = q.dtype != torch.float32
        # with out_layout "bthd" o is stored [B,T,H,D]; the op returns its [B,H,T,D] view
        view = (lambda t: t.transpose(1, 2)) if out_layout == "bthd" else (lambda t: t)
        if not any(ctx.needs_input_grad[:4]):
            # inference: no backward can follow, so no statistics or fp32 output are kept
            o, _, _ = forward_raw(q, k, v, lg, impl=_current_impl(), want_stats=False, out_layout=out_layout)
            return view(o)
        o, stats, o32 = forward_raw(q, k, v, lg, impl=_current_impl(), want_f32=lowp, out_layout=out_layout)
        ctx.save_for_backward(q, k, v, o32 if lowp else o, stats, lg)
        ctx.lowp = lowp
        ctx.gain_dtype = log_gain.dtype
        ctx.query_tile = int(query_tile)
        ctx.out_layout = out_layout
        return view(o)

    @staticmethod
    def backward(ctx, grad_y):
        if torch.is_grad_enabled():
            raise RuntimeError("CA analytic kernels support first-order gradients only")
        q, k, v, o_saved, stats, lg = ctx.saved_tensors
        want_dgain = bool(ctx.needs_input_grad[3])
        g = grad_y.to(q.dtype)
        # "bthd": the gradient of the [B,H,T,D] view of a [B,T,H,D] output, handed to the
        # kernels in that storage order (a copy only when it does not arrive that way)
        g = (g.transpose(1, 2) if ctx.out_layout == "bthd" else g).contiguous()
        # with the fp32 accumulator saved, the dtype-rounded output is not needed
        args = (q, k, v, None if ctx.lowp else o_saved, g, lg, stats)
        kw = dict(want_dgain=want_dgain, impl=_current_impl(), o_f32=o_saved if ctx.lowp else None,
                  layout=ctx.out_layout)
        det = _deterministic_requested()
        try:
            dq, dk, dv, dg = backward_raw(*args, deterministic=det, **kw)
        except RuntimeError as e:
            # torch.use_deterministic_algorithms(True, warn_only=True): warn and run the
            # ordinary backward where no deterministic kernel covers the inputs
            if not (det and "CA_ERR_UNSUPPORTED" in str(e) and torch.is_deterministic_algorithms_warn_only_enabled()):
                raise
            import warnings
            warnings.warn(f"continuum_attention backward is not deterministic here: {e}")
            dq, dk, dv, dg = backward_raw(*args, deterministic=False, **kw)
        return dq, dk, dv, (dg.to(ctx.gain_dtype) if dg is not None else None), None, None


_impl_override = {"impl": "auto"}
_det_override = {"on": False}


def _deterministic_requested() -> bool:
    """A bitwise-reproducible backward is asked for: deterministic_backward() or
    torch.use_deterministic_algorithms(True)."""
    return _det_override["on"] or torch.are_deterministic_algorithms_enabled()


class deterministic_backward:
    """Context manager: backward passes launched inside sum dQ in one fixed order, so
    dq, dk, dv and d log_gain are bitwise reproducible (bf16/f16 inputs with D = 64)."""

    def __init__(self, on: bool = True):
        self.on = bool(on)

    def __enter__(self):
        self.prev = _det_override["on"]
        _det_override["on"] = self.on
        return self

    def __exit__(self, *exc):
        _det_override["on"] = self.prev
        return False


def _current_impl() -> str:
    return _impl_override["impl"]


class use_impl:
    """Context manager selecting the kernel family ("auto", "simt", "tcgen05")."""

    def __init__(self, impl: str):
        if impl not in _IMPL_CODE:
            raise ValueError(f"impl must be one of {sorted(_IMPL_CODE)}")
        self.impl = impl

    def __enter__(self):
        self.prev = _impl_override["impl"]
        _impl_override["impl"] = self.impl
        return self

    def __exit__(self, *exc):
        _impl_override["impl"] = self.prev
        return False


def continuum_attention(q, k, v, log_gain, query_tile=64, *, out_layout="bhtd"):
    """Exact causal Continuum Attention on [B,H,T,D] tensors.

    Drop-in for ``continuum_attention`` (cuda/continuum_attention.py:768-783):
    scores ``exp(log_gain[h]) * q.k / sqrt(D)``, piecewise-linear key/value
    trajectories integrated exactly per segment, half-token caps on the first
    and last visible key, causal.  Returns [B,H,T,D] in the input dtype.

    ``out_layout="bthd"`` (no reference counterpart) stores the result [B,T,H,D]
    and returns its [B,H,T,D] view, so ``y.transpose(1, 2).reshape(B, T, H*D)``
    -- the attention output projection's input -- is free, and its gradient
    reaches the backward without a transposing copy.
    """
    return ContinuumAttentionFunction.apply(q.contiguous(), k.contiguous(), v.contiguous(), log_gain,
                                            int(query_tile), out_layout)


def continuum_attention_fixed_tau(q, k, v, tau: float = 0.30):
    """Fixed-temperature variant P (architecture.py:140-141, 175): gain 1/tau, no gain gradient."""
    if tau <= 0:
        raise ValueError("fixed_tau must be > 0")
    H = q.shape[1]
    lg = torch.full((H,), math.log(1.0 / tau), dtype=torch.float32, device=q.device)
    return ContinuumAttentionFunction.apply(q.contiguous(), k.contiguous(), v.contiguous(), lg, 64, "bhtd")
