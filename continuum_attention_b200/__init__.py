"""B200-native (sm_100a) Continuum Attention.

Public API (mirrors the reference project's operator):
    continuum_attention(q, k, v, log_gain, query_tile=64)   learned per-head gain (S/H)
    continuum_attention_fixed_tau(q, k, v, tau=0.30)        fixed temperature (P)
    ContinuumAttentionFunction                              the torch.autograd.Function
    use_impl("simt" | "tcgen05" | "auto")                   kernel-family override
    deterministic_backward(True)                            bitwise-reproducible dQ (also
                                                            under torch.use_deterministic_algorithms)

The kernels live in the native library libca_b200.so (C ABI in
include/continuum_attention_b200.h); build it with
``python -m continuum_attention_b200.build``.
"""
from .attention import (ContinuumAttentionFunction, backward_raw, continuum_attention,
                        continuum_attention_fixed_tau, deterministic_backward, forward_raw, use_impl,
                        workspace_bytes)
from ._native import CANativeError, LIB_PATH, lib

__all__ = ["continuum_attention", "continuum_attention_fixed_tau", "ContinuumAttentionFunction",
           "use_impl", "deterministic_backward", "forward_raw", "backward_raw", "workspace_bytes", "CANativeError", "LIB_PATH", "lib"]
