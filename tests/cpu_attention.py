"""Differentiable CPU stand-in for the CA operator (test-only).

Built on the oracle's tile weights, so host-side tests (decoder wiring, DDP on
gloo) can run without a GPU.  The product path never uses it.
"""
import math

import torch

from oracle.ca_oracle import ca_weights_tile


def cpu_continuum_attention(q, k, v, log_gain, query_tile=64):
    B, H, T, D = q.shape
    s = (q @ k.transpose(-2, -1)) * (log_gain.exp().view(1, H, 1, 1) / math.sqrt(D))
    w = ca_weights_tile(s.reshape(B * H, T, T), 0).reshape(B, H, T, T)
    return w.to(v.dtype) @ v
