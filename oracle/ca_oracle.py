"""CPU restatement of the Continuum Attention (CA) algorithm.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
operator in ``continuum_attention_b200``.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may
import it.  The product path never calls it and has no CPU fallback.

Parity is pinned: ``tests/test_oracle.py`` checks every function here against
the golden vectors in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by importing and running the reference itself.

Everything is vectorised torch on the CPU and computes in the dtype of its
inputs (float64 for the oracle role).  Citations name the reference file and
line range whose behaviour each function restates.

The math (one query row i, scaled scores s_j = g * q_i.k_j / sqrt(D)):

* keys/values are linearly interpolated between adjacent positions; segment
  k (key k-1 -> key k, 1 <= k <= i) with a = s_{k-1}, delta = s_k - a has
  moments  M_n = e^{a-m} J_n(delta),  J_n(x) = int_0^1 u^n e^{x u} du;
* it adds M_0 - M_1 to the weight of key k-1 and M_1 to key k;
* half-token caps 0.5 e^{s_0 - m} (key 0) and 0.5 e^{s_i - m} (key i);
* the row is normalised by its sum Z, and y_i = sum_j w_ij v_j.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch

__all__ = [
    "segment_integral_coefficients",
    "shifted_moments",
    "ca_weights_tile",
    "ca_weights",
    "ca_scores_backward_tile",
    "ca_forward",
    "ca_forward_backward",
]

# Series J_n(x) = sum_k x^k / (k! (k+n+1)) is used for |x| < 1; 20 terms leave
# a truncation error below 1/(20! * 21) ~ 2e-20, far under float64 rounding.
_SERIES_TERMS = 20


def _series_moment(x: torch.Tensor, n: int) -> torch.Tensor:
    """Unshifted J_n(x) by its power series (valid and accurate for |x| < 1)."""
    coeffs = [1.0 / (math.factorial(k) * (k + n + 1)) for k in range(_SERIES_TERMS)]
    acc = torch.full_like(x, coeffs[-1])
    for c in reversed(coeffs[:-1]):
        acc = acc * x + c
    return acc


def shifted_moments(delta: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Return z_n = e^{-max(delta,0)} * J_n(delta) for n = 0, 1, 2.

    Restates ``stable_moments`` (analytic_reference.py:12-49): closed forms
    for |delta| >= 1 and a power series for |delta| < 1.  The closed forms
    follow from integrating u^n e^{delta u} by parts; with t = |delta| and
    e = e^{-t}:
      delta >= 0: z0 = (1-e)/t, z1 = (t-1+e)/t^2, z2 = (t^2-2t+2-2e)/t^3
      delta <  0: z0 = (1-e)/t, z1 = (1-(1+t)e)/t^2, z2 = (2-(t^2+2t+2)e)/t^3
    """
    t = delta.abs()
    big = t >= 1.0
    tb = torch.where(big, t, torch.ones_like(t))
    e = torch.exp(-tb)
    z0_b = -torch.expm1(-tb) / tb
    pos = delta >= 0
    z1_b = torch.where(pos, (tb - 1.0 + e) / tb**2, (1.0 - (1.0 + tb) * e) / tb**2)
    z2_b = torch.where(pos, (tb * tb - 2.0 * tb + 2.0 - 2.0 * e) / tb**3,
                       (2.0 - (tb * tb + 2.0 * tb + 2.0) * e) / tb**3)
    xs = torch.where(big, torch.zeros_like(delta), delta)
    shift = torch.exp(-xs.clamp_min(0.0))
    z0_s = _series_moment(xs, 0) * shift
    z1_s = _series_moment(xs, 1) * shift
    z2_s = _series_moment(xs, 2) * shift
    return (torch.where(big, z0_b, z0_s), torch.where(big, z1_b, z1_s),
            torch.where(big, z2_b, z2_s))


def segment_integral_coefficients(delta: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(L, mu) of a segment: mass = e^{max(a,b)} L and mu = J1/J0.

    Restates architecture.py:32-62 via the shifted moments:
    L = z0 and mu = z1 / z0 (the shift cancels in the ratio).
    """
    z0, z1, _ = shifted_moments(delta)
    return z0, z1 / z0


def _tile_masks(Q: int, K: int, start: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    rows = torch.arange(start, start + Q, device=device).view(Q, 1)
    keys = torch.arange(K, device=device).view(1, K)
    visible = keys <= rows                       # key j visible to query i
    seg_ok = keys[:, 1:] <= rows                 # segment (j-1 -> j) visible
    return visible, seg_ok


def _tile_parts(s: torch.Tensor, start: int):
    """Shared pieces of the forward and backward for a query tile.

    s: [N, Q, K] scaled scores of queries start..start+Q-1 vs keys 0..K-1.
    Follows cuda/continuum_attention.py:622-648: mask future endpoints to the
    row max *before* any exp or difference, so future scores never overflow.
    """
    N, Q, K = s.shape
    if start + Q > K:
        raise ValueError("tile queries must see their own key (start+Q <= K)")
    visible, seg_ok = _tile_masks(Q, K, start, s.device)
    m = s.masked_fill(~visible, float("-inf")).amax(-1, keepdim=True)
    a = torch.where(seg_ok, s[..., :-1], m)
    b = torch.where(seg_ok, s[..., 1:], m)
    z0, z1, z2 = shifted_moments(b - a)
    e = torch.exp(torch.maximum(a, b) - m) * seg_ok.to(s.dtype)
    cap = torch.zeros_like(s)
    cap[..., 0] += 0.5 * torch.exp(s[..., 0] - m[..., 0])
    diag = torch.arange(start, start + Q, device=s.device)
    qidx = torch.arange(Q, device=s.device)
    cap[:, qidx, diag] += 0.5 * torch.exp(s[:, qidx, diag] - m[..., 0])
    return visible, m, e, (z0, z1, z2), cap


def ca_weights_tile(s: torch.Tensor, start: int) -> torch.Tensor:
    """Normalised CA weights for a query tile, [N, Q, K].

    Restates ``_ca_reference_weights`` (cuda/continuum_attention.py:622-648),
    which generalises ``continuous_attention_weights`` (architecture.py:65-105)
    to a query tile starting at row ``start``.
    """
    visible, m, e, (z0, z1, _), cap = _tile_parts(s, start)
    w = cap.clone()
    w[..., :-1] += e * (z0 - z1)                 # left endpoint share
    w[..., 1:] += e * z1                         # right endpoint share
    w = w * visible.to(s.dtype)
    return w / w.sum(-1, keepdim=True)


def ca_weights(logits: torch.Tensor) -> torch.Tensor:
    """Square form [..., T, T] (architecture.py:65-105)."""
    T = logits.shape[-1]
    if logits.shape[-2] != T:
        raise ValueError("square full-sequence causal logits required")
    lead = logits.shape[:-2]
    w = ca_weights_tile(logits.reshape(-1, T, T), 0)
    return w.reshape(*lead, T, T)


def ca_scores_backward_tile(s: torch.Tensor, grad_w: torch.Tensor, start: int) -> torch.Tensor:
    """Analytic VJP dL/ds of the tile weights given dL/dW, no autograd.

    Restates ``analytic_scores_backward`` (analytic_reference.py:52-75) for a
    query tile.  With g = dW - sum_k w_k dW_k and segment moments M_n, the
    left endpoint of a segment receives g_l (M0-2M1+M2) + g_r (M1-M2), the
    right endpoint g_l (M1-M2) + g_r M2, the caps add cap * g, and everything
    is divided by the row mass Z.
    """
    visible, m, e, (z0, z1, z2), cap = _tile_parts(s, start)
    Z = (e * z0).sum(-1, keepdim=True) + cap.sum(-1, keepdim=True)
    w = cap.clone()
    w[..., :-1] += e * (z0 - z1)
    w[..., 1:] += e * z1
    w = w * visible.to(s.dtype) / Z
    g = grad_w - (grad_w * w).sum(-1, keepdim=True)
    gl, gr = g[..., :-1], g[..., 1:]
    left = e * (gl * (z0 - 2.0 * z1 + z2) + gr * (z1 - z2))
    right = e * (gl * (z1 - z2) + gr * z2)
    ds = cap * g
    ds[..., :-1] += left
    ds[..., 1:] += right
    return (ds / Z).masked_fill(~visible, 0.0)


def _scale(log_gain: torch.Tensor, D: int, dtype) -> torch.Tensor:
    # cuda/continuum_attention.py:656-657: scale = exp(log_gain) * D^-0.5
    return (log_gain.detach().to(dtype).exp() * (D ** -0.5)).view(1, -1, 1, 1)


def ca_forward(q, k, v, log_gain, query_tile: int = 128, dtype=torch.float64) -> torch.Tensor:
    """y = CA(q, k, v) for [B,H,T,D] inputs, computed in ``dtype``.

    Restates ``_CAExactTiled.forward`` (cuda/continuum_attention.py:651-694):
    per query tile, scores over the causal prefix, tile weights, W @ V.
    """
    return ca_forward_backward(q, k, v, log_gain, None, query_tile, dtype)[0]


def ca_forward_backward(q, k, v, log_gain, dy, query_tile: int = 128, dtype=torch.float64):
    """Forward and (if dy is given) analytic backward, in ``dtype``.

    Restates cuda/continuum_attention.py:651-766: per query tile, recompute
    scores, dW = dY V^T, analytic dS, then dV += W^T dY, dQ += (dS*scale) K,
    dK += (dS*scale)^T Q and d log_gain += sum dS * s.
    Returns (y, dq, dk, dv, dlog_gain) with grads None when dy is None.
    """
    B, H, T, D = q.shape
    qb = q.detach().to(dtype).reshape(B * H, T, D)
    kb = k.detach().to(dtype).reshape(B * H, T, D)
    vb = v.detach().to(dtype).reshape(B * H, T, D)
    scale = _scale(log_gain, D, dtype)
    sc_bh = scale.expand(B, H, 1, 1).reshape(B * H, 1, 1)
    y = torch.empty_like(vb)
    want_grad = dy is not None
    if want_grad:
        gb = dy.detach().to(dtype).reshape(B * H, T, D)
        dq = torch.zeros_like(qb)
        dk = torch.zeros_like(kb)
        dv = torch.zeros_like(vb)
        dgain = torch.zeros(B * H, dtype=dtype)
    for start in range(0, T, query_tile):
        end = min(T, start + query_tile)
        qs, keys, vals = qb[:, start:end], kb[:, :end], vb[:, :end]
        s = torch.bmm(qs, keys.transpose(1, 2)) * sc_bh
        w = ca_weights_tile(s, start)
        y[:, start:end] = torch.bmm(w, vals)
        if want_grad:
            gys = gb[:, start:end]
            gw = torch.bmm(gys, vals.transpose(1, 2))
            ds = ca_scores_backward_tile(s, gw, start)
            dv[:, :end] += torch.bmm(w.transpose(1, 2), gys)
            dss = ds * sc_bh
            dq[:, start:end] += torch.bmm(dss, keys)
            dk[:, :end] += torch.bmm(dss.transpose(1, 2), qs)
            dgain += (ds * s).sum(dim=(1, 2))
    y = y.reshape(B, H, T, D)
    if not want_grad:
        return y, None, None, None, None
    return (y, dq.reshape(B, H, T, D), dk.reshape(B, H, T, D), dv.reshape(B, H, T, D),
            dgain.reshape(B, H).sum(0))
