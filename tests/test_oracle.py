"""Pin the CPU oracle against golden vectors produced by the reference itself.

Each fixture in tests/golden/ was written by tests/golden/make_golden.py from
the reference's own functions in float64.  The oracle (oracle/ca_oracle.py)
must reproduce them to float64 rounding; only then is it trusted as the
checker for the CUDA operator.
"""
import math
import os

import numpy as np
import pytest
import torch

from oracle import ca_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def _t(x):
    return torch.from_numpy(np.asarray(x))


def test_moments_match_reference_stable_moments():
    g = _load("moments.npz")
    z0, z1, z2 = O.shifted_moments(_t(g["delta"]))
    for got, key in ((z0, "z0"), (z1, "z1"), (z2, "z2")):
        torch.testing.assert_close(got, _t(g[key]), atol=1e-14, rtol=1e-12)
    L, mu = O.segment_integral_coefficients(_t(g["delta"]))
    torch.testing.assert_close(L, _t(g["L"]), atol=1e-14, rtol=1e-12)
    torch.testing.assert_close(mu, _t(g["mu"]), atol=1e-14, rtol=1e-12)


def test_moment_limits_and_quadrature():
    # analytic limits J_n(0) = 1/(n+1) and a trapezoid check (test_analytic_backward.py:25-39)
    z = O.shifted_moments(torch.zeros(1, dtype=torch.float64))
    for n in range(3):
        assert abs(z[n].item() - 1.0 / (n + 1)) < 1e-15
    for delta in (-12.0, -1.01, -0.8, -0.2, 0.0, 0.2, 0.8, 1.01, 12.0):
        u = torch.linspace(0, 1, 20001, dtype=torch.float64)
        wgt = (u * delta - max(delta, 0.0)).exp()
        ms = O.shifted_moments(torch.tensor(delta, dtype=torch.float64))
        for n, m in enumerate(ms):
            torch.testing.assert_close(m, torch.trapezoid(wgt * u.pow(n), u), rtol=2e-6, atol=2e-7)


def test_square_weights_and_vjp_match_reference():
    g = _load("weights_square.npz")
    keys = sorted({k.rsplit("_", 1)[0] for k in g.files})
    assert len(keys) == 30
    for key in keys:
        s, gw = _t(g[key + "_s"]), _t(g[key + "_gw"])
        w = O.ca_weights(s)
        torch.testing.assert_close(w, _t(g[key + "_w"]), atol=1e-13, rtol=1e-11, msg=key)
        T = s.shape[-1]
        ds = O.ca_scores_backward_tile(s.reshape(-1, T, T), gw.reshape(-1, T, T), 0).reshape(s.shape)
        torch.testing.assert_close(ds, _t(g[key + "_ds"]), atol=1e-11, rtol=1e-9, msg=key)


def test_tile_weights_and_vjp_match_reference_preflight_cases():
    g = _load("weights_tile.npz")
    keys = sorted({k.rsplit("_", 1)[0] for k in g.files})
    assert len(keys) == 6
    for key in keys:
        s, gw, start = _t(g[key + "_s"]), _t(g[key + "_gw"]), int(g[key + "_start"])
        w = O.ca_weights_tile(s, start)
        torch.testing.assert_close(w, _t(g[key + "_w"]), atol=1e-13, rtol=1e-11, msg=key)
        ds = O.ca_scores_backward_tile(s, gw, start)
        torch.testing.assert_close(ds, _t(g[key + "_ds"]), atol=1e-11, rtol=1e-8, msg=key)


def _check_operator(inputs, expect, tile, rtol_fwd=1e-9, rtol_bwd=1e-9):
    q, k, v, dy, lg = inputs
    y, dq, dk, dv, dg = O.ca_forward_backward(q, k, v, lg, dy, query_tile=tile)
    for name, got, ref, tol in (("y", y, expect[0], rtol_fwd), ("dq", dq, expect[1], rtol_bwd),
                                ("dk", dk, expect[2], rtol_bwd), ("dv", dv, expect[3], rtol_bwd),
                                ("dlog_gain", dg, expect[4], rtol_bwd)):
        ref = ref.to(torch.float64)
        err = (got - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
        assert err <= tol, f"{name}: normalised max error {err:.3e} > {tol:.1e}"


def test_operator_small_cases_match_reference():
    g = _load("operator_small.npz")
    names = [str(n) for n in g["__names__"]]
    assert len(names) >= 15
    for name in names:
        inp = [_t(g[f"{name}__{t}"]) for t in ("q", "k", "v", "dy", "log_gain")]
        exp = [_t(g[f"{name}__{t}"]) for t in ("y", "dq", "dk", "dv", "dlog_gain")]
        T = inp[0].shape[2]
        for tile in (7, 64, max(T, 1)):
            # fixtures store y/dq/dk/dv in float32: compare at that precision
            _check_operator(inp, exp, tile, rtol_fwd=3e-7, rtol_bwd=3e-7)


def test_operator_config1_matches_reference():
    g = _load("operator_cfg1.npz")
    inp = [_t(g[t]) for t in ("q", "k", "v", "dy", "log_gain")]
    exp = [_t(g[t]) for t in ("y", "dq", "dk", "dv", "dlog_gain")]
    assert tuple(inp[0].shape) == (2, 4, 256, 32)
    _check_operator(inp, exp, 128, rtol_fwd=3e-7, rtol_bwd=3e-7)


def test_uniform_limit_and_single_token():
    # test_acma.py:71-80: constant scores give uniform causal attention; T=1 gives w=1
    z = torch.full((2, 3, 14, 14), 4.3, dtype=torch.float64)
    w = O.ca_weights(z)
    causal = torch.ones(14, 14, dtype=torch.bool).tril()
    expect = torch.softmax(z.masked_fill(~causal, -math.inf), -1)
    torch.testing.assert_close(w, expect, atol=1e-14, rtol=1e-14)
    assert O.ca_weights(torch.tensor([[[[123.0]]]], dtype=torch.float64)).item() == 1.0


def test_extreme_logits_finite_and_shift_invariant():
    g = torch.Generator().manual_seed(5)
    s = torch.randn(1, 3, 9, 9, generator=g, dtype=torch.float64) * 150
    w = O.ca_weights(s)
    assert torch.isfinite(w).all()
    torch.testing.assert_close(w, O.ca_weights(s + 1000), atol=1e-4, rtol=1e-4)


def test_score_gradient_rows_sum_to_zero():
    # shift invariance: adding a constant to a row leaves W unchanged, so sum_j dS_ij = 0
    g = torch.Generator().manual_seed(7)
    s = torch.randn(4, 16, 40, generator=g, dtype=torch.float64) * 3
    gw = torch.randn(4, 16, 40, generator=g, dtype=torch.float64)
    ds = O.ca_scores_backward_tile(s, gw, 24)
    assert ds.sum(-1).abs().max().item() < 1e-12


def test_oracle_vjp_matches_autograd_of_oracle_weights():
    g = torch.Generator().manual_seed(9)
    s = (torch.randn(2, 12, 30, generator=g, dtype=torch.float64) * 2).requires_grad_(True)
    gw = torch.randn(2, 12, 30, generator=g, dtype=torch.float64)
    w = O.ca_weights_tile(s, 18)
    ref = torch.autograd.grad((w * gw).sum(), s)[0]
    got = O.ca_scores_backward_tile(s.detach(), gw, 18)
    torch.testing.assert_close(got, ref, atol=1e-12, rtol=1e-10)
