"""GPU tests of size-independent properties at the full BASELINE sizes, the
reference's bitwise causality checks (cuda/benchmark.py:51-82), edge cases and
the operator's error behaviour.
"""
import math

import pytest
import torch

import continuum_attention_b200 as ca
from ca_testlib import gen_inputs, norm_max_err

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _op_grads(q, k, v, lg, dy):
    q, k, v = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    lg = lg.detach().clone().requires_grad_(True)
    y = ca.continuum_attention(q, k, v, lg, 128)
    gq, gk, gv, gg = torch.autograd.grad((y.float() * dy.float()).sum(), (q, k, v, lg))
    return y.detach(), gq, gk, gv, gg


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_causal_future_perturbation_bitwise(dtype):
    # cuda/benchmark.py:54-81: future q/k/v changes leave earlier outputs bit-identical,
    # and a loss on outputs <= cut sends exactly zero gradient to future tokens
    T = 2048
    g = torch.Generator(device="cpu").manual_seed(4242)
    q = torch.randn(1, 2, T, 64, generator=g).to(DEV, dtype)
    k = torch.randn(1, 2, T, 64, generator=g).to(DEV, dtype)
    v = torch.randn(1, 2, T, 64, generator=g).to(DEV, dtype)
    rho = torch.tensor([0.0, 0.2], device=DEV)
    with torch.no_grad():
        y0 = ca.continuum_attention(q, k, v, rho, 128)
        for cut in (0, 127, 128, 1023, 1024, 2046):
            qp, kp, vp = q.clone(), k.clone(), v.clone()
            n = T - cut - 1
            qp[:, :, cut + 1:] = (torch.randn(1, 2, n, 64, generator=g) * 2.5).to(DEV, dtype)
            kp[:, :, cut + 1:] = (torch.randn(1, 2, n, 64, generator=g) * 2.5).to(DEV, dtype)
            vp[:, :, cut + 1:] = (torch.randn(1, 2, n, 64, generator=g) * 2.5).to(DEV, dtype)
            y1 = ca.continuum_attention(qp, kp, vp, rho, 128)
            assert torch.equal(y0[:, :, :cut + 1], y1[:, :, :cut + 1]), f"output leak at cut {cut}"
    for cut in (0, 127, 128, 1023, 1024, 2046):
        qt, kt, vt = (t.clone().requires_grad_(True) for t in (q, k, v))
        y = ca.continuum_attention(qt, kt, vt, rho, 128)
        gq, gk, gv = torch.autograd.grad(y[:, :, :cut + 1].float().sum(), (qt, kt, vt))
        for name, gr in (("Q", gq), ("K", gk), ("V", gv)):
            fut = gr[:, :, cut + 1:]
            if fut.numel():
                assert fut.abs().max().item() == 0.0, f"future {name} gradient at cut {cut}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gradient_identities_full_size(dtype):
    # exact identities at config-2 size:
    #   sum_j dV_j = sum_i dO_i               (rows of W sum to one)
    #   dlog_gain_h = sum_i <dQ_i, q_i> = sum_j <dK_j, k_j>   (s = scale q.k)
    q, k, v, dy = (t.to(DEV, dtype) for t in gen_inputs((2, 16, 2048, 64), 2))
    lg = torch.linspace(-0.3, 0.5, 16, device=DEV)
    y, gq, gk, gv, gg = _op_grads(q, k, v, lg, dy)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    sv = gv.double().sum(2)
    so = dy.double().sum(2)
    assert norm_max_err(sv, so) < tol
    via_q = (gq.double() * q.double()).sum(dim=(0, 2, 3))
    via_k = (gk.double() * k.double()).sum(dim=(0, 2, 3))
    assert norm_max_err(via_q, gg.double()) < tol
    assert norm_max_err(via_k, gg.double()) < tol


def test_uniform_limit_full_size():
    # constant scores (q = 0) make W exactly uniform causal attention: y_i = mean_{j<=i} v_j
    T = 2048
    v = torch.randn(2, 4, T, 64, device=DEV)
    q = torch.zeros_like(v)
    k = torch.randn_like(v)
    y = ca.continuum_attention(q, k, v, torch.zeros(4, device=DEV))
    ref = v.double().cumsum(2) / torch.arange(1, T + 1, device=DEV, dtype=torch.float64).view(1, 1, T, 1)
    assert norm_max_err(y, ref) < 1e-5


def test_linearity_in_values_and_head_sharding():
    q, k, v, _ = (t.to(DEV) for t in gen_inputs((2, 8, 1500, 64), 9))
    v2 = torch.randn_like(v)
    lg = torch.zeros(8, device=DEV)
    y1 = ca.continuum_attention(q, k, v, lg)
    y2 = ca.continuum_attention(q, k, v2, lg)
    y3 = ca.continuum_attention(q, k, 2.0 * v - 0.5 * v2, lg)
    assert norm_max_err(y3, 2.0 * y1 - 0.5 * y2) < 1e-5
    # heads are independent: running a slice of heads alone is bit-identical
    part = ca.continuum_attention(q[:, 2:5], k[:, 2:5], v[:, 2:5], lg[2:5])
    assert torch.equal(part, y1[:, 2:5])


def test_duplicate_keys_and_extreme_scores_finite():
    T = 4096
    q, k, v, dy = (t.to(DEV, torch.bfloat16) for t in gen_inputs((1, 4, T, 64), 31, qk_mag=2.0, dup_frac=0.1))
    lg = torch.full((4,), 1.0, device=DEV)       # score std ~ 4 * e
    y, gq, gk, gv, gg = _op_grads(q, k, v, lg, dy)
    for t in (y, gq, gk, gv, gg):
        assert torch.isfinite(t.float()).all()


@pytest.mark.parametrize("T", [1, 2, 3, 63, 64, 65, 127, 129, 255, 257])
def test_ragged_lengths_match_oracle(T):
    from ca_testlib import oracle, run_op, assert_fp32_parity
    q, k, v, dy = gen_inputs((1, 3, T, 64), 100 + T)
    lg = torch.tensor([0.0, 0.5, -0.5])
    outs, _ = run_op(q, k, v, lg, dy, dtype=torch.float32)
    assert_fp32_parity(outs, oracle(q, k, v, lg, dy), tag=f"T={T}")


@pytest.mark.parametrize("D", [8, 16, 32, 48, 64, 96, 128])
def test_head_dims(D):
    from ca_testlib import oracle, run_op, assert_fp32_parity
    q, k, v, dy = gen_inputs((1, 2, 150, D), 200 + D)
    lg = torch.tensor([0.0, 0.3])
    outs, _ = run_op(q, k, v, lg, dy, dtype=torch.float32)
    assert_fp32_parity(outs, oracle(q, k, v, lg, dy), tag=f"D={D}")


def test_empty_inputs():
    for shape in ((0, 2, 16, 64), (1, 2, 0, 64)):
        q = torch.zeros(shape, device=DEV, requires_grad=True)
        lg = torch.zeros(2, device=DEV, requires_grad=True)
        y = ca.continuum_attention(q, q, q, lg)
        assert y.shape == q.shape
        y.sum().backward()
        assert lg.grad is not None and torch.all(lg.grad == 0)


def test_error_behaviour():
    q = torch.randn(1, 2, 8, 64, device=DEV)
    lg = torch.zeros(2, device=DEV)
    with pytest.raises(ValueError, match="must share dtype"):
        ca.continuum_attention(q, q.half(), q, lg)
    with pytest.raises(ValueError):
        ca.continuum_attention(q, q, q, torch.zeros(3, device=DEV))
    with pytest.raises(ca.CANativeError, match="UNSUPPORTED"):
        big = torch.randn(1, 1, 8, 160, device=DEV)
        ca.continuum_attention(big, big, big, torch.zeros(1, device=DEV))
    qq = q.clone().requires_grad_(True)
    y = ca.continuum_attention(qq, qq, qq, lg)
    with pytest.raises(RuntimeError, match="first-order"):
        torch.autograd.grad(y.sum(), qq, create_graph=True)


def test_fixed_tau_matches_learned_gain_at_same_value():
    q, k, v, _ = (t.to(DEV) for t in gen_inputs((2, 4, 300, 64), 12))
    a = ca.continuum_attention_fixed_tau(q, k, v, 0.30)
    b = ca.continuum_attention(q, k, v, torch.full((4,), math.log(1 / 0.30), device=DEV))
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_inference_forward_without_statistics(dtype):
    # no input requires grad: the op runs the inference form (row statistics not
    # written) and returns exactly the training forward's output
    q, k, v, dy = gen_inputs((2, 3, 300, 64), seed=11)
    q, k, v = (t.to(DEV, dtype) for t in (q, k, v))
    lg = torch.tensor([0.0, 0.3, -0.2], device=DEV)
    with torch.no_grad():
        y_inf = ca.continuum_attention(q, k, v, lg)
    y_train = ca.continuum_attention(q.clone().requires_grad_(True), k, v, lg)
    assert torch.equal(y_inf, y_train.detach())
    o, stats, o32 = ca.forward_raw(q, k, v, lg, want_stats=False)
    assert stats is None and o32 is None and torch.equal(o, y_inf)


def test_bounded_wait_timeout_is_reported_and_context_survives():
    # a device wait on a barrier nothing completes gives up after its limit,
    # the status word reports CA_ERR_DEVICE_TIMEOUT (5), and the next calls work
    from continuum_attention_b200 import _native
    lib = _native.lib()
    lib.ca_device_status(1)
    assert lib.ca_selftest_wait_timeout(50000, None) == 0          # 50 ms limit
    assert lib.ca_device_status(1) == 5
    assert lib.ca_device_status(0) == 0
    assert lib.ca_selftest_wait_timeout(0, None) == 1
    q, k, v, dy = gen_inputs((1, 2, 200, 64), seed=5)
    q, k, v = (t.to(DEV, torch.bfloat16) for t in (q, k, v))
    lg = torch.zeros(2, device=DEV)
    y1 = ca.continuum_attention(q, k, v, lg)
    y2 = ca.continuum_attention(q, k, v, lg)
    assert torch.isfinite(y1.float()).all() and torch.equal(y1, y2)
    assert lib.ca_device_status(0) == 0


@pytest.mark.parametrize("T", [16384, 32768])
def test_long_context_rows_and_identities(T):
    # BASELINE config 3 lengths: sampled query rows (including the last) against the
    # float64 oracle on the full causal prefix, plus the exact gradient identities
    from oracle.ca_oracle import ca_weights_tile
    H = 4
    q, k, v, dy = (t.to(DEV, torch.bfloat16) for t in gen_inputs((1, H, T, 64), 41, qk_mag=2.0, dup_frac=0.1))
    lg = torch.linspace(-0.2, 0.3, H, device=DEV)
    y, gq, gk, gv, gg = _op_grads(q, k, v, lg, dy)
    assert torch.isfinite(y.float()).all() and torch.isfinite(gq.float()).all()
    rows = [0, 1, 63, 64, 127, 128, T // 2 + 5, T - 129, T - 65, T - 1]
    qd, kd, vd = (t[0].double().cpu() for t in (q, k, v))
    for h in range(H):
        scale = math.exp(float(lg[h])) / 8.0
        for i in rows:
            s = (qd[h, i:i + 1] @ kd[h, :i + 1].T) * scale          # [1, i+1]
            w = ca_weights_tile(s.unsqueeze(0), i)[0]                # row i's weights over keys 0..i
            ref = w @ vd[h, :i + 1]
            err = (y[0, h, i].double().cpu() - ref[0]).abs().max().item()
            assert err <= 4e-3 * ref.abs().max().item() + 4e-3, (h, i, err)
    sv, so = gv.double().sum(2), dy.double().sum(2)
    assert norm_max_err(sv, so) < 2e-2
    via_q = (gq.double() * q.double()).sum(dim=(0, 2, 3))
    via_k = (gk.double() * k.double()).sum(dim=(0, 2, 3))
    assert norm_max_err(via_q, gg.double()) < 2e-2
    assert norm_max_err(via_k, gg.double()) < 2e-2
