"""Helpers shared by the test files: seeded inputs, tolerance measures, fixtures.

Tolerances (from the build's stated parity bar):
  * fp32 path: normalised max error max|x - ref| / max|ref| <= 1e-5 for the
    forward output and <= 1e-4 for every gradient (dq, dk, dv, dlog_gain);
  * bf16 / fp16 inputs with fp32 accumulation: forward max|o_f32 - ref| <=
    2e-3 * rms(ref), where o_f32 is the operator's fp32 accumulator (the
    stored bf16 output is its round-to-nearest-even), and every gradient has
    cosine similarity >= 0.9999 with the reference gradient.
The reference ``ref`` is always the float64 oracle evaluated on the very
inputs the kernel saw (after any rounding to bf16/fp16).
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

FP32_FWD_TOL = 1e-5
FP32_GRAD_TOL = 1e-4
LOWP_FWD_RMS_TOL = 2e-3
LOWP_GRAD_COS = 0.9999


ZERO_REF_ABS = 1e-4   # an all-zero reference (e.g. dq at T=1) is checked as an absolute bound


def norm_max_err(x, ref) -> float:
    """max|x - ref| / max|ref|; plain max|x - ref| when the reference is all zeros."""
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    err = (x - ref).abs().max().item() if x.numel() else 0.0
    scale = ref.abs().max().item() if ref.numel() else 0.0
    return err / scale if scale > 0 else err


def rms(x) -> float:
    x = x.detach().double()
    return x.square().mean().sqrt().item()


def cosine(x, ref) -> float:
    """Cosine similarity; against an all-zero reference it is 1 iff max|x| <= ZERO_REF_ABS."""
    x = x.detach().double().cpu().flatten()
    ref = ref.detach().double().cpu().flatten()
    if ref.numel() == 0 or ref.norm().item() == 0.0:
        return 1.0 if (x.numel() == 0 or x.abs().max().item() <= ZERO_REF_ABS) else 0.0
    den = x.norm().item() * ref.norm().item()
    if den == 0.0:
        return 0.0
    return float((x @ ref).item() / den)


def gen_inputs(shape, seed, *, qk_mag=1.0, dup_frac=0.0):
    """Same recipe as tests/golden/make_golden.py:gen_inputs (fp32 CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=g) * qk_mag
    k = torch.randn(shape, generator=g) * qk_mag
    v = torch.randn(shape, generator=g)
    dy = torch.randn(shape, generator=g)
    if dup_frac > 0:
        T = shape[2]
        pick = torch.rand(T, generator=g) < dup_frac
        pick[0] = False
        for j in torch.nonzero(pick).flatten().tolist():
            k[:, :, j] = k[:, :, j - 1]
    return q.float(), k.float(), v.float(), dy.float()


def load_small_cases():
    """[(name, (q, k, v, log_gain, dy), (y, dq, dk, dv, dlog_gain))] from the golden fixture."""
    g = np.load(os.path.join(GOLD, "operator_small.npz"))
    out = []
    for name in [str(n) for n in g["__names__"]]:
        inp = [torch.from_numpy(g[f"{name}__{t}"]) for t in ("q", "k", "v", "log_gain", "dy")]
        exp = [torch.from_numpy(g[f"{name}__{t}"]) for t in ("y", "dq", "dk", "dv", "dlog_gain")]
        out.append((name, inp, exp))
    return out


def load_cfg1():
    """((q, k, v, log_gain, dy), (y, dq, dk, dv, dlog_gain)) of BASELINE config 1."""
    g = np.load(os.path.join(GOLD, "operator_cfg1.npz"))
    inp = [torch.from_numpy(g[t]) for t in ("q", "k", "v", "log_gain", "dy")]
    exp = [torch.from_numpy(g[t]) for t in ("y", "dq", "dk", "dv", "dlog_gain")]
    return inp, exp


def run_op(q, k, v, lg, dy, *, dtype, impl="auto", device="cuda"):
    """Forward (with fp32 accumulator) + backward through the native library.

    Argument order is (q, k, v, log_gain, dy), as everywhere in these tests.
    Returns (o, o_f32, dq, dk, dv, dlog_gain) as CPU tensors plus the device
    inputs actually used (rounded to ``dtype``).
    """
    from continuum_attention_b200 import backward_raw, forward_raw
    qd, kd, vd = (t.to(device=device, dtype=dtype).contiguous() for t in (q, k, v))
    dyd = dy.to(device=device, dtype=dtype).contiguous()
    lgd = lg.to(device=device, dtype=torch.float32).contiguous()
    o, stats, o32 = forward_raw(qd, kd, vd, lgd, impl=impl, want_f32=True)
    dq, dk, dv, dg = backward_raw(qd, kd, vd, o, dyd, lgd, stats, want_dgain=True, impl=impl,
                                  o_f32=o32 if dtype != torch.float32 else None)
    torch.cuda.synchronize()
    outs = [t.cpu() for t in (o, o32, dq, dk, dv, dg)]
    used = [t.cpu().double() for t in (qd, kd, vd, dyd)]
    return outs, used


def oracle(q, k, v, lg, dy, tile=256):
    from oracle.ca_oracle import ca_forward_backward
    return ca_forward_backward(q.double(), k.double(), v.double(), lg.double(), dy.double(),
                               query_tile=tile, dtype=torch.float64)


def assert_fp32_parity(outs, ref, tag=""):
    o, o32, dq, dk, dv, dg = outs
    y, rdq, rdk, rdv, rdg = ref
    e = norm_max_err(o, y)
    assert e <= FP32_FWD_TOL, f"{tag} forward normalised max error {e:.3e} > {FP32_FWD_TOL}"
    for name, a, b in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv), ("dlog_gain", dg, rdg)):
        e = norm_max_err(a, b)
        assert e <= FP32_GRAD_TOL, f"{tag} {name} normalised max error {e:.3e} > {FP32_GRAD_TOL}"


def assert_lowp_parity(outs, ref, tag="", check_round=True, lowp_dtype=torch.bfloat16):
    o, o32, dq, dk, dv, dg = outs
    y, rdq, rdk, rdv, rdg = ref
    err = (o32.double() - y).abs().max().item()
    bound = LOWP_FWD_RMS_TOL * rms(y)
    assert err <= bound, f"{tag} forward max abs error {err:.3e} > 2e-3*rms = {bound:.3e}"
    if check_round:
        assert torch.equal(o, o32.to(lowp_dtype)), f"{tag} stored output is not RNE(fp32 accumulator)"
    for name, a, b in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv), ("dlog_gain", dg, rdg)):
        c = cosine(a, b)
        assert c >= LOWP_GRAD_COS, f"{tag} {name} cosine {c:.6f} < {LOWP_GRAD_COS}"
    # the gain gradient has one entry per head: also bound its normalised error
    e = norm_max_err(dg, rdg)
    assert e <= 1e-2, f"{tag} dlog_gain normalised max error {e:.3e} > 1e-2"
