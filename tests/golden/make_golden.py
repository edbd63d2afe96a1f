"""Generate the golden fixtures in this folder by running the reference itself.

Run once, in a checkout where the reference project is available:

    python tests/golden/make_golden.py --reference <path-to-continuum-attention>

It imports the reference's own functions (``architecture.py``,
``analytic_reference.py`` and ``cuda/continuum_attention.py``) and records
their float64 outputs on seeded inputs.  The fixtures are committed; the tests
read only the ``.npz`` files and never need the reference at run time.

Fixtures:
  moments.npz        stable_moments / segment_integral_coefficients on a grid
  weights_square.npz continuous_attention_weights + analytic_scores_backward
  weights_tile.npz   _ca_reference_weights tiles + float64 autograd dS
                     (the cases of the reference's GPU preflight)
  operator_small.npz full op (y, dq, dk, dv, dlog_gain) on small shapes
  operator_cfg1.npz  full op at [2,4,256,32] fp32 inputs, seed 0, gain 1
  decoder_small.npz  the reference ContinuumDecoderLM (cuda/continuum_attention.py:
                     784-922) on the CPU in float32: state dict, a batch of bytes,
                     logits, loss and parameter gradients of a 2-layer d_model-128
                     model with non-zero per-head gains
"""
from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "cuda"))
    import architecture  # noqa: E402
    import analytic_reference  # noqa: E402
    import continuum_attention as cuda_ca  # noqa: E402
    return architecture, analytic_reference, cuda_ca


def gen_inputs(shape, seed, *, qk_mag=1.0, dup_frac=0.0):
    """Seeded fp32 q, k, v, dy (in that order) plus optional duplicated keys.

    dup_frac > 0 copies key j-1 into key j for a seeded subset of j, which
    makes adjacent score differences exactly zero.
    """
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


def reference_operator(arch, q, k, v, log_gain, dy):
    """Float64 forward + autograd backward through the reference's own weights."""
    q = q.double().requires_grad_(True)
    k = k.double().requires_grad_(True)
    v = v.double().requires_grad_(True)
    lg = log_gain.double().requires_grad_(True)
    D = q.shape[-1]
    logits = (q @ k.transpose(-2, -1)) * lg.exp().view(1, -1, 1, 1) * (D ** -0.5)
    w = arch.continuous_attention_weights(logits)
    y = w @ v
    grads = torch.autograd.grad((y * dy.double()).sum(), (q, k, v, lg))
    return [y.detach()] + [x.detach() for x in grads]


def make_moments(arch, aref):
    deltas = torch.tensor([-100., -20., -12., -3., -1.01, -1., -0.99, -0.8, -0.2, -1e-3, -1e-6,
                           0., 1e-6, 1e-3, 0.2, 0.8, 0.99, 1., 1.01, 3., 12., 20., 100.],
                          dtype=torch.float64)
    z0, z1, z2 = aref.stable_moments(deltas)
    L, mu = arch.segment_integral_coefficients(deltas)
    np.savez_compressed(os.path.join(HERE, "moments.npz"), delta=deltas.numpy(),
                        z0=z0.numpy(), z1=z1.numpy(), z2=z2.numpy(), L=L.numpy(), mu=mu.numpy())


def make_weights_square(arch, aref):
    out = {}
    g = torch.Generator().manual_seed(731)
    for T in (1, 2, 3, 7, 13, 32):
        for amp in (0.0, 0.01, 1.0, 4.0, 20.0):
            s = torch.randn(1, 2, T, T, generator=g, dtype=torch.float64) * amp
            gw = torch.randn(1, 2, T, T, generator=g, dtype=torch.float64)
            w = arch.continuous_attention_weights(s)
            ds = aref.analytic_scores_backward(s, gw, w)
            key = f"T{T}_a{amp}"
            out[key + "_s"] = s.numpy()
            out[key + "_gw"] = gw.numpy()
            out[key + "_w"] = w.numpy()
            out[key + "_ds"] = ds.numpy()
    np.savez_compressed(os.path.join(HERE, "weights_square.npz"), **out)


def make_weights_tile(cuda_ca):
    out = {}
    g = torch.Generator().manual_seed(20260814)
    cases = [(9, 0, 9, 1.0), (192, 144, 32, 1.0), (192, 160, 32, 2.5), (512, 480, 32, 2.5),
             (2048, 2040, 8, 2.5), (2048, 0, 8, 0.0)]
    for T, start, Q, mag in cases:
        K = start + Q
        s = (torch.randn(1, Q, K, generator=g) * mag).double()
        gw = torch.randn(1, Q, K, generator=g).double()
        sr = s.clone().requires_grad_(True)
        w = cuda_ca._ca_reference_weights(sr, start)
        ds = torch.autograd.grad((w * gw).sum(), sr)[0]
        key = f"T{T}_s{start}_q{Q}_m{mag}"
        out[key + "_s"] = s.numpy()
        out[key + "_gw"] = gw.numpy()
        out[key + "_w"] = w.detach().numpy()
        out[key + "_ds"] = ds.numpy()
        out[key + "_start"] = np.array(start)
    np.savez_compressed(os.path.join(HERE, "weights_tile.npz"), **out)


# (name, B, H, T, D, seed, qk_mag, dup_frac, log_gain per head or None -> zeros)
SMALL_CASES = [
    ("ca_check_1x2x9x8", 1, 2, 9, 8, 1234, 1.0, 0.0, None),
    ("preflight_1x2x17x16", 1, 2, 17, 16, 341, 1.0, 0.0, [0.0, 0.3]),
    ("t1_d64", 1, 2, 1, 64, 11, 1.0, 0.0, None),
    ("t2_d64", 1, 2, 2, 64, 12, 1.0, 0.0, None),
    ("t3_d32", 2, 1, 3, 32, 13, 1.0, 0.0, None),
    ("t7_d64", 1, 2, 7, 64, 14, 1.0, 0.0, None),
    ("t33_d64_mag2.2", 1, 2, 33, 64, 1665, 2.2, 0.0, [0.0, math.log(1 / 0.3)]),
    ("t65_d32", 2, 2, 65, 32, 16, 1.0, 0.0, None),
    ("t129_d64", 1, 2, 129, 64, 1762, 1.0, 0.0, [0.0, math.log(1 / 0.3)]),
    ("t70_d128", 1, 1, 70, 128, 18, 1.0, 0.0, None),
    ("t160_d32_mag2.5", 1, 2, 160, 32, 1825, 2.5, 0.0, [0.0, 0.2]),
    ("t200_d64_dup", 1, 1, 200, 64, 19, 2.0, 0.1, None),
    ("t256_d32_tau0.30", 1, 2, 256, 32, 1, 1.0, 0.0, [math.log(1 / 0.3)] * 2),
    ("t300_d32_std4_dup", 1, 1, 300, 32, 21, 2.0, 0.1, None),
    ("t64_d64_const", 1, 1, 64, 64, 22, 0.0, 0.0, None),
]


def make_operator_small(arch):
    out = {}
    for name, B, H, T, D, seed, mag, dup, lg in SMALL_CASES:
        q, k, v, dy = gen_inputs((B, H, T, D), seed, qk_mag=mag, dup_frac=dup)
        log_gain = torch.zeros(H) if lg is None else torch.tensor(lg, dtype=torch.float32)
        y, dq, dk, dv, dg = reference_operator(arch, q, k, v, log_gain, dy)
        for tag, x in (("q", q), ("k", k), ("v", v), ("dy", dy), ("log_gain", log_gain)):
            out[f"{name}__{tag}"] = x.numpy()
        for tag, x in (("y", y), ("dq", dq), ("dk", dk), ("dv", dv)):
            out[f"{name}__{tag}"] = x.float().numpy()
        out[f"{name}__dlog_gain"] = dg.numpy()
    out["__names__"] = np.array([c[0] for c in SMALL_CASES])
    np.savez_compressed(os.path.join(HERE, "operator_small.npz"), **out)


def make_operator_cfg1(arch):
    q, k, v, dy = gen_inputs((2, 4, 256, 32), 0)
    log_gain = torch.zeros(4)
    y, dq, dk, dv, dg = reference_operator(arch, q, k, v, log_gain, dy)
    np.savez_compressed(os.path.join(HERE, "operator_cfg1.npz"),
                        q=q.numpy(), k=k.numpy(), v=v.numpy(), dy=dy.numpy(),
                        log_gain=log_gain.numpy(),
                        y=y.float().numpy(), dq=dq.float().numpy(), dk=dk.float().numpy(),
                        dv=dv.float().numpy(), dlog_gain=dg.numpy())


DECODER_CFG = dict(vocab_size=256, block_size=64, d_model=128, n_heads=4, n_layers=2, mlp_ratio=2.0,
                   dropout=0.0, eps=1e-6, rope_theta=10000.0, grad_checkpointing=False, ca_query_tile=16)


def make_decoder(cuda_ca):
    """The reference decoder end to end on the CPU (its attention runs the CPU branch of
    _CAExactTiled through _ca_reference_weights), float32 as it trains."""
    torch.manual_seed(2024)
    cfg = cuda_ca.ContinuumDecoderConfig(**DECODER_CFG)
    model = cuda_ca.ContinuumDecoderLM(cfg)
    with torch.no_grad():
        for li, block in enumerate(model.blocks):
            block.attn.log_qk_gain.copy_(torch.tensor([0.1, -0.2, 0.3, 0.0]) * (li + 1))
    g = torch.Generator().manual_seed(4048)
    ids = torch.randint(0, 256, (2, 64), generator=g)
    out = model(ids, ids)
    out["loss"].backward()
    rec = {"ids": ids.numpy(), "logits": out["logits"].detach().numpy(), "loss": out["loss"].detach().numpy()}
    for name, t in model.state_dict().items():
        rec["param__" + name] = t.numpy()
    for name, p in model.named_parameters():
        rec["grad__" + name] = p.grad.numpy()
    rec["__config__"] = np.array(sorted(DECODER_CFG.items()), dtype=object).astype(str)
    np.savez_compressed(os.path.join(HERE, "decoder_small.npz"), **rec)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--reference", required=True, help="root of the reference project")
    p.add_argument("--only", choices=["decoder"], help="write only this fixture")
    args = p.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    arch, aref, cuda_ca = _import_reference(args.reference)
    if args.only == "decoder":
        make_decoder(cuda_ca)
        print("decoder fixture written to", HERE)
        return
    make_moments(arch, aref)
    make_weights_square(arch, aref)
    make_weights_tile(cuda_ca)
    make_operator_small(arch)
    make_operator_cfg1(arch)
    make_decoder(cuda_ca)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
