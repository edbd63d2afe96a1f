"""Operator timing at any shape: forward and backward of the public op on one GPU.

The counterpart of the reference's operator speed phase (cuda/benchmark.py:111-125,
``timed``): CUDA events around ``continuum_attention(q, k, v, log_gain)`` and around
``torch.autograd.grad`` of ``(y * dy).sum()`` for q, k, v and the gain, medians over
the repeats.  Inputs are seeded N(0,1); ``--tau`` runs the fixed-gain variant
(log_gain = log(1/tau) for every head, as ``continuum_attention_fixed_tau``).
Several input sets rotate (``--sets``) so that timed calls do not reuse the
previous call's tensors from L2 when the sets together exceed it.

    python -m continuum_attention_b200.opbench --shape 64,4,256,64 --dtype f32 --tau 0.3
"""
from __future__ import annotations

import argparse
import json
import math
import statistics

import torch

from .attention import continuum_attention, use_impl

_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def make_inputs(shape, dtype, tau, sets, seed=0, device="cuda"):
    B, H, T, D = shape
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for _ in range(sets):
        q, k, v, dy = (torch.randn(B, H, T, D, generator=g).to(device, dtype) for _ in range(4))
        if tau is None:
            lg = torch.zeros(H)
        else:
            lg = torch.full((H,), math.log(1.0 / tau))
        out.append(tuple(t.requires_grad_(True) for t in (q, k, v, lg.to(device))) + (dy,))
    return out


def timed(inputs, warmup, repeats):
    """Median forward / backward / total milliseconds of the op over the input sets."""
    def step(i):
        q, k, v, lg, dy = inputs[i % len(inputs)]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        y = continuum_attention(q, k, v, lg)
        ev[1].record()
        torch.autograd.grad((y.float() * dy.float()).sum(), (q, k, v, lg))
        ev[2].record()
        return ev

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    evs = [step(warmup + i) for i in range(repeats)]
    torch.cuda.synchronize()
    fwd = [e[0].elapsed_time(e[1]) for e in evs]
    bwd = [e[1].elapsed_time(e[2]) for e in evs]
    tot = [e[0].elapsed_time(e[2]) for e in evs]
    return {"forward_ms": statistics.median(fwd), "backward_ms": statistics.median(bwd),
            "total_ms": statistics.median(tot)}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--shape", default="2,16,2048,64", help="B,H,T,D")
    p.add_argument("--dtype", choices=sorted(_DTYPES), default="bf16")
    p.add_argument("--tau", type=float, default=None, help="fixed gain 1/tau for every head (default: gain 1)")
    p.add_argument("--kernels", choices=["auto", "simt", "tcgen05"], default="auto")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--repeats", type=int, default=20)
    p.add_argument("--sets", type=int, default=4)
    args = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("a CUDA GPU is required")
    shape = tuple(int(x) for x in args.shape.split(","))
    if len(shape) != 4:
        raise ValueError("--shape takes B,H,T,D")
    inputs = make_inputs(shape, _DTYPES[args.dtype], args.tau, max(args.sets, 1))
    with use_impl(args.kernels):
        res = timed(inputs, max(args.warmup, 1), max(args.repeats, 1))
    B, H, T, D = shape
    flops = 4.0 * B * H * T * T * D
    print(json.dumps({"shape": list(shape), "dtype": args.dtype, "tau": args.tau, "kernels": args.kernels,
                      **res, "tflops_4bht2d": flops / (res["total_ms"] * 1e-3) / 1e12}), flush=True)


if __name__ == "__main__":
    main()
