"""Loader for tests/golden/decoder_small.npz: the reference ContinuumDecoderLM
(cuda/continuum_attention.py:784-922) run on the CPU in float32 by
tests/golden/make_golden.py -- its state dict, a batch of bytes, the logits, the
loss and every parameter gradient."""
import os

import numpy as np
import torch

from continuum_attention_b200.decoder import ContinuumDecoderConfig

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decoder_small.npz")

# tolerances of the decoder comparisons: the reference's own model in float32 against
# this decoder in float32, so both carry float32 rounding through two layers; stated
# as max|x - ref| / max|ref| per tensor
LOGITS_TOL = 1e-4
LOSS_TOL = 1e-5        # relative
GRAD_TOL = 1e-3


def load():
    g = np.load(GOLD)
    cfg = {str(k): v for k, v in g["__config__"]}
    conv = {"vocab_size": int, "block_size": int, "d_model": int, "n_heads": int, "n_layers": int,
            "mlp_ratio": float, "dropout": float, "eps": float, "rope_theta": float, "ca_query_tile": int,
            "grad_checkpointing": lambda s: s == "True"}
    cfg = ContinuumDecoderConfig(**{k: conv[k](v) for k, v in cfg.items()})
    state = {k[len("param__"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("param__")}
    grads = {k[len("grad__"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("grad__")}
    return cfg, state, torch.from_numpy(g["ids"]), torch.from_numpy(g["logits"]), float(g["loss"]), grads


def nerr(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def compare(model, ids, logits_ref, loss_ref, grads_ref):
    """Forward + backward of `model` on ids; returns {name: error} for logits, loss and every gradient."""
    model.zero_grad(set_to_none=True)
    out = model(ids, ids)
    out["loss"].backward()
    errs = {"logits": nerr(out["logits"], logits_ref),
            "loss": abs(float(out["loss"].detach()) - loss_ref) / abs(loss_ref)}
    for name, p in model.named_parameters():
        errs["grad:" + name] = nerr(p.grad, grads_ref[name])
    return errs


def check(errs):
    bad = {k: v for k, v in errs.items()
           if not (v <= (LOGITS_TOL if k == "logits" else LOSS_TOL if k == "loss" else GRAD_TOL))}
    assert not bad, f"decoder differs from the reference model: {bad}"
