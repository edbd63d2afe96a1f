"""The ~5M-parameter TinyLM of the reference's small-model study, with the CA operator.

Mirrors ``architecture.TinyLM`` (architecture.py:204-245): six pre-norm blocks,
width 256, SwiGLU hidden 720, 4 heads x 64, byte vocabulary with the LM head
tied to the token embedding, learned positional embedding, RMSNorm (eps 1e-5),
Linear weights and embeddings initialised N(0, 0.02).  ``CausalAttention``
keeps the reference's variants (architecture.py:108-177):

* continuous (exact continuum attention): P (fixed tau), R (no gain), S (learned
  per-head gain from tau 1), H (learned gain from tau 0.30) -- the drop-in site
  ``self._weights(q, k, v) @ v`` (:175) is the B200 operator: the query scaling of
  ``_qkv`` (:135-145) becomes the operator's per-head log gain, so P runs with
  log(1/tau) and S/H pass their ``log_qk_gain`` parameter directly;
* softmax controls: A, B, F, G through ``F.scaled_dot_product_attention``.

``TinyLMTrainer`` runs the reference's training step (cross entropy, backward,
clip 1.0, AdamW with the geometry parameter group, benchmark.py:193-217) as one
CUDA graph: at a few thousand tokens per step the model is launch-bound, so the
whole step is captured once and replayed.
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import continuum_attention
from .rmsnorm import rms_norm as native_rms_norm
from .rmsnorm import supported as rms_norm_supported

CONTINUOUS = ("P", "R", "S", "H")
SOFTMAX = ("A", "B", "F", "G")


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) * weight (architecture.py:21-28): the native kernel
    (``rmsnorm.rms_norm``) on CUDA at the widths it covers, else torch's fused one."""

    def __init__(self, width: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.eps = eps

    def forward(self, x):
        if rms_norm_supported(x, x.dtype):
            return native_rms_norm(x, self.weight, self.eps, x.dtype)
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


class CausalAttention(nn.Module):
    def __init__(self, width: int, heads: int, seq_len: int, variant: str = "P", fixed_tau: float = 0.30,
                 attention_fn: Optional[Callable] = None):
        super().__init__()
        if variant not in CONTINUOUS + SOFTMAX:
            raise ValueError("variant must be A, B, F, G, P, R, S or H")
        if width % heads:
            raise ValueError("width must be divisible by heads")
        if fixed_tau <= 0:
            raise ValueError("fixed_tau must be > 0")
        self.variant = variant
        self.heads = heads
        self.width = width
        self.head_dim = width // heads
        self.fixed_tau = float(fixed_tau)
        self.continuous = variant in CONTINUOUS
        if variant in ("F", "G", "S", "H"):
            init_log_gain = -math.log(0.30) if variant in ("G", "H") else 0.0
            self.log_qk_gain = nn.Parameter(torch.full((heads,), init_log_gain))
        self.qkv = nn.Linear(width, 3 * width, bias=False)
        self.out = nn.Linear(width, width, bias=False)
        self.attention_fn = attention_fn or continuum_attention

    def _log_gain(self, device):
        if self.variant in ("S", "H"):
            return self.log_qk_gain
        value = math.log(1.0 / self.fixed_tau) if self.variant == "P" else 0.0
        return torch.full((self.heads,), value, device=device)

    def forward(self, x):
        B, T, _ = x.shape
        q, k, v = self.qkv(x).chunk(3, dim=-1)
        q, k, v = (t.reshape(B, T, self.heads, self.head_dim).transpose(1, 2) for t in (q, k, v))
        if self.continuous and self.attention_fn is continuum_attention:
            # stored [B,T,H,D]: the output projection below reads it without a copy
            y = continuum_attention(q, k, v, self._log_gain(x.device), 64, out_layout="bthd")
        elif self.continuous:
            y = self.attention_fn(q, k, v, self._log_gain(x.device), 64)
        else:
            if self.variant == "B":
                q = q * (1.0 / self.fixed_tau)
            elif self.variant in ("F", "G"):
                q = q * self.log_qk_gain.exp().view(1, -1, 1, 1)
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, dropout_p=0.0)
        return self.out(y.transpose(1, 2).reshape(B, T, self.width))


class SwiGLU(nn.Module):
    def __init__(self, width: int, hidden: int):
        super().__init__()
        self.gate_up = nn.Linear(width, 2 * hidden, bias=False)
        self.down = nn.Linear(hidden, width, bias=False)

    def forward(self, x):
        gate, value = self.gate_up(x).chunk(2, dim=-1)
        return self.down(F.silu(gate) * value)


class Block(nn.Module):
    def __init__(self, width, hidden, heads, seq_len, variant, fixed_tau, attention_fn=None):
        super().__init__()
        self.norm_attn = RMSNorm(width)
        self.attn = CausalAttention(width, heads, seq_len, variant, fixed_tau, attention_fn)
        self.norm_mlp = RMSNorm(width)
        self.mlp = SwiGLU(width, hidden)

    def forward(self, x):
        x = x + self.attn(self.norm_attn(x))
        return x + self.mlp(self.norm_mlp(x))


class TinyLM(nn.Module):
    """Six-layer pre-norm byte model (5,008,640 parameters for B/P/R at the defaults)."""

    def __init__(self, variant: str = "P", seq_len: int = 192, width: int = 256, hidden: int = 720,
                 heads: int = 4, fixed_tau: float = 0.30, attention_fn: Optional[Callable] = None):
        super().__init__()
        self.seq_len = seq_len
        self.variant = variant
        self.tok_embed = nn.Embedding(256, width)
        self.pos_embed = nn.Embedding(seq_len, width)
        # b0 .. b5 as in the reference, so state dicts carry the same keys
        for i in range(6):
            setattr(self, f"b{i}", Block(width, hidden, heads, seq_len, variant, fixed_tau, attention_fn))
        self.final_norm = RMSNorm(width)
        self.lm_head = nn.Linear(width, 256, bias=False)
        self.lm_head.weight = self.tok_embed.weight
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module):
        if isinstance(module, (nn.Linear, nn.Embedding)):
            torch.nn.init.normal_(module.weight, mean=0.0, std=0.02)

    def forward(self, tokens):
        _, length = tokens.shape
        if length > self.seq_len:
            raise ValueError("Sequence exceeds model seq_len")
        pos = torch.arange(length, device=tokens.device)
        x = self.tok_embed(tokens) + self.pos_embed(pos)[None, :, :]
        for i in range(6):
            x = getattr(self, f"b{i}")(x)
        return self.lm_head(self.final_norm(x))


def parameters(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters() if p.requires_grad)


def build_optimizer(model: TinyLM, lr: float = 4e-4, weight_decay: float = 0.1, geometry_lr_mult: float = 8.0,
                    capturable: bool = False):
    """AdamW(betas 0.9/0.95) with the per-head gains in their own group (benchmark.py:193-205)."""
    named = list(model.named_parameters())
    small = [p for n, p in named if n.endswith("log_qk_gain")]
    dense = [p for n, p in named if not n.endswith("log_qk_gain")]
    groups = [{"params": dense, "lr": lr, "weight_decay": weight_decay}]
    if small:
        groups.append({"params": small, "lr": lr * geometry_lr_mult, "weight_decay": 0.0})
    cuda = all(p.is_cuda for p in model.parameters())
    extra = {"capturable": True, "foreach": True} if capturable else {"fused": cuda}
    return torch.optim.AdamW(groups, betas=(0.9, 0.95), **extra)


def train_step(model: TinyLM, optimizer, x, target):
    """One reference training step; returns the loss tensor (not synchronised)."""
    logits = model(x)
    loss = F.cross_entropy(logits.reshape(-1, 256), target.reshape(-1))
    optimizer.zero_grad(set_to_none=False)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    optimizer.step()
    return loss.detach()


class TinyLMTrainer:
    """The training step captured as one CUDA graph over static batch buffers."""

    def __init__(self, model: TinyLM, batch_size: int, seq_len: int, lr: float = 4e-4,
                 weight_decay: float = 0.1, geometry_lr_mult: float = 8.0, warmup: int = 3):
        dev = next(model.parameters()).device
        self.model = model
        self.optimizer = build_optimizer(model, lr, weight_decay, geometry_lr_mult, capturable=True)
        self.x = torch.zeros(batch_size, seq_len, dtype=torch.long, device=dev)
        self.target = torch.zeros_like(self.x)
        initial = [p.detach().clone() for p in model.parameters()]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):            # allocator and kernel warm-up outside the graph
                train_step(model, self.optimizer, self.x, self.target)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = train_step(model, self.optimizer, self.x, self.target)
        # undo the warm-up updates in place (the graph holds these very tensors)
        with torch.no_grad():
            for p, p0 in zip(model.parameters(), initial):
                p.copy_(p0)
            for state in self.optimizer.state.values():
                for value in state.values():
                    if torch.is_tensor(value):
                        value.zero_()

    def step(self, x, target):
        """Copy the batch into the graph's buffers and replay one training step."""
        self.x.copy_(x, non_blocking=True)
        self.target.copy_(target, non_blocking=True)
        self.graph.replay()
        return self.loss


def _main(argv=None):
    """Training-step throughput of TinyLM (fixed-tau variant P by default, fp32 as the
    reference trains it) on one GPU, synthetic bytes, the step as one CUDA graph:
    ``python -m continuum_attention_b200.tinylm [--steps K] [--seq-len T]``.
    Prints one JSON line."""
    import argparse
    import json
    p = argparse.ArgumentParser(description=_main.__doc__)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--seq-len", type=int, default=192)
    p.add_argument("--variant", default="P")
    args = p.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(1729)
    model = TinyLM(variant=args.variant, seq_len=args.seq_len).to(dev)
    g = torch.Generator(device="cpu").manual_seed(1729)
    batch = torch.randint(0, 256, (args.batch, args.seq_len + 1), generator=g).to(dev)
    x, y = batch[:, :-1].contiguous(), batch[:, 1:].contiguous()
    trainer = TinyLMTrainer(model, batch_size=args.batch, seq_len=args.seq_len)
    for _ in range(5):
        trainer.step(x, y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        loss = trainer.step(x, y)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    print(json.dumps({"metric": f"TinyLM-{args.variant} train tokens/s", "value": args.batch * args.seq_len / (ms * 1e-3),
                      "ms_per_step": ms, "steps": args.steps, "seq_len": args.seq_len, "loss": float(loss.item()),
                      "params": parameters(model)}))


if __name__ == "__main__":
    _main()
