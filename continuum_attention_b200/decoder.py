"""CA-S byte decoder: the training workload that consumes the operator.

Mirrors ``ContinuumDecoderConfig`` / ``ContinuumDecoderLM``
(cuda/continuum_attention.py:784-922): a pre-norm decoder-only byte
Transformer whose only non-standard part is Continuum Attention with a learned
per-head score gain.  Defaults give the reference's 101,205,120 parameters
(d_model 1024, 16 heads x 64, 8 layers, 4096-wide tanh-GELU MLP, byte vocab 256,
untied embedding and head, RMSNorm, RoPE theta 1e4, residual projections
initialised with std 0.02/sqrt(2 n_layers)).

``attention_fn`` defaults to the CUDA operator; tests on machines without a GPU
pass a CPU stand-in with the same signature.  On CUDA the attention block's
input side is one native kernel (``rope.rope_qkv``: QKV unpacking fused with the
rotary embedding), the attention output is stored in the projection's input
order, and each norm is one native kernel forward (``rmsnorm``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import continuum_attention
from .gelu import gelu_tanh
from .gelu import supported as gelu_supported
from .rmsnorm import add_rms_norm, add_supported
from .rmsnorm import rms_norm as native_rms_norm
from .rmsnorm import supported as native_rms_norm_supported
from .rope import apply_rope_torch, rope_qkv


@dataclass
class ContinuumDecoderConfig:
    """Configuration of the CA-S decoder (cuda/continuum_attention.py:784-813)."""
    vocab_size: int = 256
    block_size: int = 2048
    d_model: int = 1024
    n_heads: int = 16
    n_layers: int = 8
    mlp_ratio: float = 4.0
    dropout: float = 0.0
    eps: float = 1e-6
    rope_theta: float = 10000.0
    grad_checkpointing: bool = False
    ca_query_tile: int = 64

    def __post_init__(self):
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        if (self.d_model // self.n_heads) % 2:
            raise ValueError("RoPE needs even head dimension")
        if self.n_layers <= 0 or self.block_size < 2 or self.ca_query_tile <= 0:
            raise ValueError("Invalid layer, context or CA query tile count")
        if self.dropout != 0:
            raise ValueError("The CA operator has no attention dropout; use --dropout 0.0")


class RMSNorm(nn.Module):
    """weight * x * rsqrt(mean(x^2) + eps) (cuda/continuum_attention.py:815-821).

    On CUDA with a model width the native kernels cover (128, 256, 512, 1024;
    float32 or bfloat16) it runs ``rmsnorm.rms_norm``, writing its output in the
    autocast dtype the following projection consumes; elsewhere (CPU tests, other
    widths) torch's fused ``F.rms_norm``.
    """

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        out_dtype = x.dtype
        if x.is_cuda and torch.is_autocast_enabled("cuda"):
            out_dtype = torch.get_autocast_dtype("cuda")
        if native_rms_norm_supported(x, out_dtype):
            return native_rms_norm(x, self.weight, self.eps, out_dtype)
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


def apply_rope(q, k, theta: float):
    """Rotary embedding on interleaved (even, odd) pairs (cuda/continuum_attention.py:825-835)."""
    return apply_rope_torch(q, k, theta)


class ContinuumSelfAttention(nn.Module):
    def __init__(self, dim: int, heads: int, rope_theta: float, ca_query_tile: int,
                 attention_fn: Optional[Callable] = None):
        super().__init__()
        self.heads = heads
        self.head_dim = dim // heads
        self.rope_theta = rope_theta
        self.ca_query_tile = ca_query_tile
        self.qkv = Linear(dim, 3 * dim, bias=False)
        self.out = Linear(dim, dim, bias=False)
        self.out._residual_proj = True
        # variant S: positive trainable per-head score gain g = exp(rho), starting at 1
        self.log_qk_gain = nn.Parameter(torch.zeros(heads))
        self.attention_fn = attention_fn or continuum_attention

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = rope_qkv(self.qkv(x), self.heads, self.rope_theta)
        if self.attention_fn is continuum_attention:
            # the operator stores y [B,T,H,D]: the projection's input below is a view of it
            y = continuum_attention(q, k, v, self.log_qk_gain, self.ca_query_tile, out_layout="bthd")
        else:
            y = self.attention_fn(q, k, v, self.log_qk_gain, self.ca_query_tile)
        return self.out(y.transpose(1, 2).reshape(B, T, C))


class _WeightGradFp32(torch.autograd.Function):
    """y = x W^T with W the fp32 master weight cast to bf16, as bf16 autocast runs
    nn.Linear; the backward writes dW straight out of the GEMM in fp32 (bf16
    operands, fp32 accumulate and store), where autocast stores a bf16 dW and then
    converts it to fp32 in a separate pass over the weight."""

    @staticmethod
    def forward(ctx, x, weight):
        wb = weight.to(torch.bfloat16)
        xb = x.to(torch.bfloat16)
        ctx.save_for_backward(xb, wb)
        return F.linear(xb, wb)

    @staticmethod
    def backward(ctx, dy):
        xb, wb = ctx.saved_tensors
        dy = dy.to(torch.bfloat16)
        dx = dy @ wb if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = torch.mm(dy.reshape(-1, dy.shape[-1]).t(), xb.reshape(-1, xb.shape[-1]), out_dtype=torch.float32)
        return dx, dw


class Linear(nn.Linear):
    """nn.Linear (same parameters and state-dict keys) whose bias-free bf16-autocast
    CUDA forward keeps the weight gradient in fp32 end to end (``_WeightGradFp32``);
    every other case is nn.Linear itself."""

    def forward(self, x):
        if (self.bias is None and x.is_cuda and self.weight.dtype == torch.float32
                and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16):
            return _WeightGradFp32.apply(x, self.weight)
        return super().forward(x)


class GELUMLP(nn.Module):
    def __init__(self, dim: int, ratio: float):
        super().__init__()
        hidden = int(dim * ratio)
        self.fc1 = Linear(dim, hidden, bias=False)
        self.fc2 = Linear(hidden, dim, bias=False)
        self.fc2._residual_proj = True

    def forward(self, x):
        h = self.fc1(x)
        # the native kernel pair on CUDA (same tanh approximation, fp32 arithmetic)
        a = gelu_tanh(h) if gelu_supported(h) else F.gelu(h, approximate="tanh")
        return self.fc2(a)


class CADecoderBlock(nn.Module):
    def __init__(self, cfg: ContinuumDecoderConfig, attention_fn=None):
        super().__init__()
        d = cfg.d_model
        self.norm1 = RMSNorm(d, cfg.eps)
        self.attn = ContinuumSelfAttention(d, cfg.n_heads, cfg.rope_theta, cfg.ca_query_tile, attention_fn)
        self.norm2 = RMSNorm(d, cfg.eps)
        self.mlp = GELUMLP(d, cfg.mlp_ratio)

    def forward(self, x):
        x = x + self.attn(self.norm1(x))
        return x + self.mlp(self.norm2(x))


class ContinuumDecoderLM(nn.Module):
    """Byte-level decoder; ``forward(ids, targets=None) -> {'logits', 'loss'}``."""

    def __init__(self, cfg: ContinuumDecoderConfig, attention_fn: Optional[Callable] = None):
        super().__init__()
        self.cfg = cfg
        self.byte_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.blocks = nn.ModuleList([CADecoderBlock(cfg, attention_fn) for _ in range(cfg.n_layers)])
        self.norm_f = RMSNorm(cfg.d_model, cfg.eps)
        self.lm_head = Linear(cfg.d_model, cfg.vocab_size, bias=False)   # not tied to byte_emb
        self.residual_init_scale = 1.0 / math.sqrt(2.0 * cfg.n_layers)
        self.apply(self._init_weights)

    def _init_weights(self, m):
        if isinstance(m, nn.Linear):
            std = 0.02 * self.residual_init_scale if getattr(m, "_residual_proj", False) else 0.02
            nn.init.normal_(m.weight, mean=0.0, std=std)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)

    @staticmethod
    def _add_norm(x, r, norm):
        """(x + r, norm(x + r)): one native kernel when the residual stream is float32
        and the branch output bfloat16 (bf16 autocast on CUDA), else the two steps."""
        if add_supported(x, r) and torch.is_autocast_enabled("cuda") and \
                torch.get_autocast_dtype("cuda") == torch.bfloat16:
            return add_rms_norm(x, r, norm.weight, norm.eps)
        x = x + r
        return x, norm(x)

    def forward(self, input_ids, targets=None):
        if input_ids.dim() != 2 or input_ids.shape[1] > self.cfg.block_size:
            raise ValueError("Input must be [B,T] with T<=block_size")
        x = self.byte_emb(input_ids)
        if self.cfg.grad_checkpointing and self.training:
            for block in self.blocks:
                x = torch.utils.checkpoint.checkpoint(block, x, use_reentrant=False)
            h = self.norm_f(x)
        else:
            # the blocks' residual adds run together with the norm that follows each
            # (the next block's norm1, or norm_f after the last block)
            h = self.blocks[0].norm1(x)
            for i, block in enumerate(self.blocks):
                x, h = self._add_norm(x, block.attn(h), block.norm2)
                nxt = self.blocks[i + 1].norm1 if i + 1 < len(self.blocks) else self.norm_f
                x, h = self._add_norm(x, block.mlp(h), nxt)
        logits = self.lm_head(h)
        out = {"logits": logits}
        if targets is not None:
            out["loss"] = F.cross_entropy(logits[:, :-1, :].reshape(-1, self.cfg.vocab_size),
                                          targets[:, 1:].reshape(-1), reduction="mean")
        return out


def count_parameters(model: nn.Module) -> dict:
    params = list(model.parameters())
    return {"total": sum(p.numel() for p in params),
            "trainable": sum(p.numel() for p in params if p.requires_grad)}


def _main(argv=None):
    """Training-step throughput of the CA-S decoder on one GPU, synthetic bytes:
    ``python -m continuum_attention_b200.decoder [--steps K] [--warmup W]``.
    Prints one JSON line (tokens/s, ms per step, last loss)."""
    import argparse
    import json

    from .distributed import build_adamw, train_step
    p = argparse.ArgumentParser(description=_main.__doc__)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--seq-len", type=int, default=2048)
    args = p.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(1337)
    model = ContinuumDecoderLM(ContinuumDecoderConfig(block_size=args.seq_len)).to(dev)
    opt = build_adamw(model)
    g = torch.Generator(device="cpu").manual_seed(2000)
    batch = torch.randint(0, 256, (args.batch, args.seq_len), generator=g).to(dev)
    for _ in range(args.warmup):
        train_step(model, opt, batch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    loss = None
    for _ in range(args.steps):
        loss = train_step(model, opt, batch)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    print(json.dumps({"metric": "CA-S decoder train tokens/s", "value": args.batch * args.seq_len / (ms * 1e-3),
                      "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "loss": None if loss is None else float(loss.item()),
                      "params": count_parameters(model)["total"]}))


if __name__ == "__main__":
    _main()
