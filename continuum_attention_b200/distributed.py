"""Multi-GPU plumbing for the operator and its decoder.

* The CA operator has no coupling between heads, so a [B,H,T,D] problem splits
  into B*H independent head-sequences.  ``bh_shard`` gives each rank a
  contiguous slice of the flattened B*H range; the ranks run the operator on
  their slice with no communication, and ``gather_bh`` reassembles results
  (for verification) with one all_gather.
* The CA-S decoder trains with DDP: one process per GPU, NCCL all-reduce of
  gradients (cuda/runtime.py:23-56, cuda/continuum_attention.py:1133-1139).
  ``init_distributed`` mirrors the reference's set-up (env:// rendezvous,
  device = LOCAL_RANK, seed + rank); ``train_step`` is one optimizer step with
  bf16 autocast, gradient clipping and AdamW.
"""
from __future__ import annotations

import datetime
import os
import random
from dataclasses import dataclass
from typing import Tuple

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class DistributedContext:
    rank: int
    local_rank: int
    world_size: int
    is_main: bool
    is_distributed: bool
    device: torch.device


def init_distributed(seed: int = 1337, backend: str = None, timeout_s: float = 300.0) -> DistributedContext:
    """Process-group set-up from the torchrun environment (cuda/runtime.py:23-41)."""
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    distributed = world_size > 1
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
        device = torch.device("cuda", local_rank)
    else:
        device = torch.device("cpu")
    if distributed and not dist.is_initialized():
        be = backend or ("nccl" if device.type == "cuda" else "gloo")
        kwargs = {"device_id": device} if be == "nccl" else {}
        dist.init_process_group(be, init_method="env://", timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    random.seed(seed + rank)
    torch.manual_seed(seed + rank)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed + rank)
    return DistributedContext(rank, local_rank, world_size, rank == 0, distributed, device)


def barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def cleanup() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


def bh_shard(B: int, H: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, end) of this rank's slice of the flattened B*H head-sequence range.

    Slices are contiguous and differ in size by at most one unit.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    n = B * H
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def take_bh(t: torch.Tensor, start: int, end: int) -> torch.Tensor:
    """The [1, end-start, T, D] slice of a [B,H,T,D] tensor over the flattened B*H axis."""
    B, H, T, D = t.shape
    return t.reshape(B * H, T, D)[start:end].unsqueeze(0)


def gather_bh(part: torch.Tensor, B: int, H: int, group=None) -> torch.Tensor:
    """Reassemble per-rank [1, n_r, T, D] slices into [B,H,T,D] (all ranks receive it)."""
    world = dist.get_world_size(group)
    T, D = part.shape[-2:]
    sizes = [bh_shard(B, H, world, r) for r in range(world)]
    maxn = max(e - s for s, e in sizes)
    pad = torch.zeros(1, maxn, T, D, dtype=part.dtype, device=part.device)
    pad[:, :part.shape[1]] = part
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    full = torch.cat([b[0, : e - s] for b, (s, e) in zip(bufs, sizes)], 0)
    return full.reshape(B, H, T, D)


def build_adamw(model, lr: float = 3e-4, weight_decay: float = 0.1, betas=(0.9, 0.95)):
    """AdamW as the reference builds it (cuda/runtime.py:87-88); on CUDA parameters the
    fused implementation (one kernel per step for all parameters)."""
    params = list(model.parameters())
    fused = bool(params) and all(p.is_cuda for p in params)
    return torch.optim.AdamW(params, lr=lr, weight_decay=weight_decay, betas=betas, fused=fused)


def train_step(model, optimizer, batch: torch.Tensor, amp_dtype=torch.bfloat16, grad_clip: float = 1.0):
    """One optimizer step on ``batch`` [B,T] of byte ids: autocast forward, backward
    (DDP all-reduces gradients during it), clip, AdamW.  Returns the loss tensor
    (detached, not synchronised)."""
    optimizer.zero_grad(set_to_none=True)
    dev_type = batch.device.type
    with torch.autocast(dev_type, dtype=amp_dtype, enabled=amp_dtype is not None):
        loss = model(batch, targets=batch)["loss"]
    loss.backward()
    clip_and_step(model, optimizer, grad_clip)
    return loss.detach()


def clip_and_step(model, optimizer, grad_clip: float = 1.0):
    """``clip_grad_norm_(model.parameters(), grad_clip)`` then ``optimizer.step()``.

    With a fused AdamW the clip's scaling is folded into the optimizer kernel,
    which divides each gradient by ``grad_scale`` as it reads it: one pass over
    the gradients fewer; grad_scale = 1 / min(1, grad_clip / (norm + 1e-6)).
    """
    if grad_clip and grad_clip > 0:
        if _fused_adamw(optimizer):
            grads = [p.grad for p in model.parameters() if p.grad is not None]
            norm = torch.nn.utils.get_total_norm(grads, 2.0)
            optimizer.grad_scale = torch.clamp((norm.float() + 1e-6) / grad_clip, min=1.0)
            try:
                optimizer.step()
            finally:
                del optimizer.grad_scale
            return
        torch.nn.utils.clip_grad_norm_(model.parameters(), grad_clip)
    optimizer.step()


def _fused_adamw(optimizer) -> bool:
    return (type(optimizer) is torch.optim.AdamW and not hasattr(optimizer, "grad_scale")
            and all(g.get("fused") for g in optimizer.param_groups))
