"""World-size-2 gloo tests (CPU) of the multi-GPU host logic: B*H sharding of the
operator with no data-path collective, and one DDP training step of the decoder."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from continuum_attention_b200.distributed import bh_shard, gather_bh, take_bh


def test_bh_shard_partitions_exactly():
    for B, H in ((1, 1), (2, 16), (8, 16), (3, 5)):
        for world in (1, 2, 3, 4, 8):
            ranges = [bh_shard(B, H, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == B * H
            for (s0, e0), (s1, e1) in zip(ranges, ranges[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    from continuum_attention_b200.decoder import ContinuumDecoderConfig, ContinuumDecoderLM
    from continuum_attention_b200.distributed import build_adamw, init_distributed, train_step
    from cpu_attention import cpu_continuum_attention
    from torch.nn.parallel import DistributedDataParallel as DDP

    ctx = init_distributed(seed=123, backend="gloo", timeout_s=60)
    # 1) sharded operator: each rank runs its B*H slice, one all_gather reassembles it
    g = torch.Generator().manual_seed(5)
    B, H, T, D = 2, 3, 12, 8
    q, k, v = (torch.randn(B, H, T, D, generator=g) for _ in range(3))
    lg = torch.zeros(1)
    s, e = bh_shard(B, H, world, rank)
    part = cpu_continuum_attention(take_bh(q, s, e), take_bh(k, s, e), take_bh(v, s, e), lg.expand(e - s))
    full = gather_bh(part, B, H)
    torch.save(full, os.path.join(outdir, f"sharded_{rank}.pt"))
    # 2) one DDP step of a tiny decoder; every rank must end with identical weights
    torch.manual_seed(0)
    cfg = ContinuumDecoderConfig(block_size=16, d_model=32, n_heads=2, n_layers=1)
    model = ContinuumDecoderLM(cfg, attention_fn=cpu_continuum_attention)
    ddp = DDP(model)
    opt = build_adamw(ddp, lr=1e-3)
    gb = torch.Generator().manual_seed(99)
    batch = torch.randint(0, 256, (2 * world, 16), generator=gb)[2 * rank:2 * rank + 2]
    train_step(ddp, opt, batch, amp_dtype=None)
    torch.save({k2: p.detach() for k2, p in model.state_dict().items()}, os.path.join(outdir, f"state_{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_operator_and_ddp_step_on_gloo():
    from continuum_attention_b200.decoder import ContinuumDecoderConfig, ContinuumDecoderLM
    from continuum_attention_b200.distributed import build_adamw, train_step
    from cpu_attention import cpu_continuum_attention
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, _free_port(), d), nprocs=world, join=True)
        # sharded == unsharded, on every rank
        g = torch.Generator().manual_seed(5)
        q, k, v = (torch.randn(2, 3, 12, 8, generator=g) for _ in range(3))
        ref = cpu_continuum_attention(q, k, v, torch.zeros(3))
        for r in range(world):
            torch.testing.assert_close(torch.load(os.path.join(d, f"sharded_{r}.pt")), ref, atol=1e-6, rtol=1e-6)
        # DDP step == single-process step on the concatenated batch (mean of equal local means)
        s0 = torch.load(os.path.join(d, "state_0.pt"))
        s1 = torch.load(os.path.join(d, "state_1.pt"))
        for key in s0:
            assert torch.equal(s0[key], s1[key]), key
        torch.manual_seed(0)
        cfg = ContinuumDecoderConfig(block_size=16, d_model=32, n_heads=2, n_layers=1)
        model = ContinuumDecoderLM(cfg, attention_fn=cpu_continuum_attention)
        opt = build_adamw(model, lr=1e-3)
        gb = torch.Generator().manual_seed(99)
        batch = torch.randint(0, 256, (2 * world, 16), generator=gb)
        # per-rank losses are means over 2 sequences; DDP averages the two gradients
        opt.zero_grad(set_to_none=True)
        loss = 0.5 * (model(batch[:2], targets=batch[:2])["loss"] + model(batch[2:], targets=batch[2:])["loss"])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        for key, val in model.state_dict().items():
            torch.testing.assert_close(s0[key], val, atol=1e-5, rtol=1e-4, msg=key)
