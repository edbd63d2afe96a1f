#!/usr/bin/env python3
"""Benchmark of the Continuum Attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--kernels auto|simt|tcgen05]

Workload (a "step"): one forward + backward of the CA operator on one batch of
BASELINE config 2, [B,H,T,D] = [2,16,2048,64] bf16 with q, k, v, dY ~ N(0,1)
and gain 1, causal.  Multi-GPU (torchrun, one rank per GPU): the operator
shards over B*H with no communication, so every rank processes its own batch
of the same shape (weak scaling) and ``value`` counts all ranks' work.

Metric: CA fwd+bwd TFLOP/s counting the two GEMMs per direction,
4*B*H*T^2*D per step (3.436e10 at config 2).  ``value`` is device-timed
(CUDA events, max over ranks) with inputs resident in HBM; ``e2e`` is the same
metric through the public autograd op with pinned host inputs copied in and
gradients copied out inside the timed region, consecutive steps pipelined over
a copy-in, a compute and a copy-out stream.

The line also carries "decoder": the CA-S decoder training step (BASELINE
config 4, 101,205,120 parameters, 8 x 2048 random bytes per GPU, bf16 autocast,
AdamW) in tokens/s over all ranks, with DDP over NCCL when N > 1
(``--no-decoder`` skips it), and at N=1 "tinylm": the reference's 5M-parameter
TinyLM in its fixed-tau CA variant P (fp32, batch 8, T = 192 and 512), the
training step run as one CUDA graph (``--no-tinylm`` skips it), and "config3_sharded":
BASELINE config 3 at B = 8, [8,16,16384,64], its 128 head-sequences split over the
ranks (strong scaling, ``--no-config3`` skips it).

``--impl reference`` times the reference algorithm's CPU path (the float32
restatement in oracle/, all host threads) on the same workload, one whole
config-2 batch per step with the same --steps / --warmup, and prints the same
line with "impl": "reference".  At N=1 the GPU arm's line also carries
"reference_cuda": the reference's own CUDA kernels (built from its sources into
oracle/_ref) timed at config 2 on the same GPU, outside the timed region.
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SHAPE = (2, 16, 2048, 64)
METRIC = "CA fwd+bwd TFLOP/s @[2,16,2048,64] bf16 (4*B*H*T^2*D per step)"
UNIT = "TFLOP/s"
# published reference figure: CUDA v6 on one V100, fp16, same shape, 16.603 ms per fwd+bwd (README.md:97 of the reference)
PUBLISHED_V100_V6_MS = 16.603
N_INPUT_SETS = 8   # rotating input sets, 8 x ~92 MB >> 126 MB L2


def flops_per_step(shape=SHAPE) -> float:
    B, H, T, D = shape
    return 4.0 * B * H * T * T * D


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("hbm_gbs", 6650.0)), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def _profile_traffic(kernel_tag: str):
    """dram bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    import glob
    import re
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        for line in open(path):
            m = re.match(r"\s*TRAFFIC_BYTES_PER_LAUNCH\s+(\S+)\s*=\s*([0-9.eE+]+)", line)
            if m and m.group(1) == kernel_tag:
                return float(m.group(2))
    return None


def _pci_bus_id(local: int) -> str:
    """PCI bus id of CUDA device `local` (nvidia-smi and NVML index GPUs their own way)."""
    p = torch.cuda.get_device_properties(local)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


@contextlib.contextmanager
def _gpu_local_cpus(local: int):
    """Run the block on the host CPUs NVML reports as local to GPU `local`, so that
    pinned host buffers allocated inside sit on that GPU's NUMA node; the previous
    CPU affinity is restored afterwards.  Yields whether the block runs on GPU-local
    CPUs (bound here, or the process's CPUs were all local already)."""
    old = os.sched_getaffinity(0)
    bound = False
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(_pci_bus_id(local).encode())
            words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
            cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (int(m) >> b) & 1} & old
            if cpus and cpus != old:
                os.sched_setaffinity(0, cpus)
            bound = bool(cpus)     # running on GPU-local CPUs (bound here, or already all local)
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        bound = False
    try:
        yield bound
    finally:
        os.sched_setaffinity(0, old)


def _is_float(x):
    try:
        float(x)
        return True
    except ValueError:
        return False


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", _pci_bus_id(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        power = [float(p[3]) for p in (l.split(",") for l in self.lines) if len(p) >= 9 and _is_float(p[3])]
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows),
                "power_w": statistics.median(power) if power else None}


def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(world, x: float) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_reference_sample(steps: int, warmup: int, shape=SHAPE):
    """Time the reference algorithm's CPU path (oracle restatement, float32, all host threads).

    Each step is one forward+backward of ``shape`` (default: the whole config-2 batch,
    [2,16,2048,64]).  Returns (tflops, median_s, threads, sample).
    """
    from oracle.ca_oracle import ca_forward_backward
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(2)
    q, k, v, dy = (torch.randn(shape, generator=g) for _ in range(4))
    lg = torch.zeros(shape[1])
    times = []
    for it in range(warmup + steps):
        t0 = time.perf_counter()
        ca_forward_backward(q, k, v, lg, dy, query_tile=128, dtype=torch.float32)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
    med = statistics.median(times)
    sample = (f"{list(shape)} fp32 fwd+bwd per step (oracle/ca_oracle.py, the reference's tiled CPU "
              f"algorithm restated, query tile 128), median of {len(times)}")
    return flops_per_step(shape) / med / 1e12, med, threads, sample


def _config(world: int, kernels: str):
    """The workload description both arms print (BASELINE config 2 per rank)."""
    B, H, T, D = SHAPE
    return {"workload": "CA operator fwd+bwd, BASELINE config 2 ([2,16,2048,64] bf16, gain 1, causal) "
                        "per rank; operator sharded over B*H, no collective",
            "global_batch": B * world, "seq_len": T, "heads": H, "head_dim": D,
            "parallelism": f"bh-shard x{world}", "kernels": kernels,
            "l2": f"{N_INPUT_SETS} rotating input sets (~{N_INPUT_SETS * 92} MB) > 126 MB L2",
            "vs_baseline_ref": "reference CUDA v6, 1x V100 fp16, 16.603 ms (README.md:97)"}


def run_reference_arm(args, world, rank):
    """The reference's CPU path on the host cores of rank 0 over the whole config-2 batch,
    with the same --steps and --warmup as the GPU arm (about 5-15 s per step on 8-16
    cores).  The reference itself is Python and is not present on the GPU box, so its
    restatement in oracle/ (pinned to the reference's outputs by tests/test_oracle.py)
    stands in: "kind": "port"."""
    if rank != 0:
        return
    steps, warmup = max(1, args.steps), max(0, args.warmup)
    tflops, med, threads, sample = cpu_reference_sample(steps, warmup)
    line = {
        "metric": METRIC, "value": tflops, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": med * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config(world, args.kernels),
        "cpu_baseline": {"value": tflops, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tflops, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_cuda(local):
    """The reference's own CUDA kernels (oracle/_ref, built from its sources) at config 2
    on this GPU, timed like the reference's speed phase (cuda/benchmark.py:111-125):
    CUDA events around the op and around autograd.grad, medians over 7 repeats with 2
    input sets.  None when oracle/_ref is not built."""
    from oracle import ref_cuda
    if not ref_cuda.available():
        return None
    import continuum_attention_b200 as ca
    dev = torch.device("cuda", local)
    out = {"shape": list(SHAPE), "query_tile": 128, "source": "oracle/_ref (reference sources, compiled here)"}
    runs = (("reference_prefix_v6_fp16", lambda q, k, v, lg: ref_cuda.ref_continuum_attention(q, k, v, lg, 128,
                                                                                            "prefix_v6"),
             torch.float16),
            ("reference_prefix_bf16", lambda q, k, v, lg: ref_cuda.ref_continuum_attention(q, k, v, lg, 128,
                                                                                         "prefix"),
             torch.bfloat16),
            ("ours_bf16", lambda q, k, v, lg: ca.continuum_attention(q, k, v, lg, 128), torch.bfloat16))
    for name, fn, dtype in runs:
        sets = []
        for sd in range(2):
            g = torch.Generator(device="cpu").manual_seed(1649 + sd)
            q, k, v, dy = (torch.randn(SHAPE, generator=g).to(dev, dtype) for _ in range(4))
            lg = torch.zeros(SHAPE[1], device=dev)
            sets.append(tuple(t.requires_grad_(True) for t in (q, k, v, lg)) + (dy,))

        def step(i):
            q, k, v, lg, dy = sets[i % 2]
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record()
            y = fn(q, k, v, lg)
            ev[1].record()
            torch.autograd.grad((y.float() * dy.float()).sum(), (q, k, v, lg))
            ev[2].record()
            return ev

        for i in range(2):
            step(i)
        torch.cuda.synchronize()
        evs = [step(i) for i in range(7)]
        torch.cuda.synchronize()
        med = lambda a, b: statistics.median(e[a].elapsed_time(e[b]) for e in evs)
        out[name] = {"forward_ms": med(0, 1), "backward_ms": med(1, 2), "total_ms": med(0, 2)}
        del sets
    torch.cuda.empty_cache()
    out["speedup_vs_prefix_v6_fp16"] = (out["reference_prefix_v6_fp16"]["total_ms"] /
                                        out["ours_bf16"]["total_ms"])
    return out


def _make_sets(n, device, dtype, seed):
    sets = []
    g = torch.Generator(device="cpu").manual_seed(seed)
    for _ in range(n):
        q, k, v, dy = (torch.randn(SHAPE, generator=g).to(device, dtype) for _ in range(4))
        sets.append((q, k, v, dy))
    return sets


def run_decoder(args, world, rank, local, steps: int, warmup: int):
    """CA-S decoder training step: 101,205,120 parameters, 8
    sequences x 2048 random bytes per GPU, bf16 autocast, AdamW, gradient clip 1.0,
    DDP over NCCL when world > 1 (weak scaling).  Returns a dict for the JSON line."""
    from torch.nn.parallel import DistributedDataParallel as DDP
    from continuum_attention_b200.decoder import ContinuumDecoderConfig, ContinuumDecoderLM, count_parameters
    from continuum_attention_b200.distributed import build_adamw, train_step
    dev = torch.device("cuda", local)
    torch.manual_seed(1337)                      # identical initial weights on every rank
    cfg = ContinuumDecoderConfig()
    model = ContinuumDecoderLM(cfg).to(dev)
    nparams = count_parameters(model)["total"]
    net = DDP(model, device_ids=[local], gradient_as_bucket_view=True) if world > 1 else model
    opt = build_adamw(net)
    per_gpu_batch, T = 8, cfg.block_size
    g = torch.Generator(device="cpu").manual_seed(2000 + rank)
    batches = [torch.randint(0, 256, (per_gpu_batch, T), generator=g).to(dev) for _ in range(4)]
    for i in range(warmup):
        train_step(net, opt, batches[i % 4])
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    loss = None
    for i in range(steps):
        loss = train_step(net, opt, batches[i % 4])
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(world, e0.elapsed_time(e1))
    tokens = world * per_gpu_batch * T * steps
    del net, opt, model
    torch.cuda.empty_cache()
    return {"metric": "CA-S decoder train tokens/s (BASELINE config 4)", "value": tokens / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": ms / steps, "params": nparams, "per_gpu_batch": per_gpu_batch, "seq_len": T,
            "parallelism": f"ddp{world}" if world > 1 else "single", "dtype": "bf16 autocast, fp32 master",
            "optimizer": "AdamW(lr 3e-4, wd 0.1, betas 0.9/0.95), clip 1.0", "scaling": "weak",
            "final_loss": float(loss.item()) if loss is not None else None, "data": "synthetic uniform bytes"}


def _config3_inputs(n, T, D, dev, seed):
    """n head-sequences of BASELINE config 3's input recipe: q, k ~ N(0, 2^2) (score std
    about 4), a seeded 10% of keys duplicating their left neighbour, bf16."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(1, n, T, D, generator=g) * 2).to(dev, torch.bfloat16)
    k = torch.randn(1, n, T, D, generator=g) * 2
    dup = torch.rand(T, generator=g) < 0.1
    dup[0] = False
    for j in torch.nonzero(dup).flatten().tolist():
        k[:, :, j] = k[:, :, j - 1]
    k = k.to(dev, torch.bfloat16)
    v, dy = (torch.randn(1, n, T, D, generator=g).to(dev, torch.bfloat16) for _ in range(2))
    return q, k, v, dy


def _config3_time(q, k, v, dy, steps, warmup, world, local, sample_clocks):
    """Times fwd+bwd of the public op on one slice; returns (max-over-ranks ms for all
    steps, forward ms per step, backward ms per step, clock summary or None)."""
    import continuum_attention_b200 as ca
    lg = torch.zeros(q.shape[1], device=q.device, requires_grad=True)
    stream = torch.cuda.current_stream(q.device)

    def step(ev_mid=None):
        qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
        y = ca.continuum_attention(qq, kk, vv, lg, 128)
        if ev_mid is not None:
            ev_mid.record(stream)
        return torch.autograd.grad(y, (qq, kk, vv, lg), dy)

    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps + 1)]
    clk = ClockSampler(local) if sample_clocks else None
    if clk is not None:
        clk.__enter__()
        time.sleep(0.25)
    for _ in range(warmup):   # right before the timed steps, after the sampler's start
        step()
    torch.cuda.synchronize()
    _barrier(world)
    evs[0].record(stream)
    for i in range(steps):
        step(evs[2 * i + 1])
        evs[2 * i + 2].record(stream)
    torch.cuda.synchronize()
    if clk is not None:
        time.sleep(0.1)
        clk.__exit__(None, None, None)
    ms = _max_over_ranks(world, evs[0].elapsed_time(evs[-1]))
    fwd = statistics.mean(evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(steps))
    bwd = statistics.mean(evs[2 * i + 1].elapsed_time(evs[2 * i + 2]) for i in range(steps))
    return ms, fwd, bwd, (clk.summary() if clk is not None else None)


def run_config3_sharded(world, rank, local, T: int = 16384, steps: int = 5, warmup: int = 2):
    """BASELINE config 3 across the ranks: [8,16,T,64] bf16 with q, k ~ N(0, 2^2) (score
    std about 4) and a seeded 10% of keys duplicating their left neighbour, fwd+bwd
    through the public op.  The 128 head-sequences are split into contiguous slices,
    one per rank, with no communication: the total work is fixed, so this is the
    operator's strong scaling.  The timed steps carry the SM-clock record of this rank.
    On one GPU the eighth-size slice that each of 8 ranks runs is timed as well
    ("slice_of_8"), so that the per-head-sequence cost of the two slice sizes can be
    compared on the same GPU.  Returns a dict for the JSON line."""
    from continuum_attention_b200.distributed import bh_shard
    B, H, D = 8, 16, 64
    start, end = bh_shard(B, H, world, rank)
    n = end - start
    dev = torch.device("cuda", local)
    q, k, v, dy = _config3_inputs(n, T, D, dev, 3000 + rank)
    ms, fwd, bwd, clocks = _config3_time(q, k, v, dy, steps, warmup, world, local, sample_clocks=True)
    del q, k, v, dy
    flops = 4.0 * B * H * T * T * D
    out = {"metric": f"CA fwd+bwd TFLOP/s, BASELINE config 3 at B=8 ([8,16,{T},64] bf16) over all ranks",
           "value": flops * steps / (ms * 1e-3) / 1e12, "unit": UNIT, "n_gpus": world, "steps": steps,
           "warmup": warmup, "ms_per_step": ms / steps, "forward_ms": fwd, "backward_ms": bwd,
           "head_sequences_per_rank": n, "scaling": "strong", "clocks": clocks,
           "parallelism": f"bh-shard x{world}", "data": "synthetic (score std 4, 10% duplicated keys)"}
    if world == 1:
        n8 = (B * H) // 8
        q, k, v, dy = _config3_inputs(n8, T, D, dev, 3000)
        ms8, fwd8, bwd8, clocks8 = _config3_time(q, k, v, dy, steps, warmup, 1, local, sample_clocks=True)
        del q, k, v, dy
        out["slice_of_8"] = {"head_sequences": n8, "ms_per_step": ms8 / steps, "forward_ms": fwd8,
                             "backward_ms": bwd8, "clocks": clocks8,
                             "us_per_head_sequence": 1e3 * ms8 / steps / n8,
                             "us_per_head_sequence_full": 1e3 * ms / steps / n}
    torch.cuda.empty_cache()
    return out


def run_tinylm(local, steps: int = 50):
    """TinyLM P (fixed tau 0.30, fp32 as the reference trains it) training tokens/s on
    one GPU at the reference's defaults (batch 8, T = 192) and at T = 512: the
    whole step as a CUDA graph, and eagerly for comparison."""
    from continuum_attention_b200.tinylm import TinyLM, TinyLMTrainer, build_optimizer, train_step
    dev = torch.device("cuda", local)
    out = {"metric": "TinyLM-P train tokens/s (architecture.py TinyLM, 5,008,640 params, fp32)",
           "unit": "tokens/s", "batch": 8, "data": "synthetic uniform bytes"}
    g = torch.Generator(device="cpu").manual_seed(1729)
    for T in (192, 512):
        torch.manual_seed(1729)
        model = TinyLM(variant="P", seq_len=T).to(dev)
        batch = torch.randint(0, 256, (8, T + 1), generator=g).to(dev)
        x, y = batch[:, :-1].contiguous(), batch[:, 1:].contiguous()
        trainer = TinyLMTrainer(model, batch_size=8, seq_len=T)
        for _ in range(5):
            trainer.step(x, y)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            trainer.step(x, y)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        out[f"T{T}_graph_tokens_per_s"] = 8 * T / (ms * 1e-3)
        out[f"T{T}_graph_ms_per_step"] = ms
        if T == 192:
            torch.manual_seed(1729)
            eager = TinyLM(variant="P", seq_len=T).to(dev)
            opt = build_optimizer(eager)
            for _ in range(5):
                train_step(eager, opt, x, y)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(steps):
                train_step(eager, opt, x, y)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            out["T192_eager_tokens_per_s"] = 8 * T / (ms * 1e-3)
        del trainer, model
    torch.cuda.empty_cache()
    return out


def run_ours(args, world, rank, local):
    import continuum_attention_b200 as ca
    from continuum_attention_b200 import _native
    dev = torch.device("cuda", local)
    dtype = torch.bfloat16
    B, H, T, D = SHAPE
    impl = args.kernels
    sets = _make_sets(N_INPUT_SETS, dev, dtype, seed=1000 + rank)
    lg = torch.zeros(H, device=dev)
    ws = torch.empty(ca.workspace_bytes(B, H, T, D, dtype), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i, ev_mid=None, ev_end=None):
        q, k, v, dy = sets[i % N_INPUT_SETS]
        o, stats, o32 = ca.forward_raw(q, k, v, lg, impl=impl, want_f32=True)
        nf = _native.lib().ca_last_launch_count()
        if ev_mid is not None:
            ev_mid.record(stream)
        ca.backward_raw(q, k, v, o, dy, lg, stats, want_dgain=True, impl=impl, workspace=ws, o_f32=o32)
        nb = _native.lib().ca_last_launch_count()
        if ev_end is not None:
            ev_end.record(stream)
        return nf + nb

    # Timed region 1 (the metric): K steps between two events and nothing in between.
    # An event recorded between two kernels ends the programmatic-dependent-launch
    # overlap of the second with the first (about 10 us per config-2 step), so the
    # per-call split comes from timed region 2, the same K steps with an event after
    # each forward and each backward call (the forward of step i runs between the
    # end of step i-1, or the start, and mid_i).
    ev_start, ev_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev_start2 = torch.cuda.Event(enable_timing=True)
    ev_mid = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev_end = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches = 0
    with ClockSampler(local) as clk:
        time.sleep(0.25)   # the sampler's first readings
        # warm-up right before the timed steps, so that they start on a busy GPU: the
        # W warm-up steps are split around the barrier + synchronize (the last two are
        # queued after it), so that the K timed steps queue behind running work on
        # every rank instead of starting on a GPU that the barrier left idle
        pre = max(args.warmup - 2, 1)
        for i in range(pre):
            step(i)
        torch.cuda.synchronize()
        _barrier(world)
        torch.cuda.synchronize()
        for i in range(pre, args.warmup):
            step(i)
        ev_start.record(stream)
        for i in range(args.steps):
            launches += step(args.warmup + i)
        ev_stop.record(stream)
        torch.cuda.synchronize()
        _barrier(world)
        ev_start2.record(stream)
        for i in range(args.steps):
            step(args.warmup + args.steps + i, ev_mid[i], ev_end[i])
        torch.cuda.synchronize()
        _barrier(world)
        time.sleep(0.1)
    total_ms = ev_start.elapsed_time(ev_stop)
    fwd_ms = [(ev_start2 if i == 0 else ev_end[i - 1]).elapsed_time(ev_mid[i]) for i in range(args.steps)]
    bwd_ms = [ev_mid[i].elapsed_time(ev_end[i]) for i in range(args.steps)]
    split_ms = ev_start2.elapsed_time(ev_end[-1])
    total_ms = _max_over_ranks(world, total_ms)
    ms_step = total_ms / args.steps
    value = world * flops_per_step() * args.steps / (total_ms * 1e-3) / 1e12

    # end to end: public autograd op, pinned host buffers, copies inside the timed region.
    # Three streams pipeline consecutive steps: step i's host->device copies (s_in)
    # overlap step i-1's compute, and its device->host copies (s_out) overlap step
    # i+1's; input and host-output buffers are double-buffered.  Every step still
    # moves its own inputs in and its own gradients out inside the timed region.
    # A step's inputs q, k, v, dO sit back to back in one pinned buffer and travel as
    # one copy; each gradient comes back in two halves.  With both copy directions
    # busy the whole step, that split measured 0.68 ms per step against 0.80 ms for
    # one copy per tensor each way (and 0.75-0.87 ms for finer splits): how the two
    # directions' copies interleave on the host link sets the step, not the bytes.
    with _gpu_local_cpus(local) as numa_bound:
        host = [torch.cat([t.reshape(-1) for t in sets[j]]).cpu().pin_memory() for j in range(2)]
        outs = [[torch.empty(SHAPE, dtype=dtype).pin_memory() for _ in range(3)] +
                [torch.empty(H, dtype=torch.float32).pin_memory()] for _ in range(2)]
    dev_in = [torch.empty(4 * B * H * T * D, dtype=dtype, device=dev) for _ in range(2)]

    def copy_out(hbuf, g):
        # one gradient device -> host, in two halves (the gain gradient in one piece)
        if g.numel() <= H:
            hbuf.copy_(g, non_blocking=True)
            return
        for hp, gp in zip(hbuf.view(-1).chunk(2), g.reshape(-1).chunk(2)):
            hp.copy_(gp, non_blocking=True)
    lg_req = torch.zeros(H, device=dev, requires_grad=True)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    in_used = [False, False]
    held = []   # (gradients, copy-out event) of the steps whose copies may still run

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if in_used[b]:
                s_in.wait_event(in_free[b])
            dev_in[b].copy_(host[b], non_blocking=True)
            in_ready[b].record(s_in)
        stream.wait_event(in_ready[b])
        qh, kh, vh, dy = (t.view(SHAPE) for t in dev_in[b].chunk(4))
        q, k, v = (t.detach().requires_grad_(True) for t in (qh, kh, vh))
        y = ca.continuum_attention(q, k, v, lg_req, 64)
        grads = torch.autograd.grad(y, (q, k, v, lg_req), dy)
        in_free[b].record(stream)
        in_used[b] = True
        done = torch.cuda.Event()
        done.record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for hbuf, g in zip(outs[b], grads):
                copy_out(hbuf, g)
            copied = torch.cuda.Event()
            copied.record(s_out)
        # a step's gradients are released only once the compute stream has waited
        # for their copy-out, so the allocator never hands them out while in flight
        held.append((grads, copied))
        if len(held) > 2:
            _, old_copied = held.pop(0)
            stream.wait_event(old_copied)

    e2e_steps = max(3, min(args.steps, 20)) * 2   # twice the steps: pipeline fill and drain amortised
    with ca.use_impl(impl):
        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize()
        _barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        h0 = time.perf_counter()
        for i in range(e2e_steps):
            e2e_step(i)
        host_issue_ms = (time.perf_counter() - h0) * 1e3 / e2e_steps
        tail = torch.cuda.Event()
        tail.record(s_out)
        stream.wait_event(tail)
        e1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(world, e0.elapsed_time(e1))
    e2e_value = world * flops_per_step() * e2e_steps / (e2e_ms * 1e-3) / 1e12
    elem = torch.tensor([], dtype=dtype).element_size()
    h2d = 4 * B * H * T * D * elem
    d2h = 3 * B * H * T * D * elem + H * 4

    # The e2e floor: the same per-step copies (inputs in, three gradients and the gain
    # gradient out, the same pinned buffers and streams) with no compute, both
    # directions at once -- what the host link allows per step.
    grads_dev = [torch.empty(SHAPE, dtype=dtype, device=dev) for _ in range(3)] + [torch.empty(H, device=dev)]

    def copy_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            dev_in[b].copy_(host[b], non_blocking=True)
        with torch.cuda.stream(s_out):
            for hbuf, g in zip(outs[b], grads_dev):
                copy_out(hbuf, g)

    for i in range(3):
        copy_step(i)
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    s_in.wait_event(c0)
    s_out.wait_event(c0)
    for i in range(e2e_steps):
        copy_step(i)
    d_in, d_out = torch.cuda.Event(), torch.cuda.Event()
    d_in.record(s_in)
    d_out.record(s_out)
    stream.wait_event(d_in)
    stream.wait_event(d_out)
    c1.record(stream)
    torch.cuda.synchronize()
    copy_ms = _max_over_ranks(world, c0.elapsed_time(c1)) / e2e_steps

    peak_tflops, peak_hbm, peak_kind = _peaks()
    bwd_avg = statistics.mean(bwd_ms)
    fwd_avg = statistics.mean(fwd_ms)
    dom = "backward" if bwd_avg >= fwd_avg else "forward"
    dom_ms = max(bwd_avg, fwd_avg)
    dom_flops = 2.0 * B * H * T * T * D            # two GEMMs per direction
    achieved = dom_flops / (dom_ms * 1e-3) / 1e12
    kernel_tag = f"{impl}_{dom}"
    traffic = _profile_traffic(kernel_tag)
    n_elem = B * H * T * (T + 1) / 2
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
                "frac": achieved / peak_tflops, "traffic": traffic,
                "traffic_source": "ncu capture of this kernel at this shape, fixed figure from profiles/ (not this run)",
                "kernel": f"ca_{dom} ({impl})", "peak_source": f"{peak_kind} bf16 dense burst",
                "fwd_ms": fwd_avg, "bwd_ms": bwd_avg,
                "split_source": "timed region 2: the same K steps with an event after each call "
                                f"({split_ms / args.steps:.4f} ms per step there)",
                "mufu_note": f"{n_elem:.4g} causal score elements per step; >= 2 MUFU ops each per direction"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tflops, med, threads, sample = cpu_reference_sample(2, 0)
        cpu = {"value": tflops, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
        if args.cpu_configs:
            # the other BASELINE configs the CPU path can time: config 1 and config 3 at
            # T <= 4096 (longer rows need dense T^2 score tensors of tens of GB)
            cpu["other_configs"] = {}
            for name, shp, n, w in (("config1", (2, 4, 256, 32), 5, 1), ("config3_T1024", (1, 16, 1024, 64), 3, 1),
                                    ("config3_T4096", (1, 16, 4096, 64), 2, 0)):
                tf, md, _, _ = cpu_reference_sample(n, w, shape=shp)
                cpu["other_configs"][name] = {"shape": list(shp), "ms_per_step": md * 1e3, "tflops": tf,
                                              "median_of": n}

    clocks = clk.summary()
    # The binding resource of both kernels is the special-function (MUFU) pipe and the
    # scalar issue around it, not the tensor core: >= 2 MUFU ops (exp2, reciprocal) per
    # causal score element per direction, 16 per clock per SM (nominal) at the sampled clock.
    sm_hz = (clocks["sm_mhz"] if clocks else 1965.0) * 1e6
    mufu_ops = 4.0 * n_elem
    mufu_peak = 16.0 * torch.cuda.get_device_properties(local).multi_processor_count * sm_hz
    roofline_mufu = {"bound": "mufu", "ops_per_step": mufu_ops, "achieved": mufu_ops / (ms_step * 1e-3),
                     "peak": mufu_peak, "unit": "ops/s", "frac": mufu_ops / (ms_step * 1e-3) / mufu_peak,
                     "peak_source": "nominal 16 MUFU ops/clock/SM x SMs x sampled SM clock; whole step"}
    decoder = None
    if not args.no_decoder:
        decoder = run_decoder(args, world, rank, local, steps=args.decoder_steps, warmup=3)
    tinylm = run_tinylm(local) if (world == 1 and not args.no_tinylm) else None
    config3 = None if args.no_config3 else run_config3_sharded(world, rank, local)
    ref_cuda = run_reference_cuda(local) if (world == 1 and not args.no_reference_cuda) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / (flops_per_step() / (PUBLISHED_V100_V6_MS * 1e-3) / 1e12),
            "dtype": "bf16", "data": "synthetic",
            "config": _config(world, impl),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "host_buffers_numa_local": numa_bound,
                    "copies_per_step": "h2d: q, k, v, dO as one 4-tensor copy; d2h: dq, dk, dv in two "
                                       "halves each, d log_gain in one",
                    "ms_per_step": e2e_ms / e2e_steps, "steps": e2e_steps,
                    "copy_floor_ms_per_step": copy_ms,
                    "host_issue_ms_per_step": host_issue_ms,
                    "frac_of_copy_floor": copy_ms / (e2e_ms / e2e_steps),
                    "copy_floor_note": "the same host<->device copies per step, both directions at once, "
                                       "no compute (same buffers and streams)"},
            "roofline": roofline,
            "roofline_mufu": roofline_mufu,
            # the same steps counted the FlashAttention way (2 forward + 5 backward GEMMs
            # with the backward's recompute): 7*B*H*T^2*D per step
            "value_fa_convention": {"value": value * 7.0 / 4.0, "unit": UNIT,
                                    "flop_per_step": 7.0 * B * H * T * T * D},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": launches,
            "decoder": decoder,
            "tinylm": tinylm,
            "config3_sharded": config3,
            "reference_cuda": ref_cuda,
        }
        print(json.dumps(line), flush=True)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--kernels", choices=["auto", "simt", "tcgen05"], default="auto")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-configs", action="store_true",
                   help="also time the CPU path at config 1 and config 3 (T = 1024, 4096); about a minute")
    p.add_argument("--no-decoder", action="store_true", help="skip the CA-S decoder tokens/s measurement")
    p.add_argument("--decoder-steps", type=int, default=10)
    p.add_argument("--no-tinylm", action="store_true", help="skip the TinyLM-P small-model measurement")
    p.add_argument("--no-config3", action="store_true", help="skip the config-3 strong-scaling measurement")
    p.add_argument("--no-reference-cuda", action="store_true",
                   help="skip timing the reference's CUDA kernels (oracle/_ref) at config 2")
    args = p.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world, rank, local = _dist_setup()
    try:
        if args.impl == "reference":
            run_reference_arm(args, world, rank)
        else:
            if not torch.cuda.is_available():
                raise RuntimeError("bench.py --impl ours needs a CUDA device")
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
