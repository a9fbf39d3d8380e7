#!/usr/bin/env python3
"""Headline benchmark: GPT-2 small training throughput, data parallel over N B200s.

Workload: GPT-2 small (12 layers, 12 heads, d=768, T=1024, V=50257), pure DP = N,
bf16, micro-batch 8 per GPU, grad_accum_steps 2, AdamW (lr 3e-4, wd 0.1, betas
0.9/0.95), gradient clipping at 1.0, dropout 0; synthetic uniform-random token
ids, random-init weights. Per-GPU work is fixed (weak scaling); the reported
value is the whole-job token rate  N * 8 * 1024 * 2 / step_time.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Timing: W untimed warm-up steps; then a barrier and cuda.synchronize, CUDA
events around exactly K optimizer steps on the launching stream, synchronize
and barrier again; ms/step is the maximum over ranks. Every step streams far
more than the 126 MB L2 (activations, 0.8 GB of bf16 logits per microbatch,
0.5 GB of fp32 gradients), so no flush is needed between steps. SM clocks and
throttle reasons are sampled with nvidia-smi during the timed region.

The ``e2e`` number is the same metric through the public training API
(``Engine.train_step`` with a host data loader): each step copies its input
tokens host->device from pinned memory and reads the loss back to the host,
timed on the host clock (max over ranks).

``--impl reference`` runs the unmodified reference implementation installed
in baseline/_ref through its own modules (GPT, average_gradients,
init_topology, RandomBatchLoader) doing the work of its train.py step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "train tokens/sec (device-timed, max over ranks) at 1/2/4/8 B200 vs ref NCCL build"
MODEL = dict(n_layer=12, n_head=12, n_embed=768, block_size=1024, vocab_size=50257)
MICRO_BATCH, ACCUM, SEQ = 8, 2, 1024
BASELINE_VALUE = None  # the reference publishes no throughput figure


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true", help="skip the profiler-based kernel count")
    ap.add_argument("--overlap-dp", type=int, default=0, choices=[0, 1],
                    help="reduce DP gradients block by block during the last backward (ours)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of one GPU every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.path = tempfile.mktemp(prefix=f"hb_clocks_{gpu_index}_", suffix=".csv")
        self.proc = None
        self.gpu = gpu_index

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        return {"rows": rows}


def summarize_clocks(all_rows) -> dict:
    sm, mx, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for r in all_rows:
        try:
            sm.append(float(r[1]))
            mx.append(float(r[2]))
        except ValueError:
            continue
        for name, val in zip(names, r[5:9]):
            if val.lower().startswith("active"):
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
            "samples": len(sm)}


# ---------------------------------------------------------------------------
def setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, dist.get_rank() if world > 1 else 0, local, dev


def barrier_sync(world):
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_steps(step_fn, K, world, sampler):
    barrier_sync(world)
    sampler.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        step_fn()
    e.record()
    barrier_sync(world)
    clocks = sampler.stop()
    return s.elapsed_time(e) / K, clocks


def count_launches(step_fn, prefix="hb::") -> int:
    """Kernels of ours launched by one step (torch profiler, outside the timed region)."""
    try:
        from torch.profiler import ProfilerActivity, profile
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step_fn()
            torch.cuda.synchronize()
        n = 0
        for ev in prof.events():
            if ev.device_type.name == "CUDA" and prefix in ev.name:
                n += 1
        return n
    except Exception:
        return -1


# ---------------------------------------------------------------------------
def run_ours(args, world, rank, dev):
    sys.path.insert(0, ROOT)
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.data import SyntheticLoader

    targs = build_argparser().parse_args([
        "--batch_size", str(MICRO_BATCH), "--block_size", str(SEQ), "--grad_accum_steps", str(ACCUM),
        "--n_layer", "12", "--n_head", "12", "--n_embed", "768", "--dropout", "0", "--amp", "bf16",
        "--learning_rate", "3e-4", "--weight_decay", "0.1", "--grad_clip", "1.0", "--dp", str(world),
        "--engine", "fused", "--overlap_dp", str(args.overlap_dp)])
    topo = init_topology(dp=world)
    torch.manual_seed(1337)
    cfg = GPTConfig(**MODEL, dropout=0.0)
    eng = Engine(targs, topo, dev, cfg)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    batches = [(torch.randint(0, cfg.vocab_size, (MICRO_BATCH, SEQ), device=dev, generator=g),
                torch.randint(0, cfg.vocab_size, (MICRO_BATCH, SEQ), device=dev, generator=g))
               for _ in range(ACCUM)]

    class DeviceBatches:
        B = MICRO_BATCH

        def __init__(self):
            self.i = 0

        def next_batch(self, device):
            b = batches[self.i % ACCUM]
            self.i += 1
            return b

    dl = DeviceBatches()
    step = lambda: eng.train_step(dl)
    # Launch counting runs one eager step: the captured graph replays exactly this kernel sequence.
    eng.count_step = lambda: eng._eager_step(dl)
    return eng, step, (lambda: SyntheticLoader(MICRO_BATCH, SEQ, cfg.vocab_size, seed=7, rank=rank)), "hb::"


def run_reference(args, world, rank, dev):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref, "gpt_model.py")):
        return None
    sys.path.insert(0, ref)
    import gpt_model  # noqa: E402  (reference modules, unmodified)
    import topo as rtopo
    from dp import average_gradients

    tp = rtopo.init_topology(dp=world)
    torch.manual_seed(1337)
    cfg = gpt_model.GPTConfig(**MODEL, dropout=0.0)
    model = gpt_model.GPT(cfg, topo=tp).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    batches = [(torch.randint(0, cfg.vocab_size, (MICRO_BATCH, SEQ), device=dev, generator=g),
                torch.randint(0, cfg.vocab_size, (MICRO_BATCH, SEQ), device=dev, generator=g))
               for _ in range(ACCUM)]

    class Eng:
        pass

    def train_step(loader):
        # reference train.py:414-453 with --amp bf16 (no GradScaler), pp = 1
        total_aux = torch.tensor(0.0, device=dev)
        for _ in range(ACCUM):
            x, y = loader.next_batch(dev)
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                _, loss, aux = model(x, y)
                combined = (loss + aux) / ACCUM
                total_aux = total_aux + aux.detach()
            combined.backward()
        loss_scalar = loss.detach().float()
        if tp.dp_group is not None:
            dist.all_reduce(loss_scalar, op=dist.ReduceOp.SUM, group=tp.dp_group)
            loss_scalar = loss_scalar / dist.get_world_size(group=tp.dp_group)
            dist.all_reduce(total_aux, op=dist.ReduceOp.SUM, group=tp.dp_group)
        average_gradients(model, tp.dp_group)
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss_scalar, total_aux

    class DeviceBatches:
        def __init__(self):
            self.i = 0

        def next_batch(self, device):
            b = batches[self.i % ACCUM]
            self.i += 1
            return b

    eng = Eng()
    eng.train_step = train_step
    dl = DeviceBatches()

    def make_loader():
        import train as rtrain  # reference train.py (main() is guarded)
        d = os.path.join(tempfile.gettempdir(), "hb_bench_bins")
        if rank == 0 and not os.path.exists(os.path.join(d, "fineweb_val_000000.bin")):
            import numpy as np  # uniform-random uint16 shards in the reference's .bin format
            os.makedirs(d, exist_ok=True)
            rng = np.random.default_rng(7)
            rng.integers(0, 50257, size=4_000_000, dtype=np.uint16).tofile(os.path.join(d, "fineweb_train_000001.bin"))
            rng.integers(0, 50257, size=200_000, dtype=np.uint16).tofile(os.path.join(d, "fineweb_val_000000.bin"))
        if world > 1:
            dist.barrier()
        return rtrain.RandomBatchLoader(d, "train", MICRO_BATCH, SEQ, None, seed=1337, rank=rank, dp_rank=0,
                                        dp_size=1, log_rank=1)

    return eng, (lambda: train_step(dl)), make_loader, "zzz-no-own-kernels"


def main():
    args = parse()
    world, rank, local, dev = setup()
    runner = run_ours if args.impl == "ours" else run_reference
    out = runner(args, world, rank, dev)
    if out is None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}))
        return
    eng, step, make_loader, prefix = out
    for _ in range(max(3, args.warmup)):
        step()
    ms, clk = timed_steps(step, args.steps, world, ClockSampler(local))
    ms = max_over_ranks(ms, world)
    rows = clk.get("rows", [])
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, rows)
        rows = [r for g in gathered for r in g]
    clocks = summarize_clocks(rows)
    launches = (count_launches(getattr(eng, "count_step", step), prefix)
                if (args.impl == "ours" and not args.no_launch_count) else -1)
    tokens = world * MICRO_BATCH * SEQ * ACCUM
    value = tokens / (ms / 1e3)

    e2e = None
    if not args.no_e2e:
        loader = make_loader()
        h2d = ACCUM * 2 * MICRO_BATCH * SEQ * 8
        for _ in range(2):
            l, _ = eng.train_step(loader)
            float(l.item())
        barrier_sync(world)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            l, _ = eng.train_step(loader)
            float(l.item())  # device -> host read of the step's loss
        barrier_sync(world)
        e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps, world)
        e2e = {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "ms_per_step": e2e_s * 1e3}

    if rank == 0:
        rec = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
               "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None, "dtype": "bf16",
               "data": "synthetic uniform-random GPT-2 token ids, random-init weights",
               "config": {"model": "GPT-2 small 12L/12H/768d, vocab 50257", "global_batch": world * MICRO_BATCH * ACCUM,
                          "micro_batch": MICRO_BATCH, "grad_accum_steps": ACCUM, "seq_len": SEQ,
                          "parallelism": f"dp{world}", "optimizer": "AdamW + clip 1.0",
                          "l2": "inputs larger than L2: each step streams >10 GB (activations, bf16 logits, fp32 grads)"},
               "clocks": clocks, "e2e": e2e, "gpu_launches": launches * args.steps if launches >= 0 else (0 if args.impl == "reference" else None),
               "impl": args.impl}
        print(json.dumps(rec))
    if hasattr(eng, "close"):
        eng.close()  # the captured graph must be released before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
