#!/usr/bin/env python3
"""Headline benchmark: GPT-2 small training throughput, data parallel over N B200s.

Workload: GPT-2 small (12 layers, 12 heads, d=768, T=1024, V=50257), pure DP = N,
bf16, micro-batch 8 per GPU, grad_accum_steps 2, AdamW (lr 3e-4, wd 0.1, betas
0.9/0.95), gradient clipping at 1.0, dropout 0; synthetic uniform-random token
ids, random-init weights. Per-GPU work is fixed (weak scaling); the reported
value is the whole-job token rate  N * 8 * 1024 * 2 / step_time.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--config NAME]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

``--config`` selects one of the other training configurations (same metric,
same timing; tokens/s counts dp * micro-batch * T * accumulation per step):
  gpt2m_dp2_tp4      GPT-2 medium (24L/16H/1024d), micro-batch 8, accum 2;
                     tp = N up to 4, dp2 x tp4 at 8 GPUs
  moe_dp2_ep2_tp2    MoE GPT (12L/768d, 8 experts, top-2, every 2nd block,
                     aux 0.01), micro-batch 8, accum 4; ep2 at 2 GPUs,
                     ep2 x tp2 at 4, dp2 x ep2 x tp2 at 8
  gpt2l_dp2_tp2_pp2  GPT-2 large (36L/20H/1280d), GPipe with 8 micro-batches
                     of 4; pp2 at 2 GPUs, tp2 x pp2 at 4, dp2 x tp2 x pp2 at 8
  cpu_sanity         GPT 4L/4H/128d, T=256, vocab 50257, micro-batch 8, fp32, one
                     process on the host CPU (host-timed; --profile-ops prints the
                     per-op table)

Timing: W untimed warm-up steps; then a barrier and cuda.synchronize, CUDA
events around exactly K optimizer steps on the launching stream, synchronize
and barrier again; ms/step is the maximum over ranks. Every step streams far
more than the 126 MB L2 (activations, 0.8 GB of bf16 logits per microbatch,
0.5 GB of fp32 gradients), so no flush is needed between steps. SM clocks and
throttle reasons are sampled during the timed region (NVML every 20 ms, else
nvidia-smi every 200 ms); "clocks" gives the median SM clock over all ranks'
samples and every throttle reason seen active.

The ``e2e`` number is the same metric through the public training API
(``Engine.train_step`` with a host data loader): each step copies its input
tokens host->device from pinned memory and reads the loss back to the host,
timed on the host clock (max over ranks). The loss of step i is copied
asynchronously and read once step i+1 is queued (``ScalarReader``; the last
one before the clock stops), on both arms.

``--impl reference`` runs the unmodified reference implementation installed
in baseline/_ref through its own modules (GPT or StageModule + GPipeEngine,
average_gradients, init_topology, RandomBatchLoader) doing the work of its
train.py step.
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
SEQ, VOCAB = 1024, 50257
BASELINE_VALUE = None  # the reference publishes no throughput figure


class Workload:
    """One benchmark configuration: model shape, micro-batch, accumulation and the
    (dp, ep, tp, pp) layout used at each GPU count.

    Model-parallel layouts shrink with the GPU count (the model is spread over
    fewer GPUs; below 8 GPUs dp is 1), so their per-N numbers are strong scaling
    while dp == 1 and weak scaling from there on."""

    def __init__(self, name, desc, model, micro, accum, layouts):
        self.name, self.desc, self.model, self.micro, self.accum = name, desc, model, micro, accum
        self.layouts = layouts

    def layout(self, n: int):
        if callable(self.layouts):
            return self.layouts(n)
        if n not in self.layouts:
            raise SystemExit(f"--config {self.name} runs on {sorted(self.layouts)} GPUs, not {n}")
        return self.layouts[n]

    def model_kwargs(self):
        return dict(block_size=SEQ, vocab_size=VOCAB, **self.model)


WORKLOADS = {w.name: w for w in [
    # GPT-2 small, pure data parallel: the headline configuration (default).
    Workload("gpt2s_dp", "GPT-2 small 12L/12H/768d, vocab 50257", dict(n_layer=12, n_head=12, n_embed=768),
             8, 2, lambda n: (n, 1, 1, 1)),
    # GPT-2 medium, dp2 x tp4 at 8 GPUs: column/row-parallel linears (all-gather -> GEMM, GEMM -> reduce-scatter).
    Workload("gpt2m_dp2_tp4", "GPT-2 medium 24L/16H/1024d, vocab 50257", dict(n_layer=24, n_head=16, n_embed=1024),
             8, 2, {1: (1, 1, 1, 1), 2: (1, 1, 2, 1), 4: (1, 1, 4, 1), 8: (2, 1, 4, 1)}),
    # MoE GPT: 8 experts (4x GELU MLP), top-2 softmax gate, MoE every 2nd block, aux coef 0.01; dp2 x ep2 x tp2.
    Workload("moe_dp2_ep2_tp2", "MoE GPT 12L/12H/768d, 8 experts top-2 every 2nd block, aux 0.01, vocab 50257",
             dict(n_layer=12, n_head=12, n_embed=768, num_experts=8, top_k=2, moe_freq=2, aux_loss_coef=0.01),
             8, 4, {1: (1, 1, 1, 1), 2: (1, 2, 1, 1), 4: (1, 2, 2, 1), 8: (2, 2, 2, 1)}),
    # GPT-2 large, dp2 x tp2 x pp2 GPipe with 8 micro-batches of 4 sequences.
    Workload("gpt2l_dp2_tp2_pp2", "GPT-2 large 36L/20H/1280d, vocab 50257, GPipe",
             dict(n_layer=36, n_head=20, n_embed=1280),
             4, 8, {1: (1, 1, 1, 1), 2: (1, 1, 1, 2), 4: (1, 1, 2, 2), 8: (2, 1, 2, 2)}),
]}


# CPU single-process sanity configuration (fp32, host-timed): 4L/4H/128d, T=256,
# vocab 50257, micro-batch 8, 50 AdamW iterations at lr 6e-4.
CPU_SANITY = dict(n_layer=4, n_head=4, n_embed=128, block_size=256, vocab_size=VOCAB, batch=8, lr=6e-4)


def parallelism_name(layout) -> str:
    dp, ep, tp, pp = layout
    parts = [f"dp{dp}"] + [f"{k}{v}" for k, v in (("ep", ep), ("tp", tp), ("pp", pp)) if v > 1]
    return "_".join(parts)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="gpt2s_dp", choices=sorted(WORKLOADS) + ["cpu_sanity"],
                    help="workload (default: GPT-2 small, pure data parallel; cpu_sanity: the fp32 CPU "
                         "configuration, one process, host-timed)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true", help="skip the profiler-based kernel count")
    ap.add_argument("--profile-ops", action="store_true",
                    help="cpu_sanity: print torch.profiler's per-op table of the timed steps to stderr")
    ap.add_argument("--overlap-dp", type=int, default=0, choices=[0, 1],
                    help="reduce DP gradients block by block during the last backward (ours)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, maximum SM clock, power and clock-event reasons of one GPU, sampled
    while the timed region runs.

    Primary source: NVML queries (read-only) from a background thread every 20 ms,
    so even a timed region of a few hundred milliseconds gets a dozen samples; one
    sample is taken when sampling starts and one when it stops. Fallback, when NVML
    cannot be loaded or the device not found: ``nvidia-smi -lms 200``. Rows have the
    layout of the nvidia-smi query below (reasons as "Active" / "Not Active")."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.02

    def __init__(self, gpu_index: int, uuid: str | None = None, bus_id: str | None = None, nvml=None):
        self.gpu, self.uuid, self.bus_id = gpu_index, uuid, bus_id
        self.nvml, self.handle, self.source = nvml, None, None
        self.proc, self.thread, self.rows = None, None, []

    @staticmethod
    def for_device(dev: torch.device) -> "ClockSampler":
        """Sampler of the physical GPU behind a CUDA device (found by UUID or PCI bus id,
        so it is right under CUDA_VISIBLE_DEVICES as well)."""
        uuid = bus = None
        try:
            props = torch.cuda.get_device_properties(dev)
            uuid = "GPU-" + str(props.uuid)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        except Exception:
            pass
        return ClockSampler(dev.index or 0, uuid=uuid, bus_id=bus)

    def _open_nvml(self) -> bool:
        try:
            if self.nvml is None:
                import pynvml
                self.nvml = pynvml
            self.nvml.nvmlInit()
            h = None
            for how, key in (("nvmlDeviceGetHandleByUUID", self.uuid), ("nvmlDeviceGetHandleByPciBusId", self.bus_id)):
                if h is None and key:
                    try:
                        h = getattr(self.nvml, how)(key)
                    except Exception:
                        h = None
            self.handle = h
            return h is not None
        except Exception:
            return False

    def _reasons(self):
        n = self.nvml
        for name in ("nvmlDeviceGetCurrentClocksEventReasons", "nvmlDeviceGetCurrentClocksThrottleReasons"):
            if hasattr(n, name):
                return int(getattr(n, name)(self.handle))
        return 0

    def _sample(self):
        n = self.nvml
        try:
            sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
            mx = n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM)
            pw = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
            r = self._reasons()
        except Exception:
            return
        bits = (0x8, 0x40, 0x20, 0x4)  # hw slowdown, hw thermal, sw thermal, sw power cap (nvml.h masks)
        self.rows.append([str(self.gpu), str(sm), str(mx), f"{pw:.1f}", hex(r)]
                         + ["Active" if r & b else "Not Active" for b in bits])

    def _loop(self, stop):
        while not stop.wait(self.PERIOD_S):
            self._sample()

    def start(self):
        import threading
        self.rows = []
        if self._open_nvml():
            self.source = "nvml"
            self._sample()
            self._stop = threading.Event()
            self.thread = threading.Thread(target=self._loop, args=(self._stop,), daemon=True)
            self.thread.start()
            return
        try:
            self.source = "nvidia-smi"
            self.path = tempfile.mktemp(prefix=f"hb_clocks_{self.gpu}_", suffix=".csv")
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc, self.source = None, None

    def stop(self) -> dict:
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            self.thread = None
            self._sample()
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
            return {"rows": self.rows, "source": self.source}
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
        return {"rows": rows, "source": self.source}


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
class DeviceBatches:
    """The accumulation step's micro-batches, drawn once on the device and replayed
    (device-timed region: no host->device traffic)."""

    def __init__(self, batches, B):
        self.batches, self.B, self.i = batches, B, 0

    def next_batch(self, device):
        b = self.batches[self.i % len(self.batches)]
        self.i += 1
        return b


def device_batches(w: Workload, dev, seed: int) -> DeviceBatches:
    g = torch.Generator(device=dev).manual_seed(seed)
    shape = (w.micro, SEQ)
    return DeviceBatches([(torch.randint(0, VOCAB, shape, device=dev, generator=g),
                           torch.randint(0, VOCAB, shape, device=dev, generator=g)) for _ in range(w.accum)], w.micro)


def train_flags(w: Workload, layout, overlap_dp: int = 0) -> list:
    """train.py flags of one workload and layout on the fused engine."""
    dp, ep, tp, pp = layout
    m = w.model
    flags = ["--batch_size", str(w.micro), "--block_size", str(SEQ), "--grad_accum_steps", str(w.accum),
             "--n_layer", str(m["n_layer"]), "--n_head", str(m["n_head"]), "--n_embed", str(m["n_embed"]),
             "--dropout", "0", "--amp", "bf16", "--learning_rate", "3e-4", "--weight_decay", "0.1",
             "--grad_clip", "1.0", "--dp", str(dp), "--ep", str(ep), "--tp", str(tp), "--pp", str(pp),
             "--engine", "fused", "--overlap_dp", str(overlap_dp)]
    for k in ("num_experts", "top_k", "moe_freq", "aux_loss_coef"):
        if k in m:
            flags += [f"--{k}", str(m[k])]
    return flags


def run_ours(args, w: Workload, layout, world, rank, dev):
    sys.path.insert(0, ROOT)
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.data import SyntheticLoader

    dp, ep, tp, pp = layout
    targs = build_argparser().parse_args(train_flags(w, layout, args.overlap_dp))
    topo = init_topology(dp=dp, ep=ep, tp=tp, pp=pp)
    torch.manual_seed(1337)
    cfg = GPTConfig(**w.model_kwargs(), dropout=0.0)
    eng = Engine(targs, topo, dev, cfg)
    # Ranks of one DP replica (its TP / EP / PP ranks) read the same tokens.
    dl = device_batches(w, dev, 1000 + topo.dp_rank)
    step = lambda: eng.train_step(dl)
    # Launch counting runs one eager step: the captured graph replays exactly this kernel sequence.
    eng.count_step = lambda: eng._eager_step(dl)
    return eng, step, (lambda: SyntheticLoader(w.micro, SEQ, VOCAB, seed=7, rank=topo.dp_rank)), "hb::"


def run_reference(args, w: Workload, layout, world, rank, dev):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref, "gpt_model.py")):
        return None
    sys.path.insert(0, ref)
    import gpt_model  # noqa: E402  (reference modules, unmodified)
    import topo as rtopo
    from dp import average_gradients

    dp, ep, tp, pp = layout
    tpo = rtopo.init_topology(dp=dp, ep=ep, tp=tp, pp=pp)
    torch.manual_seed(1337)
    cfg = gpt_model.GPTConfig(**w.model_kwargs(), dropout=0.0)
    aux_coef = float(w.model.get("aux_loss_coef", 0.01))
    if pp > 1:
        # The reference's pipeline cannot run under bf16 autocast: the sender's boundary is
        # the fp32 residual stream while the receiver allocates a bf16 buffer
        # (pipeline.py:217-247), so each transfer sends twice the bytes the peer expects
        # (gloo on CPU rejects it: "Received data size doesn't match expected size"; NCCL
        # gets mismatched counts). Its pipeline therefore runs in fp32, its only working mode.
        from pipeline import GPipeEngine, StageModule
        module = StageModule(cfg, tpo, tpo.pp_rank, tpo.pp).to(dev)
        pipe = GPipeEngine(module, tpo)
    else:
        module = gpt_model.GPT(cfg, topo=tpo).to(dev)
        pipe = None
    opt = torch.optim.AdamW(module.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1)
    dl = device_batches(w, dev, 1000 + tpo.dp_rank)

    class Eng:
        pass

    def train_step(loader):
        # reference train.py:400-453 with --amp bf16 (no GradScaler)
        if pipe is not None:
            loss_scalar, total_aux = pipe.forward_backward(loader, micro_batches=w.accum, device=dev, use_amp=False,
                                                           amp_dtype=torch.bfloat16, scaler=None, batch_size=w.micro,
                                                           aux_loss_coef=aux_coef)
        else:
            total_aux = torch.tensor(0.0, device=dev)
            for _ in range(w.accum):
                x, y = loader.next_batch(dev)
                with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                    _, loss, aux = module(x, y)
                    combined = (loss + aux) / w.accum
                    total_aux = total_aux + aux.detach()
                combined.backward()
            loss_scalar = loss.detach().float()
        if loss_scalar is not None and tpo.dp_group is not None:
            dist.all_reduce(loss_scalar, op=dist.ReduceOp.SUM, group=tpo.dp_group)
            loss_scalar = loss_scalar / dist.get_world_size(group=tpo.dp_group)
        if total_aux is not None and tpo.dp_group is not None:
            dist.all_reduce(total_aux, op=dist.ReduceOp.SUM, group=tpo.dp_group)
        average_gradients(module, tpo.dp_group)
        torch.nn.utils.clip_grad_norm_(module.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        if loss_scalar is None:  # pipeline stages other than the last hold no data loss
            loss_scalar = torch.zeros((), device=dev)
        return loss_scalar, total_aux

    eng = Eng()
    eng.train_step = train_step
    if pipe is not None:
        eng.dtype = "fp32"
        eng.note = ("reference pipeline in fp32: with bf16 autocast it sends an fp32 boundary into a bf16 "
                    "receive buffer (pipeline.py:217-247)")

    def make_loader():
        import train as rtrain  # reference train.py (main() is guarded)
        d = os.path.join(tempfile.gettempdir(), "hb_bench_bins")
        if rank == 0 and not os.path.exists(os.path.join(d, "fineweb_val_000000.bin")):
            import numpy as np  # uniform-random uint16 shards in the reference's .bin format
            os.makedirs(d, exist_ok=True)
            rng = np.random.default_rng(7)
            rng.integers(0, VOCAB, size=4_000_000, dtype=np.uint16).tofile(os.path.join(d, "fineweb_train_000001.bin"))
            rng.integers(0, VOCAB, size=200_000, dtype=np.uint16).tofile(os.path.join(d, "fineweb_val_000000.bin"))
        if world > 1:
            dist.barrier()
        return rtrain.RandomBatchLoader(d, "train", w.micro, SEQ, None, seed=1337, rank=tpo.dp_rank, dp_rank=0,
                                        dp_size=1, log_rank=1)

    return eng, (lambda: train_step(dl)), make_loader, "zzz-no-own-kernels"


class _PinnedReader:
    """The reference arm's copy of the deferred read-back (that arm imports nothing of
    this framework): async copy into pinned memory + event, read one step later."""

    def __init__(self):
        self.q = []
        self.slots = [torch.empty((), dtype=torch.float32, pin_memory=True) for _ in range(2)]
        self.i = 0

    def push(self, t):
        h = self.slots[self.i % 2]
        self.i += 1
        h.copy_(t.detach().float(), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.q.append((h, ev))

    def pop(self):
        h, ev = self.q.pop(0)
        ev.synchronize()
        return float(h)

    def __len__(self):
        return len(self.q)


def _scalar_reader(impl: str):
    """Deferred loss read-back of the e2e loop (same pattern on both arms)."""
    if impl == "reference":
        return _PinnedReader()
    sys.path.insert(0, ROOT)
    from heiretsu_b200.trainer import ScalarReader
    return ScalarReader(depth=2)


def cpu_batches(seed: int, n: int):
    """n (x, y) batches of the CPU configuration: int64 ids uniform in [0, V), y = x shifted by one."""
    g = torch.Generator().manual_seed(seed)
    B, T = CPU_SANITY["batch"], CPU_SANITY["block_size"]
    out = []
    for _ in range(n):
        ids = torch.randint(0, VOCAB, (B, T + 1), generator=g)
        out.append((ids[:, :-1].contiguous(), ids[:, 1:].contiguous()))
    return out


def run_cpu_sanity(args) -> dict:
    """One process on the host CPU, fp32: ``steps`` timed optimizer steps after ``warmup``
    (host clock, perf_counter), through each implementation's own training step."""
    c = CPU_SANITY
    batches = cpu_batches(1234, args.warmup + args.steps)
    it = iter(batches)

    class Feed:
        B = c["batch"]

        def next_batch(self, device):
            return next(it)

    feed = Feed()
    if args.impl == "ours":
        sys.path.insert(0, ROOT)
        from heiretsu_b200.config import GPTConfig
        from heiretsu_b200.topo import init_topology
        from heiretsu_b200.trainer import Engine, build_argparser
        flags = ["--device", "cpu", "--amp", "none", "--engine", "plain", "--batch_size", str(c["batch"]),
                 "--block_size", str(c["block_size"]), "--n_layer", str(c["n_layer"]), "--n_head", str(c["n_head"]),
                 "--n_embed", str(c["n_embed"]), "--dropout", "0", "--learning_rate", str(c["lr"])]
        targs = build_argparser().parse_args(flags)
        torch.manual_seed(1337)
        cfg = GPTConfig(n_layer=c["n_layer"], n_head=c["n_head"], n_embed=c["n_embed"], block_size=c["block_size"],
                        vocab_size=VOCAB, dropout=0.0)
        eng = Engine(targs, init_topology(dp=1), torch.device("cpu"), cfg)
        step = lambda: eng.train_step(feed)
    else:
        ref = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.exists(os.path.join(ref, "gpt_model.py")):
            return {"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}
        sys.path.insert(0, ref)
        import gpt_model  # noqa: E402  (reference modules, unmodified)
        import topo as rtopo
        tpo = rtopo.init_topology(dp=1)
        torch.manual_seed(1337)
        model = gpt_model.GPT(gpt_model.GPTConfig(n_layer=c["n_layer"], n_head=c["n_head"], n_embed=c["n_embed"],
                                                  block_size=c["block_size"], vocab_size=VOCAB, dropout=0.0),
                              topo=tpo)
        opt = torch.optim.AdamW(model.parameters(), lr=c["lr"], betas=(0.9, 0.95), weight_decay=0.1)

        def step():  # reference train.py:400-453 with --amp none, accumulation 1, one process
            x, y = feed.next_batch(None)
            _, loss, aux = model(x, y)
            (loss + aux).backward()
            torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
            opt.step()
            opt.zero_grad(set_to_none=True)
            return loss.detach(), aux
    for _ in range(args.warmup):
        step()
    prof = None
    if getattr(args, "profile_ops", False):
        from torch.profiler import ProfilerActivity, profile
        prof = profile(activities=[ProfilerActivity.CPU])
        prof.__enter__()
    t0 = time.perf_counter()
    last = None
    for _ in range(args.steps):
        last = step()
    loss = float(last[0])  # the last step's loss read back (inside the timed region)
    dt = (time.perf_counter() - t0) / args.steps
    if prof is not None:
        prof.__exit__(None, None, None)
        print(prof.key_averages().table(sort_by="self_cpu_time_total", row_limit=15), file=sys.stderr)
    tokens = c["batch"] * c["block_size"]
    return {"metric": METRIC.replace("device-timed, max over ranks", "host-timed, CPU"), "value": tokens / dt,
            "unit": "tokens/s", "n_gpus": 0, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic uniform-random GPT-2 token ids (targets = inputs shifted by one), random-init weights",
            "config": {"model": "GPT 4L/4H/128d, vocab 50257", "global_batch": c["batch"], "seq_len": c["block_size"],
                       "parallelism": "cpu", "optimizer": f"AdamW lr {c['lr']} + clip 1.0",
                       "threads": torch.get_num_threads(), "name": "cpu_sanity"},
            "final_loss": loss, "gpu_launches": 0, "impl": args.impl}


def main():
    args = parse()
    if args.config == "cpu_sanity":
        print(json.dumps(run_cpu_sanity(args)))
        return
    w = WORKLOADS[args.config]
    world, rank, local, dev = setup()
    layout = w.layout(world)
    runner = run_ours if args.impl == "ours" else run_reference
    out = runner(args, w, layout, world, rank, dev)
    if out is None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference not installed in baseline/_ref"}))
        return
    eng, step, make_loader, prefix = out
    for _ in range(max(3, args.warmup)):
        step()
    ms, clk = timed_steps(step, args.steps, world, ClockSampler.for_device(dev))
    ms = max_over_ranks(ms, world)
    rows = clk.get("rows", [])
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, rows)
        rows = [r for g in gathered for r in g]
    clocks = summarize_clocks(rows)
    clocks["source"] = clk.get("source")
    launches = (count_launches(getattr(eng, "count_step", step), prefix)
                if (args.impl == "ours" and not args.no_launch_count) else -1)
    dp = layout[0]
    tokens = dp * w.micro * SEQ * w.accum  # tokens consumed per optimizer step by the whole job
    value = tokens / (ms / 1e3)

    e2e = None
    if not args.no_e2e:
        loader = make_loader()
        h2d = w.accum * 2 * w.micro * SEQ * 8
        for _ in range(2):
            l, a = eng.train_step(loader)
            float((l if l is not None else a).item())
        reader = _scalar_reader(args.impl)
        barrier_sync(world)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            l, a = eng.train_step(loader)
            # device -> host read of every step's loss (pipeline stages before the last hold the aux
            # loss): copied asynchronously, read once the next step is queued, the last one below
            reader.push(l if l is not None else a)
            if len(reader) > 1:
                reader.pop()
        while len(reader):
            reader.pop()
        barrier_sync(world)
        e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps, world)
        e2e = {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "ms_per_step": e2e_s * 1e3}

    if rank == 0:
        rec = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
               "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True,
               "scaling": "weak" if (args.config == "gpt2s_dp" or dp > 1) else "strong",
               "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None,
               "dtype": getattr(eng, "dtype", "bf16"),
               "data": "synthetic uniform-random GPT-2 token ids, random-init weights",
               "config": {"model": w.desc, "global_batch": dp * w.micro * w.accum,
                          "micro_batch": w.micro, "grad_accum_steps": w.accum, "seq_len": SEQ,
                          "parallelism": parallelism_name(layout), "optimizer": "AdamW + clip 1.0",
                          "l2": "inputs larger than L2: each step streams >10 GB (activations, bf16 logits, fp32 grads)"},
               "clocks": clocks, "e2e": e2e, "gpu_launches": launches * args.steps if launches >= 0 else (0 if args.impl == "reference" else None),
               "impl": args.impl}
        if args.config != "gpt2s_dp":
            rec["config"]["name"] = args.config
        if getattr(eng, "note", None):
            rec["note"] = eng.note
        print(json.dumps(rec))
    if hasattr(eng, "close"):
        eng.close()  # the captured graph must be released before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
