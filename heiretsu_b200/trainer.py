"""Training driver: the reference's train.py CLI on the heiretsu_b200 engine.

Every reference flag is accepted with the same name, default and choices
(reference train.py:171-226); added flags are additive only. The loop does
the same work per step as the reference (train.py:400-524): ``grad_accum``
microbatches of forward + backward, loss all-reduce over DP, DP gradient
averaging, gradient clipping, AdamW, logging, periodic eval and checkpoints.

Two engines share this loop:

* **fused** (CUDA, bf16, configs covered by ``fused_supported``): flat fp32
  master/grad buffers, sm_100a kernels for every op, fused AdamW with global
  norm clipping, DP reduction of the flat gradient buffer.
* **plain** (CPU, fp32, fp16 AMP, or configs the fused path does not cover):
  PyTorch modules with autocast, ``average_gradients``, ``clip_grad_norm_``
  and ``torch.optim.AdamW`` -- the reference's numerics.

Deliberate differences from the reference (each a fix of a reference quirk):
the model init seed is the same on every TP rank (the TP model equals the
dense model), gradient clipping uses the global norm (``--clip_mode local``
restores per-shard clipping), EP dispatch/combine are differentiable, and the
pipeline boundary has one declared dtype.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import random
import time
from dataclasses import asdict
from datetime import timedelta
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from .config import GPTConfig
from .models.gpt import GPT
from .parallel.dp import average_gradients
from .parallel.pipeline import GPipeEngine, StageModule
from .topo import cleanup, init_topology
from .utils.ckpt import save_checkpoint
from .utils.data import RandomBatchLoader, SyntheticLoader

try:  # optional, as in the reference
    import wandb  # type: ignore

    WANDB_AVAILABLE = True
except Exception:  # pragma: no cover
    wandb = None
    WANDB_AVAILABLE = False


def build_argparser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="GPT trainer (heiretsu_b200): DP/EP/TP/PP, AMP, grad accumulation")
    # data / batching
    p.add_argument("--data_dir", type=str, default="fineweb10B")
    p.add_argument("--num_train_chunks", type=int, default=None)
    p.add_argument("--num_val_chunks", type=int, default=1)
    p.add_argument("--batch_size", type=int, default=64)
    p.add_argument("--block_size", type=int, default=512)
    p.add_argument("--eval_interval", type=int, default=1000)
    p.add_argument("--eval_iters", type=int, default=200)
    # model
    p.add_argument("--n_layer", type=int, default=6)
    p.add_argument("--n_head", type=int, default=6)
    p.add_argument("--n_embed", type=int, default=768)
    p.add_argument("--dropout", type=float, default=0.2)
    # optimisation
    p.add_argument("--max_iters", type=int, default=50000)
    p.add_argument("--learning_rate", type=float, default=3e-4)
    p.add_argument("--weight_decay", type=float, default=0.1)
    p.add_argument("--betas", type=float, nargs=2, default=(0.9, 0.95))
    p.add_argument("--grad_clip", type=float, default=1.0)
    p.add_argument("--grad_accum_steps", type=int, default=1)
    p.add_argument("--amp", type=str, choices=["none", "fp16", "bf16"], default="none")
    p.add_argument("--compile", action="store_true", help="torch.compile the plain path (the fused path ignores it)")
    p.add_argument("--device", type=str, default="auto", choices=["auto", "cpu", "cuda", "mps"])
    p.add_argument("--seed", type=int, default=1337)
    # topology
    p.add_argument("--dp", type=int, default=1)
    p.add_argument("--ep", type=int, default=1)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--dp_share_data", action="store_true")
    p.add_argument("--dist_backend", type=str, default="nccl", choices=["nccl", "gloo"])
    # MoE
    p.add_argument("--num_experts", type=int, default=0)
    p.add_argument("--top_k", type=int, default=2)
    p.add_argument("--moe_freq", type=int, default=2)
    p.add_argument("--aux_loss_coef", type=float, default=0.01)
    # wandb / checkpoints
    p.add_argument("--wandb", action="store_true")
    p.add_argument("--wandb_project", type=str, default="fineweb10B-gpt")
    p.add_argument("--wandb_entity", type=str, default=None)
    p.add_argument("--wandb_mode", type=str, default="online", choices=["online", "offline", "disabled"])
    p.add_argument("--run_name", type=str, default=None)
    p.add_argument("--save_interval", type=int, default=0)
    # additive flags
    p.add_argument("--synthetic_data", action="store_true", help="uniform-random token ids instead of .bin files")
    p.add_argument("--engine", type=str, default="auto", choices=["auto", "fused", "plain"])
    p.add_argument("--clip_mode", type=str, default="global", choices=["global", "local"])
    p.add_argument("--pp_boundary_dtype", type=str, default="fp32", choices=["fp32", "bf16"])
    p.add_argument("--pp_schedule", type=str, default="gpipe", choices=["gpipe", "1f1b"],
                   help="pp > 1: gpipe (the reference: all forwards, then all backwards) or 1f1b (one forward, "
                        "one backward; stage s holds at most pp - s micro-batches of activations)")
    p.add_argument("--pp_tie_embeddings", type=int, default=0, choices=[0, 1],
                   help="pp > 1: keep the first stage's wte and the last stage's lm_head equal (gradients summed "
                        "between the two stages), i.e. the tied dense GPT; 0 = the reference's untied stages")
    p.add_argument("--resume", type=str, default=None,
                   help="checkpoint file to load before training; 'auto' = the newest complete step in --out_dir "
                        "(or a fresh start), for jobs restarted after a failure")
    p.add_argument("--init_from", type=str, default=None,
                   help="start a new run from the weights of this checkpoint file (any shard of a step, any "
                        "layout); the optimizer and the step count start fresh")
    p.add_argument("--eval_only", action="store_true",
                   help="evaluate the (loaded) weights on --eval_iters validation batches and exit")
    p.add_argument("--out_dir", type=str, default=".")
    p.add_argument("--pg_timeout_s", type=float, default=600.0, help="process-group collective timeout")
    p.add_argument("--log_interval", type=int, default=None)
    p.add_argument("--watchdog_s", type=float, default=300.0,
                   help="multi-process runs: abort when a peer announces a failure or makes no progress "
                        "for this many seconds (0 = off)")
    p.add_argument("--device_timing", type=int, default=1, choices=[0, 1],
                   help="time each step with CUDA events and log device tokens/s (max over ranks)")
    p.add_argument("--region_timing_interval", type=int, default=0,
                   help="every N steps run the step eagerly with device timers around forward+backward, the tied "
                        "embedding sum, the TP gradient sum, the DP reduction and the optimizer; log them (max over "
                        "ranks). 0 = off")
    p.add_argument("--overlap_dp", type=int, default=0, choices=[0, 1],
                   help="reduce data-parallel gradients block by block during the last backward (fused path); "
                        "off by default: on GPT-2 small the co-running reduction slowed backward more than it hid")
    p.add_argument("--lr_schedule", type=str, default="constant", choices=["constant", "cosine"],
                   help="constant (the reference) or linear warmup then cosine decay to --min_lr at --max_iters")
    p.add_argument("--warmup_iters", type=int, default=0)
    p.add_argument("--min_lr", type=float, default=0.0)
    p.add_argument("--zero_stage", type=int, default=0, choices=[0, 1],
                   help="plain engine: 1 = shard the AdamW moments over the DP group (ZeRO stage 1)")
    p.add_argument("--activation_checkpointing", type=int, default=0, choices=[0, 1],
                   help="keep only each block's input and recompute the block in backward (plain engine; fused "
                        "engine without TP: dense blocks, not yet run on GPUs)")
    p.add_argument("--fused_tp_dropout", type=int, default=1, choices=[0, 1],
                   help="run tp > 1 with dropout > 0 on the fused engine (masks applied around the in-kernel "
                        "reduce-scatter and all-gather; default); 0 = such runs use the plain engine")
    p.add_argument("--cuda_graph", type=int, default=1, choices=[0, 1],
                   help="capture the fused training step in a CUDA graph after 2 eager steps")
    p.add_argument("--config_file", type=str, default=None,
                   help="YAML, TOML or JSON file of flag values (keys = flag names without dashes); flags given on "
                        "the command line override it")
    p.add_argument("--save_config", type=str, default=None,
                   help="write the resolved flags to this YAML/TOML/JSON file (by extension) and continue")
    return p


def _load_config_file(path: str) -> dict:
    ext = os.path.splitext(path)[1].lower()
    if ext in (".yaml", ".yml"):
        import yaml
        with open(path) as f:
            data = yaml.safe_load(f) or {}
    elif ext == ".toml":
        import tomllib
        with open(path, "rb") as f:
            data = tomllib.load(f)
    elif ext == ".json":
        with open(path) as f:
            data = json.load(f)
    else:
        raise ValueError(f"--config_file {path}: extension must be .yaml, .yml, .toml or .json")
    if not isinstance(data, dict):
        raise ValueError(f"--config_file {path}: top level must be a mapping of flag names to values")
    return data


def _coerce(action, key: str, value):
    """A config-file value as argparse would have produced it from the command line."""
    if isinstance(action, (argparse._StoreTrueAction, argparse._StoreFalseAction)):
        if not isinstance(value, bool):
            raise ValueError(f"config key {key!r}: expected true/false, got {value!r}")
        return value
    if action.nargs is not None and action.nargs not in ("?",):
        if not isinstance(value, (list, tuple)):
            raise ValueError(f"config key {key!r}: expected a list, got {value!r}")
        if isinstance(action.nargs, int) and len(value) != action.nargs:
            raise ValueError(f"config key {key!r}: expected {action.nargs} values, got {len(value)}")
        out = [action.type(v) if action.type is not None and v is not None else v for v in value]
        vals = out
    else:
        out = action.type(value) if (action.type is not None and value is not None) else value
        vals = [out]
    if action.choices is not None:
        for v in vals:
            if v not in action.choices:
                raise ValueError(f"config key {key!r}: {v!r} is not one of {list(action.choices)}")
    return tuple(out) if isinstance(out, list) and isinstance(action.default, tuple) else out


def parse_args(argv=None) -> argparse.Namespace:
    """Command-line flags, with defaults taken from ``--config_file`` when given.

    Precedence: command line > config file > built-in defaults. Unknown keys in
    the file are an error, so a typo cannot silently fall back to a default."""
    p = build_argparser()
    pre, _ = p.parse_known_args(argv)
    if pre.config_file:
        data = _load_config_file(pre.config_file)
        actions = {a.dest: a for a in p._actions if a.dest != "help"}
        unknown = sorted(k for k in data if k.replace("-", "_") not in actions)
        if unknown:
            raise ValueError(f"--config_file {pre.config_file}: unknown keys {unknown}")
        p.set_defaults(**{k.replace("-", "_"): _coerce(actions[k.replace("-", "_")], k, v) for k, v in data.items()
                          if k.replace("-", "_") not in ("config_file", "save_config")})
    args = p.parse_args(argv)
    if args.save_config and int(os.environ.get("RANK", "0")) == 0:  # one writer in a multi-process job
        save_config(args, args.save_config)
    return args


def save_config(args: argparse.Namespace, path: str) -> None:
    data = {k: (list(v) if isinstance(v, tuple) else v) for k, v in vars(args).items()
            if k not in ("config_file", "save_config")}
    ext = os.path.splitext(path)[1].lower()
    with open(path, "w") as f:
        if ext in (".yaml", ".yml"):
            import yaml
            yaml.safe_dump(data, f, sort_keys=False)
        elif ext == ".json":
            json.dump(data, f, indent=1)
        elif ext == ".toml":
            for k, v in data.items():  # flat keys: str, int, float, bool, list; None is left out
                if v is not None:
                    f.write(f"{k} = {json.dumps(v)}\n")
        else:
            raise ValueError(f"--save_config {path}: extension must be .yaml, .yml, .toml or .json")


def pick_device(arg: str):
    if arg == "auto":
        if torch.cuda.is_available():
            lr = int(os.environ.get("LOCAL_RANK", "0"))
            return torch.device("cuda", lr), lr
        if getattr(torch.backends, "mps", None) is not None and torch.backends.mps.is_available():
            return torch.device("mps"), 0  # the reference's order: cuda, then mps, then cpu (train.py:233-243)
        return torch.device("cpu"), 0
    dev = torch.device(arg)
    if dev.type == "cuda":
        lr = int(os.environ.get("LOCAL_RANK", "0")) if dev.index is None else dev.index
        return torch.device("cuda", lr), lr
    return dev, 0


def on_one_node(topo, ranks) -> bool:
    return topo.on_one_node(ranks) if hasattr(topo, "on_one_node") else True


def mp_group_of(topo):
    """Group of all ranks with this rank's dp_rank (the model-parallel replica), or None."""
    if topo.world_size == 1 or topo.tp * topo.pp * topo.ep == 1:
        return None
    groups = {}
    for d in range(topo.dp):
        ranks = [r for r in range(topo.world_size) if r // (topo.ep * topo.pp * topo.tp) == d]
        groups[d] = dist.new_group(ranks=ranks)
    return groups[topo.dp_rank]


def replication_weight(topo, tied_pp: bool = False):
    """Norm weight of each parameter: 1 / (number of model-parallel ranks holding a copy).
    With tied pipeline embeddings the first stage's wte and the last stage's lm_head are
    one parameter held twice."""

    def fn(name: str, p) -> float:
        w = 1.0
        if tied_pp and topo.pp > 1 and name in ("wte.weight", "lm_head.weight"):
            w /= 2
        tp_sharded = getattr(p, "tp_sharded", False)
        expert = ".experts." in name
        if topo.tp > 1 and not tp_sharded:
            w /= topo.tp
        if topo.ep > 1 and not expert:
            w /= topo.ep
        return w

    return fn


def mark_tp_sharded(module: torch.nn.Module) -> None:
    from .parallel.tp import ColumnParallelLinear, ColumnParallelLinearQKV, RowParallelLinear

    for m in module.modules():
        if isinstance(m, (ColumnParallelLinear, ColumnParallelLinearQKV)):
            m.weight.tp_sharded = True
            if m.bias is not None:
                m.bias.tp_sharded = True
        elif isinstance(m, RowParallelLinear):
            m.weight.tp_sharded = True


def lr_at(step: int, args) -> float:
    """Learning rate of optimizer step ``step`` (1-based). ``constant``: --learning_rate.
    ``cosine``: linear warmup over --warmup_iters steps, then cosine decay from
    --learning_rate to --min_lr at --max_iters."""
    lr = args.learning_rate
    if getattr(args, "lr_schedule", "constant") == "constant":
        return lr
    warm = max(0, int(args.warmup_iters))
    if step <= warm:
        return lr * step / warm
    span = max(1, args.max_iters - warm)
    frac = min(1.0, (step - warm) / span)
    return args.min_lr + 0.5 * (lr - args.min_lr) * (1.0 + math.cos(math.pi * frac))


class ScalarReader:
    """Reads each step's device scalar (loss) back to the host one step late.

    ``push`` starts an asynchronous copy into a pinned host slot and records an
    event; ``pop`` waits for the oldest copy and returns its value. Pushing step
    i+1 before popping step i keeps the next step queued on the GPU while the
    host waits, so reading every loss costs no idle gap between steps."""

    def __init__(self, depth: int = 2):
        self.depth = depth
        self._slots = None
        self._queue = []  # (slot index, event or None)
        self._i = 0

    def push(self, t: torch.Tensor) -> None:
        if len(self._queue) >= self.depth:
            raise RuntimeError("ScalarReader: pop before pushing more than `depth` values")
        if self._slots is None:
            pin = t.is_cuda
            self._slots = [torch.empty((), dtype=torch.float32, pin_memory=pin) for _ in range(self.depth)]
        slot = self._i % self.depth
        self._i += 1
        self._slots[slot].copy_(t.detach().float(), non_blocking=t.is_cuda)
        ev = None
        if t.is_cuda:
            ev = torch.cuda.Event()
            ev.record()
        self._queue.append((slot, ev))

    def pop(self) -> float:
        slot, ev = self._queue.pop(0)
        if ev is not None:
            ev.synchronize()
        return float(self._slots[slot])

    def __len__(self) -> int:
        return len(self._queue)


class _ListLoader:
    """Serves a fixed list of device batches in order (graph capture / replay)."""

    def __init__(self, batches):
        self.batches, self.i = batches, 0
        self.B = batches[0][0].shape[0]

    def next_batch(self, device):
        b = self.batches[self.i % len(self.batches)]
        self.i += 1
        return b


class Engine:
    """Owns the model/stage, optimizer and one training step."""

    def __init__(self, args, topo, device, cfg):
        self.args, self.topo, self.device, self.cfg = args, topo, device, cfg
        self.use_pipeline = topo.pp > 1
        if self.use_pipeline:
            self.module = StageModule(cfg, topo, topo.pp_rank, topo.pp)
        else:
            self.module = GPT(cfg, topo=topo)
        mark_tp_sharded(self.module)
        self.module.to(device)
        self.tied = None
        self.skipped_steps = 0  # plain engine: steps skipped for a non-finite gradient norm
        self.regions = None  # RegionTimer of an instrumented eager step (REGIONS), else None
        if self.use_pipeline and getattr(args, "pp_tie_embeddings", 0):
            from .parallel.pipeline import TiedEmbeddings
            self.tied = TiedEmbeddings(self.module, topo)
            self.tied.sync_weights()
        self.amp = args.amp if device.type in ("cuda", "mps") else "none"  # as train.py:354
        from .models.fused import fused_supported

        ok, why = fused_supported(cfg, topo, tp_dropout=bool(getattr(args, "fused_tp_dropout", 1)))
        want = args.engine
        if want == "fused" and not ok:
            raise ValueError(f"--engine fused: {why}")
        if want == "fused" and (device.type != "cuda" or self.amp not in ("bf16", "fp16")):
            raise ValueError("--engine fused needs --device cuda and --amp bf16 or fp16")
        self.fused = (want in ("auto", "fused")) and ok and device.type == "cuda" and self.amp in ("bf16", "fp16")
        # why an automatic choice ended on the plain engine (logged at start). --amp none
        # stays on the plain engine: it is the fp32 mode that matches the reference to 1e-4.
        self.plain_reason = None
        if not self.fused and want == "auto" and device.type == "cuda":
            self.plain_reason = why if not ok else "--amp none runs the plain fp32 engine (the fused one is 16-bit)"
        if self.fused:
            from .ops._C import load as _load
            _load()  # fail loudly if the extension is missing
        if getattr(args, "zero_stage", 0) and self.fused:
            raise ValueError("--zero_stage 1 runs on the plain engine (--engine plain); the fused engine keeps "
                             "full AdamW moments in its flat buffers")
        if getattr(args, "activation_checkpointing", 0):
            if self.fused and topo.tp > 1:
                raise ValueError("--activation_checkpointing: the fused tensor-parallel blocks keep their "
                                 "activations; use --engine plain or tp 1")
            self.module.recompute = True  # plain: torch.utils.checkpoint; fused: dense blocks rerun in backward
        self.dropout_seed = None
        if self.fused and cfg.dropout > 0:
            # Device seed of the fused dropout masks: different per DP / PP rank
            # (like the reference's per-rank torch seeds, train.py:318-328), equal
            # across TP / EP ranks, whose replicated computations must stay identical.
            base = (args.seed * 1000003 + topo.dp_rank * 7919 + topo.pp_rank * 104729) & 0x7FFFFFFF
            self.dropout_seed = torch.tensor([base], dtype=torch.int32, device=device)
            if self.use_pipeline:
                blocks = [(self.module.block_start + i, b) for i, b in enumerate(self.module.blocks)]
            else:
                blocks = list(enumerate(self.module.tr.h))
            for layer, blk in blocks:
                blk._hb_dropout = (self.dropout_seed, layer, float(cfg.dropout))
        self.mp_group = mp_group_of(topo)
        if self.fused:
            from .optim import FusedAdamW
            from .parallel.flat import FlatParams

            # The DP reduction runs over NVLink peer memory when the DP group is on one node,
            # else (a multi-node job) as NCCL all-reduces.
            use_p2p = (topo.dp > 1 and os.environ.get("HB_DP_BACKEND", "p2p") == "p2p"
                       and on_one_node(topo, topo.dp_ranks))
            from .optim import DeviceLossScaler

            self.flat = FlatParams(self.module, device, weight_of=replication_weight(topo, self.tied is not None),
                                   grad_group=topo.dp_group if use_p2p else None,
                                   tp_group=topo.tp_group if topo.tp > 1 else None,
                                   tp_sum_of=lambda n, p: topo.tp > 1 and not getattr(p, "tp_sharded", False),
                                   dtype16=torch.float16 if self.amp == "fp16" else torch.bfloat16)
            self.module.fused = True
            # fp16: activations and weight shadows in fp16, the loss scaled on the device
            # (GradScaler's rule) and unscaled inside the optimizer's clip coefficient
            fused_scaler = DeviceLossScaler(device) if self.amp == "fp16" else None
            # upstream gradient of the data loss in a training step: (loss + aux) / accumulation,
            # times the loss scale under fp16
            self.module.loss_grad_hint = 1.0 / args.grad_accum_steps
            self.module.loss_grad_scale = fused_scaler.scale_tensor if fused_scaler is not None else None
            clip_group = self.mp_group if args.clip_mode == "global" else None
            mp_symm = None
            if clip_group is not None and device.type == "cuda" and on_one_node(topo, topo.model_parallel_ranks()):
                from .parallel.symm import SymmetricBuffer
                mp_symm = SymmetricBuffer(clip_group, 16, device)
            self.optimizer = FusedAdamW(self.flat, lr=args.learning_rate, betas=args.betas,
                                        weight_decay=args.weight_decay, max_grad_norm=args.grad_clip,
                                        mp_group=clip_group, mp_symm=mp_symm, scaler=fused_scaler)
            self.scaler = fused_scaler
        elif getattr(args, "zero_stage", 0):
            from .parallel.zero import ZeroAdamW

            self.flat = None
            self.optimizer = ZeroAdamW(self.module.named_parameters(), topo.dp_group, lr=args.learning_rate,
                                       betas=tuple(args.betas), weight_decay=args.weight_decay)
            self.scaler = torch.amp.GradScaler("cuda", enabled=(self.amp == "fp16"))
        else:
            self.flat = None
            # torch's single-kernel AdamW (same update as the reference's default AdamW,
            # one pass over each parameter instead of one op per moment and parameter)
            fused_ok = device.type in ("cpu", "cuda")
            self.optimizer = torch.optim.AdamW(self.module.parameters(), lr=args.learning_rate,
                                               betas=tuple(args.betas), weight_decay=args.weight_decay,
                                               fused=fused_ok or None)
            self.scaler = torch.amp.GradScaler("cuda", enabled=(self.amp == "fp16"))
        self.amp_dtype = torch.float16 if self.amp == "fp16" else torch.bfloat16
        self.use_amp = self.amp in ("fp16", "bf16") and not self.fused
        self.forward_module = self.module
        if args.compile and not self.fused:
            self.forward_module = torch.compile(self.module)
        self.reducer = None
        if topo.dp > 1 and self.fused:
            from .parallel.grad_reduce import FlatGradReducer
            self.reducer = FlatGradReducer(self.flat, topo.dp_group, topo)
        # DP reduction overlapped with the last micro-batch's backward (fused, non-TP blocks).
        self.overlap_dp = (self.reducer is not None and self.reducer.can_overlap() and topo.tp == 1
                           and not self.use_pipeline and bool(getattr(args, "overlap_dp", 0)))
        if self.use_pipeline:
            bd = torch.float32 if args.pp_boundary_dtype == "fp32" else torch.bfloat16
            self.pipe = GPipeEngine(self.module, topo, boundary_dtype=bd,
                                    schedule=getattr(args, "pp_schedule", "gpipe"))
            self.pipe.fused_head = not args.compile
        # CUDA-graph replay of the whole fused step (forward, backward, DP
        # reduction, clipping, AdamW) once shapes are known; the first
        # GRAPH_WARMUP steps run eagerly (they also initialise lazy state).
        self.use_graph = (bool(getattr(args, "cuda_graph", 1)) and self.fused and not self.use_pipeline
                          and (self.reducer is None or self.reducer.backend == "p2p")
                          and (self.mp_group is None or args.clip_mode != "global"
                               or self.optimizer.mp_symm is not None))
        self._graph = None
        self._eager_steps = 0
        self.GRAPH_WARMUP = 2

    # -- one optimizer step ---------------------------------------------------
    def train_step(self, loader) -> tuple:
        if self.use_graph:
            batches = [loader.next_batch(self.device) for _ in range(self.args.grad_accum_steps)]
            return self._graph_step(batches)
        return self._eager_step(loader)

    def _graph_step(self, batches) -> tuple:
        if self._graph is None and self._eager_steps < self.GRAPH_WARMUP:
            self._eager_steps += 1
            return self._eager_step(_ListLoader(batches))
        if self._graph is None:
            self._static = [(x.clone(), y.clone()) for x, y in batches]
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            self.optimizer.prepare_step()
            with torch.cuda.graph(g):
                self._static_out = self._device_step(_ListLoader(self._static))
            self._graph = g
            g.replay()
        else:
            for (sx, sy), (x, y) in zip(self._static, batches):
                sx.copy_(x, non_blocking=True)
                sy.copy_(y, non_blocking=True)
            self.optimizer.prepare_step()
            self._graph.replay()
        loss, aux = self._static_out
        return self._average_scalars(loss.clone(), aux.clone())

    def _average_scalars(self, loss_scalar, aux):
        """Loss / aux all-reduce over DP (outside any captured graph: NCCL stays out of graphs)."""
        topo = self.topo
        if self.fused and topo.tp > 1 and dist.is_initialized():
            dist.all_reduce(loss_scalar, op=dist.ReduceOp.SUM, group=topo.tp_group)  # shard losses / tp
        if topo.dp_group is not None and dist.is_initialized():
            both = torch.stack([loss_scalar, aux])
            dist.all_reduce(both, op=dist.ReduceOp.SUM, group=topo.dp_group)
            both = both / topo.dp
            return both[0], both[1]
        return loss_scalar, aux

    def _device_step(self, loader) -> tuple:
        """Forward/backward of every microbatch, DP gradient reduction and optimizer (device work only;
        the DP reduction here is the fused peer-memory kernel, so a captured graph holds no NCCL call)."""
        accum = self.args.grad_accum_steps
        aux = torch.zeros((), device=self.device)
        loss_sum = torch.zeros((), device=self.device)
        for i in range(accum):
            x, y = loader.next_batch(self.device)
            _, loss, aux_mb = self.forward_module(x, y, return_logits=False)
            if i == accum - 1 and self.reducer is not None and self.overlap_dp:
                self.reducer.arm()  # reduce each block's gradients while backward continues
            combined = (loss + aux_mb) / accum
            (self.scaler.scale(combined) if self.scaler is not None else combined).backward()
            aux = aux + aux_mb.detach().float()
            loss_sum = loss_sum + loss.detach().float()
        if self.reducer is not None:
            self.reducer.finish()
        self.tp_sync_grads()
        self.optimizer.step_device()
        self.optimizer.zero_grad()
        return loss_sum / accum, aux

    def close(self) -> None:
        """Release the captured graph (before destroy_process_group) and wait for the device."""
        if self.device.type == "cuda":
            torch.cuda.synchronize()
        self._graph = None
        self._static = None
        self._static_out = None

    # Regions of an instrumented step, entered by every rank in this order.
    REGIONS = ("fwd_bwd", "tied_emb", "tp_sync", "dp_reduce", "optimizer")

    def _region(self, name: str):
        return self.regions.region(name) if self.regions is not None else contextlib.nullcontext()

    def timed_regions_step(self, loader, timer) -> tuple:
        """One eager optimizer step (the kernels a captured step replays) with device
        timers around each region in REGIONS; returns the step's (loss, aux)."""
        self.regions = timer
        try:
            return self._eager_step(loader)
        finally:
            self.regions = None

    def _eager_step(self, loader) -> tuple:
        topo = self.topo
        with self._region("fwd_bwd"):
            loss_scalar, aux = self._forward_backward(loader)
        if loss_scalar is not None and topo.dp_group is not None and dist.is_initialized():
            dist.all_reduce(loss_scalar, op=dist.ReduceOp.SUM, group=topo.dp_group)
            loss_scalar = loss_scalar / topo.dp
        if aux is not None and topo.dp_group is not None and dist.is_initialized():
            dist.all_reduce(aux, op=dist.ReduceOp.SUM, group=topo.dp_group)
            aux = aux / topo.dp
        self.sync_and_step()
        return loss_scalar, aux

    def _forward_backward(self, loader) -> tuple:
        args, topo = self.args, self.topo
        accum = args.grad_accum_steps
        if self.use_pipeline:
            loss_scalar, aux = self.pipe.forward_backward(loader, micro_batches=accum, device=self.device,
                                                          use_amp=self.use_amp, amp_dtype=self.amp_dtype,
                                                          scaler=self.scaler, batch_size=args.batch_size,
                                                          aux_loss_coef=args.aux_loss_coef)
            if self.fused and topo.tp > 1 and loss_scalar is not None and dist.is_initialized():
                dist.all_reduce(loss_scalar, op=dist.ReduceOp.SUM, group=topo.tp_group)  # shard losses / tp
        else:
            aux = torch.zeros((), device=self.device)
            loss_sum = torch.zeros((), device=self.device)
            for _ in range(accum):
                x, y = loader.next_batch(self.device)
                with torch.autocast(device_type=self.device.type, dtype=self.amp_dtype, enabled=self.use_amp):
                    # the plain path's one-node lm_head + cross-entropy is an eager optimisation;
                    # a torch.compile'd module gets the logits path to trace instead
                    _, loss, aux_mb = self.forward_module(x, y, return_logits=bool(self.args.compile)
                                                          and not self.fused)
                    combined = (loss + aux_mb) / accum
                aux = aux + aux_mb.detach().float()
                loss_sum = loss_sum + loss.detach().float()
                if self.scaler is not None and self.scaler.is_enabled():
                    self.scaler.scale(combined).backward()
                else:
                    combined.backward()
            loss_scalar = loss_sum / accum
            if self.fused and topo.tp > 1 and dist.is_initialized():
                dist.all_reduce(loss_scalar, op=dist.ReduceOp.SUM, group=topo.tp_group)
        return loss_scalar, aux

    def tp_sync_grads(self) -> None:
        """Sum the token-shard partial gradients of TP-replicated parameters over the TP group."""
        if not self.fused or self.topo.tp == 1 or self.flat.grad_symm_tp is None:
            return
        for (start, end, _), tp_sum in zip(self.flat.ranges, self.flat.tp_sum):
            if tp_sum and end > start:
                self.flat.grad_symm_tp.sum_range(start, end - start, 1.0)

    def sync_and_step(self) -> None:
        args = self.args
        with self._region("tied_emb"):
            if self.tied is not None:
                self.tied.reduce_grads()
        if self.fused:
            with self._region("tp_sync"):
                self.tp_sync_grads()
            with self._region("dp_reduce"):
                if self.reducer is not None:
                    self.reducer.reduce()
            with self._region("optimizer"):
                self.optimizer.step()
                self.optimizer.zero_grad()
            return
        if self.scaler is not None and self.scaler.is_enabled():
            self.scaler.unscale_(self.optimizer)
        with self._region("tp_sync"):
            pass  # the plain path sums TP gradients inside autograd (column-parallel backward)
        with self._region("dp_reduce"):
            average_gradients(self.module, self.topo.dp_group)
        with self._region("optimizer"):
            if args.grad_clip > 0 and not self.clip_plain(args.grad_clip):
                # Non-finite global norm (clip_mode global): every rank of the job sees it
                # (the DP average and the model-parallel norm sum carry it), so all skip.
                self.skipped_steps += 1
                if self.scaler is not None and self.scaler.is_enabled():
                    self.scaler.update(self.scaler.get_scale() * self.scaler.get_backoff_factor())
                self.optimizer.zero_grad(set_to_none=True)
                return
            if self.scaler is not None and self.scaler.is_enabled():
                self.scaler.step(self.optimizer)
                self.scaler.update()
            else:
                self.optimizer.step()
            self.optimizer.zero_grad(set_to_none=True)

    def clip_plain(self, max_norm: float) -> bool:
        """Clip the gradients to ``max_norm``. Returns False when the global norm is not
        finite (clip_mode global): the caller then skips the step on every rank, as the
        fused optimizer does and as GradScaler does for an fp16 overflow (the reference
        clips NaN gradients into the weights, train.py:446, and its GradScaler decides per
        rank). clip_mode local keeps the reference's per-shard clip and never skips."""
        params = [p for p in self.module.parameters() if p.grad is not None]
        if self.args.clip_mode == "local":
            torch.nn.utils.clip_grad_norm_(params, max_norm)
            return True
        if self.mp_group is None:
            norm = torch.nn.utils.clip_grad_norm_(params, max_norm)
            return bool(torch.isfinite(norm))
        wfn = replication_weight(self.topo, self.tied is not None)
        names = {id(p): n for n, p in self.module.named_parameters()}
        tot = torch.zeros((), device=self.device)
        for p in params:
            tot = tot + wfn(names[id(p)], p) * p.grad.detach().float().pow(2).sum()
        dist.all_reduce(tot, group=self.mp_group)
        if not bool(torch.isfinite(tot)):
            return False
        coef = torch.clamp(max_norm / (tot.sqrt() + 1e-6), max=1.0)
        for p in params:
            p.grad.detach().mul_(coef.to(p.grad.dtype))
        return True

    # -- eval -----------------------------------------------------------------
    @torch.no_grad()
    def estimate_loss(self, loader, eval_iters: int) -> Optional[float]:
        self.module.eval()
        losses = []
        for _ in range(eval_iters):
            if self.use_pipeline:
                l = self.pipe.forward_only(loader, self.args.grad_accum_steps, self.device, self.use_amp,
                                           self.amp_dtype, loader.B)
                if l is not None and self.fused and self.topo.tp > 1 and dist.is_initialized():
                    dist.all_reduce(l, group=self.topo.tp_group)  # shard losses / tp sum to the mean
                if l is not None and self.topo.dp_group is not None and dist.is_initialized():
                    dist.all_reduce(l, group=self.topo.dp_group)
                    l = l / self.topo.dp
                if l is not None:
                    losses.append(float(l.item()))
            else:
                x, y = loader.next_batch(self.device)
                with torch.autocast(device_type=self.device.type, dtype=self.amp_dtype, enabled=self.use_amp):
                    # the loss only: no [tokens, vocab] logits copy
                    _, loss, _ = self.forward_module(x, y, return_logits=bool(self.args.compile) and not self.fused)
                if self.fused and self.topo.tp > 1 and dist.is_initialized():
                    loss = loss.detach().clone()
                    dist.all_reduce(loss, group=self.topo.tp_group)  # shard losses / tp sum to the mean
                losses.append(float(loss.item()))
        self.module.train()
        return sum(losses) / len(losses) if losses else None

    # -- optimizer state by parameter name (checkpoints) ------------------------
    def optimizer_state(self) -> dict:
        """AdamW moments keyed by parameter name, for either engine (see FusedAdamW.moments_by_name)."""
        if self.fused:
            out = self.optimizer.moments_by_name()
            if self.scaler is not None:  # fp16: the device loss scale
                out["scaler"] = self.scaler.state_dict()
            return out
        if hasattr(self.optimizer, "moments_by_name"):  # ZeroAdamW: gathers the DP shards (collective)
            out = self.optimizer.moments_by_name()
            if self.scaler is not None and self.scaler.is_enabled():
                out["scaler"] = self.scaler.state_dict()
            return out
        m, v, step = {}, {}, 0
        for name, p in self.module.named_parameters():
            st = self.optimizer.state.get(p)
            if st and "exp_avg" in st:
                m[name], v[name] = st["exp_avg"].detach().cpu(), st["exp_avg_sq"].detach().cpu()
                step = int(st["step"])
        out = {"format": "by_name", "step": step, "m": m, "v": v}
        if self.scaler is not None and self.scaler.is_enabled():
            out["scaler"] = self.scaler.state_dict()
        return out

    def load_optimizer_state(self, st: dict) -> None:
        """Inverse of ``optimizer_state``; also accepts an optimizer's own ``state_dict()``."""
        if st.get("format") != "by_name":
            self.optimizer.load_state_dict(st)
            return
        if self.fused or hasattr(self.optimizer, "load_moments_by_name"):
            self.optimizer.load_moments_by_name(st)
            if "scaler" in st and self.scaler is not None and self.scaler.is_enabled():
                self.scaler.load_state_dict(st["scaler"])
            return
        for name, p in self.module.named_parameters():
            if name in st["m"]:
                self.optimizer.state[p] = {"step": torch.tensor(float(st["step"])),
                                           "exp_avg": st["m"][name].to(p.device, p.dtype).clone(),
                                           "exp_avg_sq": st["v"][name].to(p.device, p.dtype).clone()}
        if "scaler" in st and self.scaler is not None and self.scaler.is_enabled():
            self.scaler.load_state_dict(st["scaler"])

    def after_load(self) -> None:
        if self.tied is not None:
            self.tied.sync_weights()
        if self.flat is not None:
            self.flat.refresh_bf16()


def main(argv=None) -> None:
    args = parse_args(argv)
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    distributed = world_env > 1
    device, local_rank = pick_device(args.device)
    if device.type == "cuda":
        torch.cuda.set_device(local_rank)
    if distributed:
        if args.dist_backend == "nccl" and device.type != "cuda":
            raise RuntimeError("nccl backend requires CUDA; use gloo or run on CUDA.")
        kw = {"timeout": timedelta(seconds=args.pg_timeout_s)}
        if args.dist_backend == "nccl":
            kw["device_id"] = device
        store = attempt_store(kw["timeout"])
        if store is not None:
            kw.update(store=store, rank=int(os.environ["RANK"]), world_size=world_env)
        dist.init_process_group(backend=args.dist_backend, **kw)
    topo = init_topology(dp=args.dp, ep=args.ep, tp=args.tp, pp=args.pp,
                         timeout=timedelta(seconds=args.pg_timeout_s))
    rank = topo.rank

    # Same init seed on every TP rank (shards are slices of one full matrix).
    torch.manual_seed(args.seed)
    if device.type == "cuda":
        torch.cuda.manual_seed_all(args.seed)
    cfg = GPTConfig(block_size=args.block_size, n_layer=args.n_layer, n_head=args.n_head, n_embed=args.n_embed,
                    dropout=args.dropout, num_experts=args.num_experts, top_k=args.top_k, moe_freq=args.moe_freq,
                    aux_loss_coef=args.aux_loss_coef)
    engine = Engine(args, topo, device, cfg)
    module = engine.module
    start_step = 1
    resume_side = None
    if args.init_from and args.resume:
        raise ValueError("--init_from starts a new run from a checkpoint's weights; --resume continues one")
    if args.init_from:
        # New run from trained weights (fine-tuning, a changed schedule): weights only, on any
        # TP/PP/EP layout; optimizer, RNG, data position and step numbering start fresh.
        from .utils.ckpt import load_for_resume
        info = load_for_resume(module, args.init_from, topo)
        engine.after_load()
        if rank == 0:
            print(f"[init_from] weights of step {info['step']} from {args.init_from}; starting at step 1")
    if args.resume == "auto":
        # Restart after a failure (torchrun --max-restarts): the newest step every rank
        # finished writing, or a fresh start when there is none.
        from .utils.ckpt import latest_complete_checkpoint
        found = latest_complete_checkpoint(args.out_dir, topo)
        if rank == 0:
            print(f"[resume] auto: {found}" if found else f"[resume] auto: no complete checkpoint in "
                                                           f"{args.out_dir}; starting from step 1")
        args.resume = found
    if args.resume:
        from .utils.ckpt import (find_rank_state, load_for_resume, merged_optimizer_moments, reslice_moments,
                                 sidecar_path)
        info = load_for_resume(module, args.resume, topo)
        engine.after_load()
        start_step = info["step"] + 1
        restored = []
        if info["same_layout"]:
            side = sidecar_path(info["file"])
            if os.path.exists(side):
                side_obj = torch.load(side, map_location="cpu", weights_only=False)
                engine.load_optimizer_state(side_obj.get("optimizer", side_obj))
                restored.append("optimizer")
                if topo.dp == 1:
                    resume_side = side_obj  # files without per-rank state: RNG / data position of dp rank 0
        else:
            moments = merged_optimizer_moments(args.resume, info["headers"])
            if moments is not None:
                engine.load_optimizer_state(reslice_moments(module, info["full"], moments, topo.tp_rank, topo.tp))
                restored.append("optimizer (merged and re-sliced)")
        st, exact = find_rank_state(info["file"], info["step"], topo)
        if st is not None:
            resume_side = st
        if resume_side is not None and "rng" in resume_side:
            restored.append("RNG and data position" + ("" if exact or info["same_layout"] else
                                                       " (of the same DP rank)"))
        if rank == 0:
            how = "its own shard" if info["same_layout"] else "the merged shards of another TP/PP/EP layout"
            print(f"[resume] step {info['step']} from {args.resume} ({how})"
                  f"{'; ' + ', '.join(restored) if restored else '; weights only, the optimizer restarts'}")
    n_params = sum(p.numel() for p in module.parameters())
    if rank == 0:
        print(f"[model] parameters: {n_params:,} ({n_params / 1e6:.1f}M) | engine="
              f"{'fused' if engine.fused else 'plain'}")
        if engine.plain_reason:
            print(f"[engine] plain: {engine.plain_reason}")
        per_node = topo.local_world or topo.world_size
        if topo.world_size > per_node:
            dp_how = ("NVLink peer memory" if engine.reducer is not None and engine.reducer.backend == "p2p"
                      else "NCCL all-reduce")
            print(f"[nodes] {topo.world_size // per_node} nodes x {per_node} ranks | DP gradient reduction: "
                  f"{dp_how}")
        if args.num_experts > 0:
            nm = sum(1 for i in range(args.n_layer) if cfg.is_moe_layer(i))
            print(f"[MoE] num_experts={args.num_experts}, top_k={args.top_k}, moe_layers={nm}/{args.n_layer}, "
                  f"ep={args.ep}")

    data_seed = args.seed if args.dp_share_data else args.seed + topo.dp_rank
    random.seed(data_seed)
    np.random.seed(data_seed)
    torch_seed = args.seed if args.dp_share_data else args.seed + topo.dp_rank * 1000 + topo.pp_rank
    torch.manual_seed(torch_seed)
    if device.type == "cuda":
        torch.cuda.manual_seed_all(torch_seed)
    rank_for_data = 0 if args.dp_share_data else topo.dp_rank
    if args.synthetic_data:
        train_loader = SyntheticLoader(args.batch_size, args.block_size, cfg.vocab_size, seed=args.seed,
                                       rank=rank_for_data)
        val_loader = SyntheticLoader(args.batch_size, args.block_size, cfg.vocab_size, seed=args.seed + 999)
    else:
        train_loader = RandomBatchLoader(args.data_dir, "train", args.batch_size, args.block_size,
                                         args.num_train_chunks, seed=args.seed, rank=rank_for_data,
                                         dp_rank=0 if args.dp_share_data else topo.dp_rank,
                                         dp_size=1 if args.dp_share_data else topo.dp, log_rank=rank)
        val_loader = RandomBatchLoader(args.data_dir, "val", args.batch_size, args.block_size, args.num_val_chunks,
                                       seed=args.seed + 999, rank=0, dp_rank=0, dp_size=1, log_rank=rank)

    if resume_side is not None:
        from .utils.ckpt import set_rng_state
        if "rng" in resume_side:
            set_rng_state(resume_side["rng"])
        if "train_loader" in resume_side and hasattr(train_loader, "load_state_dict"):
            train_loader.load_state_dict(resume_side["train_loader"])
        if "dropout_seed" in resume_side and engine.dropout_seed is not None:
            engine.dropout_seed.fill_(int(resume_side["dropout_seed"]))
    is_main = topo.is_main
    if is_main:
        print(f"device={device} | world_size={topo.world_size} | dp={topo.dp} ep={topo.ep} tp={topo.tp} "
              f"pp={topo.pp}")
    run = None
    if is_main and args.wandb and WANDB_AVAILABLE and args.wandb_mode != "disabled":
        run = wandb.init(project=args.wandb_project, entity=args.wandb_entity or None,
                         config={**vars(args), **asdict(cfg), "device": device.type}, mode=args.wandb_mode,
                         name=args.run_name or None)
    elif is_main and args.wandb and not WANDB_AVAILABLE:
        print("wandb not available; proceeding without external logging.")

    if args.eval_only:
        # evaluate the weights as loaded (--init_from / --resume) and stop: every rank takes part
        ev = engine.estimate_loss(val_loader, args.eval_iters)
        if is_main and ev is not None:
            print(f"[eval_only] eval_loss {ev:.4f} over {args.eval_iters} batches")
            if run:
                wandb.log({"eval/loss": ev})
                run.finish()
        engine.close()
        if distributed and dist.is_initialized():
            cleanup()
        return
    module.train()
    t0 = time.time()
    wd = None
    if distributed and args.watchdog_s > 0:
        from .utils.fault import StepWatchdog, default_store
        # Keys of one attempt only: a restarted job (torchrun --max-restarts) must not read the
        # failure that ended the previous attempt.
        attempt = os.environ.get("TORCHELASTIC_RESTART_COUNT", "0")
        wd = StepWatchdog(default_store(), dist.get_rank(), dist.get_world_size(), timeout_s=args.watchdog_s,
                          prefix=f"hb_watchdog/attempt{attempt}")
    try:
        _train_loop(args, engine, module, cfg, topo, train_loader, val_loader, run, wd, t0, start_step)
    except BaseException as e:
        if wd is not None:
            wd.mark_failed(f"{type(e).__name__}: {e}")
            wd.stop()
        try:
            engine.close()
        except Exception:
            pass
        raise
    if wd is not None:
        wd.finish()
    if is_main and run:
        run.finish()
    if is_main:
        print("training finished.")
    engine.close()
    if distributed and dist.is_initialized():
        cleanup()


def attempt_store(timeout):
    """The rendezvous store of a restarted torchrun attempt, under a key prefix of its own.

    torchrun keeps its store across restarts of the worker group, and process
    groups publish their addresses under fixed keys: a rank of attempt n could
    read the address of a dead rank of an earlier attempt and fail to connect.
    From the first restart on (TORCHELASTIC_RESTART_COUNT > 0) every key goes under
    ``hb_attempt<n>/``; the first attempt uses the plain env:// rendezvous."""
    attempt = int(os.environ.get("TORCHELASTIC_RESTART_COUNT", "0") or 0)
    if attempt == 0:
        return None
    agent = os.environ.get("TORCHELASTIC_USE_AGENT_STORE") == "True"
    rank = int(os.environ["RANK"])
    base = dist.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["MASTER_PORT"]),
                         int(os.environ["WORLD_SIZE"]), is_master=(not agent and rank == 0), timeout=timeout)
    return dist.PrefixStore(f"hb_attempt{attempt}", base)


def injected_failure():
    """Host-side fault injection for recovery tests: ``HB_INJECT_FAILURE=<rank>:<step>``
    makes that rank raise at the start of that step, in the first attempt of a job only
    (TORCHELASTIC_RESTART_COUNT unset or 0), so a restarted job runs through. Nothing
    on a GPU is involved: the rank leaves between steps, with no kernel in flight."""
    spec = os.environ.get("HB_INJECT_FAILURE")
    if not spec or os.environ.get("TORCHELASTIC_RESTART_COUNT", "0") != "0":
        return None
    r, _, k = spec.partition(":")
    return int(r), int(k)


def _train_loop(args, engine, module, cfg, topo, train_loader, val_loader, run, wd, t0, start_step=1) -> None:
    from .utils.profiling import RegionTimer, rank_spread

    is_main = topo.is_main
    tokens_per_step = args.batch_size * args.block_size * args.grad_accum_steps
    last = time.time()
    log_every = args.log_interval or max(1, args.eval_interval // 10)
    timer = RegionTimer(enabled=bool(args.device_timing) and engine.device.type == "cuda")
    timed_steps = 0
    inject = injected_failure()
    for step in range(start_step, args.max_iters + 1):
        if args.lr_schedule != "constant":
            for g in engine.optimizer.param_groups:
                g["lr"] = lr_at(step, args)  # read by the next step (graph replays included)
        if wd is not None:
            wd.check()  # a failed peer is noticed here, before this step launches anything
        if inject is not None and inject == (topo.rank, step):
            raise RuntimeError(f"injected failure: rank {topo.rank} at step {step} (HB_INJECT_FAILURE)")
        region_ms = None
        spread = None  # per-rank device step times of a logging step (multi-rank runs)
        if args.region_timing_interval > 0 and step % args.region_timing_interval == 0:
            # Instrumented eager step (kept out of the dev_tok/s figure); every rank takes part.
            regions = RegionTimer(enabled=True)
            loss_scalar, aux = engine.timed_regions_step(train_loader, regions)
            region_ms = regions.summary()
            if is_main:
                print(f"step {step:6d} | regions (ms, max over ranks) "
                      + " | ".join(f"{k} {v:.3f}" for k, v in region_ms.items()))
        else:
            with timer.region("step"):
                loss_scalar, aux = engine.train_step(train_loader)
            timed_steps += 1
        if wd is not None:
            wd.beat(step)
        now = time.time()
        dt = now - last
        last = now
        eff = tokens_per_step / dt if dt > 0 else float("inf")
        if step % log_every == 0 or step == start_step:
            dev_str = ""
            if timer.enabled:
                # every rank takes part in the gather; all log on the same steps
                per_rank = [t / max(1, timed_steps) for t in timer.per_rank().get("step", [0.0])]
                step_ms = max(per_rank)
                timed_steps = 0
                if step_ms > 0:
                    dev_str = f" | dev_tok/s {topo.dp * tokens_per_step / (step_ms / 1e3):,.0f} ({step_ms:.2f} ms)"
                    if len(per_rank) > 1:
                        spread = rank_spread(per_rank)
                        dev_str += (f" | rank ms {spread['min']:.2f}..{spread['max']:.2f} "
                                    f"(slowest r{int(spread['slowest'])})")
            if is_main:
                aux_str = f" | aux_loss {aux.item():.4f}" if args.num_experts > 0 else ""
                ls = f"{loss_scalar.item():.4f}" if loss_scalar is not None else "n/a"
                lr_str = (f" | lr {engine.optimizer.param_groups[0]['lr']:.3e}"
                          if args.lr_schedule != "constant" else "")
                print(f"step {step:6d} | train_loss (mean micro) {ls}{aux_str} | eff_tok/s {eff:,.0f}{dev_str}{lr_str}")
        if is_main and run:
            log = {"train/loss_mean_micro": float(loss_scalar.item()) if loss_scalar is not None else float("nan"),
                   "opt/lr": float(engine.optimizer.param_groups[0]["lr"]), "speed/eff_tokens_per_sec": eff,
                   "amp/enabled": int(engine.amp != "none"), "amp/mode": args.amp,
                   "accum/steps": args.grad_accum_steps, "step": step}
            if region_ms:
                log.update({f"time/{k}_ms": v for k, v in region_ms.items()})
            if spread:
                log.update({"speed/rank_step_ms_min": spread["min"], "speed/rank_step_ms_median": spread["median"],
                            "speed/rank_step_ms_max": spread["max"], "speed/slowest_rank": int(spread["slowest"]),
                            "speed/rank_imbalance": spread["imbalance"]})
            if args.num_experts > 0:
                log["train/aux_loss"] = float(aux.item())
                log.update(expert_load_metrics(module))
                counts = expert_counts(module)
                if counts is not None and hasattr(wandb, "Table"):
                    table = wandb.Table(data=[[f"E{i}", float(c)] for i, c in enumerate(counts.tolist())],
                                        columns=["Expert", "Tokens"])
                    log["expert_load/distribution"] = wandb.plot.bar(table, "Expert", "Tokens",
                                                                     title=f"Expert Load (step {step})")
            wandb.log(log, step=step)
        if step % args.eval_interval == 0 or step == args.max_iters:
            ev = engine.estimate_loss(val_loader, args.eval_iters)
            if is_main and ev is not None:
                print(f"[eval] step {step} | eval_loss {ev:.4f} | elapsed {time.time() - t0:.1f}s")
                if run:
                    wandb.log({"eval/loss": ev, "step": step}, step=step)
        if args.save_interval and step % args.save_interval == 0:
            from .utils.ckpt import rng_state
            side = {"optimizer": engine.optimizer_state(), "rng": rng_state()}
            if engine.dropout_seed is not None:  # fused dropout masks continue where they stopped
                side["dropout_seed"] = int(engine.dropout_seed.item())
            if hasattr(train_loader, "state_dict"):
                side["train_loader"] = train_loader.state_dict()
            save_checkpoint(module, cfg, step, topo, args.out_dir, optimizer_state=side)
            from .utils.ckpt import save_rank_state  # every rank: its own RNG and data position
            save_rank_state(args.out_dir, step, topo, {k: side[k] for k in ("rng", "train_loader", "dropout_seed")
                                                       if k in side})
            if dist.is_initialized() and topo.world_size > 1:
                dist.barrier()  # every rank's files of this step are on disk
            if topo.rank == 0:
                from .utils.ckpt import mark_step_complete
                mark_step_complete(args.out_dir, step, topo)


def expert_counts(module):
    """Per-expert token counts [E] summed over the MoE layers, or None (reference train.py:359-370)."""
    from .models.moe import MoELayer

    total = None
    for m in module.modules():
        if isinstance(m, MoELayer) and m._expert_counts is not None:
            total = m._expert_counts.float().clone() if total is None else total + m._expert_counts.float()
    return total


def expert_load_metrics(module) -> dict:
    """Expert-load scalars of the reference's wandb log (train.py:478-494)."""
    total = expert_counts(module)
    if total is None:
        return {}
    out = {}
    s = total.sum().item()
    if s > 0:
        fr = total / s
        for i in range(total.numel()):
            out[f"expert_load/expert_{i}"] = float(total[i].item())
            out[f"expert_frac/expert_{i}"] = float(fr[i].item())
        out["expert_load/max_frac"] = float(fr.max().item())
        out["expert_load/min_frac"] = float(fr.min().item())
        out["expert_load/imbalance_ratio"] = float(fr.max().item() / max(fr.min().item(), 1e-9))
    return out
