"""Checkpoints in the reference's format (train.py:513-524), plus resume.

Model files are byte-compatible with the reference:
``{"model": state_dict, "cfg": asdict(GPTConfig), "step": int}`` and, when
sharded, a ``"topo"`` dict; names ``ckpt_{step:07d}.pt`` (tp=pp=ep=1) or
``ckpt_{step:07d}_pp{p}_ep{e}_tp{t}.pt``. Optimizer state goes to a separate
``optim_{...}.pt`` sidecar so the model files stay unchanged.
"""
from __future__ import annotations

import os
from dataclasses import asdict
from typing import Optional

import torch


def ckpt_name(step: int, topo) -> str:
    if topo.tp == 1 and topo.pp == 1 and topo.ep == 1:
        return f"ckpt_{step:07d}.pt"
    return f"ckpt_{step:07d}_pp{topo.pp_rank}_ep{topo.ep_rank}_tp{topo.tp_rank}.pt"


def save_checkpoint(module: torch.nn.Module, cfg, step: int, topo, out_dir: str = ".",
                    optimizer_state: Optional[dict] = None) -> Optional[str]:
    """Written by dp_rank 0 only (one file per (pp, ep, tp) shard)."""
    if topo.dp_rank != 0:
        return None
    sharded = not (topo.tp == 1 and topo.pp == 1 and topo.ep == 1)
    if not sharded and not topo.is_main:
        return None
    sd = {k: v.detach().cpu() for k, v in module.state_dict().items()}
    obj = {"model": sd, "cfg": asdict(cfg), "step": step}
    if sharded:
        obj["topo"] = {"dp": topo.dp, "ep": topo.ep, "tp": topo.tp, "pp": topo.pp, "pp_rank": topo.pp_rank,
                       "tp_rank": topo.tp_rank, "ep_rank": topo.ep_rank}
    path = os.path.join(out_dir, ckpt_name(step, topo))
    torch.save(obj, path)
    if optimizer_state is not None:
        torch.save(optimizer_state, sidecar_path(path))
    return path


def sidecar_path(ckpt_path: str) -> str:
    """``.../ckpt_X.pt`` -> ``.../optim_X.pt`` (optimizer / RNG / data-position state)."""
    d, b = os.path.split(ckpt_path)
    return os.path.join(d, "optim_" + (b[len("ckpt_"):] if b.startswith("ckpt_") else b))


def rng_state() -> dict:
    import random

    import numpy as np
    st = {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state()}
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        st["cuda"] = torch.cuda.get_rng_state()
    return st


def set_rng_state(st: dict) -> None:
    import random

    import numpy as np
    random.setstate(st["python"])
    np.random.set_state(st["numpy"])
    torch.set_rng_state(st["torch"])
    if "cuda" in st and torch.cuda.is_available():
        torch.cuda.set_rng_state(st["cuda"])


def load_checkpoint(module: torch.nn.Module, path: str, strict: bool = True) -> dict:
    obj = torch.load(path, map_location="cpu", weights_only=False)
    sd = obj["model"]
    # torch.compile-wrapped reference models prefix keys with `_orig_mod.`.
    sd = {k[len("_orig_mod."):] if k.startswith("_orig_mod.") else k: v for k, v in sd.items()}
    with torch.no_grad():
        module.load_state_dict(sd, strict=strict)
    return obj


# ---------------------------------------------------------------------------
# Topology changes: full (dense) state dict <-> per-rank shards
# ---------------------------------------------------------------------------
def _qkv_rows(out: int, tp_rank: int, tp: int) -> torch.Tensor:
    per = out // tp
    return torch.cat([torch.arange(i * out + tp_rank * per, i * out + (tp_rank + 1) * per) for i in range(3)])


def _full_key(local_key: str, module) -> str:
    """Map a key of a GPT / StageModule shard to the dense GPT's key."""
    from ..parallel.pipeline import StageModule

    orig = local_key  # submodule lookups use the shard's own names
    if isinstance(module, StageModule):
        if local_key.startswith("blocks."):
            rest = local_key[len("blocks."):]
            i, tail = rest.split(".", 1)
            local_key = f"tr.h.{module.block_start + int(i)}.{tail}"
        elif local_key.startswith(("wte.", "wpe.", "ln_f.")):
            local_key = "tr." + local_key
    if ".moe.expert_group.experts." in local_key:
        pre, rest = local_key.split(".moe.expert_group.experts.", 1)
        j, tail = rest.split(".", 1)
        group = module.get_submodule(f"{orig.split('.moe.')[0]}.moe.expert_group")
        local_key = f"{pre}.moe.expert_group.experts.{group.ep_rank * group.num_local_experts + int(j)}.{tail}"
    return local_key


def shard_from_full(module, full_state: dict, tp_rank: int = 0, tp: int = 1) -> dict:
    """Per-rank state dict for `module` (GPT or StageModule, any TP / EP / PP
    position) sliced from a dense GPT state dict. Slicing rules follow the
    checkpoint format: c_attn rows [Q_shard; K_shard; V_shard], column-parallel
    rows, row-parallel columns, local experts = global ep_rank*E/ep + j."""
    from ..parallel.tp import ColumnParallelLinear, ColumnParallelLinearQKV, RowParallelLinear

    kinds = {}
    for name, m in module.named_modules():
        if isinstance(m, ColumnParallelLinearQKV):
            kinds[name] = "qkv"
        elif isinstance(m, ColumnParallelLinear):
            kinds[name] = "col"
        elif isinstance(m, RowParallelLinear):
            kinds[name] = "row"
    out = {}
    for key, t in module.state_dict().items():
        full = full_state[_full_key(key, module)]
        owner, pname = key.rsplit(".", 1)
        kind = kinds.get(owner)
        if kind == "qkv":
            full = full[_qkv_rows(full.shape[0] // 3, tp_rank, tp)]
        elif kind == "col":
            per = full.shape[0] // tp
            full = full[tp_rank * per:(tp_rank + 1) * per]
        elif kind == "row" and pname == "weight":
            per = full.shape[1] // tp
            full = full[:, tp_rank * per:(tp_rank + 1) * per]
        out[key] = full.clone()
    return out


def load_from_full(module, full_state: dict, tp_rank: int = 0, tp: int = 1) -> None:
    """Load a dense GPT state dict into a shard (TP / EP / PP slicing applied)."""
    sd = shard_from_full(module, full_state, tp_rank, tp)
    with torch.no_grad():
        module.load_state_dict(sd, strict=True)
