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
        torch.save(optimizer_state, os.path.join(out_dir, "optim_" + ckpt_name(step, topo)[len("ckpt_"):]))
    return path


def load_checkpoint(module: torch.nn.Module, path: str, strict: bool = True) -> dict:
    obj = torch.load(path, map_location="cpu", weights_only=False)
    sd = obj["model"]
    # torch.compile-wrapped reference models prefix keys with `_orig_mod.`.
    sd = {k[len("_orig_mod."):] if k.startswith("_orig_mod.") else k: v for k, v in sd.items()}
    with torch.no_grad():
        module.load_state_dict(sd, strict=strict)
    return obj
