"""Checkpoints in the reference's format (train.py:513-524), plus resume.

Model files are byte-compatible with the reference:
``{"model": state_dict, "cfg": asdict(GPTConfig), "step": int}`` and, when
sharded, a ``"topo"`` dict; names ``ckpt_{step:07d}.pt`` (tp=pp=ep=1) or
``ckpt_{step:07d}_pp{p}_ep{e}_tp{t}.pt``. Optimizer state goes to a separate
``optim_{...}.pt`` sidecar so the model files stay unchanged, and each rank's
RNG states and data position to ``rstate_{step:07d}_r{rank}.pt``.

Resume (``load_for_resume``) takes any file of a step. With the same TP / PP /
EP layout every rank loads its own shard; with another layout all shards of
the step are merged into the dense GPT state dict (``merge_shards``) and
re-sliced for the new layout (weights only: the optimizer restarts).
"""
from __future__ import annotations

import json
import os
import re
from dataclasses import asdict
from typing import Dict, List, Optional, Tuple

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


def _strip_compile_prefix(sd: dict) -> dict:
    # torch.compile-wrapped reference models prefix keys with `_orig_mod.`.
    return {k[len("_orig_mod."):] if k.startswith("_orig_mod.") else k: v for k, v in sd.items()}


def load_checkpoint(module: torch.nn.Module, path: str, strict: bool = True) -> dict:
    obj = torch.load(path, map_location="cpu", weights_only=False)
    with torch.no_grad():
        module.load_state_dict(_strip_compile_prefix(obj["model"]), strict=strict)
    return obj


# ---------------------------------------------------------------------------
# Files of one checkpoint step; per-rank state
# ---------------------------------------------------------------------------
_CKPT_RE = re.compile(r"^ckpt_(\d{7})(?:_pp(\d+)_ep(\d+)_tp(\d+))?\.pt$")


def step_files(path: str) -> List[str]:
    """Every file of the checkpoint step that ``path`` belongs to: the dense file, or all
    ``ckpt_{step}_pp*_ep*_tp*.pt`` shards beside it."""
    d, b = os.path.split(path)
    m = _CKPT_RE.match(b)
    if m is None or m.group(2) is None:
        return [path]
    out = []
    for f in sorted(os.listdir(d or ".")):
        mm = _CKPT_RE.match(f)
        if mm is not None and mm.group(1) == m.group(1) and mm.group(2) is not None:
            out.append(os.path.join(d, f))
    return out


def own_shard_path(path: str, topo) -> str:
    """The file of ``path``'s step holding this rank's (pp, ep, tp) shard."""
    d, b = os.path.split(path)
    m = _CKPT_RE.match(b)
    if m is None:
        return path
    return os.path.join(d, ckpt_name(int(m.group(1)), topo))


def ckpt_layout(obj: dict) -> Tuple[int, int, int]:
    """(tp, pp, ep) a checkpoint was written with ((1, 1, 1) for a dense file)."""
    t = obj.get("topo")
    return (1, 1, 1) if t is None else (int(t["tp"]), int(t["pp"]), int(t["ep"]))


def rank_state_path(out_dir: str, step: int, rank: int) -> str:
    return os.path.join(out_dir, f"rstate_{step:07d}_r{rank}.pt")


def done_marker_path(out_dir: str, step: int) -> str:
    return os.path.join(out_dir, f"ckpt_{step:07d}.done")


def mark_step_complete(out_dir: str, step: int, topo) -> str:
    """Written by rank 0 once every rank has finished writing step ``step`` (the caller
    holds a barrier first): a crash in the middle of a save leaves no marker, so
    ``latest_complete_checkpoint`` never picks a half-written step."""
    path = done_marker_path(out_dir, step)
    tmp = path + ".tmp"
    with open(tmp, "w") as f:
        json.dump({"step": step, "layout": [topo.dp, topo.ep, topo.tp, topo.pp],
                   "file": ckpt_name(step, topo)}, f)
    os.replace(tmp, path)
    return path


def latest_complete_checkpoint(out_dir: str, topo) -> Optional[str]:
    """A checkpoint file of the newest step in ``out_dir`` with a completion marker, or
    None. The file is this rank's own shard when the layout is unchanged, else any
    shard of the step (``load_for_resume`` takes any file of a step)."""
    if not os.path.isdir(out_dir):
        return None
    steps = []
    for name in os.listdir(out_dir):
        if name.startswith("ckpt_") and name.endswith(".done"):
            try:
                steps.append(int(name[len("ckpt_"):-len(".done")]))
            except ValueError:
                continue
    for step in sorted(steps, reverse=True):
        own = os.path.join(out_dir, ckpt_name(step, topo))
        if os.path.exists(own):
            return own
        with open(done_marker_path(out_dir, step)) as f:
            other = os.path.join(out_dir, json.load(f)["file"])
        if os.path.exists(other):
            return other
    return None


def save_rank_state(out_dir: str, step: int, topo, state: dict) -> str:
    """Per-rank resume state (RNG states, data position, ...), tagged with the layout."""
    path = rank_state_path(out_dir, step, topo.rank)
    torch.save({**state, "layout": [topo.dp, topo.ep, topo.tp, topo.pp]}, path)
    return path


def load_rank_state(ckpt_path: str, step: int, topo) -> Optional[dict]:
    """This rank's state file written beside ``ckpt_path`` by a run of the same layout, or None."""
    path = rank_state_path(os.path.dirname(ckpt_path), step, topo.rank)
    if not os.path.exists(path):
        return None
    st = torch.load(path, map_location="cpu", weights_only=False)
    if list(st.get("layout", [])) != [topo.dp, topo.ep, topo.tp, topo.pp]:
        return None
    return st


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
    if not isinstance(module, StageModule) and local_key == "lm_head.weight":
        return "tr.wte.weight"  # one tied table: a state from untied pipeline stages gives its embedding
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


# ---------------------------------------------------------------------------
# Shards -> dense state dict (topology changes, dense export)
# ---------------------------------------------------------------------------
def _tp_kind(full_key: str) -> Optional[str]:
    """How a dense GPT key is split over TP ranks (tp_linear.py:87-312 layouts)."""
    if ".attn.c_attn." in full_key:
        return "qkv"
    if ".mlp.c_fc." in full_key:
        return "col"
    if full_key.endswith((".attn.c_proj.weight", ".mlp.c_proj.weight")):
        return "row"
    return None  # replicated over TP (LayerNorms, embeddings, row biases, router, experts)


def merge_shards(objs: List[dict]) -> Dict[str, torch.Tensor]:
    """Dense GPT state dict from every shard file of one checkpoint step (as loaded by
    torch.load). Pipeline stages keep their own embedding tables: ``tr.wte.weight`` comes
    from the first stage and ``lm_head.weight`` from the last (equal unless the stages
    were trained untied)."""
    from ..parallel.pipeline import _partition_layers

    cfg = objs[0]["cfg"]
    n_layer, n_exp = int(cfg["n_layer"]), int(cfg.get("num_experts", 0) or 0)
    parts: Dict[str, Dict[int, torch.Tensor]] = {}
    tp_of: Dict[str, int] = {}
    for obj in objs:
        t = obj.get("topo") or dict(tp=1, pp=1, ep=1, tp_rank=0, pp_rank=0, ep_rank=0)
        tp, pp, ep = int(t["tp"]), int(t["pp"]), int(t["ep"])
        start = _partition_layers(n_layer, pp)[int(t["pp_rank"])][0]
        for key, v in _strip_compile_prefix(obj["model"]).items():
            fk = key
            if pp > 1:
                if fk.startswith("blocks."):
                    i, tail = fk[len("blocks."):].split(".", 1)
                    fk = f"tr.h.{start + int(i)}.{tail}"
                elif fk.startswith(("wte.", "wpe.", "ln_f.")):
                    fk = "tr." + fk
            if ".moe.expert_group.experts." in fk:
                pre, rest = fk.split(".moe.expert_group.experts.", 1)
                j, tail = rest.split(".", 1)
                fk = f"{pre}.moe.expert_group.experts.{int(t['ep_rank']) * (n_exp // ep) + int(j)}.{tail}"
            parts.setdefault(fk, {})[int(t["tp_rank"])] = v
            tp_of[fk] = tp
    full: Dict[str, torch.Tensor] = {}
    for fk, by_rank in parts.items():
        kind, tp = _tp_kind(fk), tp_of[fk]
        if kind is None or tp == 1:
            full[fk] = next(iter(by_rank.values())).clone()
            continue
        if sorted(by_rank) != list(range(tp)):
            raise ValueError(f"checkpoint shards incomplete for {fk}: tp ranks {sorted(by_rank)} of {tp}")
        shards = [by_rank[r] for r in range(tp)]
        if kind == "qkv":
            per = shards[0].shape[0] // 3
            full[fk] = torch.cat([s[i * per:(i + 1) * per] for i in range(3) for s in shards])
        elif kind == "col":
            full[fk] = torch.cat(shards, 0)
        else:
            full[fk] = torch.cat(shards, 1)
    if "lm_head.weight" not in full and "tr.wte.weight" in full:
        full["lm_head.weight"] = full["tr.wte.weight"]
    if "tr.wte.weight" not in full and "lm_head.weight" in full:
        full["tr.wte.weight"] = full["lm_head.weight"]
    return full


def load_for_resume(module, path: str, topo) -> dict:
    """Load the checkpoint step that ``path`` belongs to into this rank's module.

    Returns ``{"step", "same_layout", "file"}``; ``file`` is the shard this rank read
    (same layout) or ``path``."""
    head = torch.load(path, map_location="cpu", weights_only=False)
    layout = ckpt_layout(head)
    if layout == (topo.tp, topo.pp, topo.ep):
        own = own_shard_path(path, topo) if layout != (1, 1, 1) else path
        obj = head if os.path.abspath(own) == os.path.abspath(path) else \
            torch.load(own, map_location="cpu", weights_only=False)
        with torch.no_grad():
            module.load_state_dict(_strip_compile_prefix(obj["model"]), strict=True)
        return {"step": int(obj.get("step", 0)), "same_layout": True, "file": own}
    objs = [head if os.path.abspath(f) == os.path.abspath(path) else
            torch.load(f, map_location="cpu", weights_only=False) for f in step_files(path)]
    full = merge_shards(objs)
    load_from_full(module, full, topo.tp_rank, topo.tp)
    return {"step": int(head.get("step", 0)), "same_layout": False, "file": path, "full": full,
            "headers": [{"cfg": o["cfg"], "topo": o.get("topo")} for o in objs]}


def merged_optimizer_moments(path: str, headers: List[dict]) -> Optional[dict]:
    """Dense AdamW moments of the step ``path`` belongs to, merged from every shard's
    sidecar written in the by-name format (``{"step", "m", "v"}`` keyed like the dense
    GPT state dict), or None when a sidecar is missing or in another format."""
    files = step_files(path)
    sides = []
    for f in files:
        sp = sidecar_path(f)
        if not os.path.exists(sp):
            return None
        st = torch.load(sp, map_location="cpu", weights_only=False).get("optimizer", {})
        if st.get("format") != "by_name":
            return None
        sides.append(st)
    out = {"step": int(sides[0]["step"])}
    for key in ("m", "v"):
        out[key] = merge_shards([{"model": st[key], **h} for st, h in zip(sides, headers)])
    return out


def reslice_moments(module, full_weights: dict, moments: dict, tp_rank: int, tp: int) -> dict:
    """This rank's by-name optimizer state from dense moments (parameters without
    moments start at zero)."""
    out = {"format": "by_name", "step": moments["step"]}
    names = {n for n, _ in module.named_parameters()}
    for key in ("m", "v"):
        dense = {k: moments[key].get(k, torch.zeros_like(w)) for k, w in full_weights.items()}
        local = shard_from_full(module, dense, tp_rank, tp)
        out[key] = {k: v for k, v in local.items() if k in names}
    return out


def find_rank_state(ckpt_path: str, step: int, topo) -> Tuple[Optional[dict], bool]:
    """(state, exact): this rank's own state file of the same layout (exact), or else,
    when the checkpoint's run had the same DP degree, the file of its rank with this
    rank's dp_rank and all other coordinates 0 (same data stream), or (None, False)."""
    st = load_rank_state(ckpt_path, step, topo)
    if st is not None:
        return st, True
    from ..topo import rank_from_coords
    d = os.path.dirname(ckpt_path)
    probe = rank_state_path(d, step, 0)
    if not os.path.exists(probe):
        return None, False
    lay = torch.load(probe, map_location="cpu", weights_only=False).get("layout")
    if not lay or int(lay[0]) != topo.dp:
        return None, False
    dp, ep, tp, pp = (int(x) for x in lay)
    path = rank_state_path(d, step, rank_from_coords(topo.dp_rank, 0, 0, 0, dp, ep, tp, pp))
    if not os.path.exists(path):
        return None, False
    return torch.load(path, map_location="cpu", weights_only=False), False


def main(argv=None) -> None:
    """python -m heiretsu_b200.utils.ckpt merge OUT.pt CKPT  (any file of the step):
    writes the dense checkpoint ``{"model", "cfg", "step"}`` of a sharded step."""
    import argparse

    ap = argparse.ArgumentParser(description="checkpoint tools")
    sub = ap.add_subparsers(dest="cmd", required=True)
    mg = sub.add_parser("merge", help="merge the shards of one step into a dense checkpoint")
    mg.add_argument("out")
    mg.add_argument("ckpt")
    a = ap.parse_args(argv)
    objs = [torch.load(f, map_location="cpu", weights_only=False) for f in step_files(a.ckpt)]
    full = merge_shards(objs)
    torch.save({"model": full, "cfg": objs[0]["cfg"], "step": objs[0].get("step", 0)}, a.out)
    print(f"merged {len(objs)} file(s) -> {a.out} ({len(full)} tensors)")


if __name__ == "__main__":
    main()
