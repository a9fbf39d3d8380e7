"""4-D process topology: world = dp * ep * tp * pp.

Rank layout (kept identical to the reference so that checkpoints, launch
scripts and rank-to-GPU mapping carry over; reference topo.py:1-5, :36-45):

    global_rank = dp_rank*(EP*PP*TP) + ep_rank*(PP*TP) + pp_rank*TP + tp_rank

TP is innermost, so a TP group is a set of consecutive ranks, which on one
8-GPU NVSwitch node are consecutive GPUs. Every rank calls ``new_group`` for
every group (torch requires it) in one fixed order: TP, EP, PP, DP.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from datetime import timedelta
from typing import List, Optional, Tuple

import os

import torch.distributed as dist


@dataclass
class Topology:
    dp: int
    ep: int
    tp: int
    pp: int
    rank: int
    world_size: int
    dp_rank: int
    ep_rank: int
    pp_rank: int
    tp_rank: int
    tp_group: Optional[dist.ProcessGroup]
    pp_group: Optional[dist.ProcessGroup]
    ep_group: Optional[dist.ProcessGroup]
    dp_group: Optional[dist.ProcessGroup]
    # Global ranks of every member of this rank's groups, in group-rank order.
    tp_ranks: List[int] = field(default_factory=list)
    pp_ranks: List[int] = field(default_factory=list)
    ep_ranks: List[int] = field(default_factory=list)
    dp_ranks: List[int] = field(default_factory=list)
    # Processes per node (torchrun's LOCAL_WORLD_SIZE; torchrun numbers ranks node
    # by node); 0 = every rank on one node.
    local_world: int = 0

    def node_of(self, rank: int) -> int:
        return rank // (self.local_world or self.world_size or 1)

    def on_one_node(self, ranks) -> bool:
        """Whether these global ranks share one node, i.e. one NVLink/NVSwitch domain in
        which CUDA IPC peer mappings work (the fused collectives need that)."""
        return len({self.node_of(r) for r in ranks}) <= 1

    def model_parallel_ranks(self) -> List[int]:
        """Global ranks of this rank's model-parallel replica (same dp_rank)."""
        per = self.ep * self.pp * self.tp
        return list(range(self.dp_rank * per, (self.dp_rank + 1) * per))

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1 and dist.is_initialized()

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp - 1

    @property
    def is_main(self) -> bool:
        """The logging rank: (dp, ep, tp) = 0 on the last pipeline stage (reference train.py:357)."""
        return self.dp_rank == 0 and self.ep_rank == 0 and self.tp_rank == 0 and self.is_last_stage


def coords_from_rank(rank: int, dp: int, ep: int, tp: int, pp: int) -> Tuple[int, int, int, int]:
    """global rank -> (dp_rank, ep_rank, pp_rank, tp_rank)."""
    tp_rank = rank % tp
    pp_rank = (rank // tp) % pp
    ep_rank = (rank // (tp * pp)) % ep
    dp_rank = rank // (tp * pp * ep)
    return dp_rank, ep_rank, pp_rank, tp_rank


def rank_from_coords(dp_rank: int, ep_rank: int, pp_rank: int, tp_rank: int, dp: int, ep: int, tp: int,
                     pp: int) -> int:
    """(dp_rank, ep_rank, pp_rank, tp_rank) -> global rank."""
    return ((dp_rank * ep + ep_rank) * pp + pp_rank) * tp + tp_rank


def group_members(dp: int, ep: int, tp: int, pp: int, rank: int) -> dict:
    """Global ranks of the TP/EP/PP/DP groups that contain `rank` (no torch.distributed needed)."""
    d, e, p, t = coords_from_rank(rank, dp, ep, tp, pp)
    rc = lambda dd, ee, pp_, tt: rank_from_coords(dd, ee, pp_, tt, dp, ep, tp, pp)
    return {
        "tp": [rc(d, e, p, x) for x in range(tp)],
        "ep": [rc(d, x, p, t) for x in range(ep)],
        "pp": [rc(d, e, x, t) for x in range(pp)],
        "dp": [rc(x, e, p, t) for x in range(dp)],
    }


def _all_groups(dp: int, ep: int, tp: int, pp: int):
    """Every group of every kind, in the creation order all ranks must follow."""
    rc = lambda d, e, p, t: rank_from_coords(d, e, p, t, dp, ep, tp, pp)
    tp_g = [[rc(d, e, p, t) for t in range(tp)] for d in range(dp) for e in range(ep) for p in range(pp)]
    ep_g = [[rc(d, e, p, t) for e in range(ep)] for d in range(dp) for p in range(pp) for t in range(tp)]
    pp_g = [[rc(d, e, p, t) for p in range(pp)] for d in range(dp) for e in range(ep) for t in range(tp)]
    dp_g = [[rc(d, e, p, t) for d in range(dp)] for e in range(ep) for p in range(pp) for t in range(tp)]
    return tp_g, ep_g, pp_g, dp_g


def build_groups(dp: int, ep: int, tp: int, pp: int, timeout: Optional[timedelta] = None):
    """Create all TP/EP/PP/DP groups; return this rank's (tp, pp, ep, dp) groups."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return None, None, None, None
    world = dist.get_world_size()
    if world != dp * ep * tp * pp:
        raise ValueError(f"{world} processes cannot form a dp{dp} x ep{ep} x tp{tp} x pp{pp} layout "
                         f"({dp * ep * tp * pp} ranks)")
    rank = dist.get_rank()
    mine = {}
    kw = {} if timeout is None else {"timeout": timeout}
    for kind, groups in zip(("tp", "ep", "pp", "dp"), _all_groups(dp, ep, tp, pp)):
        for ranks in groups:
            g = dist.new_group(ranks=ranks, **kw)
            if rank in ranks:
                mine[kind] = g
    return mine["tp"], mine["pp"], mine["ep"], mine["dp"]


def init_topology(dp: int, ep: int = 1, tp: int = 1, pp: int = 1, timeout: Optional[timedelta] = None) -> Topology:
    """Build the topology of the current process.

    With a single process the requested degrees collapse to 1 (dry run);
    with several processes the product must equal the world size.
    """
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    if world != dp * ep * tp * pp:
        if world == 1:
            dp = ep = tp = pp = 1
        else:
            raise ValueError(f"layout dp{dp} x ep{ep} x tp{tp} x pp{pp} needs {dp * ep * tp * pp} processes, "
                             f"the job has {world}")
    dp_rank, ep_rank, pp_rank, tp_rank = coords_from_rank(rank, dp, ep, tp, pp)
    tp_group, pp_group, ep_group, dp_group = build_groups(dp, ep, tp, pp, timeout)
    mem = group_members(dp, ep, tp, pp, rank)
    return Topology(dp=dp, ep=ep, tp=tp, pp=pp, rank=rank, world_size=world, dp_rank=dp_rank, ep_rank=ep_rank,
                    pp_rank=pp_rank, tp_rank=tp_rank, tp_group=tp_group, pp_group=pp_group, ep_group=ep_group,
                    dp_group=dp_group, tp_ranks=mem["tp"], pp_ranks=mem["pp"], ep_ranks=mem["ep"],
                    dp_ranks=mem["dp"], local_world=local_world_size(world))


def local_world_size(world: int) -> int:
    """Ranks per node from torchrun's LOCAL_WORLD_SIZE (default: all ``world`` ranks on one node)."""
    n = int(os.environ.get("LOCAL_WORLD_SIZE", world) or world)
    if n <= 0 or world % n:
        raise ValueError(f"LOCAL_WORLD_SIZE {n} does not divide the world size {world}")
    return n


def cleanup() -> None:
    """Barrier, then destroy the default process group."""
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
