"""Data-parallel reduction of the flat gradient buffer.

The flat fp32 gradient buffer (``FlatParams.grad``) is averaged over the DP
group in a few large contiguous buckets. Backends:

* ``nccl``: ``all_reduce(AVG)`` per bucket (the library baseline; also the
  gloo/CPU path, where AVG is emulated with SUM and a scale);
* ``p2p``: the fused sm_100a kernel of heiretsu_b200/csrc/comm.cu, which reads
  the peers' buckets over NVLink, sums them with the 1/dp scale applied in the
  same pass and writes the result back to every peer (no staging copies).
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from ..ops._C import load as load_ext
from .flat import FlatParams

BUCKET_ELEMS = 32 * 1024 * 1024  # 128 MB fp32 per bucket


class FlatGradReducer:
    def __init__(self, flat: FlatParams, group: Optional[dist.ProcessGroup], topo=None,
                 backend: Optional[str] = None, bucket_elems: int = BUCKET_ELEMS):
        self.flat = flat
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None and dist.is_initialized()) else 1
        self.buckets: List[Tuple[int, int]] = []
        n = flat.numel
        for s in range(0, n, bucket_elems):
            self.buckets.append((s, min(n, s + bucket_elems)))
        self.backend = backend or os.environ.get("HB_DP_BACKEND", "p2p")
        self._avg_ok = dist.is_initialized() and dist.get_backend(group) == "nccl"

        self.symm = getattr(flat, "grad_symm", None)
        if self.backend == "p2p" and self.symm is None:
            self.backend = "nccl"

    def reduce(self) -> None:
        if self.world == 1:
            return
        if self.backend == "p2p":
            # One fused kernel: reduce-scatter + 1/dp + all-gather over NVLink.
            load_ext().dp_allreduce(self.symm.ptrs, self.symm.signal_ptrs, self.symm.rank, self.flat.numel,
                                    1.0 / self.world, self.symm.counter)
            return
        g = self.flat.grad
        for s, e in self.buckets:
            chunk = g[s:e]
            if self._avg_ok:
                dist.all_reduce(chunk, op=dist.ReduceOp.AVG, group=self.group)
            else:
                dist.all_reduce(chunk, op=dist.ReduceOp.SUM, group=self.group)
                chunk.div_(self.world)
