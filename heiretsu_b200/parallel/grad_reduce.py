"""Data-parallel reduction of the flat gradient buffer.

The flat fp32 gradient buffer (``FlatParams.grad``) is averaged over the DP
group in a few large contiguous buckets. Backends:

* ``nccl``: ``all_reduce(AVG)`` per bucket (the library baseline; also the
  gloo/CPU path, where AVG is emulated with SUM and a scale);
* ``p2p``: the fused sm_100a kernel of heiretsu_b200/csrc/comm.cu, which reads
  the peers' buckets over NVLink, sums them with the 1/dp scale applied in the
  same pass and writes the result back to every peer (no staging copies).

Overlap with backward (p2p): ``arm()`` before the last micro-batch's
backward installs a per-block hook in the fused backward. When a block's
backward has been issued, its parameters' gradient ranges are final, so an
event is recorded and a side stream reduces those ranges while the main
stream continues with the next block. The side-stream kernel runs at 2 warps
per CTA, small enough to sit beside the persistent GEMM / attention CTAs.
``finish()`` reduces whatever was not covered (embeddings, final norm) and
joins the side stream. Every rank issues the same reductions in the same
order, which the kernels' epoch-tagged barriers require. All of it is
capturable in a CUDA graph (the side stream forks from and joins the
capture stream through events).
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from ..ops._C import load as load_ext
from .flat import FlatParams

BUCKET_ELEMS = 32 * 1024 * 1024  # 128 MB fp32 per bucket


def uncovered_ranges(done: List[Tuple[int, int]], n: int) -> List[Tuple[int, int]]:
    """The parts of [0, n) not covered by the (possibly overlapping) ranges in ``done``."""
    rest, pos = [], 0
    for a, b in sorted(done):
        if a > pos:
            rest.append((pos, a))
        pos = max(pos, b)
    if pos < n:
        rest.append((pos, n))
    return rest


# CTAs of each overlapped per-block reduction (0: one per SM; HB_DP_OVERLAP_BLOCKS
# overrides). Measured at 2 GPUs on GPT-2 small: one per SM 24 ms/step, 32 CTAs 27.5,
# 8 CTAs 60.6, against 21.6 for the one-shot reduction after backward.
OVERLAP_BLOCKS = int(os.environ.get("HB_DP_OVERLAP_BLOCKS", "0"))


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
        self._side = None
        self._armed = False
        self._done: List[Tuple[int, int]] = []
        self._range_cache = {}

    # -- overlap with backward ----------------------------------------------
    def can_overlap(self) -> bool:
        return self.world > 1 and self.backend == "p2p" and self.flat.device.type == "cuda"

    def _ranges_of(self, module) -> List[Tuple[int, int]]:
        """Contiguous flat-buffer ranges [start, end) holding module's parameter gradients."""
        key = id(module)
        if key not in self._range_cache:
            index = {id(p): i for i, p in enumerate(self.flat.params)}
            spans = []
            for p in module.parameters():
                i = index.get(id(p))
                if i is not None:
                    off = self.flat.offsets[i]
                    spans.append((off, off + (p.numel() + 127) // 128 * 128))
            spans.sort()
            merged: List[Tuple[int, int]] = []
            for a, b in spans:
                if merged and merged[-1][1] == a:
                    merged[-1] = (merged[-1][0], b)
                else:
                    merged.append((a, b))
            self._range_cache[key] = merged
        return self._range_cache[key]

    def arm(self) -> None:
        """Reduce each block's gradients during the coming backward pass."""
        if not self.can_overlap():
            return
        from ..models import fused as F
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.flat.device)
        self._done = []
        self._armed = True
        F.set_block_done_hook(self._on_block_done)

    def _on_block_done(self, blk) -> None:
        ranges = self._ranges_of(blk)
        if not ranges:
            return
        ev = torch.cuda.Event()
        ev.record()
        self._side.wait_event(ev)
        with torch.cuda.stream(self._side):
            for a, b in ranges:
                # 2-warp CTAs beside the backward kernels (OVERLAP_BLOCKS caps their number)
                self.symm.sum_range(a, b - a, 1.0 / self.world, threads=64, blocks=OVERLAP_BLOCKS)
        self._done.extend(ranges)

    def finish(self) -> None:
        """After backward: reduce what the overlap did not cover and join the side stream."""
        if not self._armed:
            self.reduce()
            return
        from ..models import fused as F
        F.set_block_done_hook(None)
        self._armed = False
        rest = uncovered_ranges(self._done, self.flat.numel)
        ev = torch.cuda.Event()
        ev.record()
        self._side.wait_event(ev)
        with torch.cuda.stream(self._side):
            for a, b in rest:
                self.symm.sum_range(a, b - a, 1.0 / self.world)
        torch.cuda.current_stream().wait_stream(self._side)

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
