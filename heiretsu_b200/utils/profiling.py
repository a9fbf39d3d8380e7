"""Device-side timing and NVTX annotation.

The reference times a step with the host clock only (train.py:455-459):
no device synchronisation, per rank. Here:

* ``RegionTimer`` brackets named regions with CUDA events on the current
  stream, accumulates their device time, and reports the maximum over ranks
  (one all-reduce of the per-region totals, done only when a summary is
  asked for, never inside a step).
* ``nvtx(name)`` marks a range for external profilers. It is enabled by
  ``HB_NVTX=1`` and costs one environment lookup at import otherwise. The
  fused engine wraps every sub-layer's forward and backward in one.
"""
from __future__ import annotations

import contextlib
import os
from collections import OrderedDict
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

NVTX_ENABLED = os.environ.get("HB_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx(name: str):
    if NVTX_ENABLED and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class RegionTimer:
    """Accumulated device time per named region (CUDA events; host clock on CPU)."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._pending: List[Tuple[str, object, object]] = []
        self.totals: "OrderedDict[str, float]" = OrderedDict()
        self.counts: Dict[str, int] = {}

    @contextlib.contextmanager
    def region(self, name: str):
        if not self.enabled:
            yield
            return
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            try:
                yield
            finally:
                end.record()
                self._pending.append((name, start, end))
        else:
            import time
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self._add(name, (time.perf_counter() - t0) * 1e3)

    def _add(self, name: str, ms: float) -> None:
        self.totals[name] = self.totals.get(name, 0.0) + ms
        self.counts[name] = self.counts.get(name, 0) + 1

    def collect(self) -> None:
        """Fold finished event pairs into the totals (synchronises on the last event only)."""
        if not self._pending:
            return
        self._pending[-1][2].synchronize()
        for name, s, e in self._pending:
            self._add(name, s.elapsed_time(e))
        self._pending.clear()

    def summary(self, group=None, reset: bool = True) -> Dict[str, float]:
        """Per-region total ms, maximum over the ranks of ``group`` when distributed.

        Every rank of the group must call this with the same region names."""
        self.collect()
        names = list(self.totals)
        vals = torch.tensor([self.totals[n] for n in names], dtype=torch.float64)
        if dist.is_initialized() and names:
            dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
                else torch.device("cpu")
            v = vals.to(dev)
            dist.all_reduce(v, op=dist.ReduceOp.MAX, group=group)
            vals = v.cpu()
        out = {n: float(v) for n, v in zip(names, vals)}
        if reset:
            self.totals.clear()
            self.counts.clear()
        return out


    def per_rank(self, group=None, reset: bool = True) -> Dict[str, List[float]]:
        """Per-region total ms of every rank of ``group`` (one all-gather), in group-rank
        order: the spread shows a straggler that the max alone hides.

        Every rank of the group must call this with the same region names."""
        self.collect()
        names = list(self.totals)
        vals = torch.tensor([self.totals[n] for n in names], dtype=torch.float64)
        rows = [vals]
        if dist.is_initialized() and names:
            dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
                else torch.device("cpu")
            v = vals.to(dev)
            parts = [torch.empty_like(v) for _ in range(dist.get_world_size(group))]
            dist.all_gather(parts, v, group=group)
            rows = [x.cpu() for x in parts]
        out = {n: [float(r[i]) for r in rows] for i, n in enumerate(names)}
        if reset:
            self.totals.clear()
            self.counts.clear()
        return out


def rank_spread(per_rank_ms: List[float]) -> Dict[str, float]:
    """min / median / max of per-rank times, the slowest rank and max/min (imbalance)."""
    srt = sorted(per_rank_ms)
    lo, hi = srt[0], srt[-1]
    return {"min": lo, "median": srt[len(srt) // 2], "max": hi, "slowest": float(per_rank_ms.index(hi)),
            "imbalance": hi / lo if lo > 0 else float("inf")}


def tokens_per_second(tokens_per_step_all_ranks: int, step_ms: Optional[float]) -> Optional[float]:
    return None if not step_ms else tokens_per_step_all_ranks / (step_ms / 1e3)
