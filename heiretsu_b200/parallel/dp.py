"""Data parallelism: gradient averaging over the DP group.

``average_gradients`` is the reference's API (dp.py:13-26): per-parameter
all-reduce(SUM) followed by ``/ dp``. The engine path does not use it: there
the gradients live in one flat fp32 buffer (``FlatParams``) and are reduced by
``FlatGradReducer`` in large buckets with the 1/dp scale fused into the
reduction (heiretsu_b200/csrc/comm.cu), or by NCCL when the fused kernel is
not usable (CPU / gloo, or peers without NVLink access).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def average_gradients(model: torch.nn.Module, dp_group: Optional[dist.ProcessGroup]) -> None:
    """All-reduce every ``p.grad`` over the DP group and divide by its size."""
    if dp_group is None or not dist.is_initialized() or dist.get_world_size(group=dp_group) == 1:
        return
    world = dist.get_world_size(group=dp_group)
    for p in model.parameters():
        if p.grad is None:
            continue
        dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=dp_group)
        p.grad.div_(world)
