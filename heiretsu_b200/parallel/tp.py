"""Megatron-style 1-D tensor-parallel linear layers.

Same parameter names, shard shapes and initialisation as the reference
(tp_linear.py:87-312), so that checkpoints and seeds carry over:

* ColumnParallelLinear    weight [out/tp, in], bias [out/tp]
* ColumnParallelLinearQKV weight [3*out/tp, in] = [Q_shard; K_shard; V_shard]
* RowParallelLinear       weight [out, in/tp], bias [out] (replicated, added after the reduction)

Initialisation draws the *full* matrix on the CPU and keeps this rank's slice,
so with the same seed on every TP rank the TP model equals the dense model.

These modules are the plain-PyTorch path (CPU, fp32 parity). On CUDA the model
blocks call the fused kernels in :mod:`heiretsu_b200.ops` with these modules'
parameters instead (see heiretsu_b200/models/fused.py).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn


def _ws(group: Optional[dist.ProcessGroup]) -> int:
    if group is None or not dist.is_initialized():
        return 1
    return dist.get_world_size(group=group)


def _rk(group: Optional[dist.ProcessGroup]) -> int:
    if group is None or not dist.is_initialized():
        return 0
    return dist.get_rank(group=group)


class _CopyToTP(torch.autograd.Function):
    """Identity forward; all-reduce of the input gradient in backward (reference tp_linear.py:19-34)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        if ctx.group is not None and dist.is_initialized() and _ws(ctx.group) > 1:
            g = g.contiguous()
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    """All-reduce forward; identity backward (reference tp_linear.py:37-51)."""

    @staticmethod
    def forward(ctx, x, group):
        if group is not None and dist.is_initialized() and _ws(group) > 1:
            x = x.contiguous()
            dist.all_reduce(x, op=dist.ReduceOp.SUM, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_model_parallel_region(x: torch.Tensor, tp_group) -> torch.Tensor:
    return _CopyToTP.apply(x, tp_group)


def reduce_from_model_parallel_region(x: torch.Tensor, tp_group) -> torch.Tensor:
    return _ReduceFromTP.apply(x, tp_group)


def _split_last_dim(x: torch.Tensor, tp: int) -> torch.Tensor:
    """(..., tp*d) -> (tp, ..., d)."""
    shp = x.shape[:-1] + (tp, x.shape[-1] // tp)
    return x.reshape(shp).movedim(-2, 0)


class _TPLinearBase(nn.Module):
    def _setup(self, tp_group, tp_rank, tp_world_size):
        self.tp_group = tp_group
        self.tp_world_size = tp_world_size if tp_world_size is not None else _ws(tp_group)
        self.tp_rank = tp_rank if tp_rank is not None else _rk(tp_group)


class ColumnParallelLinear(_TPLinearBase):
    """Output features sharded: W_full [out, in] -> W_shard [out/tp, in]."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, tp_group=None,
                 tp_rank: Optional[int] = None, tp_world_size: Optional[int] = None):
        super().__init__()
        self._setup(tp_group, tp_rank, tp_world_size)
        if out_features % self.tp_world_size:
            raise ValueError(f"out_features = {out_features} does not split evenly over "
                             f"{self.tp_world_size} tensor-parallel ranks")
        self.in_features, self.out_features = in_features, out_features
        self.out_per_partition = out_features // self.tp_world_size
        self.weight = nn.Parameter(torch.empty(self.out_per_partition, in_features))
        self.bias = nn.Parameter(torch.empty(self.out_per_partition)) if bias else None

    def reset_parameters(self, std: float = 0.02) -> None:
        full = torch.empty(self.out_features, self.in_features, device="cpu")
        nn.init.normal_(full, mean=0.0, std=std)
        s = self.tp_rank * self.out_per_partition
        with torch.no_grad():
            self.weight.copy_(full[s:s + self.out_per_partition].to(self.weight.device))
            if self.bias is not None:
                self.bias.zero_()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = copy_to_model_parallel_region(x, self.tp_group)
        y = torch.matmul(x, self.weight.t())
        if self.bias is not None:
            y = y + self.bias
        return y


class ColumnParallelLinearQKV(_TPLinearBase):
    """Fused QKV projection with Q, K and V each sharded by heads."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, tp_group=None,
                 tp_rank: Optional[int] = None, tp_world_size: Optional[int] = None):
        super().__init__()
        self._setup(tp_group, tp_rank, tp_world_size)
        if out_features % self.tp_world_size:
            raise ValueError(f"out_features = {out_features} does not split evenly over "
                             f"{self.tp_world_size} tensor-parallel ranks")
        self.in_features, self.out_features = in_features, out_features
        self.out_per_partition = out_features // self.tp_world_size
        self.weight = nn.Parameter(torch.empty(3 * self.out_per_partition, in_features))
        self.bias = nn.Parameter(torch.empty(3 * self.out_per_partition)) if bias else None

    def shard_rows(self) -> torch.Tensor:
        """Row indices of this rank's shard inside the full [3*out, in] matrix."""
        o, per = self.out_features, self.out_per_partition
        return torch.cat([torch.arange(i * o + self.tp_rank * per, i * o + (self.tp_rank + 1) * per)
                          for i in range(3)])

    def reset_parameters(self, std: float = 0.02) -> None:
        full = torch.empty(3 * self.out_features, self.in_features, device="cpu")
        nn.init.normal_(full, mean=0.0, std=std)
        with torch.no_grad():
            self.weight.copy_(full[self.shard_rows()].to(self.weight.device))
            if self.bias is not None:
                self.bias.zero_()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = copy_to_model_parallel_region(x, self.tp_group)
        y = torch.matmul(x, self.weight.t())
        if self.bias is not None:
            y = y + self.bias
        return y


class RowParallelLinear(_TPLinearBase):
    """Input features sharded: W_full [out, in] -> W_shard [out, in/tp]; output all-reduced."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, tp_group=None,
                 tp_rank: Optional[int] = None, tp_world_size: Optional[int] = None):
        super().__init__()
        self._setup(tp_group, tp_rank, tp_world_size)
        if in_features % self.tp_world_size:
            raise ValueError(f"in_features = {in_features} does not split evenly over "
                             f"{self.tp_world_size} tensor-parallel ranks")
        self.in_features, self.out_features = in_features, out_features
        self.in_per_partition = in_features // self.tp_world_size
        self.weight = nn.Parameter(torch.empty(out_features, self.in_per_partition))
        self.bias = nn.Parameter(torch.empty(out_features)) if bias else None

    def reset_parameters(self, std: float = 0.02) -> None:
        full = torch.empty(self.out_features, self.in_features, device="cpu")
        nn.init.normal_(full, mean=0.0, std=std)
        s = self.tp_rank * self.in_per_partition
        with torch.no_grad():
            self.weight.copy_(full[:, s:s + self.in_per_partition].to(self.weight.device))
            if self.bias is not None:
                self.bias.zero_()

    def forward(self, x: torch.Tensor, input_is_parallel: Optional[bool] = None) -> torch.Tensor:
        if input_is_parallel is None:
            input_is_parallel = x.size(-1) == self.in_per_partition
        if not input_is_parallel:
            x = _split_last_dim(x, self.tp_world_size)[self.tp_rank]
        y = torch.matmul(x, self.weight.t())
        y = reduce_from_model_parallel_region(y, self.tp_group)
        if self.bias is not None:
            y = y + self.bias
        return y
