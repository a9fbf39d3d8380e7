"""Expert-parallel token exchange (all-to-all dispatch / combine).

Unlike the reference (ep_comm.py:13-135), both directions are autograd
functions: the backward of dispatch is a combine of the gradients and vice
versa, so with ep > 1 the expert weights and the tokens receive gradients
(the reference cuts autograd there: its outputs are fresh buffers filled by a
non-differentiable all_to_all_single).

This is the host-orchestrated path (torch.distributed all_to_all_single with
variable splits). The fused GPU path writes tokens straight into the owner
rank's expert-grouped buffer over NVLink (heiretsu_b200/csrc/moe.cu).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def _a2a(x: torch.Tensor, send: List[int], recv: List[int], group) -> torch.Tensor:
    out = torch.empty((sum(recv),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_to_all_single(out, x.contiguous(), output_split_sizes=recv, input_split_sizes=send, group=group)
    return out


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send, recv, group):
        ctx.send, ctx.recv, ctx.group = send, recv, group
        return _a2a(x, send, recv, group)

    @staticmethod
    def backward(ctx, g):
        return _a2a(g, ctx.recv, ctx.send, ctx.group), None, None, None


def exchange_counts(send_counts: torch.Tensor, group) -> torch.Tensor:
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts.contiguous(), group=group)
    return recv


def all_to_all_dispatch(x: torch.Tensor, send_counts: torch.Tensor, ep_group, ep_world_size: int,
                        payload: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """Send rows of `x` (grouped by destination rank) to the EP ranks owning their experts.

    Returns (x_recv, recv_counts, payload_recv). Differentiable in `x`.
    """
    if ep_group is None or ep_world_size == 1:
        return x, send_counts, payload
    recv_counts = exchange_counts(send_counts, ep_group)
    send = send_counts.tolist()
    recv = recv_counts.tolist()
    x_recv = _AllToAll.apply(x, send, recv, ep_group)
    payload_recv = _a2a(payload, send, recv, ep_group) if payload is not None else None
    return x_recv, recv_counts, payload_recv


def all_to_all_combine(y: torch.Tensor, send_counts: torch.Tensor, recv_counts: torch.Tensor, ep_group,
                       ep_world_size: int) -> torch.Tensor:
    """Return expert outputs to the ranks the tokens came from (reverse of dispatch). Differentiable."""
    if ep_group is None or ep_world_size == 1:
        return y
    return _AllToAll.apply(y, recv_counts.tolist(), send_counts.tolist(), ep_group)


def compute_ep_send_counts(expert_indices: torch.Tensor, num_experts: int, ep_world_size: int,
                           ep_rank: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Tokens per destination EP rank and each token's destination (reference ep_comm.py:138-171)."""
    per = num_experts // ep_world_size
    ep_idx = expert_indices // per
    counts = torch.bincount(ep_idx, minlength=ep_world_size)
    return counts, ep_idx
