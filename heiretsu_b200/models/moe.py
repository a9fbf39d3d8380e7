"""Mixture-of-experts layer: top-k softmax router, load-balancing loss,
per-rank expert group and expert-parallel dispatch/combine.

Parameter names and initialisation follow the reference (moe.py:34-405) so
that checkpoints load unchanged:
``router.gate.weight`` [E, H]; ``expert_group.experts.{j}.w1.weight`` [I, H],
``.w2.weight`` [H, I] with j the *local* expert index (global = ep_rank*E/ep + j).

This module is the plain-PyTorch path. On CUDA the MoE block calls the fused
router / permutation / grouped-GEMM kernels (heiretsu_b200/models/fused.py).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..config import MoEConfig, make_moe_config  # noqa: F401  (re-export)
from ..parallel.ep import all_to_all_combine, all_to_all_dispatch


class Router(nn.Module):
    """x [N, H] -> (top_indices [N, K], top_weights [N, K] renormalised, gate_probs [N, E])."""

    def __init__(self, hidden_size: int, num_experts: int, top_k: int):
        super().__init__()
        self.num_experts, self.top_k = num_experts, top_k
        self.gate = nn.Linear(hidden_size, num_experts, bias=False)

    def forward(self, x: torch.Tensor):
        probs = F.softmax(self.gate(x), dim=-1)
        w, idx = torch.topk(probs, self.top_k, dim=-1)
        w = w / w.sum(dim=-1, keepdim=True)
        return idx, w, probs


class Expert(nn.Module):
    """GELU(tanh) MLP without biases: H -> I -> H."""

    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.w1 = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.w2 = nn.Linear(intermediate_size, hidden_size, bias=False)
        self.act = nn.GELU(approximate="tanh")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w2(self.act(self.w1(x)))


class ExpertGroup(nn.Module):
    """The E/ep experts that live on this EP rank."""

    def __init__(self, num_local_experts: int, hidden_size: int, intermediate_size: int, ep_rank: int = 0,
                 num_experts: int = 8):
        super().__init__()
        self.num_local_experts = num_local_experts
        self.ep_rank = ep_rank
        self.num_experts = num_experts
        self.expert_start_idx = ep_rank * num_local_experts
        self.experts = nn.ModuleList([Expert(hidden_size, intermediate_size) for _ in range(num_local_experts)])

    def forward(self, x_sorted: torch.Tensor, expert_counts: torch.Tensor,
                local_expert_indices: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Rows of `x_sorted` are grouped by local expert with `expert_counts` rows each."""
        if x_sorted.size(0) == 0:
            return x_sorted
        counts = expert_counts.tolist()
        outs = []
        start = 0
        for e, c in enumerate(counts):
            if c > 0:
                outs.append(self.experts[e](x_sorted[start:start + c]))
            start += c
        return torch.cat(outs, 0) if outs else x_sorted[:0]


def load_balancing_loss(gate_probs: torch.Tensor, top_indices: torch.Tensor, num_experts: int, top_k: int,
                        aux_loss_coef: float = 0.01) -> torch.Tensor:
    """alpha * E * sum_e f_e * p_e with f_e the fraction of the N*K selections
    routed to e and p_e the mean router probability of e (reference moe.py:197-242)."""
    N = gate_probs.size(0)
    counts = torch.zeros(num_experts, dtype=gate_probs.dtype, device=gate_probs.device)
    counts.scatter_add_(0, top_indices.reshape(-1), torch.ones_like(top_indices.reshape(-1), dtype=gate_probs.dtype))
    f = counts / (N * top_k)
    p = gate_probs.mean(dim=0)
    return aux_loss_coef * num_experts * (f * p).sum()


class MoELayer(nn.Module):
    """Route -> (dispatch) -> experts -> (combine) -> weighted sum over the K choices."""

    def __init__(self, config: MoEConfig, ep_group=None, ep_rank: int = 0, ep_world_size: int = 1):
        super().__init__()
        if config.num_experts % ep_world_size:
            raise ValueError(f"num_experts {config.num_experts} must be divisible by ep {ep_world_size}")
        self.config = config
        self.num_experts = config.num_experts
        self.top_k = config.top_k
        self.hidden_size = config.hidden_size
        self.aux_loss_coef = config.aux_loss_coef
        self.ep_group, self.ep_rank, self.ep_world_size = ep_group, ep_rank, ep_world_size
        self.num_local_experts = config.num_experts // ep_world_size
        self.router = Router(config.hidden_size, config.num_experts, config.top_k)
        self.expert_group = ExpertGroup(self.num_local_experts, config.hidden_size, config.intermediate_size,
                                        ep_rank=ep_rank, num_experts=config.num_experts)
        self._expert_counts: Optional[torch.Tensor] = None
        if ep_world_size > 1:
            # The EP ranks of one data replica hold identical tokens, so every
            # expert receives each token once per EP rank and its gradient sums
            # ep identical contributions: average them (the dense gradient).
            for p in self.expert_group.parameters():
                p.register_hook(lambda g, s=1.0 / ep_world_size: g * s)
                p.ep_grad_scale = 1.0 / ep_world_size

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        B, S, H = x.shape
        K = self.top_k
        xf = x.reshape(B * S, H)
        idx, w, probs = self.router(xf)
        aux = load_balancing_loss(probs, idx, self.num_experts, K, self.aux_loss_coef)
        with torch.no_grad():
            self._expert_counts = torch.bincount(idx.reshape(-1), minlength=self.num_experts).float()

        flat_idx = idx.reshape(-1)  # [N*K], token-major
        order = torch.argsort(flat_idx, stable=True)  # grouped by global expert
        x_sorted = xf.repeat_interleave(K, dim=0)[order]
        e_sorted = flat_idx[order]

        if self.ep_world_size > 1:
            # Expert-sorted order is also destination-rank-sorted (experts are
            # laid out contiguously per rank), so no second permutation is needed.
            send_counts = torch.bincount(e_sorted // self.num_local_experts, minlength=self.ep_world_size)
            x_recv, recv_counts, e_recv = all_to_all_dispatch(x_sorted, send_counts, self.ep_group,
                                                              self.ep_world_size, payload=e_sorted)
            local = e_recv - self.ep_rank * self.num_local_experts
            lorder = torch.argsort(local, stable=True)
            counts = torch.bincount(local, minlength=self.num_local_experts)
            y_l = self.expert_group(x_recv[lorder], counts)
            y_recv = torch.empty_like(y_l).index_copy(0, lorder, y_l) if y_l.numel() else y_l
            y_sorted = all_to_all_combine(y_recv, send_counts, recv_counts, self.ep_group, self.ep_world_size)
        else:
            counts = torch.bincount(e_sorted, minlength=self.num_local_experts)
            y_sorted = self.expert_group(x_sorted, counts)

        y_exp = torch.empty_like(y_sorted).index_copy(0, order, y_sorted)  # back to token-major order
        y = (y_exp.view(B * S, K, H) * w.unsqueeze(-1)).sum(dim=1)
        return y.view(B, S, H), aux
