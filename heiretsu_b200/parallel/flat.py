"""Flat parameter / gradient / 16-bit-shadow buffers.

All parameters of a module are moved into one fp32 buffer (each parameter
becomes a view, so ``state_dict`` and the module code are unchanged), with
a matching fp32 gradient buffer (``p.main_grad``) and a 16-bit shadow
(``p.w16``, bf16 or fp16) that the GEMMs read. One flat layout means one AdamW kernel, one
gradient-norm reduction and large, contiguous DP reduction buckets.

Parameters are grouped by how they are replicated across model-parallel
ranks, so the global gradient norm is a handful of range reductions:
``class_of(p)`` returns the factor by which a parameter's squared norm is
counted too often when summed over the TP x EP ranks of one replica.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Tuple

import torch

ALIGN = 128  # elements: keeps every view 256-byte aligned in bf16 and 512 in fp32


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _stack_experts(named: List[Tuple[str, torch.nn.Parameter]]) -> List[Tuple[str, torch.nn.Parameter]]:
    """Order parameters so that each MoE layer's expert weights are contiguous:
    all w1 (expert order), then all w2, at the position of the layer's first expert."""
    out: List[Tuple[str, torch.nn.Parameter]] = []
    placed = set()
    for name, p in named:
        if name in placed:
            continue
        if ".experts." in name:
            layer = name.split(".experts.")[0]
            members = [(n, q) for n, q in named if n.startswith(layer + ".experts.")]
            key = lambda nq: (nq[0].rsplit(".", 2)[-2], int(nq[0].split(".experts.")[1].split(".")[0]))
            for n, q in sorted(members, key=key):
                out.append((n, q))
                placed.add(n)
            continue
        out.append((name, p))
        placed.add(name)
    return out


class FlatParams:
    def __init__(self, module: torch.nn.Module, device: torch.device,
                 weight_of: Optional[Callable[[str, torch.nn.Parameter], float]] = None, grad_group=None,
                 tp_group=None, tp_sum_of: Optional[Callable[[str, torch.nn.Parameter], bool]] = None,
                 dtype16: torch.dtype = torch.bfloat16):
        """``dtype16``: format of the weight shadows and so of every activation of the
        fused path (bf16, or fp16 for --amp fp16).
        ``tp_sum_of(name, p)``: whether p's gradient is a per-token-shard partial
        that must be summed over the TP group (TP-replicated parameters under
        sequence-sharded TP). Parameters are grouped by (norm weight, tp_sum),
        and ``tp_sum[i]`` tells it for ``ranges[i]``."""
        named: List[Tuple[str, torch.nn.Parameter]] = []
        seen = set()
        for name, p in module.named_parameters():
            if id(p) in seen:
                continue
            seen.add(id(p))
            named.append((name, p))
        weight_of = weight_of or (lambda n, p: 1.0)
        tp_sum_of = tp_sum_of or (lambda n, p: False)
        # Group by (norm weight, TP-sum flag); stable within a group: module order.
        groups: Dict[Tuple[float, bool], List[Tuple[str, torch.nn.Parameter]]] = {}
        for name, p in named:
            groups.setdefault((float(weight_of(name, p)), bool(tp_sum_of(name, p))), []).append((name, p))
        self.ranges: List[Tuple[int, int, float]] = []  # (start, end, weight)
        self.tp_sum: List[bool] = []
        order: List[Tuple[str, torch.nn.Parameter]] = []
        total = 0
        for key in sorted(groups):
            start = total
            for name, p in _stack_experts(groups[key]):
                order.append((name, p))
                total += _align(p.numel())
            self.ranges.append((start, total, key[0]))
            self.tp_sum.append(key[1])
        self.numel = total
        self.device = device
        self.data = torch.zeros(total, device=device, dtype=torch.float32)
        # With a DP group on CUDA, the gradients live in a symmetric (peer-mapped)
        # buffer so the fused all-reduce can read and write them over NVLink.
        # The same allocation is peer-mapped in the DP group (gradient
        # averaging) and in the TP group (summing TP-replicated gradients).
        self.grad_symm = None
        self.grad_symm_tp = None
        if (grad_group is not None or tp_group is not None) and device.type == "cuda":
            from ..ops._C import load as _load
            from .symm import SymmetricBuffer
            raw = _load().raw_malloc(total * 4)
            if grad_group is not None:
                self.grad_symm = SymmetricBuffer(grad_group, total * 4, device, local_ptr=raw)
            if tp_group is not None:
                self.grad_symm_tp = SymmetricBuffer(tp_group, total * 4, device, local_ptr=raw)
            self.grad = _load().tensor_from_ptr(raw, total, torch.float32, device.index)
        else:
            self.grad = torch.zeros(total, device=device, dtype=torch.float32)
        self.data16 = torch.zeros(total, device=device, dtype=dtype16)
        self.params: List[torch.nn.Parameter] = []
        self.names: List[str] = []
        self.offsets: List[int] = []
        off = 0
        with torch.no_grad():
            for name, p in order:
                n = p.numel()
                view = self.data[off:off + n].view(p.shape)
                view.copy_(p.data.to(device))
                p.data = view
                p.main_grad = self.grad[off:off + n].view(p.shape)
                p.w16 = self.data16[off:off + n].view(p.shape)
                p.flat_owner = self
                self.params.append(p)
                self.names.append(name)
                self.offsets.append(off)
                off += _align(n)
        self.refresh_bf16()

    def stacked(self, params: List[torch.nn.Parameter]):
        """(bf16 weights, fp32 gradients) of same-shaped parameters stored back to back,
        viewed as one [len * rows, cols] matrix (the experts of one MoE layer)."""
        first = params[0]
        idx = [next(i for i, q in enumerate(self.params) if q is p) for p in params]
        n = first.numel()
        for a, b in zip(idx, idx[1:]):
            if self.offsets[b] != self.offsets[a] + n:
                raise RuntimeError("stacked parameters are not contiguous in the flat buffer")
        off = self.offsets[idx[0]]
        rows, cols = first.shape[0] * len(params), first.shape[1]
        return (self.data16[off:off + n * len(params)].view(rows, cols),
                self.grad[off:off + n * len(params)].view(rows, cols))

    def refresh_bf16(self) -> None:
        """Re-derive the 16-bit shadow from the fp32 master (after init / checkpoint load)."""
        if self.device.type == "cuda":
            from ..ops.kernels import f32_to_bf16
            f32_to_bf16(self.data, self.data16)
        else:
            self.data16.copy_(self.data)

    def zero_grad(self) -> None:
        self.grad.zero_()
