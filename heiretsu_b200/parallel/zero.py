"""ZeRO stage 1 for the plain engine: AdamW moments sharded over the DP group.

The reference keeps a full ``torch.optim.AdamW`` on every DP rank
(train.py:346-351) and lists optimizer-state sharding as future work
(README.md:128). ``ZeroAdamW`` lays the rank's parameters end to end in
``named_parameters()`` order and cuts that flat index space into ``dp`` equal
contiguous shards (a cut may fall inside a parameter). DP rank r keeps the
fp32 ``exp_avg`` / ``exp_avg_sq`` of shard r only, updates only the
parameter elements of shard r, and an all-gather over the DP group then gives
every rank every updated element. The moments take 8/dp bytes per parameter
instead of 8.

Preconditions and numerics:
* gradients are already averaged over DP (``average_gradients``), so every
  DP rank holds the same gradients and each shard's update is the one a full
  AdamW would make;
* the update is decoupled AdamW with bias correction, element for element the
  formula of ``torch.optim.AdamW`` (Loshchilov & Hutter, 2019): p *= 1 - lr*wd;
  m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*g^2;
  p -= lr/(1-b1^t) * m / (sqrt(v)/sqrt(1-b2^t) + eps);
* a parameter without a gradient is left unchanged (as torch's AdamW does);
* checkpoints stay layout-free: ``moments_by_name`` all-gathers the shards
  into whole tensors keyed by parameter name (every DP rank must call it), and
  ``load_moments_by_name`` takes this rank's shard back out of them.
"""
from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch
import torch.distributed as dist


class ZeroAdamW(torch.optim.Optimizer):
    def __init__(self, named_params, dp_group, lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1):
        named = [(n, p) for n, p in named_params if p.requires_grad]
        super().__init__([p for _, p in named], dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay))
        self.names = [n for n, _ in named]
        self.plist = [p for _, p in named]
        self.group = dp_group
        self.dp = dist.get_world_size(dp_group) if dp_group is not None else 1
        self.rank = dist.get_rank(dp_group) if dp_group is not None else 0
        self.numel = sum(p.numel() for p in self.plist)
        self.shard = max(1, math.ceil(self.numel / self.dp))
        # segments[r]: (param index, start in the param, start in shard r, length)
        self.segments: List[List[Tuple[int, int, int, int]]] = [[] for _ in range(self.dp)]
        off = 0
        for i, p in enumerate(self.plist):
            n = p.numel()
            a = off
            while a < off + n:
                r = a // self.shard
                end = min(off + n, (r + 1) * self.shard)
                self.segments[r].append((i, a - off, a - r * self.shard, end - a))
                a = end
            off += n
        dev = self.plist[0].device if self.plist else torch.device("cpu")
        self.exp_avg = torch.zeros(self.shard, device=dev, dtype=torch.float32)
        self.exp_avg_sq = torch.zeros(self.shard, device=dev, dtype=torch.float32)
        self.steps = 0

    def shard_range(self, rank: int = None) -> Tuple[int, int]:
        r = self.rank if rank is None else rank
        return r * self.shard, min(self.numel, (r + 1) * self.shard)

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            raise ValueError("ZeroAdamW.step takes no closure")
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        self.steps += 1
        bc1 = 1.0 - b1 ** self.steps
        bc2_sqrt = math.sqrt(1.0 - b2 ** self.steps)
        for i, a, s, n in self.segments[self.rank]:
            p = self.plist[i]
            if p.grad is None:
                continue
            pv = p.data.view(-1)[a:a + n]
            gv = p.grad.detach().reshape(-1)[a:a + n].float()
            m, v = self.exp_avg[s:s + n], self.exp_avg_sq[s:s + n]
            pv.mul_(1.0 - lr * wd)
            m.lerp_(gv, 1.0 - b1)
            v.mul_(b2).addcmul_(gv, gv, value=1.0 - b2)
            denom = (v.sqrt() / bc2_sqrt).add_(eps)
            pv.addcdiv_(m.to(pv.dtype), denom.to(pv.dtype), value=-lr / bc1)
        self._gather_params()

    # -- collectives ------------------------------------------------------------
    def _pack(self, r: int, fn) -> torch.Tensor:
        buf = torch.zeros(self.shard, device=self.exp_avg.device, dtype=torch.float32)
        for i, a, s, n in self.segments[r]:
            buf[s:s + n] = fn(i)[a:a + n]
        return buf

    def _all_gather(self, buf: torch.Tensor) -> List[torch.Tensor]:
        if self.dp == 1:
            return [buf]
        if buf.is_cuda:
            out = torch.empty(self.dp * self.shard, device=buf.device, dtype=buf.dtype)
            dist.all_gather_into_tensor(out, buf, group=self.group)
            return list(out.split(self.shard))
        parts = [torch.empty_like(buf) for _ in range(self.dp)]
        dist.all_gather(parts, buf, group=self.group)
        return parts

    def _gather_params(self) -> None:
        if self.dp == 1:
            return
        mine = self._pack(self.rank, lambda i: self.plist[i].data.view(-1).float())
        parts = self._all_gather(mine)
        for r, part in enumerate(parts):
            if r == self.rank:
                continue
            for i, a, s, n in self.segments[r]:
                pv = self.plist[i].data.view(-1)
                pv[a:a + n] = part[s:s + n].to(pv.dtype)

    def _full(self, shard_buf: torch.Tensor) -> List[torch.Tensor]:
        parts = self._all_gather(shard_buf)
        flat = torch.cat(parts)[:self.numel]
        out, off = [], 0
        for p in self.plist:
            out.append(flat[off:off + p.numel()].view_as(p).clone())
            off += p.numel()
        return out

    # -- checkpoints --------------------------------------------------------------
    def moments_by_name(self) -> dict:
        """Whole AdamW moments keyed by parameter name (a collective over the DP group)."""
        m = self._full(self.exp_avg)
        v = self._full(self.exp_avg_sq)
        return {"format": "by_name", "step": self.steps,
                "m": {n: t.cpu() for n, t in zip(self.names, m)},
                "v": {n: t.cpu() for n, t in zip(self.names, v)}}

    def load_moments_by_name(self, st: dict) -> None:
        self.steps = int(st["step"])
        m, v = st["m"], st["v"]
        for i, a, s, n in self.segments[self.rank]:
            name = self.names[i]
            if name in m:
                self.exp_avg[s:s + n] = m[name].reshape(-1)[a:a + n].to(self.exp_avg)
                self.exp_avg_sq[s:s + n] = v[name].reshape(-1)[a:a + n].to(self.exp_avg_sq)

    def state_bytes(self) -> int:
        return (self.exp_avg.numel() + self.exp_avg_sq.numel()) * 4

    def state_dict(self) -> Dict:  # torch.optim API: the layout-free form
        return self.moments_by_name()

    def load_state_dict(self, st: Dict) -> None:
        self.load_moments_by_name(st)
