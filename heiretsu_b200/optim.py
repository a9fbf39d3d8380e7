"""Fused AdamW with global-norm gradient clipping over a ``FlatParams`` buffer.

Semantics follow torch.optim.AdamW (decoupled weight decay applied to every
parameter, as the reference does: train.py:346-351) and
torch.nn.utils.clip_grad_norm_ (train.py:446), except that the norm is the
*global* norm over all model-parallel shards (each replicated parameter
counted once) rather than each shard's local norm.

One step = sum-of-squares reductions (one per replication class) ->
optional all-reduce of the squared norm over the model-parallel group ->
clip coefficient -> one AdamW kernel that also refreshes the 16-bit GEMM
shadow (bf16, or fp16 with a device loss scale: ``DeviceLossScaler``). Within one node the model-parallel sum runs over NVLink in a
kernel, so the whole step stays inside one captured CUDA graph. No host
synchronisation: the per-step hyper-parameters are uploaded asynchronously
from pinned memory, the coefficient stays on the device, and a non-finite norm
(fp16 overflow) skips the update inside the kernel.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from .ops import kernels as K
from .parallel.flat import FlatParams


class DeviceLossScaler:
    """Dynamic loss scaling for fp16 with torch.cuda.amp.GradScaler's rule and
    defaults (reference train.py:356, :436-452), kept on the device so a captured
    step needs no host synchronisation: ``state`` = [scale, finite steps in a row].

    ``scale(loss)`` multiplies by the device scale before backward; the optimizer
    unscales inside its clip coefficient (``K.clip_coef(..., loss_scale)``), skips
    a step whose gradient norm is not finite (the coefficient is NaN), and then
    calls ``update_after(coef)``: backoff x0.5 after a skipped step, growth x2
    after ``growth_interval`` finite steps in a row."""

    def __init__(self, device, init_scale: float = 2.0 ** 16, growth_factor: float = 2.0,
                 backoff_factor: float = 0.5, growth_interval: int = 2000):
        self.state = torch.tensor([init_scale, 0.0], device=device, dtype=torch.float32)
        self.growth_factor, self.backoff_factor, self.growth_interval = growth_factor, backoff_factor, growth_interval

    @property
    def scale_tensor(self) -> torch.Tensor:
        """The scale as a 1-element device tensor (a view: replays read the current value)."""
        return self.state[0:1]

    def scale(self, t: torch.Tensor) -> torch.Tensor:
        return t * self.state[0]

    def is_enabled(self) -> bool:
        return True

    def get_scale(self) -> float:
        return float(self.state[0].item())

    def update_after(self, coef: torch.Tensor) -> None:
        K.loss_scale_update(coef, self.state, self.growth_factor, self.backoff_factor, self.growth_interval)

    # GradScaler's checkpoint keys, so either kind of run resumes the other's scale.
    def state_dict(self) -> dict:
        st = self.state.cpu()
        return {"scale": float(st[0]), "growth_factor": self.growth_factor, "backoff_factor": self.backoff_factor,
                "growth_interval": self.growth_interval, "_growth_tracker": int(st[1])}

    def load_state_dict(self, sd: dict) -> None:
        self.state.copy_(torch.tensor([float(sd["scale"]), float(sd.get("_growth_tracker", 0))]))


class FusedAdamW:
    def __init__(self, flat: FlatParams, lr: float = 3e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1, max_grad_norm: float = 0.0, mp_group: Optional[dist.ProcessGroup] = None,
                 mp_symm=None, scaler: Optional[DeviceLossScaler] = None):
        """``mp_symm``: optional peer-mapped buffer (>= 16 bytes) over ``mp_group``;
        with it the squared norm is summed over NVLink by a kernel (graph-capturable)
        instead of an NCCL all-reduce. ``scaler``: the fp16 loss scale the gradients
        carry (unscaled in the clip coefficient, updated after each step)."""
        self.flat = flat
        self.scaler = scaler
        self.lr, self.betas, self.eps, self.wd = lr, tuple(betas), eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.mp_group = mp_group
        self.mp_symm = mp_symm
        dev = flat.device
        self._norm_slot = mp_symm.tensor(torch.float32, 4) if mp_symm is not None else None
        self.m = torch.zeros_like(flat.data)
        self.v = torch.zeros_like(flat.data)
        self.step_count = 0
        self.hyper = torch.zeros(8, device=dev, dtype=torch.float32)
        self.norm2 = torch.zeros((), device=dev, dtype=torch.float32)
        self.norm = torch.zeros((), device=dev, dtype=torch.float32)
        self.coef = torch.ones((), device=dev, dtype=torch.float32)
        self.grad_scale = 1.0
        self.param_groups = [{"lr": lr}]  # logging compatibility with torch optimizers
        # Pinned staging slots of the hyper-parameter upload; a slot is rewritten only
        # after the event behind its previous copy completed.
        self._stage = [torch.empty(8, dtype=torch.float32, pin_memory=dev.type == "cuda") for _ in range(2)]
        self._stage_ev = [None, None]

    def compute_grad_norm(self) -> torch.Tensor:
        """Global L2 norm of the gradients (device tensor), each replicated parameter counted once."""
        g = self.flat.grad
        first = True
        for start, end, wgt in self.flat.ranges:
            if end > start:
                K.sumsq(g[start:end], self.norm2, weight=wgt, accumulate=not first)
                first = False
        if first:
            self.norm2.zero_()
        if self._norm_slot is not None:
            self._norm_slot.zero_()
            self._norm_slot[0].copy_(self.norm2)
            self.mp_symm.sum_range(0, 4, 1.0)
            self.norm2.copy_(self._norm_slot[0])
        elif self.mp_group is not None and dist.is_initialized() and dist.get_world_size(self.mp_group) > 1:
            dist.all_reduce(self.norm2, group=self.mp_group)
        K.clip_coef(self.norm2, self.max_grad_norm, self.coef, self.norm,
                    self.scaler.scale_tensor if self.scaler is not None else None)
        return self.norm

    def prepare_step(self) -> None:
        """Host part of a step: advance the step count and upload the hyper-parameters.

        Kept separate from ``step_device`` so the device part can live in a
        captured CUDA graph while learning rate and bias corrections change."""
        self.step_count += 1
        lr = self.param_groups[0]["lr"]
        b1, b2 = self.betas
        vals = [lr, b1, b2, self.eps, self.wd, 1.0 - b1 ** self.step_count, math.sqrt(1.0 - b2 ** self.step_count),
                self.grad_scale]
        # Asynchronous upload from a pinned slot: a blocking copy from pageable memory would
        # synchronise the stream, and the GPU would idle while the host launches the next step.
        i = self.step_count % 2
        if self._stage_ev[i] is not None:
            self._stage_ev[i].synchronize()
        slot = self._stage[i]
        for j, v in enumerate(vals):
            slot[j] = v
        cuda = self.hyper.is_cuda
        self.hyper.copy_(slot, non_blocking=cuda)
        if cuda:
            ev = torch.cuda.Event()
            ev.record()
            self._stage_ev[i] = ev

    def step_device(self) -> None:
        """Device part of a step (no host synchronisation; graph-capturable)."""
        self.compute_grad_norm()
        K.adamw_step(self.flat.data, self.flat.grad, self.m, self.v, self.flat.data16, self.hyper, self.coef)
        if self.scaler is not None:
            self.scaler.update_after(self.coef)

    def step(self) -> None:
        self.prepare_step()
        self.step_device()

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.flat.zero_grad()

    def moments_by_name(self) -> dict:
        """AdamW state keyed by parameter name (host copies): ``{"format": "by_name",
        "step", "m": {name: tensor}, "v": {name: tensor}}``. Shaped like the parameters,
        so checkpoint tools can merge and re-slice it like the weights."""
        f = self.flat
        m, v = {}, {}
        for name, off, p in zip(f.names, f.offsets, f.params):
            n = p.numel()
            m[name] = self.m[off:off + n].view(p.shape).detach().cpu()
            v[name] = self.v[off:off + n].view(p.shape).detach().cpu()
        return {"format": "by_name", "step": self.step_count, "m": m, "v": v}

    def load_moments_by_name(self, st: dict) -> None:
        f = self.flat
        with torch.no_grad():
            for name, off, p in zip(f.names, f.offsets, f.params):
                n = p.numel()
                if name in st["m"]:
                    self.m[off:off + n].copy_(st["m"][name].reshape(-1))
                    self.v[off:off + n].copy_(st["v"][name].reshape(-1))
        self.step_count = int(st["step"])

    def state_dict(self) -> dict:
        return {"m": self.m.cpu(), "v": self.v.cpu(), "step": self.step_count, "lr": self.param_groups[0]["lr"],
                "betas": self.betas, "eps": self.eps, "weight_decay": self.wd, "names": list(self.flat.names)}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))
        self.step_count = int(sd["step"])
