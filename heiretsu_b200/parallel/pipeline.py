"""Pipeline parallelism with NCCL point-to-point: GPipe (fill / drain) and 1F1B.

Same stage partition, parameter names and default schedule as the reference
(pipeline.py:19-340): contiguous balanced layer ranges; the first stage owns
``wte``/``wpe``, the last ``ln_f``/``lm_head`` (tied only when both live on
the same stage); all M forwards, then all M backwards in reverse.

``schedule="1f1b"`` (an addition; the reference lists it as future work,
README.md:131) runs the one-forward-one-backward schedule of PipeDream-Flush
(Narayanan et al., 2021): stage s runs min(pp - s - 1, M) warm-up forwards,
then alternates one forward and one backward, then drains the remaining
backwards. It computes the same gradients as GPipe (micro-batch gradients
are summed in another order) while stage s keeps at most pp - s micro-batches
of activations instead of M.

Differences, all deliberate:

* The activation boundary travels in one declared dtype on both sides
  (``boundary_dtype``, default fp32 = the residual stream's dtype), so an AMP
  run never sends fp32 bytes into a bf16 receive buffer.
* Communication overlaps compute: the receive for microbatch m+1 is posted
  before microbatch m is computed, sends are not waited for until the end of
  the phase, and waits are stream waits (``Work.wait``), not host blocks.
* Optional tied embeddings across stages (``TiedEmbeddings``, off by
  default): the first stage's ``wte`` and the last stage's ``lm_head`` start
  equal and their gradients are summed between the two stages every step, so
  the pipeline model is the tied dense GPT. The reference unties them
  (pipeline.py:75-92), which stays the default.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..config import GPTConfig
from ..topo import rank_from_coords


def embedding_group(topo):
    """(group, first-stage rank) of this rank's {first stage, last stage} pair with the
    same (dp, ep, tp) coordinates, or None on a middle stage. Every rank creates every
    pair's group, in the same order (torch.distributed.new_group requires it)."""
    mine = None
    for d in range(topo.dp):
        for e in range(topo.ep):
            for t in range(topo.tp):
                pair = [rank_from_coords(d, e, p, t, topo.dp, topo.ep, topo.tp, topo.pp) for p in (0, topo.pp - 1)]
                g = dist.new_group(ranks=pair)
                if topo.rank in pair:
                    mine = (g, pair[0])
    return mine


class TiedEmbeddings:
    """Keeps the first stage's ``wte.weight`` and the last stage's ``lm_head.weight``
    identical: ``sync_weights`` copies the first stage's table to the last stage (start,
    checkpoint load) and ``reduce_grads`` sums the two gradients in place on both (before
    clipping and the optimizer), so both copies take the same AdamW step."""

    def __init__(self, stage: "StageModule", topo):
        if topo.pp < 2:
            raise ValueError("tied pipeline embeddings need pp >= 2")
        got = embedding_group(topo)
        self.group, self.src = got if got is not None else (None, None)
        self.param = None
        if stage.is_first:
            self.param = stage.wte.weight
        elif stage.is_last:
            self.param = stage.lm_head.weight

    def sync_weights(self) -> None:
        if self.group is not None:
            with torch.no_grad():
                dist.broadcast(self.param.data, src=self.src, group=self.group)

    def reduce_grads(self) -> None:
        if self.group is None:
            return
        g = getattr(self.param, "main_grad", None)
        if g is None:
            g = self.param.grad
        if g is None:
            g = self.param.grad = torch.zeros_like(self.param)
        dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.group)


def _partition_layers(n_layer: int, pp: int) -> List[Tuple[int, int]]:
    """Balanced contiguous [start, end) layer ranges; earlier stages take the remainder."""
    if pp <= 0:
        raise ValueError(f"pipeline degree {pp}: at least one stage is needed")
    if pp > n_layer:
        raise ValueError(f"{pp} pipeline stages cannot split {n_layer} blocks: every stage needs a block")
    base, rem = divmod(n_layer, pp)
    out, start = [], 0
    for i in range(pp):
        end = start + base + (1 if i < rem else 0)
        out.append((start, end))
        start = end
    return out


class StageModule(nn.Module):
    """The blocks of one pipeline stage plus the embedding (first) and head (last)."""

    def __init__(self, cfg: GPTConfig, topo, stage_idx: int, num_stages: int):
        super().__init__()
        from ..models.gpt import init_gpt_weights, make_block

        self.cfg = cfg
        self.stage_idx, self.num_stages = stage_idx, num_stages
        self.is_first = stage_idx == 0
        self.is_last = stage_idx == num_stages - 1
        self.tp, self.tp_rank, self.tp_group = topo.tp, topo.tp_rank, topo.tp_group
        self.ep = getattr(topo, "ep", 1)
        self.ep_rank = getattr(topo, "ep_rank", 0)
        self.ep_group = getattr(topo, "ep_group", None)
        self.topo = topo
        self.block_start, self.block_end = _partition_layers(cfg.n_layer, num_stages)[stage_idx]
        self.blocks = nn.ModuleList([
            make_block(cfg, i, self.tp_group, self.tp_rank, self.tp, self.ep_group, self.ep_rank, self.ep)
            for i in range(self.block_start, self.block_end)])
        if self.is_first:
            self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embed)
            self.wpe = nn.Embedding(cfg.block_size, cfg.n_embed)
        else:
            self.wte = None
            self.wpe = None
        if self.is_last:
            self.ln_f = nn.LayerNorm(cfg.n_embed)
            self.lm_head = nn.Linear(cfg.n_embed, cfg.vocab_size, bias=False)
        else:
            self.ln_f = None
            self.lm_head = None
        if self.is_first and self.is_last:
            self.wte.weight = self.lm_head.weight
        init_gpt_weights(self, cfg.n_layer)
        self.fused = False
        self.recompute = False  # activation checkpointing of the plain path (models.gpt.run_blocks)
        self._head_pool: list = []  # logits buffers reused by head_cross_entropy
        self.topo = topo

    # Fused tensor parallelism keeps the residual stream token-sharded: each
    # TP rank holds B/tp whole sequences, and the stage boundary is that shard
    # (sent to the same TP rank of the next stage, 1/tp of the dense bytes).
    def _fused_on(self, t: torch.Tensor) -> bool:
        """Whether this stage runs the fused kernels on `t` (a CUDA tensor)."""
        return self.fused and t.is_cuda

    def _tp_fused(self, t: torch.Tensor) -> bool:
        return self._fused_on(t) and self.tp > 1

    def boundary_batch(self, B: int) -> int:
        """Sequences per boundary tensor on this rank for a micro-batch of B."""
        return B // self.tp if self.fused and self.tp > 1 else B

    def embed(self, idx: torch.Tensor) -> torch.Tensor:
        B, T = idx.shape
        if T > self.cfg.block_size:
            raise ValueError(f"input of {T} positions exceeds the model's block_size of {self.cfg.block_size}")
        if self._fused_on(idx):
            from ..models.fused import embed_fused
            if self._tp_fused(idx):
                from ..models.fused_tp import tp_shard_rows
                r0, Ms = tp_shard_rows(self.topo, B, T)
                idx = idx.reshape(-1)[r0:r0 + Ms].view(Ms // T, T)
            return embed_fused(self.wte.weight, self.wpe.weight, idx)
        return self.wte(idx) + self.wpe(torch.arange(T, device=idx.device))[None]

    def forward_blocks(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        if self._tp_fused(x):
            from ..models.fused_tp import blocks_fused_tp, tp_supported
            Bs, T, H = x.shape
            ok, why = tp_supported(self.cfg, self.topo, Bs * self.tp, T)
            if not ok:
                raise ValueError(f"fused tensor parallelism: {why}")
            xs = x.reshape(Bs * T, H)
            xs = xs if xs.dtype == torch.float32 else xs.float()
            out, aux = blocks_fused_tp(self.blocks, xs, self.cfg, self.topo, Bs * self.tp, T)
            return out.view(Bs, T, H), aux / self.tp  # shard aux losses / tp sum to the mean
        if self._fused_on(x):
            from ..models.fused import blocks_fused
            return blocks_fused(self.blocks, x, self.cfg, recompute=self.recompute)
        from ..models.gpt import run_blocks
        return run_blocks(self.blocks, x, self.recompute)

    def forward_head(self, x: torch.Tensor, targets: Optional[torch.Tensor], want_logits: bool = True):
        if self._fused_on(x):
            from ..models.fused import head_fused
            if self._tp_fused(x):
                # this shard's mean loss / tp: the sum over the TP group is the dense mean
                Bs, T, _ = x.shape
                from ..models.fused_tp import tp_shard_rows
                r0, Ms = tp_shard_rows(self.topo, Bs * self.tp, T)
                tgt = targets.reshape(-1)[r0:r0 + Ms].view(Bs, T) if targets is not None else None
                _, loss = head_fused(self.ln_f, self.lm_head.weight, x, tgt, self.cfg.vocab_size, want_logits=False,
                                     grad_hint=getattr(self, "loss_grad_hint", 1.0) / self.tp,
                                     grad_scale=getattr(self, "loss_grad_scale", None))
                return None, (loss / self.tp if loss is not None else None)
            return head_fused(self.ln_f, self.lm_head.weight, x, targets, self.cfg.vocab_size,
                              want_logits=want_logits, grad_hint=getattr(self, "loss_grad_hint", 1.0),
                              grad_scale=getattr(self, "loss_grad_scale", None))
        x = self.ln_f(x)
        if targets is not None and not want_logits and not torch.is_autocast_enabled(x.device.type):
            from ..models.gpt import head_cross_entropy
            return None, head_cross_entropy(x, self.lm_head.weight, targets, pool=self._head_pool)
        logits = self.lm_head(x)
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1))
        return logits, loss


def one_f_one_b_plan(stage: int, pp: int, M: int) -> List[tuple]:
    """The 1F1B (PipeDream-Flush) step list of one stage.

    With W = min(pp - stage - 1, M): W warm-up forwards, then M - W rounds of one
    forward (micro-batch W + i) and one backward (micro-batch i), then the last W
    backwards; forwards and backwards each in micro-batch order. Steps:
    ``("fwd", m)``, ``("bwd", m)``; receives that the next step waits for,
    ``("recv_act", m)`` from the previous stage and ``("recv_grad", m)`` from the next;
    sends, ``("send_act", m)`` to the next stage and ``("send_grad", m)`` to the previous;
    and two batched pairs, ``("send_act+recv_grad", f, b)`` with the next stage and
    ``("send_grad+recv_act", b, f)`` with the previous one. A pair is one NCCL group,
    posted when both neighbours reach the matching pair, so transfers in opposite
    directions between two stages never wait on each other (NCCL runs each rank's
    point-to-point groups in order; ``tests/test_parallel_cpu.py`` checks the plans of
    all stages against that rule).
    """
    first, last = stage == 0, stage == pp - 1
    warm = min(pp - stage - 1, M)
    steady = M - warm
    plan: List[tuple] = []
    for m in range(warm):
        if not first:
            plan.append(("recv_act", m))
        plan.append(("fwd", m))
        plan.append(("send_act", m))
    if steady > 0 and not first:
        plan.append(("recv_act", warm))
    for i in range(steady):
        f = warm + i
        plan.append(("fwd", f))
        if not last:
            plan.append(("send_act+recv_grad", f, i))
        plan.append(("bwd", i))
        if first:
            continue
        if i == steady - 1:
            plan.append(("send_grad", i))
        else:
            plan.append(("send_grad+recv_act", i, f + 1))
    for b in range(steady, M):
        if not last:
            plan.append(("recv_grad", b))
        plan.append(("bwd", b))
        if not first:
            plan.append(("send_grad", b))
    return plan


@dataclass
class PipelineState:
    boundaries: List[torch.Tensor] = field(default_factory=list)
    recv_inputs: List[torch.Tensor] = field(default_factory=list)
    losses: List[torch.Tensor] = field(default_factory=list)
    aux_losses: List[torch.Tensor] = field(default_factory=list)


class GPipeEngine:
    """Fill/drain schedule over the stages of one pipeline group."""

    def __init__(self, stage: StageModule, topo, boundary_dtype: torch.dtype = torch.float32,
                 schedule: str = "gpipe"):
        if schedule not in ("gpipe", "1f1b"):
            raise ValueError(f"unknown pipeline schedule {schedule!r} (gpipe | 1f1b)")
        self.schedule = schedule
        # Plain (non-fused) last stage: lm_head + cross-entropy without keeping the logits
        # (models.gpt.head_cross_entropy). Off by default, so that scripts written for the
        # reference's GPipeEngine get its exact numerics; the trainer turns it on.
        self.fused_head = False
        self.max_inflight = 0  # most micro-batches whose activations were held at once (last step)
        self.stage, self.topo = stage, topo
        self.pp_rank, self.pp_size = topo.pp_rank, topo.pp
        self.is_first, self.is_last = stage.is_first, stage.is_last
        self.boundary_dtype = boundary_dtype
        self.prev_rank = self.next_rank = None
        if self.pp_size > 1:
            rc = lambda p: rank_from_coords(topo.dp_rank, topo.ep_rank, p, topo.tp_rank, topo.dp, topo.ep, topo.tp,
                                            topo.pp)
            if self.pp_rank > 0:
                self.prev_rank = rc(self.pp_rank - 1)
            if self.pp_rank < self.pp_size - 1:
                self.next_rank = rc(self.pp_rank + 1)

    # -- point-to-point -----------------------------------------------------
    def _isend(self, t: torch.Tensor, peer: int, tag: int):
        return dist.batch_isend_irecv([dist.P2POp(dist.isend, t.contiguous(), peer, tag=tag)])

    def _irecv(self, t: torch.Tensor, peer: int, tag: int):
        return dist.batch_isend_irecv([dist.P2POp(dist.irecv, t, peer, tag=tag)])

    @staticmethod
    def _wait(works) -> None:
        for w in works:
            w.wait()

    def _fwd_tag(self, m: int) -> int:
        return 1000 + m

    def _bwd_tag(self, m: int) -> int:
        return 2000 + m

    def _recv_fwd(self, m: int, B: int, S: int, H: int, device):
        buf = torch.empty((B, S, H), device=device, dtype=self.boundary_dtype)
        return buf, self._irecv(buf, self.prev_rank, self._fwd_tag(m))

    # -- schedule -------------------------------------------------------------
    def _forward_micro(self, loader, device, use_amp, amp_dtype, recv_x):
        """Forward of one micro-batch on this stage: (stage output, loss on the last stage | None, aux)."""
        idx, targets = loader.next_batch(device)
        if not self.is_last:
            targets = None
        ctx = torch.autocast(device_type=device.type, dtype=amp_dtype, enabled=use_amp and not self.stage.fused)
        with ctx:
            x = self.stage.embed(idx) if self.is_first else recv_x
            x, aux = self.stage.forward_blocks(x)
            loss = self.stage.forward_head(x, targets, want_logits=not self.fused_head)[1] if self.is_last else None
        return x, loss, aux

    def _as_input(self, buf: torch.Tensor, keep_graph: bool) -> torch.Tensor:
        x = buf.to(torch.float32) if buf.dtype != torch.float32 else buf
        if keep_graph:
            x.requires_grad_(True)
        return x

    def _run_forward(self, loader, micro_batches, device, use_amp, amp_dtype, batch_size, state, keep_graph):
        cfg = self.stage.cfg
        B, S, H = self.stage.boundary_batch(batch_size), cfg.block_size, cfg.n_embed
        pending_recv = self._recv_fwd(0, B, S, H, device) if not self.is_first else None
        sends = []
        for m in range(micro_batches):
            recv_x = None
            if not self.is_first:
                buf, works = pending_recv
                self._wait(works)
                if m + 1 < micro_batches:
                    pending_recv = self._recv_fwd(m + 1, B, S, H, device)
                recv_x = self._as_input(buf, keep_graph)
            x, loss, aux = self._forward_micro(loader, device, use_amp, amp_dtype, recv_x)
            if not self.is_last:
                out = x.detach().to(self.boundary_dtype)
                sends.append((out, self._isend(out, self.next_rank, self._fwd_tag(m))))
                if keep_graph:
                    state.boundaries.append(x)
            if keep_graph and not self.is_first:
                state.recv_inputs.append(recv_x)
            if self.is_last and loss is not None:
                state.losses.append(loss)
            state.aux_losses.append(aux)
        for _, works in sends:
            self._wait(works)
        if keep_graph:
            self.max_inflight = micro_batches

    def _backward_micro(self, boundary, loss, aux, grad, micro_batches, scaler) -> None:
        """Backward of one micro-batch: the last stage from (loss + aux) / M, the others
        from the gradient of their output (plus their own aux / M)."""
        scaled = scaler is not None and scaler.is_enabled()
        if self.is_last:
            loss_mb = (loss + aux) / micro_batches
            (scaler.scale(loss_mb) if scaled else loss_mb).backward()
        elif aux.requires_grad:
            a = aux / micro_batches
            torch.autograd.backward([boundary, scaler.scale(a) if scaled else a], [grad, None])
        else:
            boundary.backward(grad)

    def forward_backward(self, loader, micro_batches: int, device: torch.device, use_amp: bool,
                         amp_dtype: torch.dtype, scaler=None, batch_size: int = 1,
                         aux_loss_coef: float = 0.01) -> Tuple[Optional[torch.Tensor], torch.Tensor]:
        """One optimizer step's worth of forward and backward; returns (mean loss on the last stage | None, aux)."""
        if self.schedule == "1f1b":
            return self._forward_backward_1f1b(loader, micro_batches, device, use_amp, amp_dtype, scaler,
                                               batch_size)
        state = PipelineState()
        self._run_forward(loader, micro_batches, device, use_amp, amp_dtype, batch_size, state, keep_graph=True)
        total_aux = (torch.stack([a.detach().float() for a in state.aux_losses]).sum()
                     if state.aux_losses else torch.zeros((), device=device))
        if self.pp_size > 1 and dist.is_initialized() and self.topo.pp_group is not None:
            dist.all_reduce(total_aux, op=dist.ReduceOp.SUM, group=self.topo.pp_group)

        sends = []
        pending = None
        if not self.is_last:
            g0 = torch.empty_like(state.boundaries[micro_batches - 1], dtype=self.boundary_dtype)
            pending = (g0, self._irecv(g0, self.next_rank, self._bwd_tag(micro_batches - 1)))
        for m in reversed(range(micro_batches)):
            grad, boundary, loss = None, None, None
            if self.is_last:
                loss = state.losses[m]
            else:
                gbuf, works = pending
                self._wait(works)
                if m > 0:
                    nxt = torch.empty_like(state.boundaries[m - 1], dtype=self.boundary_dtype)
                    pending = (nxt, self._irecv(nxt, self.next_rank, self._bwd_tag(m - 1)))
                boundary = state.boundaries[m]
                grad = gbuf.to(boundary.dtype)
            self._backward_micro(boundary, loss, state.aux_losses[m], grad, micro_batches, scaler)
            if not self.is_first:
                gin = state.recv_inputs[m].grad.to(self.boundary_dtype)
                sends.append((gin, self._isend(gin, self.prev_rank, self._bwd_tag(m))))
        for _, works in sends:
            self._wait(works)

        if self.is_last and state.losses:
            with torch.no_grad():
                return torch.stack([l.detach().float() for l in state.losses]).mean(), total_aux.detach()
        return None, total_aux.detach()

    # -- 1F1B -------------------------------------------------------------------
    def _batch_p2p(self, ops: list) -> list:
        """Post the point-to-point ops of one step as one batch (one NCCL group): a send
        and a receive in opposite directions between two stages then cannot wait on each
        other, whatever order the two ranks reach them in."""
        return dist.batch_isend_irecv(ops) if ops else []

    def _forward_backward_1f1b(self, loader, M: int, device, use_amp, amp_dtype, scaler, batch_size):
        """Runs ``one_f_one_b_plan`` for this stage (see there for the schedule)."""
        cfg = self.stage.cfg
        B, S, H = self.stage.boundary_batch(batch_size), cfg.block_size, cfg.n_embed
        P2P = dist.P2POp
        held = []  # FIFO of (recv_x, boundary, loss, aux) for forwards whose backward is pending
        keep = []  # tensors of sends in flight, with their works
        losses, auxes = [], []
        self.max_inflight = 0
        act = None   # the received input of the next forward
        out = None   # the output of the last forward, to send
        gbuf = None  # the received gradient of the next backward
        gin = None   # the input gradient of the last backward, to send

        def new_buf():
            return torch.empty((B, S, H), device=device, dtype=self.boundary_dtype)

        for step in one_f_one_b_plan(self.pp_rank, self.pp_size, M):
            kind = step[0]
            if kind == "fwd":
                recv_x = self._as_input(act, True) if act is not None else None
                act = None
                x, loss, aux = self._forward_micro(loader, device, use_amp, amp_dtype, recv_x)
                held.append((recv_x, x, loss, aux))
                self.max_inflight = max(self.max_inflight, len(held))
                auxes.append(aux.detach().float())
                if loss is not None:
                    losses.append(loss.detach().float())
                out = None if self.is_last else x.detach().to(self.boundary_dtype)
            elif kind == "bwd":
                recv_x, x, loss, aux = held.pop(0)
                grad = gbuf.to(x.dtype) if gbuf is not None else None
                gbuf = None
                self._backward_micro(x, loss, aux, grad, M, scaler)
                gin = None if self.is_first else recv_x.grad.to(self.boundary_dtype)
            elif kind == "recv_act":
                act = new_buf()
                self._wait(self._batch_p2p([P2P(dist.irecv, act, self.prev_rank, tag=self._fwd_tag(step[1]))]))
            elif kind == "recv_grad":
                gbuf = new_buf()
                self._wait(self._batch_p2p([P2P(dist.irecv, gbuf, self.next_rank, tag=self._bwd_tag(step[1]))]))
            elif kind == "send_act":
                keep.append((out, self._batch_p2p([P2P(dist.isend, out, self.next_rank,
                                                       tag=self._fwd_tag(step[1]))])))
            elif kind == "send_grad":
                keep.append((gin, self._batch_p2p([P2P(dist.isend, gin, self.prev_rank,
                                                       tag=self._bwd_tag(step[1]))])))
            elif kind == "send_act+recv_grad":
                gbuf = new_buf()
                self._wait(self._batch_p2p([P2P(dist.isend, out, self.next_rank, tag=self._fwd_tag(step[1])),
                                            P2P(dist.irecv, gbuf, self.next_rank, tag=self._bwd_tag(step[2]))]))
                keep.append((out, []))
            elif kind == "send_grad+recv_act":
                act = new_buf()
                self._wait(self._batch_p2p([P2P(dist.isend, gin, self.prev_rank, tag=self._bwd_tag(step[1])),
                                            P2P(dist.irecv, act, self.prev_rank, tag=self._fwd_tag(step[2]))]))
                keep.append((gin, []))
            else:
                raise AssertionError(kind)
        for _, works in keep:
            self._wait(works)

        total_aux = torch.stack(auxes).sum() if auxes else torch.zeros((), device=device)
        if self.pp_size > 1 and dist.is_initialized() and self.topo.pp_group is not None:
            dist.all_reduce(total_aux, op=dist.ReduceOp.SUM, group=self.topo.pp_group)
        if self.is_last and losses:
            return torch.stack(losses).mean(), total_aux.detach()
        return None, total_aux.detach()

    @torch.no_grad()
    def forward_only(self, loader, micro_batches: int, device: torch.device, use_amp: bool, amp_dtype: torch.dtype,
                     batch_size: int) -> Optional[torch.Tensor]:
        state = PipelineState()
        self._run_forward(loader, micro_batches, device, use_amp, amp_dtype, batch_size, state, keep_graph=False)
        if self.is_last and state.losses:
            return torch.stack([l.detach().float() for l in state.losses]).mean()
        return None
