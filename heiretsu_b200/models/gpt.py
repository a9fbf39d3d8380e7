"""GPT-2 with tensor-parallel attention/MLP and optional MoE blocks.

The module tree, parameter names and initialisation order are those of the
reference (gpt_model.py:33-288) because they define the checkpoint format
(state_dict keys and shard shapes) and, with a fixed seed, the initial
weights:

    tr.wte, tr.wpe, tr.h.{i}.{ln_1, attn.c_attn, attn.c_proj, ln_2,
    mlp.c_fc, mlp.c_proj | moe.router.gate, moe.expert_group.experts.{j}.w1/w2},
    tr.ln_f, lm_head (tied to tr.wte)

Two execution paths share these parameters:

* the plain PyTorch path below (CPU, fp32 parity tests, any dtype);
* the fused sm_100a path (``heiretsu_b200.models.fused``), taken on CUDA when
  the extension is loaded and the model runs in bf16 (``model.fused = True``,
  set by ``enable_fused``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.utils.checkpoint
import torch.nn.functional as F

from ..config import GPTConfig, make_moe_config
from ..parallel.tp import ColumnParallelLinear, ColumnParallelLinearQKV, RowParallelLinear
from .moe import Expert, MoELayer

__all__ = ["GPTConfig", "AttentionTP", "MLPTP", "BlockTP", "BlockMoE", "make_block", "GPT", "init_gpt_weights"]


class AttentionTP(nn.Module):
    """Causal self-attention with heads sharded over TP ranks."""

    def __init__(self, cfg: GPTConfig, tp_group=None, tp_rank: int = 0, tp_world_size: int = 1):
        super().__init__()
        if cfg.n_embed % cfg.n_head:
            raise ValueError("n_embed must be divisible by n_head")
        if cfg.n_embed % tp_world_size:
            raise ValueError(f"n_embed = {cfg.n_embed} does not split evenly over "
                             f"{tp_world_size} tensor-parallel ranks")
        if cfg.n_head % tp_world_size:
            raise ValueError(f"n_head = {cfg.n_head} does not split evenly over "
                             f"{tp_world_size} tensor-parallel ranks")
        self.n_embed, self.n_head = cfg.n_embed, cfg.n_head
        self.tp_world_size, self.tp_rank, self.tp_group = tp_world_size, tp_rank, tp_group
        self.nh_tp = cfg.n_head // tp_world_size
        self.dh = cfg.n_embed // cfg.n_head
        self.h_tp = cfg.n_embed // tp_world_size
        self.c_attn = ColumnParallelLinearQKV(cfg.n_embed, cfg.n_embed, tp_group=tp_group, tp_rank=tp_rank,
                                              tp_world_size=tp_world_size)
        self.c_proj = RowParallelLinear(cfg.n_embed, cfg.n_embed, tp_group=tp_group, tp_rank=tp_rank,
                                        tp_world_size=tp_world_size)
        self.c_proj.NANOGPT_SCALE_INIT = 1
        self.attn_drop = nn.Dropout(cfg.dropout)
        self.resid_drop = nn.Dropout(cfg.dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, _ = x.shape
        qkv = self.c_attn(x)  # [B, S, 3*H_tp], columns = [Q | K | V], each head-major
        q, k, v = qkv.view(B, S, 3, self.nh_tp, self.dh).permute(2, 0, 3, 1, 4).unbind(0)  # [B, nh, S, dh]
        y = F.scaled_dot_product_attention(q, k, v, attn_mask=None,
                                           dropout_p=self.attn_drop.p if self.training else 0.0, is_causal=True)
        y = y.transpose(1, 2).reshape(B, S, self.h_tp)
        return self.resid_drop(self.c_proj(y, input_is_parallel=True))


class MLPTP(nn.Module):
    """c_fc (column-parallel) -> GELU(tanh) -> c_proj (row-parallel)."""

    def __init__(self, cfg: GPTConfig, tp_group=None, tp_rank: int = 0, tp_world_size: int = 1):
        super().__init__()
        self.c_fc = ColumnParallelLinear(cfg.n_embed, 4 * cfg.n_embed, tp_group=tp_group, tp_rank=tp_rank,
                                         tp_world_size=tp_world_size)
        self.gelu = nn.GELU(approximate="tanh")
        self.c_proj = RowParallelLinear(4 * cfg.n_embed, cfg.n_embed, tp_group=tp_group, tp_rank=tp_rank,
                                        tp_world_size=tp_world_size)
        self.c_proj.NANOGPT_SCALE_INIT = 1
        self.drop = nn.Dropout(cfg.dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.drop(self.c_proj(self.gelu(self.c_fc(x)), input_is_parallel=True))


class BlockTP(nn.Module):
    """Pre-LN dense block; returns (x, aux_loss=0)."""

    def __init__(self, cfg: GPTConfig, tp_group=None, tp_rank: int = 0, tp_world_size: int = 1):
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embed)
        self.attn = AttentionTP(cfg, tp_group=tp_group, tp_rank=tp_rank, tp_world_size=tp_world_size)
        self.ln_2 = nn.LayerNorm(cfg.n_embed)
        self.mlp = MLPTP(cfg, tp_group=tp_group, tp_rank=tp_rank, tp_world_size=tp_world_size)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        x = x + self.attn(self.ln_1(x))
        x = x + self.mlp(self.ln_2(x))
        return x, torch.zeros((), device=x.device, dtype=x.dtype)


class BlockMoE(nn.Module):
    """Pre-LN block whose MLP is a top-k mixture of experts; returns (x, aux_loss)."""

    def __init__(self, cfg: GPTConfig, tp_group=None, tp_rank: int = 0, tp_world_size: int = 1, ep_group=None,
                 ep_rank: int = 0, ep_world_size: int = 1):
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embed)
        self.attn = AttentionTP(cfg, tp_group=tp_group, tp_rank=tp_rank, tp_world_size=tp_world_size)
        self.ln_2 = nn.LayerNorm(cfg.n_embed)
        mcfg = make_moe_config(hidden_size=cfg.n_embed, num_experts=cfg.num_experts, top_k=cfg.top_k,
                               intermediate_mult=4, aux_loss_coef=cfg.aux_loss_coef)
        self.moe = MoELayer(mcfg, ep_group=ep_group, ep_rank=ep_rank, ep_world_size=ep_world_size)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        x = x + self.attn(self.ln_1(x))
        y, aux = self.moe(self.ln_2(x))
        return x + y, aux


def make_block(cfg: GPTConfig, layer_idx: int, tp_group=None, tp_rank: int = 0, tp_world_size: int = 1,
               ep_group=None, ep_rank: int = 0, ep_world_size: int = 1) -> nn.Module:
    """BlockMoE where (layer_idx + 1) % moe_freq == 0 and num_experts > 0, else BlockTP."""
    if cfg.is_moe_layer(layer_idx):
        return BlockMoE(cfg, tp_group, tp_rank, tp_world_size, ep_group, ep_rank, ep_world_size)
    return BlockTP(cfg, tp_group, tp_rank, tp_world_size)


def run_blocks(blocks, x: torch.Tensor, recompute: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Plain-path block loop: x through every block, returning (x, summed aux loss).

    ``recompute`` (activation checkpointing, absent from the reference, whose
    README.md:127 lists it as future work) keeps only each block's input during a
    training forward and re-runs the block in backward (non-reentrant
    ``torch.utils.checkpoint``, which restores the RNG and autocast state, so the
    dropout masks and the bf16 casts are the forward's). Collectives inside a block
    (TP all-reduces, EP all-to-alls) are re-issued in the same order on every rank.
    """
    aux_total = torch.zeros((), device=x.device, dtype=x.dtype)
    for blk in blocks:
        if recompute and blk.training and torch.is_grad_enabled():
            x, aux = torch.utils.checkpoint.checkpoint(blk, x, use_reentrant=False)
        else:
            x, aux = blk(x)
        aux_total = aux_total + aux
    return x, aux_total


class _HeadCE(torch.autograd.Function):
    """lm_head projection + mean cross-entropy in one autograd node (plain path, no autocast).

    Forward: logits = x W^T, per-row log-sum-exp, loss = mean over rows whose
    target is not ``ignore_index`` of (lse - logit[target]) (NaN when no row
    counts, like ``F.cross_entropy``). Backward turns the saved logits buffer
    into the gradient in place, (softmax - onehot) * dloss / n, and runs the two
    GEMMs. Both directions go through the rows in blocks of about 32 MB of
    logits: each block's GEMM output is reduced (forward) or turned into its
    gradient and consumed by its two GEMMs (backward) while it is still in
    cache, so the [N, V] buffer crosses DRAM about three times per step, against
    about ten for ``F.cross_entropy`` on materialised logits (log-softmax copy,
    zero-filled one-hot gradient, softmax-backward buffer). The graph can be
    differentiated once (the buffer is consumed).
    """

    BLOCK_BYTES = 32 << 20

    @staticmethod
    def _blocks(n_rows: int, n_cols: int, esz: int, cuda: bool = False):
        if cuda:  # one block: whole-matrix GEMMs suit a GPU, and its L2 is not the working set here
            return [(0, n_rows)]
        step = max(16, _HeadCE.BLOCK_BYTES // max(1, n_cols * esz))
        return [(r, min(n_rows, r + step)) for r in range(0, n_rows, step)]

    @staticmethod
    def forward(ctx, x, w, targets, ignore_index: int, pool):
        N, V = x.shape[0], w.shape[0]
        logits = None
        while pool:  # a buffer a finished backward handed back (no fresh pages to fault in)
            cand = pool.pop()
            if cand.shape == (N, V) and cand.dtype == x.dtype and cand.device == x.device:
                logits = cand
                break
        if logits is None:
            logits = torch.empty(N, V, dtype=x.dtype, device=x.device)
        lse = torch.empty(N, dtype=x.dtype, device=x.device)
        wt = w.t()
        for a, b in _HeadCE._blocks(N, V, x.element_size(), x.is_cuda):
            blk = logits[a:b]
            torch.mm(x[a:b], wt, out=blk)
            m = blk.amax(dim=1, keepdim=True)
            lse[a:b] = (blk - m).exp_().sum(dim=1).log_().add_(m.squeeze(1))
        valid = targets != ignore_index
        tgt = torch.where(valid, targets, torch.zeros_like(targets))
        picked = logits.gather(1, tgt[:, None]).squeeze(1)
        n = valid.sum().to(x.dtype)
        loss = torch.where(valid, lse - picked, torch.zeros_like(lse)).sum() / n
        ctx.save_for_backward(x, w, logits, lse, tgt, valid, n)
        ctx.consumed = False
        ctx.pool = pool
        return loss

    @staticmethod
    def backward(ctx, dloss):
        if ctx.consumed:
            raise RuntimeError("the fused lm_head/cross-entropy graph can be differentiated only once")
        ctx.consumed = True
        x, w, g, lse, tgt, valid, n = ctx.saved_tensors
        scale = torch.where(valid, dloss / n, torch.zeros_like(lse))
        dx = torch.empty_like(x)
        dw = torch.zeros_like(w)
        for a, b in _HeadCE._blocks(g.shape[0], g.shape[1], g.element_size(), g.is_cuda):
            gb = g[a:b]
            gb.sub_(lse[a:b, None]).exp_().mul_(scale[a:b, None])
            gb.scatter_add_(1, tgt[a:b, None], -scale[a:b, None])
            torch.mm(gb, w, out=dx[a:b])
            dw.addmm_(gb.t(), x[a:b])
        if ctx.pool is not None:
            ctx.pool.append(g)  # nothing else refers to the buffer: the next forward may reuse it
        return dx, dw, None, None, None


def head_cross_entropy(x: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                       pool: Optional[list] = None) -> torch.Tensor:
    """Mean cross-entropy of ``x @ w.T`` against ``targets`` without keeping the logits.

    ``pool``: a list the caller keeps; each backward puts its [N, V] buffer there and
    the next forward of the same shape takes it back, so steps stop allocating (and
    page-faulting in) a fresh logits buffer. Pipelines with several forwards in flight
    simply hold several buffers."""
    return _HeadCE.apply(x.reshape(-1, x.size(-1)), w, targets.reshape(-1), ignore_index, pool)


def init_gpt_weights(module: nn.Module, n_layer: int) -> None:
    """NanoGPT init: N(0, 0.02) everywhere, c_proj std scaled by (2L)^-0.5, zero biases.

    Applied with ``Module.apply`` (children before parents), matching the
    reference's draw order (gpt_model.py:245-258)."""

    def fn(m: nn.Module) -> None:
        if isinstance(m, (nn.Linear, ColumnParallelLinear, ColumnParallelLinearQKV, RowParallelLinear)):
            std = 0.02
            if hasattr(m, "NANOGPT_SCALE_INIT"):
                std *= (2 * n_layer) ** -0.5
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, mean=0.0, std=std)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            else:
                m.reset_parameters(std=std)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)

    module.apply(fn)


class GPT(nn.Module):
    """GPT-2 language model. ``forward(idx, targets) -> (logits, loss, aux_loss)``."""

    def __init__(self, cfg: GPTConfig, topo: Optional[object] = None):
        super().__init__()
        self.cfg = cfg
        g = lambda k, d: getattr(topo, k, d) if topo is not None else d
        tp, tp_rank, tp_group = g("tp", 1), g("tp_rank", 0), g("tp_group", None)
        ep, ep_rank, ep_group = g("ep", 1), g("ep_rank", 0), g("ep_group", None)
        self.topo = topo
        self.tr = nn.ModuleDict(dict(
            wte=nn.Embedding(cfg.vocab_size, cfg.n_embed),
            wpe=nn.Embedding(cfg.block_size, cfg.n_embed),
            h=nn.ModuleList([make_block(cfg, i, tp_group, tp_rank, tp, ep_group, ep_rank, ep)
                             for i in range(cfg.n_layer)]),
            ln_f=nn.LayerNorm(cfg.n_embed),
        ))
        self.lm_head = nn.Linear(cfg.n_embed, cfg.vocab_size, bias=False)
        self.tr.wte.weight = self.lm_head.weight  # weight tying
        init_gpt_weights(self, cfg.n_layer)
        self.fused = False  # set by heiretsu_b200.models.fused.enable_fused
        self.recompute = False  # activation checkpointing of the plain path (run_blocks)
        self._head_pool: list = []  # logits buffers reused by head_cross_entropy

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None, return_logits: bool = True):
        B, T = idx.shape
        if T > self.cfg.block_size:
            raise ValueError(f"input of {T} positions exceeds the model's block_size of {self.cfg.block_size}")
        if self.fused and idx.is_cuda:
            from .fused import gpt_forward_fused
            return gpt_forward_fused(self, idx, targets, return_logits=return_logits)
        pos = torch.arange(T, device=idx.device)
        x = self.tr.wte(idx) + self.tr.wpe(pos)[None]
        x, aux_total = run_blocks(self.tr.h, x, self.recompute)
        x = self.tr.ln_f(x)
        if targets is not None and not return_logits and not torch.is_autocast_enabled(x.device.type):
            return None, head_cross_entropy(x, self.lm_head.weight, targets, pool=self._head_pool), aux_total
        logits = self.lm_head(x)
        loss = None
        if targets is not None:
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1))
        return logits, loss, aux_total

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


# Keep the reference's import names available from this module.
_ = Expert
