"""Fused sm_100a execution of the GPT model (forward and backward).

The model is executed as three autograd functions:

* ``_Embed``  idx -> x0 = wte[idx] + wpe[t]                (fp32 residual stream)
* ``_Body``   x0 -> x_L through every block, explicit backward
* ``_Head``   x_L -> ln_f -> lm_head -> cross-entropy        (loss, fused bwd)

Inside ``_Body`` each dense block runs 6 kernels forward:

    LN1 -> QKV GEMM(+bias) -> flash attention -> proj GEMM(+bias+residual)
    LN2 -> FC GEMM(+bias, GELU; pre-activation kept) -> proj GEMM(+bias+residual)

and the mirror image backward (dgrad GEMMs with the GELU derivative fused
into the epilogue, wgrad GEMMs accumulating straight into the fp32 gradient
buffer, LayerNorm backward updating the residual gradient in place). Weights
are read through their bf16 shadows (``p.w16``); gradients are written to
``p.main_grad`` (see heiretsu_b200/parallel/flat.py), so autograd never
allocates or adds parameter gradients.

Numerics: 16-bit operands (bf16, or fp16 under ``--amp fp16``), fp32
accumulation, fp32 residual stream and fp32 LayerNorm statistics -- the same
precision split as the reference under ``torch.autocast`` (gemm in 16 bits, bias
add / LN / residual in fp32).
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch

from ..ops import gemm as G
from ..utils.profiling import nvtx
from ..ops import kernels as K

LN_EPS = 1e-5


def fused_supported(cfg, topo=None, tp_dropout: bool = True) -> Tuple[bool, str]:
    """Whether the fused path covers this configuration (else the plain path runs).

    ``tp_dropout`` = False sends tensor-parallel runs with dropout to the plain
    path (``--fused_tp_dropout 0``); by default they run fused (``models/fused_tp.py``)."""
    if cfg.n_embed % cfg.n_head or cfg.n_embed // cfg.n_head not in (16, 32, 64, 128):
        return False, "fused attention needs head_dim 16, 32, 64 or 128"
    if cfg.n_embed % 128:
        return False, "fused path needs n_embed % 128 == 0"
    if cfg.dropout > 0 and topo is not None and getattr(topo, "tp", 1) > 1 and not tp_dropout:
        return False, "fused tensor parallelism with dropout is switched off (--fused_tp_dropout 0)"
    if cfg.dropout > 0 and cfg.n_embed % 4:
        return False, "fused dropout needs n_embed % 4 == 0"
    if cfg.num_experts > 0 and topo is not None and getattr(topo, "ep", 1) > 8:
        return False, "fused expert parallelism exchanges partials over NVLink within one node (ep <= 8)"
    if topo is not None and hasattr(topo, "on_one_node"):
        # Fused TP and EP exchange through CUDA IPC peer mappings, which exist only between
        # GPUs of one node; a group that spans nodes runs the plain (NCCL) path.
        if topo.tp > 1 and not topo.on_one_node(topo.tp_ranks):
            return False, "fused tensor parallelism needs each TP group on one node (this one spans nodes)"
        if cfg.num_experts > 0 and topo.ep > 1 and not topo.on_one_node(topo.ep_ranks):
            return False, "fused expert parallelism needs each EP group on one node (this one spans nodes)"
    return True, ""


def _vpad(V: int) -> int:
    return (V + 127) // 128 * 128


# ---------------------------------------------------------------------------
class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, wte, wpe):
        ctx.save_for_backward(idx)
        ctx.wte, ctx.wpe = wte, wpe
        return K.embedding_fwd(idx, wte.detach(), wpe.detach())

    @staticmethod
    def backward(ctx, dx):
        (idx,) = ctx.saved_tensors
        K.embedding_bwd(idx, dx.contiguous(), ctx.wte.main_grad, ctx.wpe.main_grad)
        return None, None, None


def embed_fused(wte: torch.nn.Parameter, wpe: torch.nn.Parameter, idx: torch.Tensor) -> torch.Tensor:
    B, T = idx.shape
    return _Embed.apply(idx.contiguous(), wte, wpe).view(B, T, -1)


# ---------------------------------------------------------------------------
# Dropout (training only): block i uses sites 4i (attention probabilities),
# 4i+1 (attention output residual) and 4i+2 (MLP output residual), as the
# reference applies dropout (gpt_model.py:53-54, :79, :96). Every forward
# takes a snapshot of the step's device seed and then advances it, so each
# micro-batch and each graph replay draws fresh masks, and the backward
# recomputes exactly the forward's masks from the snapshot.
def _dt(blk) -> torch.dtype:
    """16-bit format of a block's activations: the format of its weight shadows
    (bf16 under --amp bf16, fp16 under --amp fp16)."""
    return blk.ln_1.weight.w16.dtype


def _dropout_of(blk):
    """(seed snapshot tensor, layer index, p) of a block in a training forward, else None."""
    d = getattr(blk, "_hb_drop_now", None)
    return d if (d is not None and blk.training) else None


def _attn_fwd(blk, x: torch.Tensor, B: int, T: int, keep: bool):
    """Attention sub-layer: x fp32 [M, H] -> x1 = x + drop(c_proj(attn(c_attn(ln_1(x)))))."""
    attn = blk.attn
    d = _dropout_of(blk)
    xn, m1, r1 = K.layernorm_fwd(x, blk.ln_1.weight, blk.ln_1.bias, LN_EPS, dtype=_dt(blk))
    qkv = G.linear_fwd(xn, attn.c_attn.weight.w16, attn.c_attn.bias)
    adrop = (d[0], 4 * d[1], d[2], 0, attn.nh_tp) if d else None
    y, lse = K.attention_fwd(qkv, B, T, attn.nh_tp, drop=adrop, head_dim=attn.dh)
    x1 = G.linear_fwd_resid(y, attn.c_proj.weight.w16, attn.c_proj.bias, x,
                            drop=(d[0], 4 * d[1] + 1, d[2], 0) if d else None)
    return x1, ((x, xn, m1, r1, qkv, y, lse, d) if keep else None)


def _mlp_fwd(blk, x1: torch.Tensor, keep: bool):
    """Dense MLP sub-layer: x2 = x1 + drop(c_proj(gelu(c_fc(ln_2(x1)))))."""
    mlp = blk.mlp
    d = _dropout_of(blk)
    xn2, m2, r2 = K.layernorm_fwd(x1, blk.ln_2.weight, blk.ln_2.bias, LN_EPS, dtype=_dt(blk))
    h, pre = G.linear_fwd_gelu(xn2, mlp.c_fc.weight.w16, mlp.c_fc.bias)
    x2 = G.linear_fwd_resid(h, mlp.c_proj.weight.w16, mlp.c_proj.bias, x1,
                            drop=(d[0], 4 * d[1] + 2, d[2], 0) if d else None)
    return x2, ((x1, xn2, m2, r2, pre, h, d) if keep else None)


def _mlp_bwd(blk, saved, dres: torch.Tensor, dres16: torch.Tensor, ws: dict):
    """In place: dres (fp32) / dres16 (16-bit) go from d(x2) to d(x1)."""
    mlp = blk.mlp
    x1, xn2, m2, r2, pre, h, d = saved
    # gradient at c_proj's output
    dout16 = K.dropout_bf16(dres, d[0], 4 * d[1] + 2, d[2], dtype=dres16.dtype) if d else dres16
    dpre = G.linear_dgrad(dout16, mlp.c_proj.weight.w16, gelu_pre=pre)
    G.linear_wgrad(dout16, h, out=mlp.c_proj.weight.main_grad, accumulate=True)
    K.colsum_bf16(dout16, mlp.c_proj.bias.main_grad)
    del dout16
    dxn2 = G.linear_dgrad(dpre, mlp.c_fc.weight.w16, f32=True)
    G.linear_wgrad(dpre, xn2, out=mlp.c_fc.weight.main_grad, accumulate=True)
    K.colsum_bf16(dpre, mlp.c_fc.bias.main_grad)
    del dpre
    K.layernorm_bwd(dxn2, x1, m2, r2, blk.ln_2.weight, dres, dres, dres16, blk.ln_2.weight.main_grad,
                    blk.ln_2.bias.main_grad, scratch=ws["ln_scratch"])


def _attn_bwd(blk, saved, dres: torch.Tensor, dres16: torch.Tensor, B: int, T: int, ws: dict):
    """In place: dres / dres16 go from d(x1) to d(x)."""
    attn = blk.attn
    x, xn, m1, r1, qkv, y, lse, d = saved
    # gradient at c_proj's output
    dout16 = K.dropout_bf16(dres, d[0], 4 * d[1] + 1, d[2], dtype=dres16.dtype) if d else dres16
    dy = G.linear_dgrad(dout16, attn.c_proj.weight.w16)
    G.linear_wgrad(dout16, y, out=attn.c_proj.weight.main_grad, accumulate=True)
    K.colsum_bf16(dout16, attn.c_proj.bias.main_grad)
    del dout16
    adrop = (d[0], 4 * d[1], d[2], 0, attn.nh_tp) if d else None
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, T, attn.nh_tp, drop=adrop, head_dim=attn.dh)
    del dy
    G.linear_wgrad(dqkv, xn, out=attn.c_attn.weight.main_grad, accumulate=True)
    K.colsum_bf16(dqkv, attn.c_attn.bias.main_grad)
    dxn = G.linear_dgrad(dqkv, attn.c_attn.weight.w16, f32=True)
    del dqkv
    K.layernorm_bwd(dxn, x, m1, r1, blk.ln_1.weight, dres, dres, dres16, blk.ln_1.weight.main_grad,
                    blk.ln_1.bias.main_grad, scratch=ws["ln_scratch"])


def _ln_scratch(M: int, H: int, device) -> torch.Tensor:
    from ..ops._C import load
    rows = load().layernorm_bwd_scratch_rows(M)
    return torch.empty(rows * 2 * H, device=device, dtype=torch.float32)


def _snapshot_dropout_seeds(blocks) -> None:
    """Give every block of this forward the current device seed (one copy),
    then advance the seed for the next forward."""
    seeds = {}
    for blk in blocks:
        cfg = getattr(blk, "_hb_dropout", None)  # (seed tensor, layer index, p)
        if cfg is None or not blk.training:
            blk._hb_drop_now = None
            continue
        seed, layer, p = cfg
        if id(seed) not in seeds:
            seeds[id(seed)] = (seed, seed.clone())
        blk._hb_drop_now = (seeds[id(seed)][1], layer, p)
    for seed, _ in seeds.values():
        seed.add_(1)


# Called after each block's backward has been issued (data-parallel gradient
# reduction overlapped with the rest of backward); None when not armed.
_BLOCK_DONE_HOOK = None


def set_block_done_hook(fn) -> None:
    global _BLOCK_DONE_HOOK
    _BLOCK_DONE_HOOK = fn


def _is_moe(blk) -> bool:
    return hasattr(blk, "moe")


class _Recompute:
    """Saved state of a dense block run without keeping its activations: the block's
    input and the dropout snapshot its forward used (backward reruns the forward)."""

    def __init__(self, x_in, drop_now):
        self.x_in, self.drop_now = x_in, drop_now


def _rerun_dense(blk, r: "_Recompute", B: int, T: int):
    """The (attention, MLP) saved tuples of a dense block, recomputed from its input
    with the forward's dropout masks (a pure function of the saved seed snapshot)."""
    prev = getattr(blk, "_hb_drop_now", None)
    blk._hb_drop_now = r.drop_now
    try:
        x1, sa = _attn_fwd(blk, r.x_in, B, T, True)
        _, sm = _mlp_fwd(blk, x1, True)
    finally:
        blk._hb_drop_now = prev
    return sa, sm


class _Body(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, blocks, B, T, recompute=False):
        from .fused_moe import moe_sublayer_fwd

        keep = x.requires_grad
        saved: List = []
        aux_total = torch.zeros((), device=x.device, dtype=torch.float32)
        _snapshot_dropout_seeds(blocks)
        for i, blk in enumerate(blocks):
            # activation checkpointing: a dense block keeps only its input (MoE blocks keep all)
            rerun = keep and recompute and not _is_moe(blk)
            x_in = x
            with nvtx(f"block{i}.attn.fwd"):
                x, sa = _attn_fwd(blk, x, B, T, keep and not rerun)
            with nvtx(f"block{i}.mlp.fwd"):
                if _is_moe(blk):
                    x, aux, sm = moe_sublayer_fwd(blk, None, x, keep)
                    aux_total = aux_total + aux
                else:
                    x, sm = _mlp_fwd(blk, x, keep and not rerun)
            saved.append(_Recompute(x_in, getattr(blk, "_hb_drop_now", None)) if rerun else (sa, sm))
        ctx.blocks, ctx.saved, ctx.B, ctx.T = blocks, saved, B, T
        return x, aux_total

    @staticmethod
    def backward(ctx, dx, daux):
        from .fused_moe import moe_sublayer_bwd

        B, T = ctx.B, ctx.T
        dres = dx.contiguous().clone()
        dres16 = K.f32_to_bf16(dres, dtype=_dt(ctx.blocks[0]))
        M, H = dres.shape
        ws = {"ln_scratch": _ln_scratch(M, H, dres.device)}
        if daux is None:
            daux = torch.zeros((), device=dres.device)
        n = len(ctx.blocks)
        for j, (blk, st) in enumerate(zip(reversed(ctx.blocks), reversed(ctx.saved))):
            if isinstance(st, _Recompute):
                with nvtx(f"block{n - 1 - j}.recompute"):
                    st = _rerun_dense(blk, st, B, T)
            sa, sm = st
            with nvtx(f"block{n - 1 - j}.mlp.bwd"):
                if _is_moe(blk):
                    moe_sublayer_bwd(blk, None, sm, dres, dres16, daux, ws["ln_scratch"])
                else:
                    _mlp_bwd(blk, sm, dres, dres16, ws)
            with nvtx(f"block{n - 1 - j}.attn.bwd"):
                _attn_bwd(blk, sa, dres, dres16, B, T, ws)
            if _BLOCK_DONE_HOOK is not None:
                _BLOCK_DONE_HOOK(blk)
        ctx.saved = None
        return dres, None, None, None, None


def blocks_fused(blocks, x: torch.Tensor, cfg, recompute: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Run a list of blocks (dense or MoE) on x [B, T, H]; returns (fp32 x, summed MoE aux loss).
    ``recompute``: dense blocks keep only their input and rerun their forward in backward."""
    B, T, H = x.shape
    x2 = x.reshape(B * T, H)
    if x2.dtype != torch.float32:
        x2 = x2.float()
    out, aux = _Body.apply(x2.contiguous(), list(blocks), B, T, bool(recompute))
    return out.view(B, T, H), aux


# ---------------------------------------------------------------------------
# Single-pass cross-entropy (forward and gradient in one kernel while each logit
# row is in L2): the default, measured 12% faster than the two-kernel pair on a
# B200 at 8192 x 50304 (416 vs 471 us); HB_CE_FUSED=0 selects the pair.
CE_FUSED = os.environ.get("HB_CE_FUSED", "1") == "1"


class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, ln_w, ln_b, wte, targets, V, want_logits, grad_hint=1.0, grad_scale=None):
        M, H = x.shape
        Vp = _vpad(V)
        dt = wte.w16.dtype
        xn, mean, rstd = K.layernorm_fwd(x, ln_w, ln_b, LN_EPS, dtype=dt)
        logits = torch.empty(M, Vp, device=x.device, dtype=dt)
        G.gemm(xn, wte.w16, logits, Vp, G.EPI_BF16, False, False)
        logits_out = logits[:, :V].float() if want_logits else None
        if targets is None:
            ctx.mark_non_differentiable(logits_out) if logits_out is not None else None
            return torch.zeros((), device=x.device), logits_out
        # rows the mean runs over (targets equal to ignore_index count for nothing, as in
        # F.cross_entropy): the gradient scale is dloss / n_valid, like the forward's mean
        n_valid = (targets != -100).sum().float().clamp_min_(1.0).reshape(1)
        ctx.ce_fused = CE_FUSED and not want_logits
        if ctx.ce_fused:
            # the gradient is written now, scaled for the upstream gradient the caller expects
            # (grad_hint, times the fp16 loss scale the caller multiplies the loss by);
            # backward corrects it only if the actual one differs
            expected = torch.full((1,), float(grad_hint), device=x.device, dtype=torch.float32)
            if grad_scale is not None:
                expected = expected * grad_scale
            loss, lse = K.cross_entropy_fused_(logits, V, targets, (expected / n_valid).contiguous())
            n_valid = expected
        else:
            loss, lse, _ = K.cross_entropy_fwd(logits, V, targets)
        ctx.save_for_backward(x, xn, mean, rstd, logits, lse, targets, n_valid)
        ctx.ln_w, ctx.ln_b, ctx.wte, ctx.V = ln_w, ln_b, wte, V
        if logits_out is not None:
            ctx.mark_non_differentiable(logits_out)
        return loss, logits_out

    @staticmethod
    def backward(ctx, dloss, _dlogits):
        x, xn, mean, rstd, logits, lse, targets, n_valid = ctx.saved_tensors
        V = ctx.V
        M, H = x.shape
        if ctx.ce_fused:  # n_valid holds the expected upstream gradient here
            dl = K.cross_entropy_rescale_(logits, dloss.reshape(1).float().contiguous(), n_valid)
        else:
            dl = K.cross_entropy_bwd_(logits, V, targets, lse, (dloss.reshape(1).float() / n_valid).contiguous(), 1.0)
        dlv = dl[:, :V]
        dxn = G.linear_dgrad(dlv, ctx.wte.w16, f32=True)
        G.linear_wgrad(dl, xn, out=ctx.wte.main_grad, accumulate=True, n_rows=V)
        dx = torch.empty_like(x)
        dx16 = torch.empty(x.shape, device=x.device, dtype=xn.dtype)
        zero = torch.zeros_like(x)
        K.layernorm_bwd(dxn, x, mean, rstd, ctx.ln_w, zero, dx, dx16, ctx.ln_w.main_grad, ctx.ln_b.main_grad)
        return dx, None, None, None, None, None, None, None, None


def head_fused(ln_f, wte: torch.nn.Parameter, x: torch.Tensor, targets: Optional[torch.Tensor], V: int,
               want_logits: bool = True, grad_hint: float = 1.0, grad_scale: Optional[torch.Tensor] = None):
    """ln_f -> lm_head (tied to wte) -> cross-entropy. Returns (logits fp32 | None, loss | None).

    ``grad_hint`` / ``grad_scale``: the upstream gradient the caller will send (a float,
    times an optional device scalar such as the fp16 loss scale)."""
    B, T, H = x.shape
    x2 = x.reshape(B * T, H)
    if x2.dtype != torch.float32:
        x2 = x2.float()
    t = targets.reshape(-1).contiguous() if targets is not None else None
    loss, logits = _Head.apply(x2.contiguous(), ln_f.weight, ln_f.bias, wte, t, V, want_logits, grad_hint,
                               grad_scale)
    if logits is not None:
        logits = logits.view(B, T, V)
    return logits, (loss if targets is not None else None)


def gpt_forward_fused(model, idx: torch.Tensor, targets: Optional[torch.Tensor], return_logits: bool = True):
    cfg = model.cfg
    topo = getattr(model, "topo", None)
    if topo is not None and getattr(topo, "tp", 1) > 1:
        return _gpt_forward_fused_tp(model, idx, targets)
    x = embed_fused(model.tr.wte.weight, model.tr.wpe.weight, idx)
    x, aux = blocks_fused(model.tr.h, x, cfg, recompute=getattr(model, "recompute", False))
    logits, loss = head_fused(model.tr.ln_f, model.lm_head.weight, x, targets, cfg.vocab_size,
                              want_logits=return_logits, grad_hint=getattr(model, "loss_grad_hint", 1.0),
                              grad_scale=getattr(model, "loss_grad_scale", None))
    return logits, loss, aux


def _gpt_forward_fused_tp(model, idx, targets):
    """Tensor-parallel forward on this rank's token shard (whole sequences).

    The returned loss is this shard's mean loss divided by tp, so that the sum
    over the TP group is the dense model's mean loss (and the gradients match)."""
    from .fused_tp import blocks_fused_tp, tp_shard_rows, tp_supported

    cfg, topo = model.cfg, model.topo
    B, T = idx.shape
    ok, why = tp_supported(cfg, topo, B, T)
    if not ok:
        raise ValueError(f"fused tensor parallelism: {why}")
    r0, Ms = tp_shard_rows(topo, B, T)
    Bs = Ms // T
    idx_s = idx.reshape(-1)[r0:r0 + Ms].view(Bs, T)
    x = embed_fused(model.tr.wte.weight, model.tr.wpe.weight, idx_s)
    x, aux = blocks_fused_tp(model.tr.h, x.reshape(Ms, -1), cfg, topo, B, T)
    tgt = targets.reshape(-1)[r0:r0 + Ms].view(Bs, T) if targets is not None else None
    logits, loss = head_fused(model.tr.ln_f, model.lm_head.weight, x.view(Bs, T, -1), tgt, cfg.vocab_size,
                              want_logits=False, grad_hint=getattr(model, "loss_grad_hint", 1.0) / topo.tp,
                              grad_scale=getattr(model, "loss_grad_scale", None))
    # Each TP rank routes only its token shard; the shard aux losses / tp sum to
    # the mean over shards (the dense aux uses all tokens at once).
    return None, (loss / topo.tp if loss is not None else None), aux / topo.tp


def enable_fused(module: torch.nn.Module, cfg, topo=None) -> bool:
    """Switch a GPT / StageModule to the fused path if the config is covered.

    Requires parameters already flattened (``p.w16`` / ``p.main_grad``)."""
    ok, why = fused_supported(cfg, topo)
    if ok:
        module.fused = True
    return ok
