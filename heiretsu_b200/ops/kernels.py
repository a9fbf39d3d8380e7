"""Thin Python wrappers over the extension's non-GEMM kernels.

Every wrapper allocates its outputs (unless given) with the PyTorch caching
allocator on the current stream and launches exactly one sm_100a kernel
sequence; nothing here falls back to a PyTorch implementation.
"""
from __future__ import annotations

from typing import Optional

import torch

from ._C import load


def _ext():
    return load()


# ---------------------------------------------------------------------------
# LayerNorm
# ---------------------------------------------------------------------------
def layernorm_fwd(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5,
                  dtype: torch.dtype = torch.bfloat16):
    """fp32 x [M, H] -> (y [M, H] in the 16-bit ``dtype`` (bf16 or fp16), mean [M], rstd [M])."""
    M = x.numel() // x.shape[-1]
    y = torch.empty(x.shape, device=x.device, dtype=dtype)
    mean = torch.empty(M, device=x.device, dtype=torch.float32)
    rstd = torch.empty(M, device=x.device, dtype=torch.float32)
    _ext().layernorm_fwd(x, w, b, y, mean, rstd, eps)
    return y, mean, rstd


def layernorm_bwd(dy, x, mean, rstd, w, dres_in, dres, dres16, dgamma, dbeta, scratch=None, dy_srcs: int = 1):
    """dres = dres_in + dLN/dx(dy); dres16 = 16-bit(dres); dgamma/dbeta (fp32) += partials.

    With ``dy_srcs > 1`` the output gradient is the sum of that many [M, H]
    slots of ``dy`` (the receive buffer of a reduce-scatter)."""
    H = x.shape[-1]
    M = x.numel() // H
    if scratch is None:
        rows = _ext().layernorm_bwd_scratch_rows(M)
        scratch = torch.empty(rows * 2 * H, device=x.device, dtype=torch.float32)
    _ext().layernorm_bwd(dy, x, mean, rstd, w, dres_in, dres, dres16, scratch, dgamma, dbeta, dy_srcs)


def resid_sum_ln(x, parts, nsrc, bias, x_new, w=None, b=None, y=None, mean=None, rstd=None, eps: float = 1e-5):
    """x_new = x + sum of `nsrc` 16-bit partial slots + bias; optionally y = LN(x_new) (16-bit, the slots' format)."""
    _ext().resid_sum_ln(x, parts, nsrc, bias, x_new, w, b, y, mean, rstd, eps)


def colsum_bf16(x: torch.Tensor, out: torch.Tensor) -> None:
    """out (fp32) += column sums of 16-bit (bf16 or fp16) x [M, N]."""
    _ext().colsum_bf16(x, out)


# ---------------------------------------------------------------------------
# Cross-entropy
# ---------------------------------------------------------------------------
def cross_entropy_fwd(logits: torch.Tensor, V: int, targets: torch.Tensor, ignore_index: int = -100):
    """16-bit logits [M, Vp] -> (mean loss (0-d fp32), lse [M], per-row loss [M])."""
    M = logits.shape[0]
    lse = torch.empty(M, device=logits.device, dtype=torch.float32)
    rows = torch.empty(M, device=logits.device, dtype=torch.float32)
    mean = torch.empty((), device=logits.device, dtype=torch.float32)
    _ext().cross_entropy_fwd(logits, V, targets, ignore_index, lse, rows, mean)
    return mean, lse, rows


def cross_entropy_fused_(logits: torch.Tensor, V: int, targets: torch.Tensor, scale: torch.Tensor,
                         ignore_index: int = -100):
    """Forward and gradient in one pass: returns (mean loss, lse) and leaves
    (softmax - onehot) * scale in ``logits`` (columns >= V zeroed); ``scale`` fp32 [1]."""
    M = logits.shape[0]
    lse = torch.empty(M, device=logits.device, dtype=torch.float32)
    rows = torch.empty(M, device=logits.device, dtype=torch.float32)
    mean = torch.empty((), device=logits.device, dtype=torch.float32)
    _ext().cross_entropy_fused(logits, V, targets, ignore_index, lse, rows, mean, scale)
    return mean, lse


def cross_entropy_rescale_(g: torch.Tensor, actual: torch.Tensor, expected: torch.Tensor) -> torch.Tensor:
    """In place g *= actual / expected (fp32 [1] device scalars); nothing happens when equal."""
    _ext().cross_entropy_rescale(g, actual, expected)
    return g


def cross_entropy_bwd_(logits, V, targets, lse, scale: Optional[torch.Tensor], scale_mul: float,
                       ignore_index: int = -100) -> torch.Tensor:
    """In place: logits <- (softmax - onehot) * scale * scale_mul (columns >= V zeroed)."""
    _ext().cross_entropy_bwd(logits, V, targets, ignore_index, lse, scale, scale_mul)
    return logits


# ---------------------------------------------------------------------------
# Embedding
# ---------------------------------------------------------------------------
def embedding_fwd(idx: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor) -> torch.Tensor:
    B, T = idx.shape
    out = torch.empty(B * T, wte.shape[1], device=idx.device, dtype=torch.float32)
    _ext().embedding_fwd(idx, wte, wpe, out)
    return out


def embedding_bwd(idx, dx, dwte: Optional[torch.Tensor], dwpe: Optional[torch.Tensor]) -> None:
    _ext().embedding_bwd(idx, dx, dwte, dwpe)


# ---------------------------------------------------------------------------
# Optimizer pieces
# ---------------------------------------------------------------------------
def sumsq(x: torch.Tensor, out: torch.Tensor, weight: float = 1.0, accumulate: bool = False, scratch=None):
    """out (0-d fp32) (+)= weight * sum(x^2), deterministic two-pass."""
    if scratch is None:
        scratch = torch.empty(_ext().sumsq_scratch_size(), device=x.device, dtype=torch.float32)
    _ext().sumsq(x, scratch, weight, out, accumulate)


def clip_coef(norm2: torch.Tensor, max_norm: float, coef: torch.Tensor, norm: Optional[torch.Tensor] = None,
              loss_scale: Optional[torch.Tensor] = None):
    """coef = min(1, max_norm / norm) (NaN when the norm is not finite). With ``loss_scale``
    (fp32 device scalar S) the gradients hold S * g: the norm is unscaled and coef carries 1/S."""
    _ext().clip_coef(norm2, max_norm, coef, norm, loss_scale)


def loss_scale_update(coef: torch.Tensor, state: torch.Tensor, growth: float = 2.0, backoff: float = 0.5,
                      interval: int = 2000) -> None:
    """Dynamic loss scale on the device: state = [scale, finite steps in a row] (fp32)."""
    _ext().loss_scale_update(coef, state, growth, backoff, interval)


def adamw_step(p, grad, m, v, p16, hyper, coef=None):
    _ext().adamw_step(p, grad, m, v, p16, hyper, coef)


def f32_to_bf16(x: torch.Tensor, y: Optional[torch.Tensor] = None, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """fp32 -> 16-bit copy (into ``y``, else a new tensor of ``dtype``: bf16 or fp16)."""
    if y is None:
        y = torch.empty(x.shape, device=x.device, dtype=dtype)
    _ext().f32_to_bf16(x, y)
    return y


# ---------------------------------------------------------------------------
# Attention (causal; head_dim 16, 32, 64 or 128)
# ---------------------------------------------------------------------------
def attention_fwd(qkv: torch.Tensor, B: int, T: int, nh: int, out: Optional[torch.Tensor] = None, drop=None,
                  head_dim: int = 64):
    """qkv [B*T, 3*nh*dh] (bf16 or fp16) -> (y [B*T, nh*dh] same format, nlse fp32 [B, nh, Tpad]), dh = head_dim.

    nlse = -log2(sum_k 2^(s_k * log2(e) / sqrt(dh))) per query row: the negated
    log2-domain log-sum-exp, kept in the form the backward kernel consumes.
    Natural-log LSE = -nlse * ln(2).

    ``drop = (seed_tensor, site, p, h0, nh_total)`` applies dropout to the
    attention probabilities (mask of heads h0 .. h0+nh-1 of nh_total; see
    ops/dropout_ref.py); the backward must get the same ``drop``."""
    Tpad = (T + 127) // 128 * 128
    if out is None:
        out = torch.empty(B * T, nh * head_dim, device=qkv.device, dtype=qkv.dtype)
    lse = torch.empty(B, nh, Tpad, device=qkv.device, dtype=torch.float32)
    d_seed, d_site, d_p, h0, nht = drop if drop is not None else (None, 0, 0.0, 0, 0)
    _ext().attention_fwd(qkv, B, T, nh, out, lse, d_seed, int(d_site), float(d_p), int(h0), int(nht), int(head_dim))
    return out, lse


def attention_bwd(qkv, out, dout, lse, B, T, nh, dqkv: Optional[torch.Tensor] = None, drop=None,
                  head_dim: int = 64):
    """Returns dqkv [B*T, 3*nh*dh] in qkv's format (columns [dQ | dK | dV])."""
    Tpad = (T + 127) // 128 * 128
    if dqkv is None:
        dqkv = torch.empty(B * T, 3 * nh * head_dim, device=qkv.device, dtype=qkv.dtype)
    dvec = torch.empty(B, nh, Tpad, device=qkv.device, dtype=torch.float32)
    dq_acc = torch.empty(B * T, nh * max(head_dim, 64), device=qkv.device, dtype=torch.float32)
    d_seed, d_site, d_p, h0, nht = drop if drop is not None else (None, 0, 0.0, 0, 0)
    _ext().attention_bwd(qkv, out, dout, lse, B, T, nh, dvec, dq_acc, dqkv, d_seed, int(d_site), float(d_p), int(h0),
                         int(nht), int(head_dim))
    return dqkv


def dropout_bf16(g: torch.Tensor, seed: torch.Tensor, site: int, p: float, row0: int = 0,
                 out: Optional[torch.Tensor] = None, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """16-bit(g * mask) for residual dropout site ``site`` (g fp32 [M, H]; out bf16 or fp16)."""
    if out is None:
        out = torch.empty(g.shape, device=g.device, dtype=dtype)
    _ext().dropout_bf16(g, out, seed, int(site), float(p), int(row0))
    return out
