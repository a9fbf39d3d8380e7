"""Autoregressive sampling from a trained GPT, with a key/value cache.

The reference has no inference path (its README covers training only); this
adds one on the plain modules, so it runs on any device and on tensor- or
expert-parallel ranks: the column/row-parallel layers and the MoE all-to-alls
work on any token count, and every rank of a TP/EP group computes the same
logits, so ranks that sample with equally seeded generators pick the same
tokens and stay in lockstep.

Decoding: one prefill forward over the prompt fills each layer's cache with
K and V of the rank's heads; each new token then runs the blocks on one
position, attending to the cached keys. ``kv_cache=False`` re-runs the whole
context every step (the window cropped to ``block_size``), which is the
oracle of the tests.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn.functional as F


class KVCache:
    """K and V of every layer, [B, heads of this rank, block_size, head_dim]."""

    def __init__(self, model, batch: int, device, dtype):
        cfg = model.cfg
        self.k: List[torch.Tensor] = []
        self.v: List[torch.Tensor] = []
        for blk in model.tr.h:
            a = blk.attn
            self.k.append(torch.zeros(batch, a.nh_tp, cfg.block_size, a.dh, device=device, dtype=dtype))
            self.v.append(torch.zeros(batch, a.nh_tp, cfg.block_size, a.dh, device=device, dtype=dtype))
        self.len = 0


def _attn_cached(attn, x: torch.Tensor, ck: torch.Tensor, cv: torch.Tensor, pos: int) -> torch.Tensor:
    """Attention of positions pos .. pos+S-1 over the cached keys 0 .. pos+S-1 (no dropout)."""
    B, S, _ = x.shape
    qkv = attn.c_attn(x)
    q, k, v = qkv.view(B, S, 3, attn.nh_tp, attn.dh).permute(2, 0, 3, 1, 4).unbind(0)
    ck[:, :, pos:pos + S] = k
    cv[:, :, pos:pos + S] = v
    keys, vals = ck[:, :, :pos + S], cv[:, :, :pos + S]
    if S == 1:
        y = F.scaled_dot_product_attention(q, keys, vals)
    else:  # query i (absolute position pos + i) sees keys 0 .. pos + i
        allowed = torch.ones(S, pos + S, dtype=torch.bool, device=x.device).tril(diagonal=pos)
        y = F.scaled_dot_product_attention(q, keys, vals, attn_mask=allowed)
    y = y.transpose(1, 2).reshape(B, S, attn.h_tp)
    return attn.c_proj(y, input_is_parallel=True)


@torch.no_grad()
def _forward_cached(model, idx: torch.Tensor, cache: KVCache) -> torch.Tensor:
    """Logits of the last position of ``idx`` (the tokens after ``cache.len``)."""
    B, S = idx.shape
    pos = cache.len
    x = model.tr.wte(idx) + model.tr.wpe(torch.arange(pos, pos + S, device=idx.device))[None]
    for blk, ck, cv in zip(model.tr.h, cache.k, cache.v):
        x = x + _attn_cached(blk.attn, blk.ln_1(x), ck, cv, pos)
        h = blk.ln_2(x)
        x = x + (blk.moe(h)[0] if hasattr(blk, "moe") else blk.mlp(h))
    cache.len = pos + S
    return model.lm_head(model.tr.ln_f(x[:, -1:, :]))[:, -1, :]


def _pick(logits: torch.Tensor, temperature: float, top_k: Optional[int], generator) -> torch.Tensor:
    if temperature <= 0:
        return logits.argmax(dim=-1, keepdim=True)
    logits = logits.float() / temperature
    if top_k is not None and top_k < logits.size(-1):
        kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    probs = torch.softmax(logits, dim=-1)
    return torch.multinomial(probs, 1, generator=generator)


@torch.no_grad()
def generate(model, idx: torch.Tensor, max_new_tokens: int, temperature: float = 1.0, top_k: Optional[int] = None,
             generator: Optional[torch.Generator] = None, kv_cache: bool = True) -> torch.Tensor:
    """Extend ``idx`` [B, T0] by ``max_new_tokens`` sampled tokens; returns [B, T0 + new].

    ``temperature <= 0`` picks the most likely token. With ``kv_cache`` the total
    length must fit in ``block_size``; without it the context is cropped to the
    last ``block_size`` tokens, as training saw them."""
    cfg = model.cfg
    was_training, was_fused = model.training, getattr(model, "fused", False)
    model.eval()
    model.fused = False  # plain modules: any sequence length, fp32 master weights
    try:
        if kv_cache:
            if idx.size(1) + max_new_tokens > cfg.block_size:
                raise ValueError(f"prompt {idx.size(1)} + {max_new_tokens} new tokens > block_size {cfg.block_size}"
                                 " (use kv_cache=False to slide the window)")
            cache = KVCache(model, idx.size(0), idx.device, model.tr.wte.weight.dtype)
            logits = _forward_cached(model, idx, cache)
            for i in range(max_new_tokens):
                nxt = _pick(logits, temperature, top_k, generator)
                idx = torch.cat([idx, nxt], dim=1)
                if i + 1 < max_new_tokens:
                    logits = _forward_cached(model, nxt, cache)
            return idx
        for _ in range(max_new_tokens):
            ctx = idx[:, -cfg.block_size:]
            logits, _, _ = model(ctx)
            nxt = _pick(logits[:, -1, :], temperature, top_k, generator)
            idx = torch.cat([idx, nxt], dim=1)
        return idx
    finally:
        model.train(was_training)
        model.fused = was_fused
