"""PyTorch restatement of the counter-based dropout masks of csrc/dropout.cuh.

Element pairs are hashed: pair index n -> 32 bits; the low 16 bits decide
element 2n, the high 16 bits element 2n+1 (kept when >= thresh, thresh =
round(p * 65536); kept values are scaled by 1 / (1 - p)).

Index conventions (pair index = element index // 2):
  residual dropout of a sub-layer output [M, H] (rows offset by ``row0``
    for token shards): element = (row0 + row) * H + col
  attention probabilities, head h of nh_total, batch b, query q, key k:
    element = ((b * nh_total + h) * T + q) * T + k
"""
from __future__ import annotations

import torch

M32 = 0xFFFFFFFF


def _u32(x: torch.Tensor) -> torch.Tensor:
    return x & M32


def lowbias32(x: torch.Tensor) -> torch.Tensor:
    x = _u32(x)
    x = x ^ (x >> 16)
    x = _u32(x * 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _u32(x * 0x846CA68B)
    x = x ^ (x >> 16)
    return x


def _lowbias32_int(x: int) -> int:
    return int(lowbias32(torch.tensor([x], dtype=torch.int64))[0])


def site_key(seed: int, site: int) -> int:
    return _lowbias32_int((seed & M32) ^ _lowbias32_int((site * 0x9E3779B9 + 0x85EBCA6B) & M32))


def pair_bits(key: int, pair: torch.Tensor) -> torch.Tensor:
    lo = pair & M32
    hi = pair >> 32
    return lowbias32(lo ^ key ^ _u32(hi * 0xC2B2AE35))


def multipliers(seed: int, site: int, elem: torch.Tensor, p: float) -> torch.Tensor:
    """Float multipliers (0 or 1/(1-p)) for int64 element indices."""
    thresh = int(round(p * 65536))
    bits = pair_bits(site_key(seed, site), elem >> 1)
    u = torch.where((elem & 1) == 0, bits & 0xFFFF, bits >> 16)
    return torch.where(u >= thresh, torch.tensor(1.0 / (1.0 - p), dtype=torch.float64),
                       torch.tensor(0.0, dtype=torch.float64))


def residual_mask(seed: int, site: int, M: int, H: int, p: float, row0: int = 0) -> torch.Tensor:
    r = torch.arange(M, dtype=torch.int64)[:, None] + row0
    c = torch.arange(H, dtype=torch.int64)[None, :]
    return multipliers(seed, site, r * H + c, p)


def attention_mask(seed: int, site: int, B: int, nh: int, T: int, p: float, h0: int = 0,
                   nh_total: int = None) -> torch.Tensor:
    """[B, nh, T, T] multipliers for heads h0 .. h0+nh-1 of nh_total."""
    nh_total = nh_total or nh
    b = torch.arange(B, dtype=torch.int64)[:, None, None, None]
    h = torch.arange(nh, dtype=torch.int64)[None, :, None, None] + h0
    q = torch.arange(T, dtype=torch.int64)[None, None, :, None]
    k = torch.arange(T, dtype=torch.int64)[None, None, None, :]
    return multipliers(seed, site, ((b * nh_total + h) * T + q) * T + k, p)
