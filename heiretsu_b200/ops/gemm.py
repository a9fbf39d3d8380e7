"""Python wrappers of the tcgen05 GEMM (heiretsu_b200/csrc/gemm_kernel.cuh).

Three layouts cover every linear layer of the model without transposed
copies (reference einsums: tp_linear.py:148, :224, :301):

* ``linear_fwd``   y[M,N]  = x[M,K] @ W[N,K]^T   (+ bias, GELU or residual)
* ``linear_dgrad`` dx[M,K] = dy[M,N] @ W[N,K]    (optionally times GELU'(pre))
* ``linear_wgrad`` dW[N,K] (+)= dy[M,N]^T @ x[M,K]
"""
from __future__ import annotations

import os

from typing import Optional

import torch

from ._C import load

EPI_BF16 = 0
EPI_BF16_GELU = 1
EPI_F32 = 2
EPI_F32_ACC = 3
EPI_F32_RESID = 4
EPI_BF16_DGELU = 5


_BN_OVERRIDE = int(os.environ.get("HB_GEMM_BN", "0"))  # 128 / 192 / 256 forces one tile width (comparisons)


def _bn(n: int) -> int:
    """Output tile width: 256 when N is large enough to keep every SM busy at M = 8k, else 128."""
    if _BN_OVERRIDE:
        return _BN_OVERRIDE
    return 256 if n >= 2048 else 128


def _bn_f32_out(n: int) -> int:
    """Tile width for fp32-output GEMMs (residual forward, fp32 dgrad): 192 for
    768-class widths, where it measured 4-6% faster than 128 (4 tiles across
    instead of 6, less shared-memory operand traffic per MMA); bf16-output and
    weight-gradient GEMMs measured slower with 192 and keep _bn."""
    if _BN_OVERRIDE:
        return _BN_OVERRIDE
    if n % 192 == 0 and 576 <= n <= 1536:
        return 192
    return _bn(n)


def gemm(a, b, c, n, epi, a_mn, b_mn, bias=None, aux=None, resid=None, block_n=None, ag=None, rs=None, grp=None,
         drop=None, cmb=None):
    """D = A.B^T-style GEMM (see module doc). ``ag = (src_ptrs, flags, rank, rows)`` turns on
    the in-kernel all-gather of A's token shards; ``rs = (dst_ptrs, rank, rows)`` stores each
    output tile into its token owner's receive slot (reduce-scatter epilogue);
    ``grp = (mode, offsets, n_groups, b_off, c_off)`` runs an expert-grouped GEMM;
    ``drop = (seed_tensor, site, p, row0)`` applies residual dropout in the F32Resid epilogue;
    ``cmb = (slot_ptrs, inv, weights, K, tokens)`` adds the expert-parallel combine to a row-grouped
    16-bit GEMM: each output row, times its routing weight, goes to slot (k, t) of every EP rank."""
    ag_src, ag_flags, ag_rank, ag_rows = ag if ag is not None else ([], None, 0, 0)
    rs_dst, rs_rank, rs_rows = rs if rs is not None else ([], 0, 0)
    g_mode, g_off, g_n, g_b, g_c = grp if grp is not None else (0, None, 0, 0, 0)
    d_seed, d_site, d_p, d_row0 = drop if drop is not None else (None, 0, 0.0, 0)
    c_dst, c_inv, c_w, c_k, c_n = cmb if cmb is not None else ([], None, None, 0, 0)
    load().gemm(a, b, c, int(n), int(epi), bool(a_mn), bool(b_mn), bias, aux, resid,
                int(block_n if block_n is not None else _bn(n)), list(ag_src), ag_flags, int(ag_rank),
                int(ag_rows), list(rs_dst), int(rs_rank), int(rs_rows), int(g_mode), g_off, int(g_n), int(g_b),
                int(g_c), d_seed, int(d_site), float(d_p), int(d_row0), list(c_dst), c_inv, c_w, int(c_k), int(c_n))
    return c


def linear_fwd(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
               out: Optional[torch.Tensor] = None, n: Optional[int] = None) -> torch.Tensor:
    """y = x @ w^T + bias in x's 16-bit format. `n` may exceed w.shape[0] (rows beyond are zero)."""
    M = x.shape[0]
    N = int(n if n is not None else w.shape[0])
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=x.dtype)
    return gemm(x, w, out, N, EPI_BF16, False, False, bias=bias)


def linear_fwd_gelu(x, w, bias, *, out=None, pre=None):
    """Returns (gelu(x @ w^T + b), x @ w^T + b), both in x's 16-bit format."""
    M, N = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=x.dtype)
    if pre is None:
        pre = torch.empty(M, N, device=x.device, dtype=x.dtype)
    gemm(x, w, out, N, EPI_BF16_GELU, False, False, bias=bias, aux=pre)
    return out, pre


def linear_fwd_resid(x, w, bias, resid, *, out=None, drop=None):
    """fp32 out = resid + dropout(x @ w^T + bias) (out may be resid itself; ``drop`` as in gemm)."""
    N = w.shape[0]
    if out is None:
        out = torch.empty_like(resid)
    return gemm(x, w, out, N, EPI_F32_RESID, False, False, bias=bias, resid=resid, drop=drop,
                block_n=_bn_f32_out(N))


def linear_dgrad(dy, w, *, out=None, gelu_pre=None, f32=False):
    """dx = dy @ w (w: [N, K]); with `gelu_pre`, dx *= gelu'(gelu_pre)."""
    M, K = dy.shape[0], w.shape[1]
    if gelu_pre is not None:
        epi, dt = EPI_BF16_DGELU, dy.dtype
    else:
        epi, dt = (EPI_F32, torch.float32) if f32 else (EPI_BF16, dy.dtype)
    if out is None:
        out = torch.empty(M, K, device=dy.device, dtype=dt)
    return gemm(dy, w, out, K, epi, False, True, aux=gelu_pre, block_n=_bn_f32_out(K) if epi == EPI_F32 else None)


def linear_wgrad(dy, x, *, out=None, accumulate=False, n_rows=None):
    """dW[N,K] (+)= dy[:, :N]^T @ x in fp32; `n_rows` limits N (e.g. an unpadded vocab)."""
    N = int(n_rows if n_rows is not None else dy.shape[1])
    K = x.shape[1]
    if out is None:
        out = torch.zeros(N, K, device=dy.device, dtype=torch.float32)
        accumulate = False
    a = dy if N == dy.shape[1] else dy[:, :N]
    # Kernel view: D[n, k] = sum_m A(n, m) B(k, m) with A = dy and B = x both
    # stored with the reduction (token) dimension outermost: MN-major.
    return gemm(a, x, out, K, EPI_F32_ACC if accumulate else EPI_F32, True, True)
