"""Fused tensor-parallel execution (sm_100a kernels + NVLink peer memory).

Same math as the reference's Megatron TP (tp_linear.py:19-312): column-parallel
QKV / FC with the input replicated, row-parallel projections whose partial
outputs are summed over the TP group. The B200 form keeps the residual stream
sharded by tokens between the TP GEMMs (sequence parallelism), which turns
each all-reduce into a reduce-scatter plus the next layer's all-gather, and
fuses both into the GEMMs:

* AG -> GEMM: the column-parallel GEMM gathers the token shards of its input
  from the peers inside the kernel (heiretsu_b200/csrc/gemm_kernel.cuh,
  ``ag_copy_units``) while it already multiplies the rows that have arrived.
* GEMM -> RS: the row-parallel GEMM stores each partial output tile straight
  into the owning rank's receive slot over NVLink; ``resid_sum_ln`` then sums
  the slots with the bias and the residual and applies the next LayerNorm.

Backward mirrors it: dgrad of a row-parallel layer is AG -> GEMM (with the
GELU derivative fused), dgrad of a column-parallel layer is GEMM -> RS into
fp32 slots consumed by the LayerNorm backward. Weight gradients use the
gathered activations kept from forward. Parameters replicated over TP
(LayerNorms, row-parallel biases, embeddings) accumulate token-shard partial
gradients, summed over the group once per step (``tp_sync_grads``).

Dropout (on by default; ``--fused_tp_dropout 0`` sends such runs to the plain engine) uses the masks of the single-GPU
fused path, indexed by global head and global token row, so every TP rank
draws distinct masks from the one seed: the attention kernels take the
rank's first head (h0 = tp_rank * heads per rank), and a residual site sums
the partial outputs with the bias, keeps bf16(mask * sum) and adds it to the
fp32 residual shard (token rows from tp_rank * Ms). Backward masks the
residual-gradient shard into the gather source before the all-gather GEMM,
so both the weight gradient and the bias column sum see the masked gradient.

Ordering between ranks uses device barriers (bounded waits) on the TP group:
before every gather (sources written) and after every scatter (partials
delivered); gather sources alternate between two buffers so a rank never
overwrites a shard a peer may still be reading.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from ..ops import gemm as G
from ..ops import kernels as K
from ..ops._C import load as _ext

LN_EPS = 1e-5


class TPComm:
    """Symmetric buffers and barriers of one TP group for one activation shape."""

    def __init__(self, topo, Ms: int, H: int, device: torch.device, dtype: torch.dtype = torch.bfloat16):
        from ..parallel.symm import SymmetricBuffer

        g = topo.tp_group
        self.tp, self.rank, self.Ms, self.H = topo.tp, topo.tp_rank, Ms, H
        self.dtype = dtype  # 16-bit format of the gathered / reduce-scattered activations
        self.src = [SymmetricBuffer(g, Ms * H * 2, device) for _ in range(2)]
        self.recv16 = SymmetricBuffer(g, self.tp * Ms * H * 2, device)
        self.recv32 = SymmetricBuffer(g, self.tp * Ms * H * 4, device)
        self.flags = torch.zeros(self.tp * Ms // 128 + 1, dtype=torch.int32, device=device)
        self.zero32 = None  # [Ms, H] fp32 zeros: the residual input of a dropout site's partial sum

    def zeros(self) -> torch.Tensor:
        if self.zero32 is None:
            self.zero32 = torch.zeros(self.Ms, self.H, dtype=torch.float32, device=self.src[0].device)
        return self.zero32

    def barrier(self) -> None:
        self.src[0].barrier()

    def src_view(self, i: int) -> torch.Tensor:
        return self.src[i].tensor(self.dtype, self.Ms * self.H).view(self.Ms, self.H)

    def recv16_all(self) -> torch.Tensor:
        return self.recv16.tensor(self.dtype, self.tp * self.Ms * self.H).view(self.tp * self.Ms, self.H)

    def recv32_all(self) -> torch.Tensor:
        return self.recv32.tensor(torch.float32, self.tp * self.Ms * self.H).view(self.tp * self.Ms, self.H)

    def ag(self, i: int):
        return (self.src[i].ptrs, self.flags, self.rank, self.Ms)

    def rs16(self):
        return (self.recv16.ptrs, self.rank, self.Ms)

    def rs32(self):
        return (self.recv32.ptrs, self.rank, self.Ms)


_COMMS = {}


def get_comm(topo, Ms: int, H: int, device, dtype: torch.dtype = torch.bfloat16) -> TPComm:
    key = (id(topo.tp_group), Ms, H, str(device), dtype)
    if key not in _COMMS:
        _COMMS[key] = TPComm(topo, Ms, H, device, dtype)
    return _COMMS[key]


def _empty(*shape, dtype, device=None):
    return torch.empty(*shape, dtype=dtype, device=device)


def _resid_dropout(comm: TPComm, x_s: torch.Tensor, bias, d, site: int) -> torch.Tensor:
    """x_s + bf16(mask * (sum of the TP partial outputs + bias)): a residual dropout site on the
    token shard (global token rows from tp_rank * Ms, so the mask is the single-GPU one)."""
    t = torch.empty_like(x_s)
    K.resid_sum_ln(comm.zeros(), comm.recv16_all(), comm.tp, bias, t)
    kept = K.dropout_bf16(t, d[0], site, d[2], row0=comm.rank * comm.Ms, dtype=comm.dtype)
    return x_s + kept.float()


def _attn_drop(attn, comm: TPComm, d):
    return (d[0], 4 * d[1], d[2], comm.rank * attn.nh_tp, attn.nh_tp * comm.tp) if d else None


def tp_block_fwd(blk, comm: TPComm, x_s: torch.Tensor, B: int, T: int, keep: bool):
    """x_s: fp32 residual token shard [Ms, H] -> next residual shard; returns (x2_s, aux | None, saved)."""
    from .fused import _dropout_of

    attn, mlp = blk.attn, getattr(blk, "mlp", None)
    tp, Ms, H = comm.tp, comm.Ms, comm.H
    M = tp * Ms
    dev = x_s.device
    nh = attn.nh_tp
    ext = _ext()
    d = _dropout_of(blk)  # (seed snapshot, layer, p) in a training forward with dropout, else None
    # LN1 -> gather source 0
    xn_s = comm.src_view(0)
    m1 = _empty(Ms, dtype=torch.float32, device=dev)
    r1 = _empty(Ms, dtype=torch.float32, device=dev)
    ext.layernorm_fwd(x_s, blk.ln_1.weight, blk.ln_1.bias, xn_s, m1, r1, LN_EPS)
    comm.barrier()
    xn_full = _empty(M, H, dtype=comm.dtype, device=dev)
    n_qkv = 3 * attn.h_tp
    qkv = _empty(M, n_qkv, dtype=comm.dtype, device=dev)
    G.gemm(xn_full, attn.c_attn.weight.w16, qkv, n_qkv, G.EPI_BF16, False, False, bias=attn.c_attn.bias,
           ag=comm.ag(0))
    y, lse = K.attention_fwd(qkv, B, T, nh, drop=_attn_drop(attn, comm, d), head_dim=attn.dh)
    G.gemm(y, attn.c_proj.weight.w16, comm.recv16_all(), H, G.EPI_BF16, False, False, rs=comm.rs16())
    comm.barrier()
    x1_s = _empty(Ms, H, dtype=torch.float32, device=dev)
    if hasattr(blk, "moe"):
        # MoE sub-layer on this rank's tokens: no TP communication (experts are TP-replicated).
        from .fused_moe import moe_sublayer_fwd

        if d:
            x1_s = _resid_dropout(comm, x_s, attn.c_proj.bias, d, 4 * d[1] + 1)
        else:
            K.resid_sum_ln(x_s, comm.recv16_all(), tp, attn.c_proj.bias, x1_s)
        x2_s, aux, sm = moe_sublayer_fwd(blk, None, x1_s, keep)
        saved = ((x_s, m1, r1, xn_full, qkv, y, lse), sm, d) if keep else None
        return x2_s, aux, saved
    xn2_s = comm.src_view(1)
    m2 = _empty(Ms, dtype=torch.float32, device=dev)
    r2 = _empty(Ms, dtype=torch.float32, device=dev)
    if d:
        x1_s = _resid_dropout(comm, x_s, attn.c_proj.bias, d, 4 * d[1] + 1)
        ext.layernorm_fwd(x1_s, blk.ln_2.weight, blk.ln_2.bias, xn2_s, m2, r2, LN_EPS)
    else:
        K.resid_sum_ln(x_s, comm.recv16_all(), tp, attn.c_proj.bias, x1_s, blk.ln_2.weight, blk.ln_2.bias, xn2_s,
                       m2, r2, LN_EPS)
    comm.barrier()
    xn2_full = _empty(M, H, dtype=comm.dtype, device=dev)
    n_fc = mlp.c_fc.out_per_partition
    h = _empty(M, n_fc, dtype=comm.dtype, device=dev)
    pre = _empty(M, n_fc, dtype=comm.dtype, device=dev)
    G.gemm(xn2_full, mlp.c_fc.weight.w16, h, n_fc, G.EPI_BF16_GELU, False, False, bias=mlp.c_fc.bias, aux=pre,
           ag=comm.ag(1))
    G.gemm(h, mlp.c_proj.weight.w16, comm.recv16_all(), H, G.EPI_BF16, False, False, rs=comm.rs16())
    comm.barrier()
    if d:
        x2_s = _resid_dropout(comm, x1_s, mlp.c_proj.bias, d, 4 * d[1] + 2)
    else:
        x2_s = _empty(Ms, H, dtype=torch.float32, device=dev)
        K.resid_sum_ln(x1_s, comm.recv16_all(), tp, mlp.c_proj.bias, x2_s)
    saved = ((x_s, m1, r1, xn_full, qkv, y, lse), (x1_s, m2, r2, xn2_full, pre, h), d) if keep else None
    return x2_s, None, saved


def tp_block_bwd(blk, comm: TPComm, saved, dres: torch.Tensor, k: int, B: int, T: int, ln_scratch,
                 daux: Optional[torch.Tensor] = None) -> int:
    """dres: fp32 residual-gradient shard (updated in place); its bf16 copy is in gather source k.
    Returns the gather source holding the bf16 copy of the new dres."""
    attn, mlp = blk.attn, getattr(blk, "mlp", None)
    tp, Ms, H = comm.tp, comm.Ms, comm.H
    M = tp * Ms
    dev = dres.device
    nh = attn.nh_tp
    (x_s, m1, r1, xn_full, qkv, y, lse), sm, d = saved
    if hasattr(blk, "moe"):
        from .fused_moe import moe_sublayer_bwd

        k = 1 - k
        moe_sublayer_bwd(blk, None, sm, dres, comm.src_view(k), daux, ln_scratch)
        return _tp_attn_bwd(blk, comm, (x_s, m1, r1, xn_full, qkv, y, lse), dres, k, B, T, ln_scratch, d)
    x1_s, m2, r2, xn2_full, pre, h = sm
    n_fc = mlp.c_fc.out_per_partition
    # --- MLP: x2 = x1 + drop(RS(c_proj(gelu(c_fc(AG(ln_2(x1)))))))
    if d:  # the gathered gradient of c_proj's output is the masked residual gradient
        K.dropout_bf16(dres, d[0], 4 * d[1] + 2, d[2], row0=comm.rank * Ms, out=comm.src_view(k))
    comm.barrier()
    dx2_full = _empty(M, H, dtype=comm.dtype, device=dev)
    dpre = _empty(M, n_fc, dtype=comm.dtype, device=dev)
    G.gemm(dx2_full, mlp.c_proj.weight.w16, dpre, n_fc, G.EPI_BF16_DGELU, False, True, aux=pre, ag=comm.ag(k))
    G.linear_wgrad(dx2_full, h, out=mlp.c_proj.weight.main_grad, accumulate=True)
    K.colsum_bf16(comm.src_view(k), mlp.c_proj.bias.main_grad)  # token-shard partial; summed over TP per step
    G.gemm(dpre, mlp.c_fc.weight.w16, comm.recv32_all(), H, G.EPI_F32, False, True, rs=comm.rs32())
    G.linear_wgrad(dpre, xn2_full, out=mlp.c_fc.weight.main_grad, accumulate=True)
    K.colsum_bf16(dpre, mlp.c_fc.bias.main_grad)
    del dpre, dx2_full
    comm.barrier()
    k = 1 - k
    K.layernorm_bwd(comm.recv32_all(), x1_s, m2, r2, blk.ln_2.weight, dres, dres, comm.src_view(k),
                    blk.ln_2.weight.main_grad, blk.ln_2.bias.main_grad, scratch=ln_scratch, dy_srcs=tp)
    return _tp_attn_bwd(blk, comm, (x_s, m1, r1, xn_full, qkv, y, lse), dres, k, B, T, ln_scratch, d)


def _tp_attn_bwd(blk, comm: TPComm, saved, dres: torch.Tensor, k: int, B: int, T: int, ln_scratch, d=None) -> int:
    """Attention sub-layer backward: x1 = x + drop(RS(c_proj(attn(c_attn(AG(ln_1(x)))))))."""
    attn = blk.attn
    tp, Ms, H = comm.tp, comm.Ms, comm.H
    M = tp * Ms
    dev = dres.device
    nh = attn.nh_tp
    x_s, m1, r1, xn_full, qkv, y, lse = saved
    if d:
        K.dropout_bf16(dres, d[0], 4 * d[1] + 1, d[2], row0=comm.rank * Ms, out=comm.src_view(k))
    comm.barrier()
    dx1_full = _empty(M, H, dtype=comm.dtype, device=dev)
    dy = _empty(M, attn.h_tp, dtype=comm.dtype, device=dev)
    G.gemm(dx1_full, attn.c_proj.weight.w16, dy, attn.h_tp, G.EPI_BF16, False, True, ag=comm.ag(k))
    G.linear_wgrad(dx1_full, y, out=attn.c_proj.weight.main_grad, accumulate=True)
    K.colsum_bf16(comm.src_view(k), attn.c_proj.bias.main_grad)
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, T, nh, drop=_attn_drop(attn, comm, d), head_dim=attn.dh)
    del dy, dx1_full
    G.linear_wgrad(dqkv, xn_full, out=attn.c_attn.weight.main_grad, accumulate=True)
    K.colsum_bf16(dqkv, attn.c_attn.bias.main_grad)
    G.gemm(dqkv, attn.c_attn.weight.w16, comm.recv32_all(), H, G.EPI_F32, False, True, rs=comm.rs32())
    del dqkv
    comm.barrier()
    k = 1 - k
    K.layernorm_bwd(comm.recv32_all(), x_s, m1, r1, blk.ln_1.weight, dres, dres, comm.src_view(k),
                    blk.ln_1.weight.main_grad, blk.ln_1.bias.main_grad, scratch=ln_scratch, dy_srcs=tp)
    return k


class _TPBody(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_s, blocks, comm, B, T):
        from .fused import _snapshot_dropout_seeds

        keep = x_s.requires_grad
        saved = []
        aux_total = torch.zeros((), device=x_s.device, dtype=torch.float32)
        _snapshot_dropout_seeds(blocks)
        comm.barrier()
        for blk in blocks:
            x_s, aux, s = tp_block_fwd(blk, comm, x_s, B, T, keep)
            if aux is not None:
                aux_total = aux_total + aux
            saved.append(s)
        ctx.blocks, ctx.saved, ctx.comm, ctx.B, ctx.T = blocks, saved, comm, B, T
        return x_s, aux_total

    @staticmethod
    def backward(ctx, dx, daux):
        comm = ctx.comm
        if daux is None:
            daux = torch.zeros((), device=dx.device)
        dres = dx.contiguous().clone()
        comm.barrier()
        K.f32_to_bf16(dres, comm.src_view(0))
        rows = _ext().layernorm_bwd_scratch_rows(comm.Ms)
        ln_scratch = torch.empty(rows * 2 * comm.H, device=dres.device, dtype=torch.float32)
        k = 0
        for blk, s in zip(reversed(ctx.blocks), reversed(ctx.saved)):
            k = tp_block_bwd(blk, comm, s, dres, k, ctx.B, ctx.T, ln_scratch, daux)
        ctx.saved = None
        return dres, None, None, None, None


def tp_shard_rows(topo, B: int, T: int) -> Tuple[int, int]:
    """(first row, row count) of this TP rank's token shard of the [B*T] tokens."""
    Ms = B * T // topo.tp
    return topo.tp_rank * Ms, Ms


def tp_supported(cfg, topo, B: int, T: int) -> Tuple[bool, str]:
    tp = topo.tp
    if tp > 8:
        return False, "TP group larger than one NVSwitch node"
    if B % tp:
        return False, "batch size must be divisible by tp (token shards hold whole sequences)"
    if (B * T // tp) % 128:
        return False, "tokens per TP rank must be a multiple of 128"
    if cfg.n_embed % tp or (cfg.n_head // tp) < 1:
        return False, "heads must divide over tp"
    return True, ""


def blocks_fused_tp(blocks, x_s: torch.Tensor, cfg, topo, B: int, T: int):
    """Returns (x_L token shard, aux loss of this shard's MoE layers)."""
    comm = get_comm(topo, x_s.shape[0], x_s.shape[1], x_s.device, blocks[0].ln_1.weight.w16.dtype)
    return _TPBody.apply(x_s.contiguous(), list(blocks), comm, B, T)
