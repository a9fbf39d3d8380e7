"""Fused mixture-of-experts sub-layer (router, permutation, grouped expert GEMMs, combine).

Forward, for the LayerNorm output xn [N, H] of this rank's tokens:

    route      logits = xn Wg^T -> softmax -> top-k -> renormalise; per-expert
               counts, padded segment offsets, row positions and the
               load-balancing aux loss (moe.cu; no host synchronisation)
    gather     xp[pos[t, k]] = xn[t]                 (expert-grouped, 128-padded)
    expert 1   hp = GELU(xp W1_e^T)                  (row-grouped tcgen05 GEMM)
    expert 2   yp = hp W2_e^T                        (row-grouped tcgen05 GEMM)
    combine    x_new[t] = x[t] + sum_k round16(w[t, k] yp[pos[t, k]])   (fp32 sum, k ascending)

The local experts' w1 (and w2) are stored back to back in the flat parameter
buffer, so each grouped GEMM reads one [E*I, H] weight matrix and picks the
expert's block from the m-block's segment. Backward mirrors every step; the
weight gradients use the reduction-grouped GEMM (tile = expert, m, n) over
exactly that expert's rows. Semantics are the reference's MoELayer
(moe.py:245-405) with routing weights and aux loss differentiable.

Expert parallelism (ep > 1). The EP ranks of one data replica hold the same
tokens (the reference shards data by DP rank only, train.py:322), so no
token ever has to travel: every EP rank routes all of its tokens (the router
is replicated), gathers only the rows of its own experts (window
[e0, e0 + E/ep) of the padded segments) and runs those experts once. The
combine's exchange happens inside the second expert GEMM: its epilogue
writes each output row (rounded to 16 bits, the value yp holds), times the
row's routing weight, as 16 bits into slot k, row t of every EP rank's
peer-mapped slot buffer (the (token, k) of a row comes from the inverse map
the gather records). Each (t, k) is owned by exactly one rank, so every slot
row is written once. After one bounded NVLink barrier, every rank adds
x + slot 0 + ... + slot K-1 in that order (moe_slots_reduce), so every
replica gets the same bits, and they are the bits of the one-GPU combine,
which rounds the same terms to 16 bits: the forward does not depend on ep. In
backward the combine needs no traffic (every rank holds the full
gradient). The input gradients of the local experts and the routing-weight
gradients of the local slots are summed over NVLink (peer_sum) before the
replicated router backward. Compared with the reference's two all-to-alls
per layer (moe.py:349-386; every token sent once per EP rank), each token
is processed once, and each rank sends (ep-1)/ep of its K x N x H 16-bit
slot rows over NVLink from the GEMM epilogue, with no separate combine pass.
"""
from __future__ import annotations


import torch

from ..ops import gemm as G
from ..ops import kernels as K
from ..ops._C import load as _ext

LN_EPS = 1e-5
PAD = 128


def _stacks(moe, flat=None):
    ex = moe.expert_group.experts
    flat = flat or ex[0].w1.weight.flat_owner
    w1, g1 = flat.stacked([e.w1.weight for e in ex])
    w2, g2 = flat.stacked([e.w2.weight for e in ex])
    return w1, g1, w2, g2


def _window(moe):
    """(first global expert of this rank, one past its last, global expert count)."""
    El = moe.num_local_experts
    e0 = moe.ep_rank * El
    return e0, e0 + El, moe.num_experts


class _EPBuffers:
    """Peer-mapped buffers of one MoE layer over its EP group: the forward
    combine slots (K x N x H, 16-bit; slot k row t receives token t's k-th
    expert output, scaled by its routing weight, from the rank that owns that
    expert) and the backward sums (N x H input gradient + N x K routing-weight
    gradient, fp32). Each call site owns its buffer, which is what makes one
    barrier per exchange sufficient."""

    def __init__(self, moe, N: int, H: int, K: int, device, dtype: torch.dtype):
        from ..parallel.symm import SymmetricBuffer
        self.N, self.H, self.K, self.dtype = N, H, K, dtype
        self.nb = (N * H + N * K + 3) // 4 * 4
        # Two slot buffers used in turn by consecutive forwards: a rank that is one
        # forward ahead (evaluation runs forwards back to back, with no backward
        # barrier in between) writes the other buffer while a peer still reads.
        self.slots = [SymmetricBuffer(moe.ep_group, K * N * H * 2, device) for _ in range(2)]
        self.turn = 0
        self.bwd = SymmetricBuffer(moe.ep_group, self.nb * 4, device)
        self.rank = self.bwd.rank

    def next_slots(self):
        """The slot buffer of the coming forward."""
        b = self.slots[self.turn]
        self.turn ^= 1
        return b

    def slot_tensor(self, b) -> torch.Tensor:
        return b.tensor(self.dtype, self.K * self.N * self.H).view(self.K, self.N, self.H)

    def bwd_parts(self):
        t = self.bwd.tensor(torch.float32, self.nb)
        NH = self.N * self.H
        return t, t[:NH].view(self.N, self.H), t[NH:NH + self.N * self.K].view(self.N, self.K)


def _ep_buffers(moe, N: int, H: int, K: int, device, dtype: torch.dtype = torch.bfloat16) -> _EPBuffers:
    cache = moe.__dict__.setdefault("_hb_ep_buffers", {})
    key = (N, H, K, str(device), dtype)
    if key not in cache:
        cache[key] = _EPBuffers(moe, N, H, K, device, dtype)
    return cache[key]


def _peer_sum(buf, addend, dst, n: int) -> None:
    _ext().peer_sum(buf.ptrs, buf.signal_ptrs, buf.rank, addend, dst, n, buf.counter)


def moe_route_and_experts(moe, xn2: torch.Tensor, flat=None):
    """Router + permutation + the two grouped expert GEMMs for 16-bit xn2 [N, H] (bf16 or fp16),
    over this rank's experts.

    Returns (aux, state) where state holds everything combine / backward need."""
    ext = _ext()
    N, H = xn2.shape
    e0, e1, E = _window(moe)
    El = e1 - e0
    Kk = moe.top_k
    I = moe.config.intermediate_size
    dev = xn2.device
    probs = torch.empty(N, E, device=dev, dtype=torch.float32)
    topi = torch.empty(N, Kk, device=dev, dtype=torch.int32)
    topw = torch.empty(N, Kk, device=dev, dtype=torch.float32)
    counts = torch.empty(E, device=dev, dtype=torch.int32)
    probsum = torch.empty(E, device=dev, dtype=torch.float32)
    off = torch.empty(E + 1, device=dev, dtype=torch.int32)
    aux = torch.empty((), device=dev, dtype=torch.float32)
    pos = torch.empty(N * Kk, device=dev, dtype=torch.int32)
    ext.moe_route(xn2, moe.router.gate.weight, Kk, moe.aux_loss_coef, probs, topi, topw, counts, probsum, off, aux,
                  pos)
    with torch.no_grad():
        moe._expert_counts = counts  # diagnostics (reference moe.py:329-332)
    if El == E:
        off_l = off
    else:
        off_l = torch.empty(El + 1, device=dev, dtype=torch.int32)
        ext.moe_local_offsets(off, e0, El, off_l)
    # capacity of this rank's rows: every local segment padded to 128 rows
    R = (N * Kk + El * (PAD - 1) + PAD - 1) // PAD * PAD
    xp = torch.zeros(R, H, device=dev, dtype=xn2.dtype)
    ep = moe.ep_world_size
    inv = torch.empty(R, device=dev, dtype=torch.int32) if ep > 1 else None
    ext.moe_gather(xn2, pos, Kk, xp, off, e0, e1, inv)
    w1, _, w2, _ = _stacks(moe, flat)
    hp = torch.empty(R, I, device=dev, dtype=xn2.dtype)
    prep = torch.empty(R, I, device=dev, dtype=xn2.dtype)
    G.gemm(xp, w1, hp, I, G.EPI_BF16_GELU, False, False, aux=prep, grp=(1, off_l, El, I, 0))
    yp = torch.empty(R, H, device=dev, dtype=xn2.dtype)
    cmb = None
    if ep > 1:
        # the second expert GEMM also performs the combine's exchange: each output row,
        # times its routing weight, goes straight into slot (k, t) of every EP rank
        slots = _ep_buffers(moe, N, H, Kk, dev, xn2.dtype).next_slots()
        cmb = (slots.ptrs, inv, topw, Kk, N)
        moe._hb_slots_now = slots
    G.gemm(hp, w2, yp, H, G.EPI_BF16, False, False, grp=(1, off_l, El, H, 0), cmb=cmb)
    return aux, (probs, topi, topw, counts, off, off_l, pos, xp, hp, prep, yp)


def moe_combine_fwd(moe, state, x1: torch.Tensor) -> torch.Tensor:
    """x2 = x1 + sum_k w_k y_k (over all experts of all EP ranks)."""
    ext = _ext()
    probs, topi, topw, counts, off, off_l, pos, xp, hp, prep, yp = state
    e0, e1, E = _window(moe)
    x2 = torch.empty_like(x1)
    if moe.ep_world_size == 1:
        ext.moe_combine(yp, pos, topw, x1, x2, off, e0, e1)
        return x2
    N, H = x1.shape
    buf = _ep_buffers(moe, N, H, moe.top_k, x1.device, yp.dtype)
    slots = moe._hb_slots_now  # the buffer the expert GEMM of this forward filled
    slots.barrier()  # every rank's expert GEMM has written its slot rows
    ext.moe_slots_reduce(x1, buf.slot_tensor(slots), moe.top_k, x2)
    return x2


def moe_experts_bwd(moe, xn2: torch.Tensor, state, dx_res: torch.Tensor, daux: torch.Tensor, flat=None):
    """Backward of route + experts + combine. dx_res: fp32 gradient of the
    combined output [N, H]. Returns dxn2 (fp32 [N, H]) and accumulates the
    expert and gate weight gradients."""
    ext = _ext()
    probs, topi, topw, counts, off, off_l, pos, xp, hp, prep, yp = state
    N, H = xn2.shape
    e0, e1, E = _window(moe)
    El = e1 - e0
    Kk = moe.top_k
    I = moe.config.intermediate_size
    R = xp.shape[0]
    dev = xn2.device
    ep = moe.ep_world_size
    w1, g1, w2, g2 = _stacks(moe, flat)
    if ep > 1:
        buf = _ep_buffers(moe, N, H, Kk, dev, xn2.dtype)
        whole, dxn2_part, dw = buf.bwd_parts()
    else:
        dxn2_part = torch.empty(N, H, device=dev, dtype=torch.float32)
        dw = torch.empty(N, Kk, device=dev, dtype=torch.float32)
    dyp = torch.zeros(R, H, device=dev, dtype=xn2.dtype)
    ext.moe_combine_bwd(dx_res, yp, pos, topw, dyp, dw, off, e0, e1)
    dprep = torch.empty(R, I, device=dev, dtype=xn2.dtype)
    G.gemm(dyp, w2, dprep, I, G.EPI_BF16_DGELU, False, True, aux=prep, grp=(1, off_l, El, H, 0))
    G.gemm(dyp, hp, g2, I, G.EPI_F32_ACC, True, True, grp=(2, off_l, El, 0, H))
    dxp = torch.empty(R, H, device=dev, dtype=torch.float32)
    G.gemm(dprep, w1, dxp, H, G.EPI_F32, False, True, grp=(1, off_l, El, I, 0))
    G.gemm(dprep, xp, g1, H, G.EPI_F32_ACC, True, True, grp=(2, off_l, El, 0, I))
    del dyp, dprep
    ext.moe_unpermute(dxp, pos, Kk, dxn2_part, off, e0, e1)
    del dxp
    if ep > 1:
        # input and routing-weight gradients of every rank's experts, summed over NVLink
        summed = torch.empty(buf.nb, device=dev, dtype=torch.float32)
        _peer_sum(buf.bwd, None, summed, buf.nb)
        dxn2 = summed[:N * H].view(N, H)
        dw = summed[N * H:N * H + N * Kk].view(N, Kk)
    else:
        dxn2 = dxn2_part
    Ep = (E + 7) // 8 * 8  # row stride of the logits gradient: 16-byte aligned for TMA
    dlog = torch.zeros(N, Ep, device=dev, dtype=xn2.dtype)
    ext.moe_router_bwd(probs, topi, topw, dw, daux.reshape(1).float().contiguous(), counts, moe.aux_loss_coef,
                       moe.router.gate.weight, dlog, dxn2)
    G.gemm(dlog[:, :E], xn2, moe.router.gate.weight.main_grad, H, G.EPI_F32_ACC, True, True)
    return dxn2


def moe_sublayer_fwd(blk, flat, x1: torch.Tensor, keep: bool):
    """x1: fp32 residual [N, H] -> (x2 = x1 + MoE(ln_2(x1)) fp32, aux (0-d), saved)."""
    moe = blk.moe
    xn2, m2, r2 = K.layernorm_fwd(x1, blk.ln_2.weight, blk.ln_2.bias, LN_EPS, dtype=blk.ln_2.weight.w16.dtype)
    aux, state = moe_route_and_experts(moe, xn2, flat)
    x2 = moe_combine_fwd(moe, state, x1)
    saved = (x1, xn2, m2, r2, state) if keep else None
    return x2, aux, saved

def moe_sublayer_bwd(blk, flat, saved, dres: torch.Tensor, dres16: torch.Tensor, daux: torch.Tensor, ln_scratch):
    """In place: dres / dres16 go from d(x2) to d(x1)."""
    x1, xn2, m2, r2, state = saved
    dxn2 = moe_experts_bwd(blk.moe, xn2, state, dres, daux, flat)
    K.layernorm_bwd(dxn2, x1, m2, r2, blk.ln_2.weight, dres, dres, dres16, blk.ln_2.weight.main_grad,
                    blk.ln_2.bias.main_grad, scratch=ln_scratch)
