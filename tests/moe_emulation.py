"""PyTorch stand-ins for the fused MoE sub-layer's kernels (csrc/moe.cu and the
expert-grouped GEMM modes), for CPU tests of models/fused_moe.py's host
orchestration: routing, padded expert windows, the inverse slot map, the
grouped expert GEMMs, the one-GPU combine, the expert-parallel combine written
from the second expert GEMM into every rank's slot buffer, and the backward.

Each stand-in restates the kernel's contract in PyTorch (fp32 arithmetic, the
same 16-bit roundings at the same points, the same in-place outputs). The
expert-parallel peer buffers become local tensors summed over the EP group with
gloo collectives at the points where the kernels meet at a device barrier. The
kernels themselves are tested against fp32 oracles on the GPU; these stand-ins
test only the code around them.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F

PAD = 128  # expert segments are padded to this many rows (csrc/moe.cu kPad)


def _r16(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Round to the 16-bit format and widen back to fp32."""
    return x.to(dtype).float()


# ---- csrc/moe.cu ------------------------------------------------------------
class FakeMoEExt:
    @staticmethod
    def moe_route(x, wg, K, coef, probs, topi, topw, counts, probsum, off, aux, pos):
        N = x.shape[0]
        E = wg.shape[0]
        p = torch.softmax(x.float() @ wg.float().t(), dim=-1)
        w, i = torch.topk(p, K, dim=-1)  # largest first
        w = w / w.sum(dim=-1, keepdim=True)
        probs.view(N, E).copy_(p)
        topi.view(N, K).copy_(i.int())
        topw.view(N, K).copy_(w)
        cnt = torch.bincount(i.reshape(-1), minlength=E)
        counts.copy_(cnt.int())
        probsum.copy_(p.sum(dim=0))
        o = torch.zeros(E + 1, dtype=torch.int64)
        o[1:] = torch.cumsum((cnt + PAD - 1) // PAD * PAD, dim=0)
        off.copy_(o.int())
        aux.copy_(coef * E * ((cnt.float() / (N * K)) * (p.sum(dim=0) / N)).sum())
        flat = i.reshape(-1)
        rows = torch.empty(N * K, dtype=torch.int64)
        for e in range(E):  # token-major order inside each expert's segment
            slots = (flat == e).nonzero().view(-1)
            rows[slots] = o[e] + torch.arange(slots.numel())
        pos.copy_(rows.int())

    @staticmethod
    def moe_local_offsets(off, e0, n, out):
        out[:n + 1].copy_(off[e0:e0 + n + 1] - off[e0])

    @staticmethod
    def moe_gather(x, pos, K, xp, off, e0, e1, inv=None):
        lo, hi = int(off[e0]), int(off[e1])
        slots = torch.arange(pos.numel())
        r = pos.long()
        m = (r >= lo) & (r < hi)
        if inv is not None:
            inv.fill_(-1)
            inv[r[m] - lo] = slots[m].int()
        xp[r[m] - lo] = x[slots[m] // K]

    @staticmethod
    def _window_rows(pos, N, K, off, e0, e1):
        lo, hi = int(off[e0]), int(off[e1])
        r = pos.long().view(N, K)
        return r - lo, (r >= lo) & (r < hi)

    @staticmethod
    def moe_combine(yp, pos, topw, resid, out, off, e0, e1):
        N, H = out.shape
        K = topw.shape[1]
        rows, m = FakeMoEExt._window_rows(pos, N, K, off, e0, e1)
        acc = resid.clone() if resid is not None else torch.zeros(N, H)
        for k in range(K):  # k ascending, each weighted term rounded to 16 bits
            term = _r16(topw[:, k:k + 1] * yp[rows[:, k].clamp(min=0)].float(), yp.dtype)
            acc[m[:, k]] += term[m[:, k]]
        out.copy_(acc)

    @staticmethod
    def moe_slots_reduce(x, slots, K, out):
        acc = x.clone()
        for k in range(K):
            acc += slots[k].float()
        out.copy_(acc)

    @staticmethod
    def moe_combine_bwd(dy, yp, pos, topw, dyp, dw, off, e0, e1):
        N = dy.shape[0]
        K = topw.shape[1]
        rows, m = FakeMoEExt._window_rows(pos, N, K, off, e0, e1)
        dw.zero_()
        for k in range(K):
            t = m[:, k].nonzero().view(-1)
            rr = rows[t, k]
            dw[t, k] = (dy[t] * yp[rr].float()).sum(dim=-1)
            dyp[rr] = (topw[t, k:k + 1] * dy[t]).to(dyp.dtype)

    @staticmethod
    def moe_unpermute(dxp, pos, K, dx, off, e0, e1):
        N = dx.shape[0]
        rows, m = FakeMoEExt._window_rows(pos, N, K, off, e0, e1)
        acc = torch.zeros_like(dx)
        for k in range(K):
            t = m[:, k].nonzero().view(-1)
            acc[t] += dxp[rows[t, k]]
        dx.copy_(acc)

    @staticmethod
    def moe_router_bwd(probs, topi, topw, dw, daux, counts, coef, wg, dlogits, dx):
        N, E = probs.shape
        K = topi.shape[1]
        idx = topi.long()
        dp = (daux.reshape(-1)[0] * coef * E * (counts.float() / (N * K)) / N).expand(N, E).clone()
        S = probs.gather(1, idx).sum(dim=1, keepdim=True)
        dot = (dw * topw).sum(dim=1, keepdim=True)
        dp.scatter_add_(1, idx, (dw - dot) / S)
        dl = probs * (dp - (probs * dp).sum(dim=1, keepdim=True))
        dlogits[:, :E].copy_(dl.to(dlogits.dtype))
        dx += dl @ wg.float()


# ---- the GEMM forms the MoE sub-layer uses (csrc/gemm_kernel.cuh) ---------------
EPI_BF16, EPI_BF16_GELU, EPI_F32, EPI_F32_ACC, EPI_F32_RESID, EPI_BF16_DGELU = range(6)


def _gelu_grad(x):
    x = x.detach().requires_grad_(True)
    with torch.enable_grad():
        (g,) = torch.autograd.grad(F.gelu(x, approximate="tanh").sum(), x)
    return g


def _epilogue(d, epi, c, aux, bias, out_rows, cmb, row0):
    """Apply the epilogue of D (fp32) to rows out_rows of C (and AUX)."""
    if bias is not None:
        d = d + bias.float()
    if epi == EPI_BF16:
        c[out_rows] = d.to(c.dtype)
        if cmb is not None:
            _combine_push(cmb, d.to(c.dtype), row0)
    elif epi == EPI_BF16_GELU:
        pre = d.to(c.dtype)
        aux[out_rows] = pre
        c[out_rows] = F.gelu(pre.float(), approximate="tanh").to(c.dtype)
    elif epi == EPI_F32:
        c[out_rows] = d
    elif epi == EPI_F32_ACC:
        c[out_rows] += d
    elif epi == EPI_BF16_DGELU:
        c[out_rows] = (d * _gelu_grad(aux[out_rows].float())).to(c.dtype)
    else:
        raise NotImplementedError(epi)


def _combine_push(cmb, y16, row0):
    """Expert-parallel combine epilogue: row p (window row row0 + p) with routing
    slot i = inv[row] = t * K + k goes, as 16-bit(w_i * y_row), to slot (k, t) of
    every EP rank's buffer (here: this rank's contribution, summed at the barrier)."""
    slots, inv, w, K, N = cmb
    i = inv[row0:row0 + y16.shape[0]].long()
    m = i >= 0
    t, k = i[m] // K, i[m] % K
    slots.contrib[k, t] = _r16(w.reshape(-1)[i[m]].unsqueeze(1) * y16[m].float(), slots.contrib.dtype).to(
        slots.contrib.dtype)


def moe_gemm(a, b, c, n, epi, a_mn, b_mn, bias=None, aux=None, resid=None, block_n=None, ag=None, rs=None, grp=None,
             drop=None, cmb=None):
    """C = A' B'^T with A' = A (or A^T when a_mn) and B' = B (or B^T when b_mn);
    ``grp = (1, offsets, groups, b_rows, 0)``: rows of A in segment g use B's rows
    [g * b_rows, (g+1) * b_rows); ``grp = (2, offsets, groups, 0, c_rows)``: the
    reduction runs over segment g only, into C's rows [g * c_rows, (g+1) * c_rows)."""
    assert ag is None and rs is None and drop is None and resid is None

    def a_(x):
        return x.float().t() if a_mn else x.float()

    def b_(x):
        return x.float().t() if b_mn else x.float()

    if grp is None or grp[0] == 0:
        d = a_(a) @ b_(b).t()
        if d.shape[1] < c.shape[1] and epi == EPI_BF16:  # n beyond B's rows: zero columns
            d = F.pad(d, (0, c.shape[1] - d.shape[1]))
        _epilogue(d, epi, c, aux, bias, slice(0, d.shape[0]), cmb, 0)
        return c
    mode, off, groups, b_rows, c_rows = grp
    off = [int(v) for v in off[:groups + 1]]
    for g in range(groups):
        lo, hi = off[g], off[g + 1]
        if hi == lo:
            continue
        if mode == 1:
            d = a_(a)[lo:hi] @ b_(b[g * b_rows:(g + 1) * b_rows]).t()
            _epilogue(d, epi, c, aux, bias, slice(lo, hi), cmb, lo)
        else:
            d = a_(a)[:, lo:hi] @ b_(b)[:, lo:hi].t()
            _epilogue(d, epi, c, aux, bias, slice(g * c_rows, (g + 1) * c_rows), None, 0)
    return c


# ---- expert-parallel buffers (peer memory) as gloo collectives ------------------
class FakeSlots:
    """One combine slot buffer [K, N, H]: the rows this rank's GEMM pushed; the
    barrier sums the ranks' contributions (each (k, t) is written by one rank)."""

    def __init__(self, group, K, N, H, dtype):
        self.group = group
        self.contrib = torch.zeros(K, N, H, dtype=dtype)
        self.full = None

    @property
    def ptrs(self):  # stands in for the peer pointer table
        return self

    def barrier(self):
        s = self.contrib.float()
        dist.all_reduce(s, group=self.group)
        self.full = s.to(self.contrib.dtype)


class FakeEPBuffers:
    def __init__(self, moe, N, H, K, dtype):
        self.N, self.H, self.K, self.dtype = N, H, K, dtype
        self.group = moe.ep_group
        self.nb = (N * H + N * K + 3) // 4 * 4
        self.slots = [FakeSlots(self.group, K, N, H, dtype) for _ in range(2)]
        self.turn = 0
        self.bwd = self
        self.t = torch.zeros(self.nb)

    def next_slots(self):
        b = self.slots[self.turn]
        self.turn ^= 1
        b.contrib.zero_()  # the real buffers are overwritten in full by every forward
        return b

    def slot_tensor(self, b):
        return b.full

    def bwd_parts(self):
        NH = self.N * self.H
        return self.t, self.t[:NH].view(self.N, self.H), self.t[NH:NH + self.N * self.K].view(self.N, self.K)


def _peer_sum(buf, addend, dst, n):
    s = buf.t[:n].clone()
    dist.all_reduce(s, group=buf.group)
    dst[:n].copy_(s if addend is None else s + addend[:n])


def emulate_moe(setattr_fn) -> None:
    """Install the stand-ins on models/fused_moe.py, after fused_emulation's own
    (``emulate`` or ``emulate_tp``), whose GEMM stand-in keeps the dense forms."""
    import heiretsu_b200.models.fused_moe as FM
    from heiretsu_b200.ops import gemm as G

    setattr_fn(FM, "_ext", lambda: FakeMoEExt)
    prev = G.gemm  # the stand-in already installed for the dense forms (plain or TP)

    def gemm(a, b, c, n, epi, a_mn, b_mn, bias=None, aux=None, resid=None, block_n=None, ag=None, rs=None,
             grp=None, drop=None, cmb=None):
        if grp is not None or cmb is not None or a_mn:  # the expert-grouped and weight-gradient forms
            return moe_gemm(a, b, c, n, epi, a_mn, b_mn, bias=bias, aux=aux, grp=grp, cmb=cmb)
        return prev(a, b, c, n, epi, a_mn, b_mn, bias=bias, aux=aux, resid=resid, block_n=block_n, ag=ag, rs=rs,
                    grp=grp, drop=drop)

    setattr_fn(G, "gemm", gemm)
    cache = {}

    def ep_buffers(moe, N, H, K, device, dtype=torch.bfloat16):
        key = (id(moe), N, H, K, dtype)
        if key not in cache:
            cache[key] = FakeEPBuffers(moe, N, H, K, dtype)
        return cache[key]

    setattr_fn(FM, "_ep_buffers", ep_buffers)
    setattr_fn(FM, "_peer_sum", _peer_sum)
