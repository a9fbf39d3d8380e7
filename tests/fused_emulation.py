"""PyTorch stand-ins for the sm_100a kernel wrappers, for CPU tests of the fused
engine's host orchestration.

The fused path (models/fused.py) is Python that sequences kernel calls, saves
tensors between forward and backward, and (with activation checkpointing)
reruns forwards. Its kernels run only on a B200, but its sequencing can be
checked on the CPU: ``emulate(monkeypatch)`` replaces every wrapper in
``heiretsu_b200.ops.kernels`` and ``heiretsu_b200.ops.gemm`` that the single-GPU
fused path calls with an fp32 PyTorch restatement of the same contract (same
argument conventions, same in-place outputs, the same dropout masks through
``ops/dropout_ref.py``). The kernels themselves are tested against fp32
oracles on the GPU; these stand-ins test only the code around them.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from heiretsu_b200.ops import dropout_ref as DR


def _seed(t) -> int:
    return int(t.reshape(-1)[0].item())


def _gelu(x):
    return F.gelu(x, approximate="tanh")


def _gelu_grad(x):
    x = x.detach().requires_grad_(True)
    with torch.enable_grad():
        y = _gelu(x)
        (g,) = torch.autograd.grad(y.sum(), x)
    return g


# ---- GEMM -------------------------------------------------------------------
def linear_fwd(x, w, bias=None, *, out=None, n=None):
    N = int(n if n is not None else w.shape[0])
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    if N > y.shape[1]:
        y = F.pad(y, (0, N - y.shape[1]))
    y = y.to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def linear_fwd_gelu(x, w, bias, *, out=None, pre=None):
    p = (x.float() @ w.float().t() + bias.float()).to(x.dtype).float()
    return _gelu(p).to(x.dtype), p.to(x.dtype)


def linear_fwd_resid(x, w, bias, resid, *, out=None, drop=None):
    y = x.float() @ w.float().t() + bias.float()
    if drop is not None:
        seed, site, p, row0 = drop
        y = y * DR.residual_mask(_seed(seed), site, y.shape[0], y.shape[1], p, row0).float()
    r = resid + y
    if out is not None:
        out.copy_(r)
        return out
    return r


def linear_dgrad(dy, w, *, out=None, gelu_pre=None, f32=False):
    d = dy.float() @ w.float()
    if gelu_pre is not None:
        return (d * _gelu_grad(gelu_pre.float())).to(dy.dtype)
    return d if f32 else d.to(dy.dtype)


def linear_wgrad(dy, x, *, out=None, accumulate=False, n_rows=None):
    N = int(n_rows if n_rows is not None else dy.shape[1])
    g = dy[:, :N].float().t() @ x.float()
    if out is None:
        return g
    if accumulate:
        out.add_(g)
    else:
        out.copy_(g)
    return out


def gemm(a, b, c, n, epi, a_mn, b_mn, bias=None, aux=None, resid=None, block_n=None, ag=None, rs=None, grp=None,
         drop=None):
    """Only the plain bf16 C = A B^T form (the lm_head) is used on the single-GPU path."""
    assert epi == 0 and not a_mn and not b_mn and ag is None and rs is None and grp is None
    y = a.float() @ b.float().t()
    c[:, :y.shape[1]].copy_(y.to(c.dtype))
    if c.shape[1] > y.shape[1]:
        c[:, y.shape[1]:].zero_()
    return c


# ---- LayerNorm, dropout, conversions ------------------------------------------
def layernorm_fwd(x, w, b, eps=1e-5, dtype=torch.bfloat16):
    mean = x.mean(-1)
    rstd = torch.rsqrt(x.var(-1, unbiased=False) + eps)
    y = (x - mean[:, None]) * rstd[:, None] * w + b
    return y.to(dtype), mean, rstd


def layernorm_bwd(dy, x, mean, rstd, w, dres_in, dres, dres16, dgamma, dbeta, scratch=None, dy_srcs=1):
    H = x.shape[-1]
    g = dy.float().reshape(dy_srcs, -1, H).sum(0) if dy_srcs > 1 else dy.float()
    xh = (x - mean[:, None]) * rstd[:, None]
    dgamma.add_((g * xh).sum(0))
    dbeta.add_(g.sum(0))
    gw = g * w
    dx = rstd[:, None] * (gw - gw.mean(-1, keepdim=True) - xh * (gw * xh).mean(-1, keepdim=True))
    new = dres_in + dx
    dres.copy_(new)
    dres16.copy_(new.to(dres16.dtype))


def dropout_bf16(g, seed, site, p, row0=0, out=None, dtype=torch.bfloat16):
    m = DR.residual_mask(_seed(seed), site, g.shape[0], g.shape[1], p, row0).float()
    y = (g.float() * m).to(out.dtype if out is not None else dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def f32_to_bf16(x, out=None, dtype=torch.bfloat16):
    if out is None:
        return x.to(dtype)
    out.copy_(x)
    return out


def colsum_bf16(x, out):
    out.add_(x.float().sum(0))


# ---- attention ------------------------------------------------------------------
def _qkv(qkv, B, T, nh, dh=64):
    q, k, v = qkv.float().view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4).unbind(0)
    return q, k, v


def _attn(q, k, v, T, drop, B, nh):
    s = (q @ k.transpose(-1, -2)) / (q.shape[-1] ** 0.5)
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1), float("-inf"))
    p = torch.softmax(s, -1)
    if drop is not None:
        seed, site, pr, h0, nht = drop
        p = p * DR.attention_mask(_seed(seed), site, B, nh, T, pr, h0, nht).float()
    return p @ v


def attention_fwd(qkv, B, T, nh, out=None, drop=None, head_dim=64):
    q, k, v = _qkv(qkv, B, T, nh, head_dim)
    y = _attn(q, k, v, T, drop, B, nh).transpose(1, 2).reshape(B * T, nh * head_dim)
    lse = torch.zeros(B, nh, (T + 127) // 128 * 128)
    return y.bfloat16(), lse


def attention_bwd(qkv, out, dout, lse, B, T, nh, dqkv=None, drop=None, head_dim=64):
    q, k, v = (t.detach().requires_grad_(True) for t in _qkv(qkv, B, T, nh, head_dim))
    with torch.enable_grad():
        y = _attn(q, k, v, T, drop, B, nh).transpose(1, 2).reshape(B * T, nh * head_dim)
        dq, dk, dv = torch.autograd.grad(y, (q, k, v), dout.float())
    d = torch.stack([dq, dk, dv]).permute(1, 3, 0, 2, 4).reshape(B * T, 3 * nh * head_dim)
    return d.bfloat16()


# ---- loss, embedding, optimizer ------------------------------------------------
def cross_entropy_fwd(logits, V, targets, ignore_index=-100):
    lf = logits[:, :V].float()
    lse = torch.logsumexp(lf, -1)
    valid = targets != ignore_index
    t = torch.where(valid, targets, torch.zeros_like(targets))
    rows = torch.where(valid, lse - lf.gather(1, t[:, None]).squeeze(1), torch.zeros_like(lse))
    mean = rows.sum() / valid.sum().clamp_min(1)
    return mean, lse, rows


def cross_entropy_bwd_(logits, V, targets, lse, scale, scale_mul, ignore_index=-100):
    lf = logits[:, :V].float()
    valid = targets != ignore_index
    s = (scale.reshape(-1)[0] if scale is not None else 1.0) * scale_mul
    g = torch.exp(lf - lse[:, None])
    t = torch.where(valid, targets, torch.zeros_like(targets))
    g.scatter_add_(1, t[:, None], -torch.ones(g.shape[0], 1))
    g = g * torch.where(valid, s, torch.zeros_like(lse))[:, None]
    logits.zero_()
    logits[:, :V].copy_(g.bfloat16())
    return logits


def cross_entropy_fused_(logits, V, targets, scale, ignore_index=-100):
    mean, lse, _ = cross_entropy_fwd(logits, V, targets, ignore_index)
    cross_entropy_bwd_(logits, V, targets, lse, scale, 1.0, ignore_index)
    return mean, lse


def cross_entropy_rescale_(g, actual, expected):
    if not torch.equal(actual, expected):
        g.copy_((g.float() * (actual / expected)).bfloat16())
    return g


def embedding_fwd(idx, wte, wpe):
    B, T = idx.shape
    return (wte[idx] + wpe[:T][None]).reshape(B * T, -1)


def embedding_bwd(idx, dx, dwte, dwpe):
    B, T = idx.shape
    d = dx.reshape(B, T, -1)
    if dwte is not None:
        dwte.index_add_(0, idx.reshape(-1), d.reshape(B * T, -1))
    if dwpe is not None:
        dwpe[:T].add_(d.sum(0))


def sumsq(x, out, weight=1.0, accumulate=False):
    v = weight * x.float().pow(2).sum()
    if accumulate:
        out.add_(v)
    else:
        out.copy_(v)


def clip_coef(norm2, max_norm, coef, norm=None, loss_scale=None):
    inv_s = 1.0 / loss_scale.reshape(-1)[0] if loss_scale is not None else torch.ones(())
    n = norm2.sqrt() * inv_s
    if norm is not None:
        norm.copy_(n)
    c = torch.clamp(max_norm / (n + 1e-6), max=1.0) if max_norm > 0 else torch.ones(())
    coef.copy_(torch.where(torch.isfinite(n), c * inv_s, torch.full((), float("nan"))))


def loss_scale_update(coef, state, growth=2.0, backoff=0.5, interval=2000):
    if math.isnan(float(coef)):
        state[0] *= backoff
        state[1] = 0.0
    else:
        state[1] += 1.0
        if state[1] >= interval:
            state[0] *= growth
            state[1] = 0.0


def adamw_step(p, g, m, v, p16, hyper, coef):
    lr, b1, b2, eps, wd, bc1, bc2s, gs = hyper.tolist()
    c = float(coef)
    if not math.isfinite(c):
        return
    gg = g * c * gs
    p.mul_(1 - lr * wd)
    m.mul_(b1).add_(gg, alpha=1 - b1)
    v.mul_(b2).addcmul_(gg, gg, value=1 - b2)
    p.addcdiv_(m, (v.sqrt() / bc2s).add_(eps), value=-lr / bc1)
    if p16 is not None:
        p16.copy_(p)


KERNELS = ["layernorm_fwd", "layernorm_bwd", "dropout_bf16", "f32_to_bf16", "colsum_bf16", "attention_fwd",
           "attention_bwd", "cross_entropy_fwd", "cross_entropy_bwd_", "cross_entropy_fused_",
           "cross_entropy_rescale_", "embedding_fwd", "embedding_bwd", "sumsq", "clip_coef", "loss_scale_update",
           "adamw_step"]
GEMMS = ["linear_fwd", "linear_fwd_gelu", "linear_fwd_resid", "linear_dgrad", "linear_wgrad", "gemm"]


def emulate(monkeypatch) -> None:
    import heiretsu_b200.models.fused as FZ
    from heiretsu_b200.ops import gemm as G
    from heiretsu_b200.ops import kernels as K

    mod = globals()
    for name in KERNELS:
        monkeypatch.setattr(K, name, mod[name])
    for name in GEMMS:
        monkeypatch.setattr(G, name, mod[name])
    monkeypatch.setattr(FZ, "_ln_scratch", lambda M, H, device: torch.empty(0))


# ---- fused tensor parallelism (gloo ranks) -----------------------------------------
class FakeTPComm:
    """Stand-in of models/fused_tp.TPComm on gloo ranks: the same buffers as local
    tensors; the in-kernel all-gather and reduce-scatter of the GEMM become
    all_gather calls in ``tp_gemm``; barriers are no-ops (gloo calls block)."""

    def __init__(self, topo, Ms, H, dtype=torch.bfloat16):
        self.tp, self.rank, self.Ms, self.H, self.group = topo.tp, topo.tp_rank, Ms, H, topo.tp_group
        self.dtype = dtype
        self.src = [torch.zeros(Ms, H, dtype=dtype) for _ in range(2)]
        self.r16 = torch.zeros(self.tp * Ms, H, dtype=dtype)
        self.r32 = torch.zeros(self.tp * Ms, H, dtype=torch.float32)
        self.zero32 = None

    def barrier(self):
        pass

    def zeros(self):
        if self.zero32 is None:
            self.zero32 = torch.zeros(self.Ms, self.H)
        return self.zero32

    def src_view(self, i):
        return self.src[i]

    def recv16_all(self):
        return self.r16

    def recv32_all(self):
        return self.r32

    def ag(self, i):
        return ("ag", i, self)

    def rs16(self):
        return ("rs", self)

    def rs32(self):
        return ("rs", self)


def _all_gather(t, group):
    import torch.distributed as dist

    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, t.contiguous(), group=group)
    return parts


def tp_gemm(a, b, c, n, epi, a_mn, b_mn, bias=None, aux=None, resid=None, block_n=None, ag=None, rs=None,
            grp=None, drop=None):
    """The GEMM forms of the fused TP path: C = A B^T (b_mn False) or A B (b_mn True), with
    bias, GELU (pre-activation to ``aux``) or dGELU (times GELU'(aux)) epilogues, an
    all-gather of A's token shards (``ag``) and a reduce-scatter of C into the owners'
    receive slots (``rs``)."""
    assert grp is None and drop is None and not a_mn
    if ag is not None:
        _, i, comm = ag
        a.copy_(torch.cat(_all_gather(comm.src[i], comm.group)))
    y = a.float() @ (b.float() if b_mn else b.float().t())
    if bias is not None:
        y = y + bias.float()
    if epi == 1:
        aux.copy_(y.bfloat16())
        y = _gelu(y)
    elif epi == 5:
        y = y * _gelu_grad(aux.float())
    if rs is not None:
        _, comm = rs
        out = y.to(c.dtype)
        for src, part in enumerate(_all_gather(out, comm.group)):
            c[src * comm.Ms:(src + 1) * comm.Ms].copy_(part[comm.rank * comm.Ms:(comm.rank + 1) * comm.Ms])
        return c
    c[:, :y.shape[1]].copy_(y.to(c.dtype))
    return c


def resid_sum_ln(x, parts, nsrc, bias, x_new, w=None, b=None, y=None, mean=None, rstd=None, eps=1e-5):
    Ms = x.shape[0]
    s = x + parts.float().reshape(nsrc, Ms, -1).sum(0) + bias
    x_new.copy_(s)
    if w is not None:
        yy, mm, rr = layernorm_fwd(s, w, b, eps)
        y.copy_(yy)
        mean.copy_(mm)
        rstd.copy_(rr)


class _FakeExt:
    @staticmethod
    def layernorm_fwd(x, w, b, y, mean, rstd, eps):
        yy, mm, rr = layernorm_fwd(x, w, b, eps)
        y.copy_(yy)
        mean.copy_(mm)
        rstd.copy_(rr)

    @staticmethod
    def layernorm_bwd_scratch_rows(M):
        return 1


def emulate_tp(setattr_fn) -> None:
    """Everything ``emulate`` replaces, plus the TP communication layer and GEMM forms.
    ``setattr_fn(obj, name, value)`` installs a replacement (monkeypatch.setattr or a
    plain setattr in a spawned rank)."""
    import heiretsu_b200.models.fused as FZ
    import heiretsu_b200.models.fused_tp as FT
    from heiretsu_b200.ops import gemm as G
    from heiretsu_b200.ops import kernels as K

    mod = globals()
    for name in KERNELS:
        setattr_fn(K, name, mod[name])
    for name in GEMMS:
        setattr_fn(G, name, mod[name])
    setattr_fn(G, "gemm", tp_gemm)
    setattr_fn(K, "resid_sum_ln", resid_sum_ln)
    setattr_fn(FZ, "_ln_scratch", lambda M, H, device: torch.empty(0))
    setattr_fn(FT, "_ext", lambda: _FakeExt)
    comms = {}

    def get_comm(topo, Ms, H, device, dtype=torch.bfloat16):
        key = (id(topo.tp_group), Ms, H, dtype)
        if key not in comms:
            comms[key] = FakeTPComm(topo, Ms, H, dtype)
        return comms[key]

    setattr_fn(FT, "get_comm", get_comm)
