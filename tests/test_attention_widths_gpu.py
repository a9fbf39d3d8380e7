"""Causal attention at head widths other than 64 against fp32 PyTorch.

head_dim 128 runs its own tcgen05 kernels (the reference's default model,
--n_head 6 --n_embed 768, has 128-wide heads); 16 and 32 run the 64-wide
kernels on zero-padded heads. Forward output and the Q/K/V gradients are
compared with F.scaled_dot_product_attention in fp32 on the same bf16 inputs,
including sequence lengths that are not multiples of the 128-row tile; with
dropout, against the PyTorch restatement of the mask (ops/dropout_ref.py).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return (a.float() - b.float()).norm().item() / (b.float().norm().item() + 1e-12)


@pytest.mark.parametrize("dh", [128, 32, 16])
@pytest.mark.parametrize("B,T,nh", [(2, 256, 2), (1, 1024, 6), (2, 200, 3), (1, 130, 2)])
def test_attention_width_fwd_bwd(dh, B, T, nh):
    from heiretsu_b200.ops import kernels as K
    from heiretsu_b200.ops._C import check_status

    torch.manual_seed(7)
    H = nh * dh
    qkv = torch.randn(B * T, 3 * H, device="cuda").bfloat16()
    y, lse = K.attention_fwd(qkv, B, T, nh, head_dim=dh)
    torch.cuda.synchronize()
    check_status()
    q, k, v = (t.float().detach().requires_grad_(True) for t in
               qkv.view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4).unbind(0))
    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    ref2 = ref.transpose(1, 2).reshape(B * T, H)
    assert (y.float() - ref2).abs().max().item() < 2e-2
    # the LSE handed to the backward: -nlse * ln 2 is the natural-log log-sum-exp
    s = (q @ k.transpose(-1, -2)) / dh ** 0.5
    s = s.masked_fill(torch.ones(T, T, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    want_lse = torch.logsumexp(s, -1)
    got_lse = -lse[:, :, :T] * 0.6931471805599453
    assert (got_lse - want_lse).abs().max().item() < 2e-2
    dy = torch.randn(B * T, H, device="cuda").bfloat16()
    ref2.backward(dy.float())
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, T, nh, head_dim=dh)
    torch.cuda.synchronize()
    check_status()
    d = dqkv.float().view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4)
    for i, (name, g) in enumerate((("q", q.grad), ("k", k.grad), ("v", v.grad))):
        e = (d[i] - g).abs().max().item()
        scale = g.abs().max().item()
        assert e <= 3e-2 * scale + 1e-3, (dh, name, e, scale)


@pytest.mark.parametrize("dh", [128, 32])
def test_attention_width_dropout(dh):
    from heiretsu_b200.ops import kernels as K
    from heiretsu_b200.ops._C import check_status
    from heiretsu_b200.ops.dropout_ref import attention_mask

    torch.manual_seed(1)
    B, T, nh, p, site, sval = 2, 256, 2, 0.25, 12, 777
    H = nh * dh
    qkv = (0.5 * torch.randn(B * T, 3 * H, device="cuda")).bfloat16()
    seed = torch.tensor([sval], dtype=torch.int32, device="cuda")
    drop = (seed, site, p, 0, nh)
    y, lse = K.attention_fwd(qkv, B, T, nh, drop=drop, head_dim=dh)
    dy = torch.randn_like(y)
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, T, nh, drop=drop, head_dim=dh)
    torch.cuda.synchronize()
    check_status()
    q, k, v = (t.float().detach().requires_grad_(True) for t in
               qkv.view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4).unbind(0))
    s = q @ k.transpose(-1, -2) / dh ** 0.5
    causal = torch.ones(T, T, device="cuda", dtype=torch.bool).tril()
    prob = torch.softmax(s.masked_fill(~causal, float("-inf")), dim=-1)
    mask = attention_mask(sval, site, B, nh, T, p).float().cuda()
    o = (prob * mask) @ v
    assert _rel(y, o.permute(0, 2, 1, 3).reshape(B * T, H)) < 2e-2
    o.backward(dy.float().view(B, T, nh, dh).permute(0, 2, 1, 3))
    dq, dk, dv = dqkv.view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4).unbind(0)
    assert _rel(dq, q.grad) < 3e-2
    assert _rel(dk, k.grad) < 3e-2
    assert _rel(dv, v.grad) < 3e-2


def test_reference_default_model_runs_fused():
    """--n_head 6 --n_embed 768 (head_dim 128): the fused model's loss and gradients
    against the plain fp32 model on the same weights."""
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.fused import fused_supported
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.ops._C import check_status
    from heiretsu_b200.parallel.flat import FlatParams

    cfg = GPTConfig(block_size=512, vocab_size=50257, n_layer=2, n_head=6, n_embed=768, dropout=0.0)
    assert fused_supported(cfg)[0]
    torch.manual_seed(0)
    ref = GPT(cfg).cuda()
    torch.manual_seed(0)
    fz = GPT(cfg).cuda()
    flat = FlatParams(fz, torch.device("cuda"))
    fz.fused = True
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randint(0, cfg.vocab_size, (2, 512), device="cuda", generator=g)
    y = torch.randint(0, cfg.vocab_size, (2, 512), device="cuda", generator=g)
    _, lr, _ = ref(x, y)
    lr.backward()
    _, lf, _ = fz(x, y, return_logits=False)
    lf.backward()
    torch.cuda.synchronize()
    check_status()
    assert abs(lf.item() - lr.item()) < 2e-2, (lf.item(), lr.item())
    rp = dict(ref.named_parameters())
    bad = []
    for n, p in fz.named_parameters():
        rel = (p.main_grad - rp[n].grad).norm().item() / (rp[n].grad.norm().item() + 1e-8)
        if rel > 5e-2:
            bad.append((n, rel))
    assert not bad, bad
    del flat
