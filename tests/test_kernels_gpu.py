"""Numerics of the non-GEMM sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def K():
    from heiretsu_b200.ops import kernels
    return kernels


def check():
    from heiretsu_b200.ops._C import check_status
    check_status()


@pytest.mark.parametrize("M,H", [(8192, 768), (300, 1024), (17, 128), (64, 32)])
def test_layernorm_fwd_bwd(M, H):
    torch.manual_seed(0)
    x = torch.randn(M, H, device="cuda") * 2 + 0.5
    w = torch.randn(H, device="cuda")
    b = torch.randn(H, device="cuda")
    y, mean, rstd = K().layernorm_fwd(x, w, b)
    check()
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    br = b.clone().requires_grad_(True)
    yr = F.layer_norm(xr, (H,), wr, br, 1e-5)
    # bf16 output: relative rounding 2^-8 of |y| (|y| up to ~6 here)
    assert ((y.float() - yr).abs() / (yr.abs() + 1.0)).max().item() < 1e-2
    dy = torch.randn(M, H, device="cuda")
    yr.backward(dy)
    dres_in = torch.randn(M, H, device="cuda")
    dres = torch.empty_like(dres_in)
    dres16 = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    dg = torch.zeros(H, device="cuda")
    db = torch.ones(H, device="cuda")
    K().layernorm_bwd(dy, x, mean, rstd, w, dres_in, dres, dres16, dg, db)
    check()
    assert torch.allclose(dres, dres_in + xr.grad, atol=1e-3, rtol=1e-3)
    assert (dres16.float() - dres).abs().max().item() <= 1e-2 * dres.abs().max().item()
    assert torch.allclose(dg, wr.grad, atol=1e-2, rtol=1e-3)
    assert torch.allclose(db, 1 + br.grad, atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("M,V", [(512, 50257), (64, 128), (33, 1000)])
def test_cross_entropy(M, V):
    torch.manual_seed(1)
    Vp = (V + 127) // 128 * 128
    logits = torch.zeros(M, Vp, device="cuda", dtype=torch.bfloat16)
    logits[:, :V] = (torch.randn(M, V, device="cuda") * 3).bfloat16()
    t = torch.randint(0, V, (M,), device="cuda")
    loss, lse, rows = K().cross_entropy_fwd(logits, V, t)
    check()
    lr = logits[:, :V].float().requires_grad_(True)
    ref = F.cross_entropy(lr, t)
    assert abs(loss.item() - ref.item()) < 1e-4 * max(1.0, abs(ref.item()))
    ref.backward(torch.tensor(0.5, device="cuda"))
    K().cross_entropy_bwd_(logits, V, t, lse, torch.tensor([0.5], device="cuda"), 1.0 / M)
    check()
    assert (logits[:, :V].float() - lr.grad).abs().max().item() < 2e-3 / M + 1e-6 * 0 + 4e-3 * lr.grad.abs().max().item()
    if Vp > V:
        assert logits[:, V:].float().abs().max().item() == 0.0


def test_embedding():
    torch.manual_seed(2)
    B, T, V, H = 4, 256, 1000, 768
    idx = torch.randint(0, V, (B, T), device="cuda")
    wte = torch.randn(V, H, device="cuda")
    wpe = torch.randn(T, H, device="cuda")
    out = K().embedding_fwd(idx, wte, wpe)
    check()
    ref = wte[idx] + wpe[None]
    assert torch.allclose(out.view(B, T, H), ref)
    dx = torch.randn(B * T, H, device="cuda")
    dwte = torch.zeros_like(wte)
    dwpe = torch.zeros_like(wpe)
    K().embedding_bwd(idx, dx, dwte, dwpe)
    check()
    rwte = torch.zeros_like(wte).index_add_(0, idx.reshape(-1), dx)
    assert torch.allclose(dwte, rwte, atol=1e-4)
    assert torch.allclose(dwpe, dx.view(B, T, H).sum(0), atol=1e-4)


@pytest.mark.parametrize("M,N", [(8192, 3072), (1000, 768), (333, 138)])
def test_colsum(M, N):
    torch.manual_seed(3)
    x = torch.randn(M, N, device="cuda").bfloat16()
    out = torch.ones(N, device="cuda")
    K().colsum_bf16(x, out)
    check()
    assert torch.allclose(out, 1 + x.float().sum(0), atol=1e-2, rtol=1e-4)


def test_adamw_matches_torch():
    from heiretsu_b200.optim import FusedAdamW
    from heiretsu_b200.parallel.flat import FlatParams

    torch.manual_seed(4)
    m1 = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.LayerNorm(96), torch.nn.Linear(96, 40)).cuda()
    m2 = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.LayerNorm(96), torch.nn.Linear(96, 40)).cuda()
    m2.load_state_dict(m1.state_dict())
    flat = FlatParams(m2, torch.device("cuda"))
    opt1 = torch.optim.AdamW(m1.parameters(), lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    opt2 = FusedAdamW(flat, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0)
    for _ in range(4):
        x = torch.randn(32, 64, device="cuda")
        l1 = m1(x).pow(2).mean()
        l1.backward()
        torch.nn.utils.clip_grad_norm_(m1.parameters(), 1.0)
        opt1.step()
        opt1.zero_grad()
        with torch.no_grad():
            xx = x.clone().requires_grad_(False)
        l2 = m2(xx).pow(2).mean()
        grads = torch.autograd.grad(l2, list(m2.parameters()))
        for p, g in zip(m2.parameters(), grads):
            p.main_grad.copy_(g)
        opt2.step()
        opt2.zero_grad()
    check()
    for (n, a), b in zip(m1.named_parameters(), m2.parameters()):
        assert torch.allclose(a, b, atol=1e-5, rtol=1e-4), n
        assert torch.allclose(b.w16.float(), b, atol=1e-2, rtol=1e-2), n


def test_adamw_skips_a_nonfinite_step():
    """A NaN anywhere in the flat gradient makes the clip coefficient NaN, and the
    AdamW kernel then leaves weights, moments and the bf16 shadow untouched."""
    from heiretsu_b200.optim import FusedAdamW
    from heiretsu_b200.parallel.flat import FlatParams

    torch.manual_seed(5)
    m = torch.nn.Sequential(torch.nn.Linear(64, 96), torch.nn.LayerNorm(96), torch.nn.Linear(96, 40)).cuda()
    flat = FlatParams(m, torch.device("cuda"))
    opt = FusedAdamW(flat, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0)

    def step(poison):
        flat.grad.normal_()
        if poison:
            flat.grad[flat.grad.numel() // 3] = float("nan")
        opt.step()
        opt.zero_grad()
        torch.cuda.synchronize()

    step(False)
    before = (flat.data.clone(), opt.m.clone(), opt.v.clone(), flat.data16.clone())
    step(True)
    check()
    assert torch.isnan(opt.coef).item()
    after = (flat.data, opt.m, opt.v, flat.data16)
    assert all(torch.equal(a, b) for a, b in zip(before, after))
    step(False)
    check()
    assert not torch.equal(before[0], flat.data) and bool(torch.isfinite(flat.data).all())


@pytest.mark.parametrize("B,T,nh", [(2, 256, 2), (1, 1024, 4), (2, 200, 3), (8, 1024, 12)])
def test_attention_fwd_bwd(B, T, nh):
    torch.manual_seed(5)
    H = nh * 64
    qkv = (torch.randn(B * T, 3 * H, device="cuda")).bfloat16()
    y, lse = K().attention_fwd(qkv, B, T, nh)
    check()
    q, k, v = qkv.float().view(B, T, 3, nh, 64).permute(2, 0, 3, 1, 4).unbind(0)
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    ref2 = ref.transpose(1, 2).reshape(B * T, H)
    err = (y.float() - ref2).abs().max().item()
    assert err < 2e-2, err
    dy = torch.randn(B * T, H, device="cuda").bfloat16()
    ref2.backward(dy.float())
    dqkv = K().attention_bwd(qkv, y, dy, lse, B, T, nh)
    check()
    d = dqkv.float().view(B, T, 3, nh, 64).permute(2, 0, 3, 1, 4)
    for i, (name, g) in enumerate((("q", q.grad), ("k", k.grad), ("v", v.grad))):
        e = (d[i] - g).abs().max().item()
        scale = g.abs().max().item()
        assert e <= 3e-2 * scale + 1e-3, (name, e, scale)


def test_attention_fwd_growing_scores():
    """Keys of the later tiles score far above the earlier ones (K scaled by 5 from
    key 384 on), so the running row max grows by more than the forward's rescale
    threshold several tiles in: the O-in-TMEM forward must rescale its accumulator.
    Checked, with the LSE the backward consumes, against fp32 torch."""
    torch.manual_seed(9)
    B, T, nh = 2, 1024, 4
    H = nh * 64
    x = torch.randn(B, T, 3, H, device="cuda")
    x[:, 384:, 1] *= 5.0
    qkv = x.reshape(B * T, 3 * H).bfloat16()
    y, lse = K().attention_fwd(qkv, B, T, nh)
    check()
    q, k, v = qkv.float().view(B, T, 3, nh, 64).permute(2, 0, 3, 1, 4).unbind(0)
    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B * T, H)
    err = (y.float() - ref).abs().max().item()
    assert err < 2e-2, err
    s = (q @ k.transpose(-1, -2)) / 8.0
    s = s.masked_fill(torch.ones(T, T, device="cuda", dtype=torch.bool).triu(1), float("-inf"))
    lse_ref = torch.logsumexp(s, dim=-1) / math.log(2.0)  # log2 domain
    got = -lse[:, :, :T]
    assert (got - lse_ref).abs().max().item() < 2e-2 * lse_ref.abs().max().item() + 1e-2


@pytest.mark.parametrize("single_pass", [False, True])
def test_cross_entropy_rejects_out_of_range_targets(single_pass):
    """A target outside [0, V) (not ignore_index) is no class: the kernel reads no
    logit for it, reports a bad argument in the status word, and makes that row's
    loss NaN (and, in the single pass, its gradient), as F.cross_entropy refuses it."""
    from heiretsu_b200.ops._C import check_status

    torch.manual_seed(6)
    M, V = 64, 1000
    Vp = 1024
    logits = torch.zeros(M, Vp, device="cuda", dtype=torch.bfloat16)
    logits[:, :V] = torch.randn(M, V, device="cuda").bfloat16()
    t = torch.randint(0, V, (M,), device="cuda")
    t[5] = V + 3
    if single_pass:
        scale = torch.full((1,), 1.0 / M, device="cuda")
        loss, _ = K().cross_entropy_fused_(logits, V, t, scale)
    else:
        loss, _, rows = K().cross_entropy_fwd(logits, V, t)
        assert bool(torch.isnan(rows[5])) and bool(torch.isfinite(rows[:5]).all())
    torch.cuda.synchronize()
    assert bool(torch.isnan(loss))
    with pytest.raises(RuntimeError, match="bad argument"):
        check_status()
    if single_pass:
        assert bool(torch.isnan(logits[5].float()).any()) and bool(torch.isfinite(logits[4].float()).all())


def test_attention_trace_buffer_too_small_is_not_written():
    """A trace buffer with fewer rows than the launch has CTAs turns tracing off for
    that launch (each CTA writes its own row): nothing is written, before or past it."""
    from heiretsu_b200.ops._C import load

    ext = load()
    B, T, nh = 2, 1024, 4  # forward grid: B * nh * 4 query-tile pairs = 32 CTAs
    qkv = torch.randn(B * T, 3 * nh * 64, device="cuda").bfloat16()
    backing = torch.full((64, 80), 7, dtype=torch.int64, device="cuda")
    small = backing[:16]  # 16 rows < 32 CTAs
    ext.attention_set_trace(small)
    try:
        K().attention_fwd(qkv, B, T, nh)
        torch.cuda.synchronize()
    finally:
        ext.attention_set_trace(None)
    check()
    assert bool((backing == 7).all())
    full = torch.zeros(32, 80, dtype=torch.int64, device="cuda")
    ext.attention_set_trace(full)
    try:
        K().attention_fwd(qkv, B, T, nh)
        torch.cuda.synchronize()
    finally:
        ext.attention_set_trace(None)
    assert bool((full[:, 0] > 0).all())  # every CTA stamped its start


def test_embedding_rejects_out_of_range_tokens():
    """A token id outside [0, V) names no row: the forward reads nothing for it, makes
    its output row NaN and reports a bad argument; the backward adds nothing for it."""
    from heiretsu_b200.ops._C import check_status

    torch.manual_seed(8)
    B, T, V, H = 2, 64, 100, 128
    idx = torch.randint(0, V, (B, T), device="cuda")
    idx[1, 7] = V + 5
    idx[0, 3] = -2
    wte = torch.randn(V, H, device="cuda")
    wpe = torch.randn(T, H, device="cuda")
    out = K().embedding_fwd(idx, wte, wpe).view(B, T, H)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="bad argument"):
        check_status()
    assert bool(torch.isnan(out[1, 7]).all()) and bool(torch.isnan(out[0, 3]).all())
    good = torch.ones(B, T, dtype=torch.bool, device="cuda")
    good[1, 7] = good[0, 3] = False
    ref = wte[idx.clamp(0, V - 1)] + wpe[None]
    assert torch.allclose(out[good], ref[good])
    dwte = torch.zeros(V, H, device="cuda")
    dx = torch.randn(B * T, H, device="cuda")
    K().embedding_bwd(idx, dx, dwte, None)
    check()
    ref_dwte = torch.zeros(V, H, device="cuda")
    ref_dwte.index_add_(0, idx.view(-1)[good.view(-1)], dx[good.view(-1)])
    assert torch.allclose(dwte, ref_dwte, atol=1e-5)
    with pytest.raises(RuntimeError, match="position table"):
        K().embedding_fwd(torch.zeros(1, T + 1, dtype=torch.long, device="cuda"), wte, wpe)
