"""Fused dropout against fp32 PyTorch references that rebuild the same masks
(ops/dropout_ref.py restates the counter-based hash)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return (a.float() - b.float()).norm().item() / (b.float().norm().item() + 1e-12)


def test_residual_dropout_epilogue_and_gradient_mask():
    from heiretsu_b200.ops import gemm as G
    from heiretsu_b200.ops import kernels as K
    from heiretsu_b200.ops._C import check_status
    from heiretsu_b200.ops.dropout_ref import residual_mask

    torch.manual_seed(0)
    M, Kd, N, p, site = 512, 256, 384, 0.2, 7
    x = torch.randn(M, Kd, device="cuda").bfloat16()
    w = (0.05 * torch.randn(N, Kd, device="cuda")).bfloat16()
    b = torch.randn(N, device="cuda")
    r = torch.randn(M, N, device="cuda")
    seed = torch.tensor([12345], dtype=torch.int32, device="cuda")
    out = G.linear_fwd_resid(x, w, b, r, drop=(seed, site, p, 0))
    torch.cuda.synchronize()
    check_status()
    mask = residual_mask(12345, site, M, N, p).float().cuda()
    ref = r + mask * (x.float() @ w.float().t() + b)
    assert _rel(out, ref) < 1e-2
    assert torch.all((out - r)[mask == 0] == 0)  # dropped elements carry the residual only
    assert abs((mask == 0).float().mean().item() - p) < 0.01

    g = torch.randn(M, N, device="cuda")
    assert torch.equal(K.dropout_bf16(g, seed, site, p), (g * mask).bfloat16())
    mask2 = residual_mask(12345, site, M, N, p, row0=M).float().cuda()
    assert torch.equal(K.dropout_bf16(g, seed, site, p, row0=M), (g * mask2).bfloat16())
    assert not torch.equal(mask, mask2)


def test_attention_dropout_matches_reference():
    from heiretsu_b200.ops import kernels as K
    from heiretsu_b200.ops._C import check_status
    from heiretsu_b200.ops.dropout_ref import attention_mask

    torch.manual_seed(1)
    B, T, nh, p, site, sval = 2, 256, 2, 0.25, 12, 777
    H = nh * 64
    qkv = (0.5 * torch.randn(B * T, 3 * H, device="cuda")).bfloat16()
    seed = torch.tensor([sval], dtype=torch.int32, device="cuda")
    drop = (seed, site, p, 0, nh)
    y, lse = K.attention_fwd(qkv, B, T, nh, drop=drop)
    dy = torch.randn_like(y)
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, T, nh, drop=drop)
    torch.cuda.synchronize()
    check_status()

    q, k, v = (t.float().detach().requires_grad_(True) for t in
               qkv.view(B, T, 3, nh, 64).permute(2, 0, 3, 1, 4).unbind(0))
    s = q @ k.transpose(-1, -2) / 8.0
    causal = torch.ones(T, T, device="cuda", dtype=torch.bool).tril()
    prob = torch.softmax(s.masked_fill(~causal, float("-inf")), dim=-1)
    mask = attention_mask(sval, site, B, nh, T, p).float().cuda()
    o = (prob * mask) @ v
    y_ref = o.permute(0, 2, 1, 3).reshape(B * T, H)
    assert _rel(y, y_ref) < 2e-2
    o.backward(dy.float().view(B, T, nh, 64).permute(0, 2, 1, 3))
    dq, dk, dv = dqkv.view(B, T, 3, nh, 64).permute(2, 0, 3, 1, 4).unbind(0)
    assert _rel(dq, q.grad) < 3e-2
    assert _rel(dk, k.grad) < 3e-2
    assert _rel(dv, v.grad) < 3e-2


def test_fused_engine_with_dropout_trains():
    """GPT-2-style model with dropout 0.1 on the fused engine: graph-captured steps
    advance the device seed (fresh masks), losses stay finite and fall on a fixed batch."""
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.utils.data import SyntheticLoader

    args = build_argparser().parse_args([
        "--batch_size", "4", "--block_size", "256", "--grad_accum_steps", "2", "--n_layer", "2", "--n_head", "2",
        "--n_embed", "128", "--dropout", "0.1", "--amp", "bf16", "--engine", "fused", "--learning_rate", "1e-3"])
    torch.manual_seed(0)
    cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=2, n_head=2, n_embed=128, dropout=0.1)
    eng = Engine(args, init_topology(dp=1), torch.device("cuda"), cfg)
    assert eng.fused and eng.dropout_seed is not None
    x, y = SyntheticLoader(4, 256, 1000, seed=3).next_batch(torch.device("cuda"))

    class _Fixed:
        def next_batch(self, device):
            return x, y

    s0 = int(eng.dropout_seed.item())
    losses = [float(eng.train_step(_Fixed())[0].item()) for _ in range(8)]
    torch.cuda.synchronize()
    assert int(eng.dropout_seed.item()) == s0 + 8 * 2  # one advance per micro-batch forward, graph replays too
    assert all(v == v for v in losses) and losses[-1] < losses[0] - 0.3, losses
    eng.module.eval()
    with torch.no_grad():
        a = eng.module(x, y, return_logits=False)[1].item()
        b = eng.module(x, y, return_logits=False)[1].item()
    assert a == b  # no dropout in eval
    eng.close()
