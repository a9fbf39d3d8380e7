"""Fused MoE (router, device-side permutation, grouped tcgen05 expert GEMMs, combine)
against an fp32 PyTorch emulation of the same sub-layer.

The emulation is fed the fused path's own bf16 LayerNorm output through a
straight-through estimator, so both route every token identically and only
the kernels' numerics are compared (near-uniform random routers would
otherwise flip top-k choices under bf16 rounding).
"""
import copy

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return (a.float() - b.float()).norm().item() / (b.float().norm().item() + 1e-12)


@pytest.mark.parametrize("E,K,N", [(8, 2, 1024), (4, 1, 384), (8, 2, 200)])
def test_fused_moe_sublayer_matches_torch(E, K, N):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.fused_moe import moe_sublayer_bwd, moe_sublayer_fwd
    from heiretsu_b200.models.gpt import BlockMoE
    from heiretsu_b200.ops._C import check_status, load
    from heiretsu_b200.parallel.flat import FlatParams

    H = 128
    cfg = GPTConfig(block_size=256, vocab_size=100, n_layer=2, n_head=2, n_embed=H, num_experts=E, top_k=K)
    torch.manual_seed(0)
    blk = BlockMoE(cfg).cuda()
    with torch.no_grad():
        blk.moe.router.gate.weight.mul_(5.0)
        for p in blk.parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    ref = copy.deepcopy(blk)
    FlatParams(blk, torch.device("cuda"))
    x1 = torch.randn(N, H, device="cuda")
    x2, aux, saved = moe_sublayer_fwd(blk, None, x1, keep=True)
    torch.cuda.synchronize()
    check_status()
    xn2_bf = saved[1]
    xr = x1.clone().requires_grad_(True)
    xn = F.layer_norm(xr, (H,), ref.ln_2.weight, ref.ln_2.bias, 1e-5)
    xn_st = xn + (xn2_bf.float() - xn).detach()
    y, aux_r = ref.moe(xn_st.view(1, N, H))
    x2_r = xr + y[0]
    topi_fused = saved[4][1].long()
    probs_r = torch.softmax(xn_st.detach() @ ref.moe.router.gate.weight.t(), -1)
    _, topi_r = torch.topk(probs_r, K, -1)
    assert torch.equal(topi_fused, topi_r), "routing differs"
    assert _rel(x2 - x1, x2_r - xr) < 2e-2
    assert abs(aux.item() - aux_r.item()) < 1e-4 * max(1.0, abs(aux_r.item()))
    # backward
    dres = torch.randn(N, H, device="cuda")
    ((x2_r * dres).sum() + aux_r).backward()
    dres_f = dres.clone()
    dres16 = dres_f.bfloat16()
    scratch = torch.empty(load().layernorm_bwd_scratch_rows(N) * 2 * H, device="cuda")
    moe_sublayer_bwd(blk, None, saved, dres_f, dres16, torch.ones((), device="cuda"), scratch)
    torch.cuda.synchronize()
    check_status()
    assert _rel(dres_f, xr.grad) < 3e-2
    rp = dict(ref.named_parameters())
    for n, p in blk.named_parameters():
        if n.startswith(("ln_1", "attn")):
            continue
        assert _rel(p.main_grad, rp[n].grad) < 4e-2, n


def test_fused_moe_model_trains():
    """Fused MoE GPT overfitting one fixed batch: the first loss equals the plain
    path's, and both trajectories fall together."""
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.utils.data import SyntheticLoader

    out = {}
    for engine in ("plain", "fused"):
        args = build_argparser().parse_args([
            "--batch_size", "4", "--block_size", "256", "--grad_accum_steps", "1", "--n_layer", "2", "--n_head", "2",
            "--n_embed", "128", "--dropout", "0", "--amp", "bf16", "--engine", engine, "--num_experts", "4",
            "--learning_rate", "1e-3"])
        torch.manual_seed(0)
        cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=2, n_head=2, n_embed=128, dropout=0.0,
                        num_experts=4, top_k=2, moe_freq=2)
        eng = Engine(args, init_topology(dp=1), torch.device("cuda"), cfg)
        assert eng.fused == (engine == "fused")
        x, y = SyntheticLoader(4, 256, 1000, seed=3).next_batch(torch.device("cuda"))

        class _Fixed:
            def next_batch(self, device):
                return x, y

        loader = _Fixed()
        losses = []
        for _ in range(8):
            l, a = eng.train_step(loader)
            losses.append(float(l.item()))
        out[engine] = losses
        eng.close()
    f, p = out["fused"], out["plain"]
    assert abs(f[0] - p[0]) < 3e-2, (f[0], p[0])
    assert all(v == v for v in f) and f[-1] < f[0] - 0.3, f
    assert abs(f[-1] - p[-1]) < 0.1, (f, p)
