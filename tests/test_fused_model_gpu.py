"""The fused sm_100a GPT path against the plain fp32 PyTorch path on the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _models(n_layer=2, n_embed=128, n_head=2, V=1000, T=256, seed=0):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.parallel.flat import FlatParams

    cfg = GPTConfig(block_size=T, vocab_size=V, n_layer=n_layer, n_head=n_head, n_embed=n_embed, dropout=0.0)
    torch.manual_seed(seed)
    ref = GPT(cfg).cuda()
    torch.manual_seed(seed)
    fz = GPT(cfg).cuda()
    flat = FlatParams(fz, torch.device("cuda"))
    fz.fused = True
    return cfg, ref, fz, flat


@pytest.mark.parametrize("n_layer,n_embed,n_head,V,T", [(2, 128, 2, 1000, 256), (2, 768, 12, 50257, 1024)])
def test_fused_loss_and_grads(n_layer, n_embed, n_head, V, T):
    from heiretsu_b200.ops._C import check_status

    cfg, ref, fz, flat = _models(n_layer, n_embed, n_head, V, T)
    B = 2
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randint(0, V, (B, T), device="cuda", generator=g)
    y = torch.randint(0, V, (B, T), device="cuda", generator=g)
    _, loss_r, _ = ref(x, y)
    loss_r.backward()
    _, loss_f, _ = fz(x, y, return_logits=False)
    loss_f.backward()
    torch.cuda.synchronize()
    check_status()
    assert abs(loss_f.item() - loss_r.item()) < 2e-2, (loss_f.item(), loss_r.item())
    rp = dict(ref.named_parameters())
    bad = []
    for n, p in fz.named_parameters():
        gr = rp[n].grad
        gf = p.main_grad
        denom = gr.norm().item() + 1e-8
        rel = (gf - gr).norm().item() / denom
        if rel > 5e-2:
            bad.append((n, rel))
    assert not bad, bad


def test_fused_grads_with_ignored_targets():
    """Targets equal to -100 (F.cross_entropy's ignore_index) count for nothing: the
    loss and the gradients are means over the remaining rows only."""
    from heiretsu_b200.ops._C import check_status

    cfg, ref, fz, flat = _models()
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randint(0, 1000, (2, 256), device="cuda", generator=g)
    y = torch.randint(0, 1000, (2, 256), device="cuda", generator=g)
    y[0, :100] = -100
    _, loss_r, _ = ref(x, y)
    loss_r.backward()
    _, loss_f, _ = fz(x, y, return_logits=False)
    loss_f.backward()
    torch.cuda.synchronize()
    check_status()
    assert abs(loss_f.item() - loss_r.item()) < 2e-2, (loss_f.item(), loss_r.item())
    rp = dict(ref.named_parameters())
    bad = []
    for n, p in fz.named_parameters():
        gr, gf = rp[n].grad, p.main_grad
        rel = (gf - gr).norm().item() / (gr.norm().item() + 1e-8)
        if rel > 5e-2:
            bad.append((n, rel))
    assert not bad, bad


def test_fused_logits_match():
    cfg, ref, fz, flat = _models()
    x = torch.randint(0, 1000, (2, 256), device="cuda")
    with torch.no_grad():
        lr, _, _ = ref(x)
        lf, _, _ = fz(x)
    assert (lr - lf).abs().max().item() < 5e-2


def test_cuda_graph_step_matches_eager():
    """Graph-captured training steps give the same losses as eager steps."""
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.utils.data import SyntheticLoader

    losses = {}
    for graph in (0, 1):
        args = build_argparser().parse_args([
            "--batch_size", "2", "--block_size", "256", "--grad_accum_steps", "2", "--n_layer", "2", "--n_head", "2",
            "--n_embed", "128", "--dropout", "0", "--amp", "bf16", "--engine", "fused", "--cuda_graph", str(graph)])
        torch.manual_seed(0)
        cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=2, n_head=2, n_embed=128, dropout=0.0)
        eng = Engine(args, init_topology(dp=1), torch.device("cuda"), cfg)
        loader = SyntheticLoader(2, 256, 1000, seed=3)
        out = []
        for _ in range(6):
            l, _ = eng.train_step(loader)
            out.append(float(l.item()))
        losses[graph] = out
    assert all(abs(a - b) < 2e-3 for a, b in zip(losses[0], losses[1])), losses
    assert losses[1][-1] < losses[1][0]
