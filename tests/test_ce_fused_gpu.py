"""Single-pass cross-entropy (the default; HB_CE_FUSED=0 selects two kernels): one kernel writes the loss terms
and the gradient while each logit row is in L2. It must equal the two-kernel
path (forward, then the in-place gradient), also with ignored targets, and the
backward correction must rescale the gradient when the upstream gradient is not
the expected one."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_single_pass_equals_two_kernels():
    from heiretsu_b200.ops import kernels as K
    from heiretsu_b200.ops._C import check_status

    g = torch.Generator(device="cuda").manual_seed(0)
    M, V, Vp = 1024, 50257, 50304
    base = torch.zeros(M, Vp, device="cuda", dtype=torch.bfloat16)
    base[:, :V] = (3 * torch.randn(M, V, device="cuda", generator=g)).bfloat16()
    t = torch.randint(0, V, (M,), device="cuda", generator=g)
    t[:37] = -100
    n = float((t != -100).sum().item())

    a = base.clone()
    loss_a, lse_a, _ = K.cross_entropy_fwd(a, V, t)
    K.cross_entropy_bwd_(a, V, t, lse_a, torch.full((1,), 1.0 / n, device="cuda"), 1.0)
    b = base.clone()
    loss_b, lse_b = K.cross_entropy_fused_(b, V, t, torch.full((1,), 1.0 / n, device="cuda"))
    torch.cuda.synchronize()
    check_status()
    assert torch.allclose(lse_a, lse_b, rtol=0, atol=1e-6)
    assert abs(loss_a.item() - loss_b.item()) < 1e-6
    assert torch.equal(a, b)

    c = b.clone()
    one = torch.ones(1, device="cuda")
    K.cross_entropy_rescale_(c, one, one)
    assert torch.equal(c, b)  # equal scalars: untouched
    K.cross_entropy_rescale_(c, 2 * one, one)
    assert torch.equal(c, (2 * b.float()).bfloat16())


@pytest.mark.parametrize("upstream", [1.0, 0.5])
def test_fused_model_with_single_pass_ce(upstream):
    import heiretsu_b200.models.fused as FZ
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.parallel.flat import FlatParams

    cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=2, n_head=2, n_embed=128, dropout=0.0)
    gx = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randint(0, 1000, (2, 256), device="cuda", generator=gx)
    y = torch.randint(0, 1000, (2, 256), device="cuda", generator=gx)
    grads, losses = [], []
    default = FZ.CE_FUSED
    for single in (False, True):
        torch.manual_seed(0)
        m = GPT(cfg).cuda()
        flat = FlatParams(m, torch.device("cuda"))
        m.fused = True
        FZ.CE_FUSED = single
        try:
            _, loss, _ = m(x, y, return_logits=False)  # grad_hint 1.0: upstream 0.5 takes the correction
            (upstream * loss).backward()
        finally:
            FZ.CE_FUSED = default
        torch.cuda.synchronize()
        losses.append(loss.item())
        grads.append({n: p.main_grad.clone() for n, p in m.named_parameters()})
        del flat
    assert abs(losses[0] - losses[1]) < 1e-6
    for n in grads[0]:
        ref, got = grads[0][n], grads[1][n]
        assert (got - ref).norm().item() <= 1e-2 * (ref.norm().item() + 1e-8), n
