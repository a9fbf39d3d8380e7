"""The plain path's fused lm_head + cross-entropy against F.cross_entropy on logits."""
import pytest
import torch
import torch.nn.functional as F

from heiretsu_b200.models.gpt import head_cross_entropy


@pytest.mark.parametrize("ignore_some", [False, True])
def test_head_ce_matches_torch(ignore_some):
    g = torch.Generator().manual_seed(0)
    N, H, V = 96, 32, 1000
    x = torch.randn(4, N // 4, H, generator=g, dtype=torch.float64, requires_grad=True)
    w = torch.randn(V, H, generator=g, dtype=torch.float64, requires_grad=True)
    t = torch.randint(0, V, (4, N // 4), generator=g)
    if ignore_some:
        t[0, :5] = -100
    loss = head_cross_entropy(x, w, t)
    (2.5 * loss).backward()
    gx, gw = x.grad.clone(), w.grad.clone()
    x.grad = w.grad = None
    ref = F.cross_entropy((x @ w.t()).reshape(-1, V), t.reshape(-1))
    (2.5 * ref).backward()
    assert torch.allclose(loss, ref, rtol=1e-12, atol=1e-12)
    assert torch.allclose(gx, x.grad, rtol=1e-10, atol=1e-12)
    assert torch.allclose(gw, w.grad, rtol=1e-10, atol=1e-12)


def test_head_ce_all_ignored_is_nan_and_single_backward():
    x = torch.randn(3, 8, requires_grad=True)
    w = torch.randn(20, 8, requires_grad=True)
    assert torch.isnan(head_cross_entropy(x, w, torch.full((3,), -100)))
    loss = head_cross_entropy(x, w, torch.tensor([1, 2, 3]))
    loss.backward(retain_graph=True)
    with pytest.raises(RuntimeError, match="only once"):
        loss.backward()


def test_gpt_forward_without_logits_matches():
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT

    torch.manual_seed(0)
    m = GPT(GPTConfig(block_size=32, vocab_size=96, n_layer=2, n_head=2, n_embed=32, dropout=0.0))
    x = torch.randint(0, 96, (2, 32))
    y = torch.randint(0, 96, (2, 32))
    logits, l1, _ = m(x, y)
    l1.backward()
    g1 = {n: p.grad.clone() for n, p in m.named_parameters()}
    m.zero_grad()
    none, l2, _ = m(x, y, return_logits=False)
    l2.backward()
    assert none is None and logits is not None
    assert abs(l1.item() - l2.item()) < 1e-6
    for n, p in m.named_parameters():
        assert torch.allclose(g1[n], p.grad, atol=1e-6, rtol=1e-5), n
