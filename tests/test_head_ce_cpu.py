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


def test_head_ce_buffer_pool():
    """Backward hands its logits buffer to the pool and the next forward takes it; two
    forwards in flight (a pipeline) hold two buffers; every result stays exact."""
    g = torch.Generator().manual_seed(4)
    N, H, V = 32, 16, 300
    w = torch.randn(V, H, generator=g, dtype=torch.float64, requires_grad=True)
    pool = []

    def ref(x, t):
        w.grad = None
        xr = x.detach().clone().requires_grad_(True)
        F.cross_entropy((xr @ w.t()), t).backward()
        return xr.grad, w.grad.clone()

    xs = [torch.randn(N, H, generator=g, dtype=torch.float64, requires_grad=True) for _ in range(4)]
    ts = [torch.randint(0, V, (N,), generator=g) for _ in range(4)]
    expect = [ref(x, t) for x, t in zip(xs, ts)]
    w.grad = None
    l0 = head_cross_entropy(xs[0], w, ts[0], pool=pool)
    l0.backward()
    assert len(pool) == 1
    buf = pool[0].data_ptr()
    gw0 = w.grad.clone()
    w.grad = None
    l1 = head_cross_entropy(xs[1], w, ts[1], pool=pool)
    assert not pool  # taken back
    l1.backward()
    assert pool[0].data_ptr() == buf
    gw1 = w.grad.clone()
    w.grad = None
    l2 = head_cross_entropy(xs[2], w, ts[2], pool=pool)  # two in flight: the second one allocates
    l3 = head_cross_entropy(xs[3], w, ts[3], pool=pool)
    l3.backward()
    gw3 = w.grad.clone()
    w.grad = None
    l2.backward()
    gw2 = w.grad.clone()
    assert len(pool) == 2
    for i, gw in enumerate([gw0, gw1, gw2, gw3]):
        assert torch.allclose(xs[i].grad, expect[i][0], rtol=1e-10, atol=1e-12), i
        assert torch.allclose(gw, expect[i][1], rtol=1e-10, atol=1e-12), i
