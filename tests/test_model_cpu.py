"""fp32 CPU parity of the model against the reference (same seed -> same weights, logits, losses)."""
import pytest
import torch

from oracle import have_reference, load_reference

from heiretsu_b200.config import GPTConfig
from heiretsu_b200.models.gpt import GPT

pytestmark = pytest.mark.skipif(not have_reference(), reason="reference not available")


def small_cfg(**kw):
    base = dict(block_size=64, vocab_size=128, n_layer=3, n_head=4, n_embed=32, dropout=0.0)
    base.update(kw)
    return base


def build_pair(seed=1234, **kw):
    R = load_reference()
    torch.manual_seed(seed)
    ref = R.gpt_model.GPT(R.gpt_model.GPTConfig(**small_cfg(**kw)))
    torch.manual_seed(seed)
    ours = GPT(GPTConfig(**small_cfg(**kw)))
    return ref, ours


@pytest.mark.parametrize("moe", [False, True])
def test_same_seed_same_state_dict(moe):
    kw = dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}
    ref, ours = build_pair(**kw)
    rs, os_ = ref.state_dict(), ours.state_dict()
    assert list(rs.keys()) == list(os_.keys())
    for k in rs:
        assert rs[k].shape == os_[k].shape, k
        assert torch.equal(rs[k], os_[k]), k


@pytest.mark.parametrize("moe", [False, True])
def test_forward_backward_parity(moe):
    kw = dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}
    ref, ours = build_pair(**kw)
    g = torch.Generator().manual_seed(0)
    x = torch.randint(0, 128, (2, 64), generator=g)
    y = torch.randint(0, 128, (2, 64), generator=g)
    lr, loss_r, aux_r = ref(x, y)
    lo, loss_o, aux_o = ours(x, y)
    assert (lr - lo).abs().max().item() <= 1e-4
    assert abs(loss_r.item() - loss_o.item()) <= 1e-5
    assert abs(aux_r.item() - aux_o.item()) <= 1e-6
    (loss_r + aux_r).backward()
    (loss_o + aux_o).backward()
    ro = dict(ours.named_parameters())
    for n, p in ref.named_parameters():
        assert p.grad is not None and ro[n].grad is not None, n
        assert (p.grad - ro[n].grad).abs().max().item() <= 1e-5, n


def test_training_loss_curve_matches_reference():
    """5 AdamW steps with clipping: same losses as the reference's update rule."""
    ref, ours = build_pair()
    opt_r = torch.optim.AdamW(ref.parameters(), lr=6e-4, betas=(0.9, 0.95), weight_decay=0.1)
    opt_o = torch.optim.AdamW(ours.parameters(), lr=6e-4, betas=(0.9, 0.95), weight_decay=0.1)
    g = torch.Generator().manual_seed(5)
    for _ in range(5):
        x = torch.randint(0, 128, (4, 64), generator=g)
        y = torch.randint(0, 128, (4, 64), generator=g)
        lr_ = []
        for m, opt in ((ref, opt_r), (ours, opt_o)):
            _, loss, aux = m(x, y)
            (loss + aux).backward()
            torch.nn.utils.clip_grad_norm_(m.parameters(), 1.0)
            opt.step()
            opt.zero_grad(set_to_none=True)
            lr_.append(loss.item())
        assert abs(lr_[0] - lr_[1]) <= 1e-4, lr_


def test_block_size_guard():
    _, ours = build_pair()
    with pytest.raises(ValueError):
        ours(torch.zeros(1, 65, dtype=torch.long))
