"""Activation checkpointing (``--activation_checkpointing 1``) on the plain engine.

Recomputing each block in backward must change nothing: the same loss and the
same gradients as keeping the activations, with dropout on (the recompute sees
the forward's RNG state) and with collectives inside the blocks (TP, EP).
"""
import pytest
import torch

from dist_util import run_ranks
from test_parallel_cpu import _worker_curve

from heiretsu_b200.config import GPTConfig
from heiretsu_b200.models.gpt import GPT
from heiretsu_b200.parallel.pipeline import StageModule


def _grads(model, x, y, seed):
    torch.manual_seed(seed)
    _, loss, aux = model(x, y)
    (loss + aux).backward()
    return loss.item(), {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}


@pytest.mark.parametrize("moe", [False, True])
def test_recompute_same_loss_and_grads(moe):
    kw = dict(block_size=32, vocab_size=96, n_layer=4, n_head=4, n_embed=32, dropout=0.1)
    if moe:
        kw.update(num_experts=4, top_k=2, moe_freq=2)
    g = torch.Generator().manual_seed(3)
    x = torch.randint(0, 96, (4, 32), generator=g)
    y = torch.randint(0, 96, (4, 32), generator=g)
    torch.manual_seed(5)
    base = GPT(GPTConfig(**kw))
    torch.manual_seed(5)
    ck = GPT(GPTConfig(**kw))
    ck.recompute = True
    l0, g0 = _grads(base, x, y, 17)
    l1, g1 = _grads(ck, x, y, 17)
    assert l0 == l1
    assert g0.keys() == g1.keys()
    for n in g0:
        assert torch.allclose(g0[n], g1[n], atol=1e-6, rtol=0), n


def test_recompute_keeps_only_block_inputs():
    """With recompute, the saved-for-backward tensors of a stage are a fraction of the
    eager ones (counted with saved-tensor hooks)."""
    from heiretsu_b200.topo import Topology

    topo = Topology(dp=1, ep=1, tp=1, pp=1, rank=0, world_size=1, dp_rank=0, ep_rank=0, pp_rank=0, tp_rank=0,
                    tp_group=None, pp_group=None, ep_group=None, dp_group=None)
    cfg = GPTConfig(block_size=32, vocab_size=96, n_layer=4, n_head=4, n_embed=32, dropout=0.0)
    torch.manual_seed(0)
    stage = StageModule(cfg, topo, 0, 1)
    x = torch.randint(0, 96, (4, 32))

    def saved_bytes(recompute):
        stage.recompute = recompute
        total = [0]

        def pack(t):
            total[0] += t.numel() * t.element_size()
            return t

        with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
            h = stage.embed(x)
            stage.forward_blocks(h)
        return total[0]

    eager, ck = saved_bytes(False), saved_bytes(True)
    assert ck * 4 < eager, (ck, eager)


@pytest.mark.parametrize("dp,tp,pp,ep,moe,extra", [
    (1, 2, 1, 1, False, ()),
    (1, 1, 1, 2, True, ()),
    (1, 2, 2, 1, False, ("--pp_schedule", "1f1b")),
])
def test_recompute_training_follows_dense(dp, tp, pp, ep, moe, extra):
    """Five AdamW steps with --activation_checkpointing 1 on TP / EP / PP gloo ranks follow
    the single-process loss curve of the model without recompute."""
    res = run_ranks(_worker_curve, dp * tp * pp * ep, dp, tp, pp, 2, 5, 0, ep, moe,
                    ("--activation_checkpointing", "1") + tuple(extra))
    checked = 0
    for losses, ref in res:
        if losses[0] is None:
            continue
        checked += 1
        for a, b in zip(losses, ref):
            assert abs(a - b) < 1e-4, (losses, ref)
    assert checked >= 1
