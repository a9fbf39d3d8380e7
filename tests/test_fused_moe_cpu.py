"""The fused MoE sub-layer's host orchestration (models/fused_moe.py) on the CPU,
with its kernels replaced by PyTorch stand-ins (tests/moe_emulation.py, on top
of tests/fused_emulation.py): routing and padded expert windows, the grouped
expert GEMMs, the one-GPU combine and the backward against the plain MoE model,
expert parallelism on 2 gloo ranks (each rank runs its own experts; the second
expert GEMM's combine pushes rows into every rank's slot buffer; the backward
sums partial input gradients) against the one-process fused run, and expert x
tensor parallelism (ep2 x tp2, 4 gloo ranks, MoE sub-layers on TP token
shards) against dp2 x tp2 with every expert on every rank. The kernels
themselves are covered by the GPU tests."""
import torch

from fused_emulation import emulate
from moe_emulation import emulate_moe

from heiretsu_b200.config import GPTConfig
from heiretsu_b200.models.gpt import GPT

CFG = dict(block_size=64, vocab_size=200, n_layer=2, n_head=2, n_embed=128, dropout=0.0, num_experts=4, top_k=2,
           moe_freq=2)


def _model(cfg, topo=None, full=None):
    from heiretsu_b200.parallel.flat import FlatParams
    from heiretsu_b200.trainer import mark_tp_sharded, replication_weight
    from heiretsu_b200.utils.ckpt import load_from_full

    torch.manual_seed(0)
    m = GPT(cfg, topo=topo)
    if full is None:
        with torch.no_grad():  # decisive routing: no near-ties between the 2nd and 3rd expert
            for blk in m.tr.h:
                if hasattr(blk, "moe"):
                    blk.moe.router.gate.weight.mul_(20.0)
    else:
        load_from_full(m, full)
        mark_tp_sharded(m)
    flat = FlatParams(m, torch.device("cpu"), weight_of=replication_weight(topo) if topo is not None else None)
    m.fused = True
    return m, flat


def _batch(B=2):
    g = torch.Generator().manual_seed(5)
    return torch.randint(0, 200, (B, 64), generator=g), torch.randint(0, 200, (B, 64), generator=g)


def _fused_step(m, x, y):
    from heiretsu_b200.models.fused import gpt_forward_fused

    _, loss, aux = gpt_forward_fused(m, x, y, return_logits=False)
    (loss + aux).backward()
    return loss.item(), aux.item(), {n: p.main_grad.clone() for n, p in m.named_parameters()}


def test_emulated_fused_moe_matches_the_plain_model(monkeypatch):
    emulate(monkeypatch)
    emulate_moe(monkeypatch.setattr)
    cfg = GPTConfig(**CFG)
    x, y = _batch()
    m, flat = _model(cfg)
    full = {k: v.detach().clone() for k, v in m.state_dict().items()}
    loss_f, aux_f, grads_f = _fused_step(m, x, y)
    plain = GPT(cfg)
    plain.load_state_dict(full)
    _, loss_p, aux_p = plain(x, y)
    (loss_p + aux_p).backward()
    assert abs(loss_f - loss_p.item()) < 2e-2
    assert abs(aux_f - aux_p.item()) < 1e-3 * max(1.0, abs(aux_p.item()))
    for n, p in plain.named_parameters():
        rel = (grads_f[n] - p.grad).norm().item() / (p.grad.norm().item() + 1e-8)
        assert rel < 5e-2, (n, rel)
    # every expert of the MoE block took tokens, so each grouped GEMM segment was exercised
    counts = [blk.moe._expert_counts for blk in m.tr.h if hasattr(blk, "moe")][0]
    assert bool((counts > 0).all()), counts


def _worker_ep(rank, world):
    import torch.distributed as dist

    from fused_emulation import emulate_tp

    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.ckpt import shard_from_full

    emulate_tp(setattr)
    emulate_moe(setattr)
    cfg = GPTConfig(**CFG)
    x, y = _batch()
    one, f1 = _model(cfg)
    full = {k: v.detach().clone() for k, v in one.state_dict().items()}
    l1, a1, g1 = _fused_step(one, x, y)

    topo = init_topology(dp=1, ep=world)
    model, flat = _model(cfg, topo, full)
    results = []
    for _ in range(2):  # the second pass reuses both slot buffers
        flat.zero_grad()
        le, ae, ge = _fused_step(model, x, y)
        expect = shard_from_full(model, {**full, **g1})
        worst = max(((ge[n] - expect[n]).norm() / (expect[n].norm() + 1e-8)).item()
                    for n, _ in model.named_parameters())
        results.append((abs(le - l1), abs(ae - a1), worst))
    dist.barrier()
    return results


def test_emulated_fused_ep2_matches_one_process():
    """Expert parallelism over 2 gloo ranks: the forward is the one-process fused
    forward bit for bit (the slots hold the terms the one-GPU combine adds, in the
    same order) and the gradients agree up to the order of the backward's sums."""
    from dist_util import run_ranks

    for per_pass in run_ranks(_worker_ep, 2):
        for dloss, daux, worst in per_pass:
            assert dloss == 0.0 and daux == 0.0, (dloss, daux)
            assert worst < 1e-4, worst


def _worker_ep_tp(rank, world):
    import torch.distributed as dist

    from fused_emulation import emulate_tp

    from heiretsu_b200.topo import init_topology

    emulate_tp(setattr)
    emulate_moe(setattr)
    cfg = GPTConfig(**dict(CFG, n_layer=4))
    x, y = _batch(B=4)
    one, _ = _model(cfg)
    full = {k: v.detach().clone() for k, v in one.state_dict().items()}

    def run(topo):
        from heiretsu_b200.parallel.flat import FlatParams
        from heiretsu_b200.trainer import mark_tp_sharded, replication_weight
        from heiretsu_b200.utils.ckpt import load_from_full

        torch.manual_seed(0)
        model = GPT(cfg, topo=topo)
        load_from_full(model, full, topo.tp_rank, topo.tp)
        mark_tp_sharded(model)
        flat = FlatParams(model, torch.device("cpu"), weight_of=replication_weight(topo))
        model.fused = True
        for _ in range(2):  # the second pass reuses both slot buffers
            flat.zero_grad()
            _, loss_s, aux_s = gpt_forward_fused(model, x, y, return_logits=False)
            (loss_s + aux_s).backward()
            for p in model.parameters():  # token-shard partials of TP-replicated parameters
                if not getattr(p, "tp_sharded", False):
                    dist.all_reduce(p.main_grad, group=topo.tp_group)
        lt = loss_s.detach().clone()
        dist.all_reduce(lt, group=topo.tp_group)
        return model, lt.item()

    from heiretsu_b200.models.fused import gpt_forward_fused

    topo_ep = init_topology(dp=1, ep=2, tp=2)
    model_ep, loss_ep = run(topo_ep)
    topo_tp = init_topology(dp=2, tp=2)  # same TP partner and token shard for every rank, all experts
    model_tp, loss_tp = run(topo_tp)
    tp_grads = {n: p.main_grad for n, p in model_tp.named_parameters()}
    E_l = cfg.num_experts // 2
    worst = 0.0
    for n, p in model_ep.named_parameters():
        ref = n
        if ".experts." in n:
            pre, rest = n.split(".experts.", 1)
            j, tail = rest.split(".", 1)
            ref = f"{pre}.experts.{topo_ep.ep_rank * E_l + int(j)}.{tail}"
        worst = max(worst, ((p.main_grad - tp_grads[ref]).norm() / (tp_grads[ref].norm() + 1e-8)).item())
    dist.barrier()
    return abs(loss_ep - loss_tp), worst


def test_emulated_fused_ep2_tp2_matches_tp2():
    """Expert x tensor parallelism (ep2 x tp2, 4 gloo ranks; the TP blocks run on token
    shards and each EP pair shares one) against dp2 x tp2 with every expert on every
    rank: same token shards, same TP partners, so the forward agrees bit for bit."""
    from dist_util import run_ranks

    for dloss, worst in run_ranks(_worker_ep_tp, 4):
        assert dloss == 0.0, dloss
        assert worst < 1e-4, worst
