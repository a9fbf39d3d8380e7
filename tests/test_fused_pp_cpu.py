"""Fused pipeline stages on the CPU: the stage modules' fused embedding, blocks
and head (kernels replaced by the PyTorch stand-ins of tests/fused_emulation.py)
driven by the GPipe and 1F1B schedules on 2 gloo ranks, against one process
running the same fused model over the same micro-batches. The kernels are
covered by the GPU tests; this checks the host side of fused pipeline
parallelism: boundary tensors and their gradients, the fused head's gradient
scale under accumulation, and the schedules' ordering."""
import pytest
import torch

from heiretsu_b200.config import GPTConfig

CFG = dict(block_size=64, vocab_size=200, n_layer=4, n_head=2, n_embed=128, dropout=0.0)


def _batch(seed, B):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 200, (B, 64), generator=g), torch.randint(0, 200, (B, 64), generator=g)


def _worker_pp(rank, world, schedule, accum, tp):
    from fused_emulation import emulate_tp

    from heiretsu_b200.models.fused import gpt_forward_fused
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.parallel.flat import FlatParams
    from heiretsu_b200.parallel.pipeline import GPipeEngine, StageModule
    from heiretsu_b200.topo import init_topology
    import torch.distributed as dist

    from heiretsu_b200.trainer import mark_tp_sharded, replication_weight
    from heiretsu_b200.utils.ckpt import load_from_full, shard_from_full

    emulate_tp(setattr)
    setattr(StageModule, "_fused_on", lambda self, t: self.fused)  # the stand-ins run on CPU tensors
    cfg = GPTConfig(**CFG)
    B = 2 * tp  # fused TP wants 128-token multiples per TP rank
    batches = [_batch(300 + m, B) for m in range(accum)]

    torch.manual_seed(0)
    one = GPT(cfg)
    full = {k: v.detach().clone() for k, v in one.state_dict().items()}
    FlatParams(one, torch.device("cpu"))
    one.fused = True
    one.loss_grad_hint = 1.0 / accum
    tot = 0.0
    for x, y in batches:
        _, l, a = gpt_forward_fused(one, x, y, return_logits=False)
        ((l + a) / accum).backward()
        tot += l.item() / accum
    g1 = {n: p.main_grad.clone() for n, p in one.named_parameters()}

    topo = init_topology(dp=1, tp=tp, pp=world // tp)
    stage = StageModule(cfg, topo, topo.pp_rank, topo.pp)
    load_from_full(stage, full, topo.tp_rank, topo.tp)
    mark_tp_sharded(stage)
    FlatParams(stage, torch.device("cpu"), weight_of=replication_weight(topo))
    stage.fused = True
    stage.loss_grad_hint = 1.0 / accum

    class Loader:
        def __init__(self):
            self.i = 0

        def next_batch(self, device):
            b = batches[self.i % accum]
            self.i += 1
            return b

    eng = GPipeEngine(stage, topo, schedule=schedule)
    eng.fused_head = True
    loss, _ = eng.forward_backward(Loader(), accum, torch.device("cpu"), False, torch.bfloat16, None, B)
    if tp > 1:  # token-shard partials of TP-replicated parameters; shard losses
        for p in stage.parameters():
            if not getattr(p, "tp_sharded", False):
                dist.all_reduce(p.main_grad, group=topo.tp_group)
        if loss is not None:
            loss = loss.detach().clone()
            dist.all_reduce(loss, group=topo.tp_group)
    expect = shard_from_full(stage, {**full, **g1}, topo.tp_rank, topo.tp)
    worst = 0.0
    for n, p in stage.named_parameters():
        if n in ("wte.weight", "lm_head.weight"):
            continue  # untied across stages: checked jointly below
        worst = max(worst, ((p.main_grad - expect[n]).norm() / (expect[n].norm() + 1e-8)).item())
    out = {"loss_err": abs(loss.item() - tot) if loss is not None else 0.0, "worst": worst,
           "tied_dense": expect["wte.weight" if stage.is_first else "lm_head.weight"].clone(),
           "tp_rank": topo.tp_rank}
    if stage.is_first:
        out["wte_grad"] = stage.wte.weight.main_grad.clone()
    if stage.is_last:
        out["head_grad"] = stage.lm_head.weight.main_grad.clone()
    return out


@pytest.mark.parametrize("schedule,accum,tp", [("gpipe", 2, 1), ("1f1b", 3, 1), ("1f1b", 1, 1), ("1f1b", 2, 2)])
def test_emulated_fused_pipeline_matches_one_process(schedule, accum, tp):
    """pp2 (and pp2 x tp2 on 4 ranks: the TP blocks run on token shards and the stage
    boundary is each TP rank's shard). With TP the row-parallel outputs are summed
    as 16-bit partials, as on the GPU, so gradients agree to bf16 noise (the fused TP
    test's tolerance); without TP to fp32 summation order."""
    from dist_util import run_ranks

    tol = 1e-4 if tp == 1 else 2e-2
    res = run_ranks(_worker_pp, 2 * tp, schedule, accum, tp)
    for r in res:
        assert r["loss_err"] < (1e-5 if tp == 1 else 1e-3), r["loss_err"]
        assert r["worst"] < tol, r["worst"]
    for t in range(tp):  # the untied embedding and head together carry the tied gradient
        first = [r for r in res if "wte_grad" in r and r["tp_rank"] == t][0]
        last = [r for r in res if "head_grad" in r and r["tp_rank"] == t][0]
        tied = first["wte_grad"] + last["head_grad"]
        rel = ((tied - first["tied_dense"]).norm() / first["tied_dense"].norm()).item()
        assert rel < tol, rel
