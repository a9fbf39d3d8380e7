"""Multi-process (gloo, CPU) parity of every parallelism against the dense model.

The oracle is a dense fp32 GPT; each rank loads its shard of the same weights
(TP slices, EP local experts, PP stages) and must reproduce the dense loss
and the matching slices of the dense gradients.
"""
import pytest
import torch

from dist_util import run_ranks

CFG = dict(block_size=32, vocab_size=96, n_layer=4, n_head=4, n_embed=32, dropout=0.0)


def _batch(seed, B=4, T=32, V=96):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, V, (B, T), generator=g), torch.randint(0, V, (B, T), generator=g)


def _dense(cfg_kw, seed=11):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT

    torch.manual_seed(seed)
    m = GPT(GPTConfig(**cfg_kw))
    return m


def _dense_grads(cfg_kw, x, y):
    m = _dense(cfg_kw)
    _, loss, aux = m(x, y)
    (loss + aux).backward()
    return m.state_dict(), {n: p.grad.clone() for n, p in m.named_parameters()}, loss.item()


def _worker_tp_dp(rank, world, dp, tp, moe, ep):
    import torch.distributed as dist

    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.parallel.dp import average_gradients
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.ckpt import load_from_full, shard_from_full

    cfg_kw = dict(CFG, **(dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}))
    topo = init_topology(dp=dp, ep=ep, tp=tp)
    # every DP rank gets its own batch; the dense oracle sees their concatenation
    xs = [_batch(100 + d) for d in range(dp)]
    x, y = xs[topo.dp_rank]
    # Dense oracle: the mean over DP ranks of the dense model on each rank's
    # batch (the MoE aux loss is per rank, as in the reference, and is not
    # linear in the token statistics, so it differs from the aux loss of the
    # concatenated batch).
    per = [_dense_grads(cfg_kw, bx, by) for bx, by in xs]
    full_state = per[0][0]
    dense_grads = {k: sum(g[k] for _, g, _ in per) / dp for k in per[0][1]}
    dense_loss = sum(l for _, _, l in per) / dp
    model = GPT(GPTConfig(**cfg_kw), topo=topo)
    load_from_full(model, full_state, topo.tp_rank, topo.tp)
    _, loss, aux = model(x, y)
    (loss + aux).backward()
    average_gradients(model, topo.dp_group)
    lt = loss.detach().clone()
    if topo.dp_group is not None:
        dist.all_reduce(lt, group=topo.dp_group)
        lt /= topo.dp
    # compare every gradient with the matching slice of the dense gradient
    dense_grad_sd = {k: dense_grads[k] for k in dense_grads}
    expect = shard_from_full(model, {**full_state, **dense_grad_sd}, topo.tp_rank, topo.tp)
    errs = {}
    for n, p in model.named_parameters():
        errs[n] = (p.grad - expect[n]).abs().max().item() if p.grad is not None else float("inf")
    return abs(lt.item() - dense_loss), max(errs.values()), max(errs, key=errs.get)


@pytest.mark.parametrize("dp,tp,moe,ep", [(2, 1, False, 1), (1, 2, False, 1), (2, 2, False, 1), (1, 1, True, 2),
                                          (1, 2, True, 2), (2, 2, True, 2),  # the 8-rank MoE 4-D layout
                                          (4, 1, False, 1), (1, 4, False, 1), (2, 1, True, 4)])
def test_parallel_matches_dense(dp, tp, moe, ep):
    world = dp * tp * ep
    res = run_ranks(_worker_tp_dp, world, dp, tp, moe, ep)
    for rank, (dloss, gerr, worst) in enumerate(res):
        assert dloss < 1e-5, (rank, dloss)
        assert gerr < 1e-5, (rank, gerr, worst)


def _worker_pp(rank, world, pp, tp, accum, dp=1, ep=1, moe=False, schedule="gpipe"):
    import torch.distributed as dist

    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.parallel.dp import average_gradients
    from heiretsu_b200.parallel.pipeline import GPipeEngine, StageModule
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.ckpt import load_from_full, shard_from_full

    cfg_kw = dict(CFG, **(dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}))
    topo = init_topology(dp=dp, ep=ep, tp=tp, pp=pp)
    per_dp = [[_batch(200 + 10 * d + m) for m in range(accum)] for d in range(dp)]
    batches = per_dp[topo.dp_rank]

    class L:
        B = 4

        def __init__(self):
            self.i = 0

        def next_batch(self, device):
            b = batches[self.i % accum]
            self.i += 1
            return b

    # Dense oracle: for each DP rank, the mean over its microbatches of loss
    # (+ aux) accumulated; gradients and losses then averaged over DP ranks.
    grads, tot = None, 0.0
    for d in range(dp):
        dense = _dense(cfg_kw)
        full_state = dense.state_dict()
        for x, y in per_dp[d]:
            _, l, a = dense(x, y)
            ((l + a) / accum).backward()
            tot += l.item() / accum / dp
        g = {n: p.grad.clone() / dp for n, p in dense.named_parameters()}
        grads = g if grads is None else {k: grads[k] + g[k] for k in g}
    stage = StageModule(GPTConfig(**cfg_kw), topo, topo.pp_rank, topo.pp)
    load_from_full(stage, full_state, topo.tp_rank, topo.tp)
    eng = GPipeEngine(stage, topo, schedule=schedule)
    loss, _ = eng.forward_backward(L(), accum, torch.device("cpu"), False, torch.bfloat16, None, 4)
    average_gradients(stage, topo.dp_group)
    if loss is not None and topo.dp_group is not None:
        loss = loss.detach().clone()
        dist.all_reduce(loss, group=topo.dp_group)
        loss /= topo.dp
    expect = shard_from_full(stage, {**full_state, **grads}, topo.tp_rank, topo.tp)
    errs = []
    for n, p in stage.named_parameters():
        e = expect[n]
        if n in ("wte.weight", "lm_head.weight") and pp > 1:
            continue  # untied across stages: checked jointly below
        errs.append((p.grad - e).abs().max().item())
    out = {"loss_err": abs(loss.item() - tot) if loss is not None else 0.0, "gerr": max(errs) if errs else 0.0}
    if stage.is_first:
        out["wte_grad"] = stage.wte.weight.grad.clone()
    if stage.is_last:
        out["head_grad"] = stage.lm_head.weight.grad.clone()
    out["tied_dense"] = grads["tr.wte.weight"].clone()
    out["stage"], out["inflight"] = topo.pp_rank, eng.max_inflight
    return out


# Layouts of the reference suite (tests/run_full_suite.sh:35-65): pp, tp, dp, ep, moe.
@pytest.mark.parametrize("pp,tp,dp,ep,moe", [(2, 1, 1, 1, False), (2, 2, 1, 1, False), (4, 1, 1, 1, False),
                                             (2, 1, 2, 1, False), (2, 2, 2, 1, False), (2, 2, 1, 2, True)])
def test_pipeline_matches_dense(pp, tp, dp, ep, moe):
    res = run_ranks(_worker_pp, pp * tp * dp * ep, pp, tp, 2, dp, ep, moe)
    for r in res:
        assert r["loss_err"] < 1e-5
        assert r["gerr"] < 1e-5
    first = [r for r in res if "wte_grad" in r][0]
    last = [r for r in res if "head_grad" in r][0]
    tied = first["wte_grad"] + last["head_grad"]
    assert (tied - first["tied_dense"]).abs().max().item() < 1e-5


@pytest.mark.parametrize("pp,tp,dp,ep,moe,accum", [(2, 1, 1, 1, False, 4), (4, 1, 1, 1, False, 6),
                                                   (4, 1, 1, 1, False, 2), (2, 2, 1, 1, False, 3),
                                                   (2, 1, 2, 1, False, 4), (2, 1, 1, 2, True, 4)])
def test_1f1b_matches_dense(pp, tp, dp, ep, moe, accum):
    """The 1F1B schedule gives the dense model's loss and gradients (also with fewer
    micro-batches than stages), and stage s never holds more than pp - s micro-batches
    of activations (GPipe holds all of them)."""
    res = run_ranks(_worker_pp, pp * tp * dp * ep, pp, tp, accum, dp, ep, moe, "1f1b")
    for r in res:
        assert r["loss_err"] < 1e-5
        assert r["gerr"] < 1e-5
        assert r["inflight"] == min(pp - r["stage"], accum), r
    first = [r for r in res if "wte_grad" in r][0]
    last = [r for r in res if "head_grad" in r][0]
    assert ((first["wte_grad"] + last["head_grad"]) - first["tied_dense"]).abs().max().item() < 1e-5


def _worker_curve(rank, world, dp, tp, pp, accum, steps, tie=0, ep=1, moe=False, extra=()):
    """Five optimizer steps of the training engine (AdamW, global-norm clip) on
    this layout; returns the logged losses and those of a single-process dense
    engine fed the concatenation of the DP ranks' micro-batches."""
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.utils.ckpt import load_from_full

    moe_kw = dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}
    cfg_kw = dict(CFG, **moe_kw)
    cfg = GPTConfig(**cfg_kw)
    flags = ["--batch_size", "4", "--block_size", "32", "--grad_accum_steps", str(accum), "--n_layer", "4",
             "--n_head", "4", "--n_embed", "32", "--learning_rate", "3e-3", "--grad_clip", "0.5",
             "--engine", "plain", "--amp", "none", "--device", "cpu"]
    for k, v in moe_kw.items():
        flags += [f"--{k}", str(v)]
    data = {(s, m, d): _batch(1000 + 97 * s + 13 * m + d) for s in range(steps) for m in range(accum)
            for d in range(dp)}

    class Feed:
        def __init__(self, dps):
            self.dps, self.i = dps, 0
            self.B = 4 * len(dps)

        def next_batch(self, device):
            s, m = divmod(self.i, accum)
            self.i += 1
            xs = [data[(s, m, d)] for d in self.dps]
            return torch.cat([x for x, _ in xs]), torch.cat([y for _, y in xs])

    full_state = _dense(cfg_kw).state_dict()
    # dense single-process reference on the concatenated DP batches
    eargs = build_argparser().parse_args(flags + ["--dp", "1"])
    ref = Engine(eargs, _single_topo(), torch.device("cpu"), cfg)
    load_from_full(ref.module, full_state)
    if pp > 1 and not tie:
        # Pipeline stages keep separate embedding and lm_head copies (the reference's
        # GPipe layout, pipeline.py:36-143), so the oracle unties them too.
        m = ref.module
        m.lm_head.weight = torch.nn.Parameter(m.tr.wte.weight.detach().clone())
        ref.optimizer = torch.optim.AdamW(m.parameters(), lr=eargs.learning_rate, betas=tuple(eargs.betas),
                                          weight_decay=eargs.weight_decay)
    feed = Feed(list(range(dp)))
    ref_losses = [float(ref.train_step(feed)[0]) for _ in range(steps)]

    topo = init_topology(dp=dp, ep=ep, tp=tp, pp=pp)
    args = build_argparser().parse_args(flags + ["--dp", str(dp), "--ep", str(ep), "--tp", str(tp), "--pp", str(pp),
                                                 "--pp_tie_embeddings", str(tie)] + list(extra))
    eng = Engine(args, topo, torch.device("cpu"), cfg)
    load_from_full(eng.module, full_state, topo.tp_rank, topo.tp)
    if tie and eng.module.is_last:
        with torch.no_grad():
            eng.module.lm_head.weight.normal_()  # after_load must restore it from the first stage
    eng.after_load()
    feed = Feed([topo.dp_rank])
    losses = []
    for _ in range(steps):
        loss, _ = eng.train_step(feed)
        losses.append(None if loss is None else float(loss))
    return losses, ref_losses


def _single_topo():
    from heiretsu_b200.topo import Topology

    return Topology(dp=1, ep=1, tp=1, pp=1, rank=0, world_size=1, dp_rank=0, ep_rank=0, pp_rank=0, tp_rank=0,
                    tp_group=None, pp_group=None, ep_group=None, dp_group=None)


@pytest.mark.parametrize("dp,tp,pp,tie,ep,moe", [(2, 2, 1, 0, 1, False), (1, 2, 2, 0, 1, False),
                                                  (2, 1, 2, 0, 1, False), (1, 2, 2, 1, 1, False),
                                                  (2, 1, 2, 1, 1, False), (1, 1, 1, 0, 2, True),
                                                  (1, 2, 1, 0, 2, True), (1, 1, 2, 0, 2, True)])
def test_five_step_loss_curve_matches_dense(dp, tp, pp, tie, ep, moe):
    """Untied pipeline stages (the reference's layout) follow an untied dense model;
    with --pp_tie_embeddings 1 they follow the tied dense GPT itself. Expert-parallel
    ranks of one replica see the same tokens, so an EP run (dp = 1) follows the
    single-process MoE model."""
    res = run_ranks(_worker_curve, dp * tp * pp * ep, dp, tp, pp, 2, 5, tie, ep, moe)
    checked = 0
    for losses, ref in res:
        assert ref[-1] < ref[0]
        if losses[0] is None:  # pipeline stages before the last log no loss
            continue
        checked += 1
        for a, b in zip(losses, ref):
            assert abs(a - b) < 1e-4, (losses, ref)
    assert checked >= 1


@pytest.mark.parametrize("dp,tp,pp,tie", [(1, 2, 2, 1), (2, 1, 2, 0)])
def test_1f1b_training_follows_dense(dp, tp, pp, tie):
    """--pp_schedule 1f1b through the trainer: five AdamW steps with clipping follow the
    single-process loss curve (four micro-batches, so the steady state is exercised)."""
    res = run_ranks(_worker_curve, dp * tp * pp, dp, tp, pp, 4, 5, tie, 1, False, ("--pp_schedule", "1f1b"))
    checked = 0
    for losses, ref in res:
        if losses[0] is None:
            continue
        checked += 1
        for a, b in zip(losses, ref):
            assert abs(a - b) < 1e-4, (losses, ref)
    assert checked >= 1


def _ops(stage, step):
    """(peer stage, direction, kind, micro-batch) of each transfer of a 1F1B plan step."""
    k = step[0]
    if k == "recv_act":
        return [(stage - 1, "recv", "act", step[1])]
    if k == "recv_grad":
        return [(stage + 1, "recv", "grad", step[1])]
    if k == "send_act":
        return [(stage + 1, "send", "act", step[1])]
    if k == "send_grad":
        return [(stage - 1, "send", "grad", step[1])]
    if k == "send_act+recv_grad":
        return [(stage + 1, "send", "act", step[1]), (stage + 1, "recv", "grad", step[2])]
    if k == "send_grad+recv_act":
        return [(stage - 1, "send", "grad", step[1]), (stage - 1, "recv", "act", step[2])]
    return None  # compute


@pytest.mark.parametrize("pp", range(1, 9))
def test_1f1b_plans_cannot_deadlock(pp):
    """Simulate every stage's 1F1B plan under NCCL's rule (a rank runs its point-to-point
    groups in order; a group ends once every transfer's counterpart is posted by the peer)
    for M = 1..12 micro-batches: every plan runs to the end, sends and receives pair up in
    order on every link, and stage s never holds more than pp - s forwards."""
    from heiretsu_b200.parallel.pipeline import one_f_one_b_plan

    for M in range(1, 13):
        plans = [one_f_one_b_plan(s, pp, M) for s in range(pp)]
        pos = [0] * pp
        while True:
            moved = False
            current = [plans[s][pos[s]] if pos[s] < len(plans[s]) else None for s in range(pp)]
            posted = [set() for _ in range(pp)]
            for s, st in enumerate(current):
                for op in (_ops(s, st) or []) if st is not None else []:
                    posted[s].add(op)
            for s, st in enumerate(current):
                if st is None:
                    continue
                ops = _ops(s, st)
                done = ops is None or all(
                    (s, "recv" if d == "send" else "send", kind, m) in posted[peer] for peer, d, kind, m in ops)
                if done:
                    pos[s] += 1
                    moved = True
            if not moved:
                break
        assert pos == [len(p) for p in plans], (pp, M, pos)
        for s, plan in enumerate(plans):
            f = [st[1] for st in plan if st[0] == "fwd"]
            b = [st[1] for st in plan if st[0] == "bwd"]
            assert f == list(range(M)) and b == list(range(M))
            held = peak = 0
            for st in plan:
                held += {"fwd": 1, "bwd": -1}.get(st[0], 0)
                peak = max(peak, held)
            assert peak == min(pp - s, M)
            for kind, d, nb in (("act", "send", s + 1), ("grad", "send", s - 1), ("act", "recv", s - 1),
                                ("grad", "recv", s + 1)):
                seq = [m for st in plan for peer, dd, k, m in (_ops(s, st) or []) if k == kind and dd == d]
                assert seq == sorted(seq)
                if 0 <= nb < pp:
                    other = [m for st in plans[nb] for peer, dd, k, m in (_ops(nb, st) or [])
                             if k == kind and dd != d]
                    assert seq == other, (s, kind, d)
