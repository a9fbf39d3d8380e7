"""The fused engine's host orchestration on the CPU, with the kernel wrappers
replaced by PyTorch stand-ins (tests/fused_emulation.py): forward/backward
sequencing and saved tensors against the plain model, activation
checkpointing (rerun forwards with the saved dropout snapshot), the
single-pass cross-entropy with its backward correction, and rows whose
target is ignored. The kernels themselves are covered by the GPU tests."""
import pytest
import torch

from fused_emulation import emulate

from heiretsu_b200.config import GPTConfig
from heiretsu_b200.models.gpt import GPT

CFG = dict(block_size=64, vocab_size=200, n_layer=3, n_head=2, n_embed=128)


def _fused(dropout=0.0, recompute=False):
    from heiretsu_b200.parallel.flat import FlatParams

    torch.manual_seed(0)
    m = GPT(GPTConfig(**CFG, dropout=dropout))
    flat = FlatParams(m, torch.device("cpu"))
    m.fused = True
    m.recompute = recompute
    if dropout > 0:
        seed = torch.tensor([77], dtype=torch.int32)
        for layer, blk in enumerate(m.tr.h):
            blk._hb_dropout = (seed, layer, dropout)
    return m, flat


def _step(m, x, y, upstream=1.0):
    from heiretsu_b200.models.fused import gpt_forward_fused

    _, loss, _ = gpt_forward_fused(m, x, y, return_logits=False)
    (upstream * loss).backward()
    return loss.item(), {n: p.main_grad.clone() for n, p in m.named_parameters()}


def _batch(ignore=False):
    g = torch.Generator().manual_seed(5)
    x = torch.randint(0, 200, (2, 64), generator=g)
    y = torch.randint(0, 200, (2, 64), generator=g)
    if ignore:
        y[1, :20] = -100
    return x, y


def _close(a, b, tol):
    for n in a:
        assert (a[n] - b[n]).norm().item() <= tol * (b[n].norm().item() + 1e-8), n


@pytest.mark.parametrize("ignore", [False, True])
def test_emulated_fused_path_matches_the_plain_model(monkeypatch, ignore):
    emulate(monkeypatch)
    x, y = _batch(ignore)
    m, flat = _fused()
    loss_f, grads_f = _step(m, x, y)
    torch.manual_seed(0)
    plain = GPT(GPTConfig(**CFG, dropout=0.0))
    _, loss_p, _ = plain(x, y)
    loss_p.backward()
    assert abs(loss_f - loss_p.item()) < 2e-2
    _close(grads_f, {n: p.grad for n, p in plain.named_parameters()}, 5e-2)


@pytest.mark.parametrize("dropout", [0.0, 0.2])
def test_emulated_recompute_gives_the_same_gradients(monkeypatch, dropout):
    emulate(monkeypatch)
    x, y = _batch()
    l0, g0 = _step(_fused(dropout)[0], x, y)
    m1, flat1 = _fused(dropout, recompute=True)
    l1, g1 = _step(m1, x, y)
    assert l0 == l1
    _close(g1, g0, 1e-6)
    if dropout:  # the masks were really applied: a run without dropout differs
        _, gn = _step(_fused(0.0)[0], x, y)
        assert any((gn[n] - g0[n]).norm() > 1e-3 * g0[n].norm() for n in g0)


@pytest.mark.parametrize("upstream", [1.0, 0.5])
@pytest.mark.parametrize("ignore", [False, True])
def test_emulated_single_pass_cross_entropy(monkeypatch, upstream, ignore):
    import heiretsu_b200.models.fused as FZ

    emulate(monkeypatch)
    x, y = _batch(ignore)
    monkeypatch.setattr(FZ, "CE_FUSED", False)  # the two-kernel path as the reference
    l0, g0 = _step(_fused()[0], x, y, upstream)
    monkeypatch.setattr(FZ, "CE_FUSED", True)
    m1, flat1 = _fused()
    l1, g1 = _step(m1, x, y, upstream)  # grad_hint 1.0: upstream 0.5 goes through the correction
    assert abs(l0 - l1) < 1e-6
    _close(g1, g0, 1e-2)


def test_emulated_grad_hint_skips_the_correction(monkeypatch):
    """With the hint equal to the upstream gradient (1 / accumulation in the trainer), the
    backward correction is a no-op and the gradients equal the two-kernel path's."""
    import heiretsu_b200.models.fused as FZ

    emulate(monkeypatch)
    calls = []
    real = FZ.K.cross_entropy_rescale_

    def spy(g, actual, expected):
        calls.append(bool(torch.equal(actual, expected)))
        return real(g, actual, expected)

    monkeypatch.setattr(FZ.K, "cross_entropy_rescale_", spy)
    x, y = _batch()
    monkeypatch.setattr(FZ, "CE_FUSED", False)  # the two-kernel path as the reference
    l0, g0 = _step(_fused()[0], x, y, 0.5)
    monkeypatch.setattr(FZ, "CE_FUSED", True)
    m1, flat1 = _fused()
    m1.loss_grad_hint = 0.5
    l1, g1 = _step(m1, x, y, 0.5)
    assert calls == [True]
    _close(g1, g0, 1e-2)


def _worker_tp(rank, world, dropout):
    import torch.distributed as dist

    from fused_emulation import emulate_tp

    from heiretsu_b200.models.fused import gpt_forward_fused
    from heiretsu_b200.parallel.flat import FlatParams
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import mark_tp_sharded
    from heiretsu_b200.utils.ckpt import load_from_full, shard_from_full

    emulate_tp(setattr)
    topo = init_topology(dp=1, tp=world)
    cfg = GPTConfig(**dict(CFG, n_layer=2), dropout=dropout)
    g = torch.Generator().manual_seed(9)
    x = torch.randint(0, 200, (4, 64), generator=g)
    y = torch.randint(0, 200, (4, 64), generator=g)

    def with_dropout(m):
        if dropout > 0:
            seed = torch.tensor([31], dtype=torch.int32)
            for layer, blk in enumerate(m.tr.h):
                blk._hb_dropout = (seed, layer, dropout)

    torch.manual_seed(0)
    one = GPT(cfg)
    full = {k: v.detach().clone() for k, v in one.state_dict().items()}
    f1 = FlatParams(one, torch.device("cpu"))
    one.fused = True
    with_dropout(one)
    _, l1, _ = gpt_forward_fused(one, x, y, return_logits=False)
    l1.backward()
    g1 = {n: p.main_grad.clone() for n, p in one.named_parameters()}

    model = GPT(cfg, topo=topo)
    load_from_full(model, full, topo.tp_rank, topo.tp)
    mark_tp_sharded(model)
    flat = FlatParams(model, torch.device("cpu"))
    model.fused = True
    with_dropout(model)
    _, ls, _ = gpt_forward_fused(model, x, y, return_logits=False)
    ls.backward()
    for p in model.parameters():  # token-shard partials of TP-replicated parameters
        if not getattr(p, "tp_sharded", False):
            dist.all_reduce(p.main_grad, group=topo.tp_group)
    lt = ls.detach().clone()
    dist.all_reduce(lt, group=topo.tp_group)
    expect = shard_from_full(model, {**full, **g1}, topo.tp_rank, topo.tp)
    worst = max(((p.main_grad - expect[n]).norm() / (expect[n].norm() + 1e-8)).item()
                for n, p in model.named_parameters())
    del f1, flat
    return abs(lt.item() - l1.item()), worst


@pytest.mark.parametrize("dropout", [0.0, 0.2])
def test_emulated_fused_tp_matches_one_process(dropout):
    """Fused TP orchestration on 2 gloo ranks (all-gather / reduce-scatter GEMM forms
    emulated) against the one-process fused run: with dropout the masks must be the
    single-GPU ones (global head and token-row indices) for the two to agree."""
    from dist_util import run_ranks

    for dloss, worst in run_ranks(_worker_tp, 2, dropout):
        assert dloss < 2e-2, dloss
        assert worst < 5e-2, worst


def test_device_loss_scaler_rule(monkeypatch):
    """fp16 loss scaling of the fused optimizer, with the kernels emulated: a scaled
    gradient steps exactly like the unscaled one (1/S folded into the clip
    coefficient), a non-finite gradient skips the step and halves S, and S doubles
    after growth_interval finite steps in a row."""
    import torch.nn as nn

    from fused_emulation import emulate
    from heiretsu_b200.optim import DeviceLossScaler, FusedAdamW
    from heiretsu_b200.parallel.flat import FlatParams

    emulate(monkeypatch)
    torch.manual_seed(0)
    ref_m, m = nn.Linear(8, 4), nn.Linear(8, 4)
    m.load_state_dict(ref_m.state_dict())
    f_ref = FlatParams(ref_m, torch.device("cpu"))
    f = FlatParams(m, torch.device("cpu"))
    opt_ref = FusedAdamW(f_ref, lr=1e-2, max_grad_norm=0.5)
    sc = DeviceLossScaler(torch.device("cpu"), init_scale=1024.0, growth_interval=3)
    opt = FusedAdamW(f, lr=1e-2, max_grad_norm=0.5, scaler=sc)
    g = torch.randn(f.numel)
    f_ref.grad.copy_(g)
    f.grad.copy_(g * 1024.0)
    opt_ref.step()
    opt.step()
    assert torch.allclose(f.data, f_ref.data, atol=1e-6)
    assert sc.get_scale() == 1024.0
    before = f.data.clone()
    f.grad.fill_(float("inf"))
    opt.step()
    assert torch.equal(before, f.data) and sc.get_scale() == 512.0
    for _ in range(3):
        f.grad.copy_(g * sc.get_scale())
        opt.step()
    assert sc.get_scale() == 1024.0
    st = sc.state_dict()
    assert st["scale"] == 1024.0 and st["_growth_tracker"] == 0
