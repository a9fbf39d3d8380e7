"""CPU unit tests: MoE pieces, CLI parity, checkpoint round trips, data loader, topology."""
import os
import re

import pytest
import torch

from oracle import have_reference, load_reference, ref_dir

from heiretsu_b200.config import GPTConfig
from heiretsu_b200.models.gpt import GPT
from heiretsu_b200.models.moe import Expert, MoELayer, Router, load_balancing_loss, make_moe_config


def test_router_shapes_and_normalisation():
    r = Router(64, 8, 2)
    idx, w, probs = r(torch.randn(8, 64))
    assert idx.shape == (8, 2) and w.shape == (8, 2) and probs.shape == (8, 8)
    assert idx.min() >= 0 and idx.max() < 8
    assert torch.allclose(w.sum(-1), torch.ones(8))
    assert torch.allclose(probs.sum(-1), torch.ones(8))


def test_expert_and_aux_loss():
    assert Expert(64, 256)(torch.randn(10, 64)).shape == (10, 64)
    probs = torch.softmax(torch.randn(16, 4), -1)
    aux = load_balancing_loss(probs, torch.randint(0, 4, (16, 2)), 4, 2, 0.01)
    assert aux.shape == () and aux.item() >= 0


@pytest.mark.skipif(not have_reference(), reason="reference not available")
def test_moe_layer_matches_reference():
    R = load_reference()
    torch.manual_seed(3)
    ref = R.moe.MoELayer(R.moe.make_moe_config(32, num_experts=4, top_k=2))
    torch.manual_seed(3)
    ours = MoELayer(make_moe_config(32, num_experts=4, top_k=2))
    ours.load_state_dict(ref.state_dict())
    x = torch.randn(2, 16, 32, requires_grad=True)
    x2 = x.detach().clone().requires_grad_(True)
    yr, ar = ref(x)
    yo, ao = ours(x2)
    assert torch.allclose(yr, yo, atol=1e-6) and torch.allclose(ar, ao, atol=1e-7)
    (yr.sum() + ar).backward()
    (yo.sum() + ao).backward()
    assert torch.allclose(x.grad, x2.grad, atol=1e-5)
    for (n, a), b in zip(ref.named_parameters(), ours.parameters()):
        assert torch.allclose(a.grad, b.grad, atol=1e-5), n


@pytest.mark.skipif(not have_reference(), reason="reference not available")
def test_cli_accepts_every_reference_flag():
    """Every reference flag exists with the same default and choices."""
    import argparse

    src = open(os.path.join(ref_dir(), "train.py")).read()
    body = src[src.index("p = argparse.ArgumentParser("):src.index("args = p.parse_args()")]
    ns = {"argparse": argparse}
    import textwrap

    exec(textwrap.dedent("    " + body), ns)  # the reference's own parser
    ref = ns["p"]
    from heiretsu_b200.trainer import build_argparser

    ours = {a.dest: a for a in build_argparser()._actions}
    for act in ref._actions:
        if act.dest == "help":
            continue
        assert act.dest in ours, act.dest
        o = ours[act.dest]
        assert o.default == act.default or tuple(o.default or ()) == tuple(act.default or ()), act.dest
        assert (o.choices or None) == (act.choices or None), act.dest


@pytest.mark.skipif(not have_reference(), reason="reference not available")
def test_checkpoint_round_trips_with_reference(tmp_path):
    from types import SimpleNamespace

    from heiretsu_b200.utils.ckpt import load_checkpoint, save_checkpoint

    R = load_reference()
    kw = dict(block_size=32, vocab_size=64, n_layer=2, n_head=2, n_embed=32)
    torch.manual_seed(0)
    ours = GPT(GPTConfig(**kw))
    topo = SimpleNamespace(dp=1, ep=1, tp=1, pp=1, dp_rank=0, ep_rank=0, tp_rank=0, pp_rank=0, is_main=True)
    path = save_checkpoint(ours, GPTConfig(**kw), 7, topo, str(tmp_path))
    assert os.path.basename(path) == "ckpt_0000007.pt"
    obj = torch.load(path, weights_only=False)
    assert set(obj) == {"model", "cfg", "step"} and obj["step"] == 7
    ref = R.gpt_model.GPT(R.gpt_model.GPTConfig(**obj["cfg"]))
    ref.load_state_dict(obj["model"])
    x = torch.randint(0, 64, (2, 32))
    assert torch.allclose(ref(x)[0], ours(x)[0], atol=1e-6)
    # reference -> ours (through the reference's own save layout)
    torch.manual_seed(1)
    ref2 = R.gpt_model.GPT(R.gpt_model.GPTConfig(**kw))
    p2 = tmp_path / "ref.pt"
    torch.save({"model": ref2.state_dict(), "cfg": obj["cfg"], "step": 1}, p2)
    ours2 = GPT(GPTConfig(**kw))
    load_checkpoint(ours2, str(p2))
    assert torch.allclose(ref2(x)[0], ours2(x)[0], atol=1e-6)


@pytest.mark.skipif(not have_reference(), reason="reference not available")
def test_bin_loader_matches_reference(tmp_path):
    import importlib.util
    import sys

    from heiretsu_b200.utils.data import RandomBatchLoader, write_synthetic_bins

    write_synthetic_bins(str(tmp_path), vocab_size=500, train_tokens=20000, val_tokens=5000, seed=1, num_train=2)
    load_reference()
    spec = importlib.util.spec_from_file_location("ref_train", os.path.join(ref_dir(), "train.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    a = mod.RandomBatchLoader(str(tmp_path), "train", 4, 16, None, seed=5, rank=1, dp_rank=1, dp_size=2, log_rank=1)
    b = RandomBatchLoader(str(tmp_path), "train", 4, 16, None, seed=5, rank=1, dp_rank=1, dp_size=2, log_rank=1)
    for _ in range(3):
        xa, ya = a.next_batch("cpu")
        xb, yb = b.next_batch("cpu")
        assert torch.equal(xa, xb) and torch.equal(ya, yb)


def test_topology_layout():
    from heiretsu_b200.topo import coords_from_rank, group_members, rank_from_coords

    for world in [(2, 1, 2, 2), (1, 2, 2, 2), (2, 2, 1, 2)]:
        dp, ep, tp, pp = world
        n = dp * ep * tp * pp
        for r in range(n):
            d, e, p, t = coords_from_rank(r, dp, ep, tp, pp)
            assert rank_from_coords(d, e, p, t, dp, ep, tp, pp) == r
            g = group_members(dp, ep, tp, pp, r)
            assert r in g["tp"] and r in g["dp"] and r in g["ep"] and r in g["pp"]
            assert g["tp"] == list(range(r - t, r - t + tp))  # TP ranks are consecutive
    if have_reference():
        R = load_reference()
        for r in range(16):
            assert R.topo.coords_from_rank(r, 2, 2, 2, 2) == coords_from_rank(r, 2, 2, 2, 2)


def test_cpu_trainer_runs_and_loss_drops(tmp_path):
    from heiretsu_b200.trainer import main

    main(["--device", "cpu", "--synthetic_data", "--n_layer", "2", "--n_head", "2", "--n_embed", "32",
          "--block_size", "32", "--batch_size", "4", "--max_iters", "3", "--eval_interval", "3", "--eval_iters", "1",
          "--dropout", "0", "--save_interval", "3", "--out_dir", str(tmp_path)])
    assert (tmp_path / "ckpt_0000003.pt").exists()


def test_region_timer_and_nvtx_cpu():
    import time

    from heiretsu_b200.utils.profiling import RegionTimer, nvtx, tokens_per_second

    t = RegionTimer()
    for _ in range(3):
        with t.region("a"), nvtx("a"):
            time.sleep(0.002)
    with t.region("b"):
        pass
    s = t.summary()
    assert set(s) == {"a", "b"} and s["a"] >= 5.0 and s["b"] >= 0.0
    assert t.summary() == {}  # reset after a summary
    assert abs(tokens_per_second(1000, 500.0) - 2000.0) < 1e-9
    assert RegionTimer(enabled=False).summary() == {}


def _timer_max_worker(rank, world):
    from heiretsu_b200.utils.profiling import RegionTimer

    t = RegionTimer()
    t._add("step", 10.0 * (rank + 1))
    return t.summary()["step"]


def test_region_timer_max_over_ranks():
    from dist_util import run_ranks

    assert run_ranks(_timer_max_worker, 2) == [20.0, 20.0]


def _timer_per_rank_worker(rank, world):
    from heiretsu_b200.utils.profiling import RegionTimer, rank_spread

    t = RegionTimer()
    t._add("step", [12.0, 30.0, 10.0][rank])
    pr = t.per_rank()["step"]
    return pr, rank_spread(pr)


def test_region_timer_per_rank_spread():
    """Per-rank step times (all-gather) and their spread: the straggler is named."""
    from dist_util import run_ranks

    for pr, sp in run_ranks(_timer_per_rank_worker, 3):
        assert pr == [12.0, 30.0, 10.0]
        assert sp["min"] == 10.0 and sp["max"] == 30.0 and sp["median"] == 12.0 and sp["slowest"] == 1.0
        assert abs(sp["imbalance"] - 3.0) < 1e-12


def test_roofline_fractions(tmp_path):
    import json

    from heiretsu_b200.utils.roofline import fractions, fused_target_ms, load_peaks, render

    fb = load_peaks(str(tmp_path / "absent.json"))
    assert fb.label == "of fallback" and fb.hbm_gbs == 6650.0
    p = tmp_path / "peaks.json"
    p.write_text(json.dumps({"hbm_gbs": 7000.0, "bf16_tflops": {"value": 1600.0}, "bf16_tflops_sustained": 1450.0}))
    pk = load_peaks(str(p))
    assert pk.label == "of measured" and pk.bf16_tflops == 1600.0 and pk.hbm_gbs == 7000.0
    rows = fractions([{"op": "gemm", "name": "x", "ms": 1.0, "tflops": 800.0, "ref_tflops": 1200.0},
                      {"op": "layernorm", "name": "bwd", "ms": 0.05, "gbs": 3500.0}], pk)
    assert abs(rows[0]["frac"] - 0.5) < 1e-12 and abs(rows[0]["ref_frac"] - 0.75) < 1e-12
    assert abs(rows[1]["frac"] - 0.5) < 1e-12
    assert "of measured" in render(rows)
    # 1 TFLOP at 1.6 PFLOP/s = 0.625 ms < 770 MB at 770 GB/s = 1 ms: the link bounds it
    assert abs(fused_target_ms(1e12, 770e6, pk) - 1.0) < 1e-9
    assert abs(fused_target_ms(3.2e12, 770e6, pk) - 2.0) < 1e-9


def test_dropout_reference_hash():
    import torch

    from heiretsu_b200.ops.dropout_ref import lowbias32, residual_mask

    def py_lowbias32(x):
        x &= 0xFFFFFFFF
        x ^= x >> 16
        x = (x * 0x7FEB352D) & 0xFFFFFFFF
        x ^= x >> 15
        x = (x * 0x846CA68B) & 0xFFFFFFFF
        x ^= x >> 16
        return x

    vals = [0, 1, 2, 12345, 0xFFFFFFFF, 0x80000000, 987654321]
    assert lowbias32(torch.tensor(vals, dtype=torch.int64)).tolist() == [py_lowbias32(v) for v in vals]
    m = residual_mask(7, 3, 256, 128, 0.2)
    assert set(torch.unique(m).tolist()) == {0.0, 1.25}
    assert abs((m == 0).double().mean().item() - 0.2) < 0.01
    assert not torch.equal(m, residual_mask(8, 3, 256, 128, 0.2))  # seed changes the mask
    assert not torch.equal(m, residual_mask(7, 4, 256, 128, 0.2))  # so does the site


def test_uncovered_ranges():
    from heiretsu_b200.parallel.grad_reduce import uncovered_ranges

    assert uncovered_ranges([], 10) == [(0, 10)]
    assert uncovered_ranges([(2, 4), (6, 8)], 10) == [(0, 2), (4, 6), (8, 10)]
    assert uncovered_ranges([(0, 5), (3, 10)], 10) == []
    assert uncovered_ranges([(6, 8), (0, 2)], 8) == [(2, 6)]


def test_flat_params_grouping_and_block_ranges():
    import torch

    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.parallel.flat import ALIGN, FlatParams
    from heiretsu_b200.parallel.grad_reduce import FlatGradReducer

    cfg = GPTConfig(block_size=16, vocab_size=64, n_layer=2, n_head=2, n_embed=32, num_experts=4, top_k=2,
                    moe_freq=2)
    torch.manual_seed(0)
    m = GPT(cfg)
    before = {n: p.detach().clone() for n, p in m.named_parameters()}
    # three classes: expert weights (weight 1, summed over TP), LayerNorms (0.5, summed), the rest (0.5, not)
    weight_of = lambda n, p: 1.0 if ".experts." in n else 0.5
    tp_sum_of = lambda n, p: ".experts." in n or ".ln_" in n
    flat = FlatParams(m, torch.device("cpu"), weight_of=weight_of, tp_sum_of=tp_sum_of)
    assert [(w, t) for (_, _, w), t in zip(flat.ranges, flat.tp_sum)] == [(0.5, False), (0.5, True), (1.0, True)]
    for (a, b, w), t in zip(flat.ranges, flat.tp_sum):
        for n, p, off in zip(flat.names, flat.params, flat.offsets):
            if a <= off < b:
                assert weight_of(n, p) == w and tp_sum_of(n, p) == t
                assert off % ALIGN == 0
    for n, p in m.named_parameters():  # values survive the move into the flat buffer
        assert torch.equal(p.detach(), before[n])
    # the experts of the MoE layer are stored back to back (one grouped-GEMM weight matrix)
    ex = m.tr.h[1].moe.expert_group.experts
    w1, g1 = flat.stacked([e.w1.weight for e in ex])
    assert w1.shape == (4 * ex[0].w1.weight.shape[0], ex[0].w1.weight.shape[1])
    assert torch.equal(w1[: ex[0].w1.weight.shape[0]], ex[0].w1.weight.detach().bfloat16())

    # per-block gradient ranges of the overlapped reducer: sorted, disjoint, covering every parameter
    red = FlatGradReducer.__new__(FlatGradReducer)
    red.flat, red._range_cache = flat, {}
    for blk in m.tr.h:
        rs = red._ranges_of(blk)
        assert rs == sorted(rs) and all(a < b for a, b in rs)
        assert all(b1 <= a2 for (_, b1), (a2, _) in zip(rs, rs[1:]))
        idx = {id(p): i for i, p in enumerate(flat.params)}
        for p in blk.parameters():
            off = flat.offsets[idx[id(p)]]
            assert any(a <= off and off + p.numel() <= b for a, b in rs)


def test_dropout_seed_snapshots():
    import torch

    from heiretsu_b200.models.fused import _dropout_of, _snapshot_dropout_seeds

    class Blk(torch.nn.Module):
        pass

    seed = torch.tensor([41], dtype=torch.int32)
    blocks = [Blk(), Blk(), Blk()]
    for i, b in enumerate(blocks[:2]):
        b._hb_dropout = (seed, i, 0.1)
    _snapshot_dropout_seeds(blocks)
    assert int(seed.item()) == 42  # advanced once per forward, not per block
    d0, d1 = _dropout_of(blocks[0]), _dropout_of(blocks[1])
    assert d0[0] is d1[0] and int(d0[0].item()) == 41 and (d0[1], d1[1]) == (0, 1)
    assert _dropout_of(blocks[2]) is None  # no dropout configured
    for b in blocks:
        b.eval()
    _snapshot_dropout_seeds(blocks)
    assert int(seed.item()) == 42 and all(_dropout_of(b) is None for b in blocks)  # eval: off, no advance


def test_gemm_tile_width_policy():
    from heiretsu_b200.ops import gemm as g

    assert g._bn(50304) == 256 and g._bn(2304) == 256 and g._bn(768) == 128 and g._bn(136) == 128
    assert g._bn_f32_out(768) == 192 and g._bn_f32_out(1536) == 192
    assert g._bn_f32_out(384) == 128 and g._bn_f32_out(3072) == 256 and g._bn_f32_out(1000) == 128


def test_commbench_work_and_roofline():
    from heiretsu_b200.parallel import commbench as C
    from heiretsu_b200.utils.roofline import Peaks

    # reduce-scatter + all-gather moves 2 (N-1)/N of the buffer per GPU and direction
    assert C.dp_reduce_bytes(1000, 8) == 2 * 7 / 8 * 4000
    assert C.dp_reduce_bytes(1000, 2) == 4000
    f, b = C.tp_ag_gemm_work(8192, 3072, 1024, 4)
    assert f == 2 * 8192 * 768 * 1024 and b == 0.75 * 8192 * 1024 * 2
    f, b = C.tp_gemm_rs_work(8192, 1024, 4096, 4)
    assert f == 2 * 8192 * 1024 * 1024 and b == 0.75 * 8192 * 1024 * 2
    assert C.ep_combine_bytes(8192, 768, 2) == 8192 * 768 * 4
    peaks = Peaks(6650.0, 1590.0, 1400.0, "of fallback")
    rows = C.attach_roofline([dict(case="dp_reduce", shape="x", ms=2.0, ref_ms=4.0, flops=0.0,
                                   nvlink_bytes=770e9 * 1e-3)], peaks)
    r = rows[0]
    assert abs(r["target_ms"] - 1.0) < 1e-9 and abs(r["frac"] - 0.5) < 1e-9 and abs(r["ref_frac"] - 0.25) < 1e-9
    assert abs(r["nvlink_gbs"] - 385.0) < 1e-6
    assert "of fallback" in r["label"] and "| dp_reduce |" in C.table(rows)


def test_region_timing_step(tmp_path, capsys):
    from heiretsu_b200.trainer import Engine, main

    main(["--device", "cpu", "--synthetic_data", "--n_layer", "2", "--n_head", "2", "--n_embed", "32",
          "--block_size", "32", "--batch_size", "4", "--max_iters", "4", "--eval_interval", "100",
          "--eval_iters", "1", "--dropout", "0", "--log_interval", "1", "--region_timing_interval", "2",
          "--out_dir", str(tmp_path)])
    lines = [l for l in capsys.readouterr().out.splitlines() if "regions (ms" in l]
    assert len(lines) == 2 and lines[0].startswith("step      2") and lines[1].startswith("step      4")
    for name in Engine.REGIONS:
        assert f"| {name} " in lines[0] or f") {name} " in lines[0], lines[0]


def test_fused_adamw_hyper_upload_values():
    """prepare_step writes [lr, b1, b2, eps, wd, 1-b1^t, sqrt(1-b2^t), grad_scale] for step t
    through its staging slots (host part only; the kernels need a GPU)."""
    import math
    import types

    import torch

    from heiretsu_b200.optim import FusedAdamW

    flat = types.SimpleNamespace(device=torch.device("cpu"), data=torch.zeros(16), grad=torch.zeros(16), ranges=[])
    opt = FusedAdamW(flat, lr=2e-3, betas=(0.8, 0.9), eps=1e-7, weight_decay=0.05)
    for t in (1, 2, 3):
        opt.prepare_step()
        want = torch.tensor([2e-3, 0.8, 0.9, 1e-7, 0.05, 1 - 0.8 ** t, math.sqrt(1 - 0.9 ** t), 1.0])
        assert torch.allclose(opt.hyper, want), (t, opt.hyper)


def test_lr_schedule(capsys, tmp_path):
    import math

    from heiretsu_b200.trainer import build_argparser, lr_at, main

    a = build_argparser().parse_args(["--learning_rate", "1e-3", "--lr_schedule", "cosine", "--warmup_iters", "4",
                                      "--min_lr", "1e-4", "--max_iters", "14"])
    assert lr_at(1, a) == 2.5e-4 and lr_at(4, a) == 1e-3
    assert abs(lr_at(9, a) - (1e-4 + 0.5 * 9e-4 * (1 + math.cos(math.pi * 0.5)))) < 1e-12
    assert abs(lr_at(14, a) - 1e-4) < 1e-12
    c = build_argparser().parse_args(["--learning_rate", "1e-3"])
    assert lr_at(7, c) == 1e-3  # the reference's constant rate by default
    main(["--device", "cpu", "--synthetic_data", "--n_layer", "1", "--n_head", "2", "--n_embed", "32",
          "--block_size", "16", "--batch_size", "2", "--max_iters", "3", "--eval_interval", "100", "--eval_iters",
          "1", "--log_interval", "1", "--learning_rate", "1e-3", "--lr_schedule", "cosine", "--warmup_iters", "2",
          "--out_dir", str(tmp_path)])
    lrs = [l.split("| lr ")[1] for l in capsys.readouterr().out.splitlines() if "| lr " in l]
    assert lrs == ["5.000e-04", "1.000e-03", "0.000e+00"], lrs


def test_node_locality_of_groups(monkeypatch):
    """Ranks are numbered node by node (torchrun): on two 8-GPU nodes, TP/EP/PP groups of a
    dp2 x ep2 x tp2 x pp2 job stay on one node, its DP groups span both; the fused path is
    kept only for groups on one node (CUDA IPC peer mappings), DP falls back to NCCL."""
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.fused import fused_supported
    from heiretsu_b200.topo import Topology, coords_from_rank, group_members, local_world_size

    def topo(rank, dp, ep, tp, pp, per_node):
        d, e, p, t = coords_from_rank(rank, dp, ep, tp, pp)
        m = group_members(dp, ep, tp, pp, rank)
        return Topology(dp=dp, ep=ep, tp=tp, pp=pp, rank=rank, world_size=dp * ep * tp * pp, dp_rank=d, ep_rank=e,
                        pp_rank=p, tp_rank=t, tp_group=None, pp_group=None, ep_group=None, dp_group=None,
                        tp_ranks=m["tp"], pp_ranks=m["pp"], ep_ranks=m["ep"], dp_ranks=m["dp"],
                        local_world=per_node)

    moe = GPTConfig(block_size=64, vocab_size=128, n_layer=2, n_head=2, n_embed=128, dropout=0.0, num_experts=4)
    for r in range(16):
        t = topo(r, 2, 2, 2, 2, 8)
        assert t.on_one_node(t.tp_ranks) and t.on_one_node(t.ep_ranks) and t.on_one_node(t.pp_ranks)
        assert not t.on_one_node(t.dp_ranks)
        assert t.on_one_node(t.model_parallel_ranks())
        assert fused_supported(moe, t)[0]
    # tp4 over nodes of 2 GPUs: the TP group spans nodes -> plain path
    t = topo(0, 1, 1, 4, 1, 2)
    ok, why = fused_supported(moe, t)
    assert not ok and "spans nodes" in why
    t = topo(0, 1, 4, 1, 1, 2)
    ok, why = fused_supported(moe, t)
    assert not ok and "EP group" in why
    # single node: local_world 0 (unset) means everything is on one node
    t = topo(3, 8, 1, 1, 1, 0)
    assert t.on_one_node(t.dp_ranks)
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    assert local_world_size(16) == 8
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "3")
    with pytest.raises(ValueError):
        local_world_size(16)
    monkeypatch.delenv("LOCAL_WORLD_SIZE")
    assert local_world_size(4) == 4


def test_fused_tp_dropout_is_default():
    """tp > 1 with dropout runs the fused engine unless --fused_tp_dropout 0."""
    import types

    from heiretsu_b200.models.fused import fused_supported
    from heiretsu_b200.trainer import build_argparser

    cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=2, n_head=4, n_embed=256, dropout=0.1)
    topo = types.SimpleNamespace(dp=1, ep=1, tp=2, pp=1)
    assert fused_supported(cfg, topo)[0]
    ok, why = fused_supported(cfg, topo, tp_dropout=False)
    assert not ok and "--fused_tp_dropout 0" in why
    assert build_argparser().parse_args([]).fused_tp_dropout == 1
    assert fused_supported(cfg, types.SimpleNamespace(dp=2, ep=1, tp=1, pp=1))[0]  # DP with dropout: fused


def test_gelu_reciprocal_seed_constant():
    """The epilogue's reciprocal seed K - bits(d): K is the equal-ripple constant
    0x7E800000 + round((2 sqrt 6 - 4) 2^23), and its seed error over a whole binade
    (every fp32 mantissa) stays below (5 - 2 sqrt 6) / 2 plus rounding."""
    import math
    import re

    import numpy as np

    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "heiretsu_b200", "csrc", "common.cuh")).read()
    k = int(re.search(r"__int_as_float\((0x[0-9A-Fa-f]+) - __float_as_int\(d\)\)", src).group(1), 16)
    c = 2 * math.sqrt(6) - 4
    assert k == 0x7E800000 + round(c * 2 ** 23)
    bits = (np.int64(127) << 23) | np.arange(2 ** 23, dtype=np.int64)
    d = bits.astype(np.int32).view(np.float32).astype(np.float64)
    r = (np.int64(k) - bits).astype(np.int32).view(np.float32).astype(np.float64)
    seed_err = np.abs(r * d - 1).max()
    assert seed_err <= (5 - 2 * math.sqrt(6)) / 2 + 1e-6
    assert seed_err ** 4 < 7e-6  # two Newton steps square the error twice


def test_exp2_fma_derivation():
    """exp2_fma (common.cuh), restated in numpy float32: nearest-integer split by the
    1.5 * 2^23 shift, degree-5 Taylor series of 2^f on [-1/2, 1/2], exponent-field
    scaling. Its coefficients are (ln 2)^k / k!, and its relative error stays under the
    Lagrange remainder bound (ln(2)/2)^6 / 6! * 2 < 5e-6 plus float32 rounding."""
    import math
    import re

    import numpy as np

    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "heiretsu_b200", "csrc", "common.cuh")).read()
    body = src[src.index("float exp2_fma(float x)"):src.index("sigmoid_2u_fma")]
    coefs = [float(c) for c in re.findall(r"([0-9]\.[0-9]+e-?[0-9]+)f", body)]
    want = [(math.log(2) ** k) / math.factorial(k) for k in (5, 4, 3, 2, 1)]
    assert len(coefs) == 5 and all(abs(a - b) <= 1e-7 * b for a, b in zip(coefs, want))
    f32 = np.float32
    x = np.concatenate([np.linspace(-125, 64, 2_000_001, dtype=np.float64),
                        np.random.default_rng(0).uniform(-125, 64, 200_000)]).astype(np.float32)
    t = (x + f32(12582912.0)).astype(np.float32)
    f = (x - (t - f32(12582912.0))).astype(np.float32)
    p = np.float32(coefs[0])
    for c in coefs[1:] + [1.0]:
        p = (f.astype(np.float64) * p + c).astype(np.float32)  # one rounding per step, as fmaf
    n = t.view(np.int32) - 0x4B400000
    got = (p.view(np.int32) + (n << 23)).view(np.float32).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 5e-6 + 4e-7, rel.max()


def test_attention_trace_reports():
    """Phase arithmetic of the attention trace reports on hand-made stamps."""
    import numpy as np

    from heiretsu_b200.ops.attn_trace import backward_report, forward_report

    t = np.zeros((4, 80), dtype=np.int64)  # two live CTAs, two empty rows
    for c in range(2):
        base = 1000 * (c + 1)
        t[c, 0], t[c, 1], t[c, 2] = base, base + 100, base + 5000
        for g in (0, 1):
            for j in range(2):
                s = base + 200 + 1000 * j
                t[c, 8 + 24 * g + j], t[c, 16 + 24 * g + j] = s, s + 10
                t[c, 56 + 8 * g + j], t[c, 24 + 24 * g + j] = s + 110, s + 600
    r = forward_report(t)
    assert r["ctas"] == 2 and r["span_us"] == 6.0 and r["first_load_ns"] == 100.0
    first = r["tiles"][0]
    assert (first["softmax_ns"], first["max_pass_ns"], first["turnaround_ns"]) == (600.0, 100.0, 400.0)
    assert len(r["tiles"]) == 4 and "turnaround_ns" in r["tiles"][1]  # j = 1 still has a slot for j + 1

    b = np.zeros((2, 80), dtype=np.int64)
    b[0, 0], b[0, 1], b[0, 2] = 10, 30, 9010
    for i in range(3):
        for g in (0, 1):
            r0 = 100 + 2000 * i + 50 * g
            b[0, 24 + 24 * g + i], b[0, 40 + 24 * g + i] = r0, r0 + 1500
            if i > 0:
                b[0, 32 + 24 * g + i] = r0 + 700
    rb = backward_report(b)
    tile1 = [x for x in rb["tiles"] if x["g"] == 1 and x["i"] == 1][0]
    assert (tile1["softmax_ns"], tile1["wait_prev_mma_ns"], tile1["turnaround_ns"]) == (1500.0, 700.0, 500.0)
    assert rb["span_us"] == 9.0
