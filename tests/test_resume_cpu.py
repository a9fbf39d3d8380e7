"""Exact resume: a run resumed from its step-2 checkpoint (model, optimizer
sidecar with AdamW moments, RNG states and data position) reproduces the
uninterrupted run's step-4 weights bit for bit (CPU, plain engine, dropout on)."""
import os

import torch


def _args(out_dir, extra):
    return ["--device", "cpu", "--synthetic_data", "--n_layer", "2", "--n_head", "2", "--n_embed", "32",
            "--block_size", "16", "--batch_size", "2", "--grad_accum_steps", "2", "--dropout", "0.1",
            "--eval_interval", "1000", "--eval_iters", "1", "--out_dir", str(out_dir), "--seed", "7"] + extra


def test_resume_reproduces_uninterrupted_run(tmp_path):
    from heiretsu_b200.trainer import main

    a, b = tmp_path / "a", tmp_path / "b"
    a.mkdir()
    b.mkdir()
    main(_args(a, ["--max_iters", "4", "--save_interval", "2"]))
    assert (a / "ckpt_0000002.pt").exists() and (a / "optim_0000002.pt").exists()
    side = torch.load(a / "optim_0000002.pt", weights_only=False)
    assert {"optimizer", "rng", "train_loader"} <= set(side)
    main(_args(b, ["--max_iters", "4", "--save_interval", "4", "--resume", os.fspath(a / "ckpt_0000002.pt")]))
    full = torch.load(a / "ckpt_0000004.pt", weights_only=False)
    resumed = torch.load(b / "ckpt_0000004.pt", weights_only=False)
    assert resumed["step"] == 4
    for k, v in full["model"].items():
        assert torch.equal(v, resumed["model"][k]), k


def test_resume_without_sidecar_loads_weights(tmp_path):
    from heiretsu_b200.trainer import main

    a, b = tmp_path / "a", tmp_path / "b"
    a.mkdir()
    b.mkdir()
    main(_args(a, ["--max_iters", "2", "--save_interval", "2"]))
    os.remove(a / "optim_0000002.pt")  # a checkpoint written by the reference has no sidecar
    main(_args(b, ["--max_iters", "3", "--save_interval", "3", "--resume", os.fspath(a / "ckpt_0000002.pt")]))
    assert torch.load(b / "ckpt_0000003.pt", weights_only=False)["step"] == 3


def test_init_from_loads_weights_only(tmp_path):
    """--init_from: the new run starts from the checkpoint's weights at step 1 with a fresh
    optimizer; its first step's loss is the loss of those weights, not of a new init."""
    from heiretsu_b200.trainer import main

    a, b, c = tmp_path / "a", tmp_path / "b", tmp_path / "c"
    for d in (a, b, c):
        d.mkdir()
    main(_args(a, ["--max_iters", "3", "--save_interval", "3", "--learning_rate", "1e-2"]))
    for d, extra in ((b, ["--init_from", os.fspath(a / "ckpt_0000003.pt")]), (c, [])):
        main(_args(d, ["--max_iters", "1", "--save_interval", "1", "--dropout", "0"] + extra))
    trained = torch.load(a / "ckpt_0000003.pt", weights_only=False)["model"]
    tuned = torch.load(b / "ckpt_0000001.pt", weights_only=False)
    fresh = torch.load(c / "ckpt_0000001.pt", weights_only=False)["model"]
    assert tuned["step"] == 1 and not (b / "optim_0000003.pt").exists()
    # one AdamW step with fresh moments moves every weight by at most ~lr (3e-4) from the trained one
    for k, v in trained.items():
        assert (tuned["model"][k] - v).abs().max().item() < 1e-3, k
    assert max((fresh[k] - v).abs().max().item() for k, v in trained.items()) > 1e-2


def test_eval_only_reports_the_loaded_weights(tmp_path, capsys):
    """--eval_only with --init_from prints the evaluation of the checkpoint's weights and trains nothing."""
    import re

    from heiretsu_b200.trainer import main

    a = tmp_path / "a"
    a.mkdir()
    main(_args(a, ["--max_iters", "4", "--save_interval", "4", "--eval_interval", "4", "--eval_iters", "3",
                   "--learning_rate", "1e-2"]))
    out = capsys.readouterr().out
    trained = float(re.search(r"\[eval\] step 4 \| eval_loss ([0-9.]+)", out).group(1))
    main(_args(tmp_path, ["--eval_only", "--eval_iters", "3", "--init_from", os.fspath(a / "ckpt_0000004.pt")]))
    out = capsys.readouterr().out
    got = float(re.search(r"\[eval_only\] eval_loss ([0-9.]+)", out).group(1))
    assert abs(got - trained) < 1e-3, (got, trained)
    assert not list(tmp_path.glob("ckpt_*.pt"))


def _pp_main(rank, world, out_dir):
    from heiretsu_b200.trainer import main

    main(["--device", "cpu", "--dist_backend", "gloo", "--synthetic_data", "--pp", "2", "--n_layer", "2",
          "--n_head", "2", "--n_embed", "32", "--block_size", "16", "--batch_size", "2", "--grad_accum_steps", "2",
          "--dropout", "0", "--max_iters", "2", "--eval_interval", "2", "--eval_iters", "1", "--save_interval", "2",
          "--out_dir", out_dir, "--pg_timeout_s", "60"])
    return sorted(os.listdir(out_dir))


def test_pipeline_trainer_runs_eval_and_saves_shards(tmp_path):
    from dist_util import run_ranks_raw

    res = run_ranks_raw(_pp_main, 2, str(tmp_path), init=False, timeout=240)
    assert all(status == "ok" for status, _ in res), res
    files = res[0][1]
    assert "ckpt_0000002_pp0_ep0_tp0.pt" in files and "ckpt_0000002_pp1_ep0_tp0.pt" in files, files


def _main_ranks(rank, world, out_dir, extra):
    from heiretsu_b200.trainer import main

    main(["--device", "cpu", "--dist_backend", "gloo", "--synthetic_data", "--n_layer", "2", "--n_head", "2",
          "--n_embed", "32", "--block_size", "16", "--batch_size", "2", "--grad_accum_steps", "2", "--dropout",
          "0.1", "--eval_interval", "1000", "--eval_iters", "1", "--out_dir", out_dir, "--seed", "7",
          "--pg_timeout_s", "60"] + extra)
    return sorted(os.listdir(out_dir))


def test_sharded_resume_reproduces_uninterrupted_run(tmp_path):
    """dp2 x tp2 on gloo ranks: each rank reloads its own shard, the optimizer sidecar and
    its own RNG states / data position, and step 4 matches the uninterrupted run bit for bit."""
    from dist_util import run_ranks_raw

    a, b = tmp_path / "a", tmp_path / "b"
    a.mkdir()
    b.mkdir()
    lay = ["--dp", "2", "--tp", "2"]
    res = run_ranks_raw(_main_ranks, 4, str(a), lay + ["--max_iters", "4", "--save_interval", "2"], init=False,
                        timeout=240)
    assert all(st == "ok" for st, _ in res), res
    assert {f"rstate_0000002_r{r}.pt" for r in range(4)} <= set(res[0][1])
    res = run_ranks_raw(_main_ranks, 4, str(b), lay + ["--max_iters", "4", "--save_interval", "4", "--resume",
                                                         os.fspath(a / "ckpt_0000002_pp0_ep0_tp1.pt")],
                        init=False, timeout=240)
    assert all(st == "ok" for st, _ in res), res
    for t in range(2):
        full = torch.load(a / f"ckpt_0000004_pp0_ep0_tp{t}.pt", weights_only=False)
        resumed = torch.load(b / f"ckpt_0000004_pp0_ep0_tp{t}.pt", weights_only=False)
        for k, v in full["model"].items():
            assert torch.equal(v, resumed["model"][k]), (t, k)


_MOE_CFG = dict(block_size=16, vocab_size=64, n_layer=4, n_head=4, n_embed=32, dropout=0.0, num_experts=4,
                top_k=2, moe_freq=2)


def _dense_state():
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT

    torch.manual_seed(3)
    return GPT(GPTConfig(**_MOE_CFG)).state_dict()


def _save_shards(rank, world, out_dir):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.parallel.pipeline import StageModule
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.ckpt import load_from_full, save_checkpoint

    topo = init_topology(dp=1, ep=2, tp=2, pp=2)
    cfg = GPTConfig(**_MOE_CFG)
    stage = StageModule(cfg, topo, topo.pp_rank, topo.pp)
    load_from_full(stage, _dense_state(), topo.tp_rank, topo.tp)
    return save_checkpoint(stage, cfg, 5, topo, out_dir)


def _reshard(rank, world, shard_file, tp, pp):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.parallel.pipeline import StageModule
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import mark_tp_sharded
    from heiretsu_b200.utils.ckpt import load_for_resume, shard_from_full

    topo = init_topology(dp=1, tp=tp, pp=pp)
    cfg = GPTConfig(**_MOE_CFG)
    m = StageModule(cfg, topo, topo.pp_rank, topo.pp) if pp > 1 else GPT(cfg, topo=topo)
    mark_tp_sharded(m)
    info = load_for_resume(m, shard_file, topo)
    want = shard_from_full(m, _dense_state(), topo.tp_rank, topo.tp)
    bad = [k for k, v in m.state_dict().items() if not torch.equal(v, want[k])]
    return info["step"], info["same_layout"], bad


def test_merge_and_resume_on_another_layout(tmp_path):
    """Shards of an ep2 x tp2 x pp2 MoE model merge back into the dense state dict exactly;
    tp2 and tp2 x pp2 runs (and a dense process) resume from them with the right slices."""
    from dist_util import run_ranks

    from heiretsu_b200.utils.ckpt import load_for_resume, main as ckpt_main, merge_shards, step_files

    paths = run_ranks(_save_shards, 8, str(tmp_path))
    shard = paths[0]
    files = step_files(shard)
    assert len(files) == 8
    merged = merge_shards([torch.load(f, weights_only=False) for f in files])
    dense = _dense_state()
    assert set(merged) == set(dense)
    for k, v in dense.items():
        assert torch.equal(merged[k], v), k
    for tp, pp in ((2, 1), (2, 2)):
        for step, same, bad in run_ranks(_reshard, tp * pp, shard, tp, pp):
            assert step == 5 and not same and not bad, bad
    # dense export and a single-process load
    out = tmp_path / "dense.pt"
    ckpt_main(["merge", str(out), shard])
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.topo import init_topology

    m = GPT(GPTConfig(**_MOE_CFG))
    info = load_for_resume(m, str(out), init_topology(dp=1))
    assert info["same_layout"] and info["step"] == 5
    for k, v in dense.items():
        assert torch.equal(m.state_dict()[k], v), k


def _main_plain(rank, world, out_dir, extra):
    from heiretsu_b200.trainer import main

    main(["--device", "cpu", "--dist_backend", "gloo", "--synthetic_data", "--n_layer", "4", "--n_head", "2",
          "--n_embed", "32", "--block_size", "16", "--batch_size", "2", "--grad_accum_steps", "2", "--dropout", "0",
          "--eval_interval", "1000", "--eval_iters", "1", "--out_dir", out_dir, "--seed", "3", "--learning_rate",
          "3e-3", "--pg_timeout_s", "60"] + extra)


def test_resume_on_another_layout_continues_the_run(tmp_path):
    """A tied tp2 x pp2 run saved at step 2, resumed by one dense process (weights, AdamW
    moments merged from the four shard sidecars and re-sliced, data position of dp rank
    0), reaches the tp2 x pp2 run's own step-4 weights; a weights-only resume does not."""
    from dist_util import run_ranks_raw

    from heiretsu_b200.trainer import main
    from heiretsu_b200.utils.ckpt import merge_shards, step_files

    a, b, c = tmp_path / "a", tmp_path / "b", tmp_path / "c"
    for d in (a, b, c):
        d.mkdir()
    lay = ["--tp", "2", "--pp", "2", "--pp_tie_embeddings", "1"]
    res = run_ranks_raw(_main_plain, 4, str(a), lay + ["--max_iters", "4", "--save_interval", "2"], init=False,
                        timeout=300)
    assert all(st == "ok" for st, _ in res), res
    shard2 = os.fspath(a / "ckpt_0000002_pp1_ep0_tp1.pt")
    single = ["--device", "cpu", "--synthetic_data", "--n_layer", "4", "--n_head", "2", "--n_embed", "32",
              "--block_size", "16", "--batch_size", "2", "--grad_accum_steps", "2", "--dropout", "0",
              "--eval_interval", "1000", "--eval_iters", "1", "--seed", "3", "--learning_rate", "3e-3",
              "--max_iters", "4", "--save_interval", "4", "--resume", shard2]
    main(single + ["--out_dir", str(b)])
    ref = merge_shards([torch.load(f, weights_only=False) for f in step_files(os.fspath(a / "ckpt_0000004_pp0_ep0_tp0.pt"))])
    got = torch.load(b / "ckpt_0000004.pt", weights_only=False)["model"]
    err = max((got[k] - ref[k]).abs().max().item() for k in ref)
    assert err < 2e-5, err
    for f in step_files(shard2):  # weights only: the optimizer restarts
        os.remove(os.path.join(os.path.dirname(f), "optim_" + os.path.basename(f)[len("ckpt_"):]))
    main(single + ["--out_dir", str(c)])
    got_c = torch.load(c / "ckpt_0000004.pt", weights_only=False)["model"]
    err_c = max((got_c[k] - ref[k]).abs().max().item() for k in ref)
    assert err_c > 50 * max(err, 1e-7), (err, err_c)
