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
