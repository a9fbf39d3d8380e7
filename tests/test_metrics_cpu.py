"""The wandb payload carries the reference's keys (train.py:469-511), MoE
expert-load diagnostics included; checked with a recording stand-in module."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_wandb_keys_match_reference(tmp_path):
    out = tmp_path / "calls.json"
    env = dict(os.environ, HB_FAKE_WANDB_OUT=str(out), OMP_NUM_THREADS="1",
               PYTHONPATH=os.pathsep.join([os.path.join(ROOT, "tests", "fake_wandb"), ROOT]))
    code = ("from heiretsu_b200.trainer import main; main(['--device', 'cpu', '--synthetic_data', '--n_layer', '2', "
            "'--n_head', '2', '--n_embed', '32', '--block_size', '16', '--batch_size', '2', '--max_iters', '2', "
            "'--eval_interval', '2', '--eval_iters', '1', '--num_experts', '4', '--top_k', '2', '--wandb', "
            "'--wandb_mode', 'offline', '--log_interval', '1', '--dropout', '0'])")
    r = subprocess.run([sys.executable, "-c", code], cwd=str(tmp_path), env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    calls = json.loads(out.read_text())
    assert "init" in calls[0] and calls[-1] == {"finish": True}
    logs = [c["log"] for c in calls if "log" in c]
    train = [l for l in logs if "train/loss_mean_micro" in l]
    assert len(train) == 2
    for key in ["opt/lr", "speed/eff_tokens_per_sec", "amp/enabled", "amp/mode", "accum/steps", "train/aux_loss",
                "expert_load/expert_0", "expert_frac/expert_3", "expert_load/max_frac", "expert_load/min_frac",
                "expert_load/imbalance_ratio", "expert_load/distribution"]:
        assert key in train[0], key
    assert abs(sum(train[0][f"expert_frac/expert_{i}"] for i in range(4)) - 1.0) < 1e-5
    assert any("eval/loss" in l for l in logs)
