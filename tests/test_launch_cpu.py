"""The bash launcher end to end on CPU: 2 gloo ranks, synthetic data, a checkpoint at the end."""
import os
import socket
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_run_train_sh_dp2_cpu(tmp_path):
    env = dict(os.environ, DP="2", SYNTHETIC="1", DEVICE="cpu", DIST_BACKEND="gloo", AMP="none", N_LAYER="1",
               N_HEAD="2", N_EMBED="32", BLOCK_SIZE="16", BATCH_SIZE="2", GRAD_ACCUM="1", MAX_ITERS="3",
               EVAL_INTERVAL="3", EVAL_ITERS="1", SAVE_INTERVAL="3", SAVE_PATH=str(tmp_path), DROPOUT="0",
               MASTER_PORT=str(_port()), JOB_TIMEOUT="240", OMP_NUM_THREADS="1")
    r = subprocess.run(["bash", os.path.join(ROOT, "run_train.sh")], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    assert "training finished." in r.stdout
    assert "[eval] step 3" in r.stdout
    assert sorted(p.name for p in tmp_path.glob("ckpt_*.pt")), list(tmp_path.iterdir())
