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


def test_run_train_sh_two_nodes_cpu(tmp_path):
    """NNODES=2: the same launcher command on two 'nodes' (two torchrun agents on this host,
    one gloo rank each) forms one dp2 job; run settings come from a CONFIG_FILE."""
    cfg = tmp_path / "run.yaml"
    cfg.write_text("n_layer: 1\nn_head: 2\nn_embed: 32\nblock_size: 16\nbatch_size: 2\nmax_iters: 3\n"
                   "eval_interval: 3\neval_iters: 1\ndropout: 0.0\nsynthetic_data: true\n")
    base = dict(os.environ, DP="2", NNODES="2", DEVICE="cpu", DIST_BACKEND="gloo", AMP="none", GRAD_ACCUM="1",
                SAVE_INTERVAL="3", SAVE_PATH=str(tmp_path), MASTER_PORT=str(_port()), JOB_TIMEOUT="240",
                OMP_NUM_THREADS="1", CONFIG_FILE=str(cfg),
                # launcher defaults that the file must override: command-line values only come from the file
                N_LAYER="", N_HEAD="", N_EMBED="", BLOCK_SIZE="", BATCH_SIZE="", MAX_ITERS="", EVAL_INTERVAL="",
                EVAL_ITERS="", DROPOUT="")
    procs = [subprocess.Popen(["bash", os.path.join(ROOT, "run_train.sh")], cwd=ROOT,
                              env=dict(base, NODE_RANK=str(n)), stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                              text=True) for n in range(2)]
    outs = [p.communicate(timeout=300) for p in procs]
    for p, (out, err) in zip(procs, outs):
        assert p.returncode == 0, (out[-2000:], err[-3000:])
    assert "training finished." in outs[0][0]
    assert "[eval] step 3" in outs[0][0]


def test_restart_after_failure_resumes_exactly(tmp_path):
    """MAX_RESTARTS=1: rank 1 raises at step 5 (host-side injection, after the step-4
    checkpoint); torchrun restarts both ranks, which resume from the newest complete
    checkpoint (RESUME=auto) and finish; the step-6 weights equal an uninterrupted run's."""
    import torch

    def run(out, **extra):
        env = dict(os.environ, DP="2", SYNTHETIC="1", DEVICE="cpu", DIST_BACKEND="gloo", AMP="none", N_LAYER="1",
                   N_HEAD="2", N_EMBED="32", BLOCK_SIZE="16", BATCH_SIZE="2", GRAD_ACCUM="2", MAX_ITERS="6",
                   EVAL_INTERVAL="100", EVAL_ITERS="1", SAVE_INTERVAL="2", SAVE_PATH=str(out), DROPOUT="0.1",
                   MASTER_PORT=str(_port()), JOB_TIMEOUT="280", OMP_NUM_THREADS="1", **extra)
        return subprocess.run(["bash", os.path.join(ROOT, "run_train.sh")], cwd=ROOT, env=env, capture_output=True,
                              text=True, timeout=300)

    clean = run(tmp_path / "clean")
    assert clean.returncode == 0, (clean.stdout[-2000:], clean.stderr[-3000:])
    hit = run(tmp_path / "hit", MAX_RESTARTS="1", HB_INJECT_FAILURE="1:5")
    assert hit.returncode == 0, (hit.stdout[-2000:], hit.stderr[-3000:])
    assert "injected failure: rank 1 at step 5" in hit.stderr
    assert "[resume] auto: no complete checkpoint" in hit.stdout  # the first attempt starts fresh
    assert "[resume] step 4 from" in hit.stdout
    assert "training finished." in hit.stdout
    assert sorted(p.name for p in (tmp_path / "hit").glob("*.done")) == [
        "ckpt_0000002.done", "ckpt_0000004.done", "ckpt_0000006.done"]
    a = torch.load(tmp_path / "clean" / "ckpt_0000006.pt", weights_only=False)["model"]
    b = torch.load(tmp_path / "hit" / "ckpt_0000006.pt", weights_only=False)["model"]
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
