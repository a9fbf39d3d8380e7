"""Failure detection, tested by injecting failures on the host among gloo CPU
ranks: a rank that raises, a rank that stalls, a rank that leaves before a
collective, and a point-to-point message that is never sent. No GPU is used."""
import time

import pytest

from dist_util import run_ranks_raw


def _announced(rank, world):
    from heiretsu_b200.utils.fault import PeerFailure, StepWatchdog, default_store

    wd = StepWatchdog(default_store(), rank, world, timeout_s=60, poll_s=0.05)
    t0 = time.monotonic()
    try:
        for step in range(1, 400):
            wd.check()
            if rank == 1 and step == 3:
                raise RuntimeError("injected failure")
            time.sleep(0.02)
            wd.beat(step)
    except PeerFailure as e:
        return ("peer_failure", e.rank, time.monotonic() - t0)
    except RuntimeError as e:
        wd.mark_failed(str(e))
        return ("raised", rank, 0.0)
    finally:
        wd.stop()
    return ("finished", -1, 0.0)


def test_announced_failure_reaches_peer():
    res = run_ranks_raw(_announced, 2)
    assert res[1] == ("ok", ("raised", 1, 0.0))
    status, (kind, who, dt) = res[0]
    assert status == "ok" and kind == "peer_failure" and who == 1 and dt < 10


def _stall(rank, world):
    from heiretsu_b200.utils.fault import PeerFailure, StepWatchdog, default_store

    wd = StepWatchdog(default_store(), rank, world, timeout_s=1.0, poll_s=0.05)
    try:
        for step in range(1, 400):
            wd.check()
            if rank == 1 and step == 3:
                time.sleep(4.0)  # stalls without beating
                return ("stalled",)
            time.sleep(0.02)
            wd.beat(step)
    except PeerFailure as e:
        return ("peer_failure", e.rank, "no progress" in e.reason)
    finally:
        wd.stop()
    return ("finished",)


def test_stalled_rank_times_out():
    res = run_ranks_raw(_stall, 2)
    assert res[0] == ("ok", ("peer_failure", 1, True))
    assert res[1] == ("ok", ("stalled",))


def _finish_is_not_a_stall(rank, world):
    from heiretsu_b200.utils.fault import StepWatchdog, default_store

    wd = StepWatchdog(default_store(), rank, world, timeout_s=0.5, poll_s=0.05)
    for step in range(1, 4):
        wd.check()
        wd.beat(step)
    if rank == 1:
        wd.finish()
        return "done"
    time.sleep(1.5)  # rank 1 is silent but finished: no failure
    wd.check()
    wd.finish()
    return "done"


def test_finished_peer_is_not_flagged():
    assert [r[1] for r in run_ranks_raw(_finish_is_not_a_stall, 2)] == ["done", "done"]


def _leaves_before_collective(rank, world):
    import torch
    import torch.distributed as dist

    if rank == 1:
        return "left"  # process ends: its sockets close
    time.sleep(0.5)
    t0 = time.monotonic()
    try:
        dist.all_reduce(torch.ones(4))
    except Exception as e:
        return ("error", type(e).__name__, time.monotonic() - t0)
    return ("completed",)


def test_collective_with_departed_rank_errors():
    res = run_ranks_raw(_leaves_before_collective, 2, pg_timeout_s=5.0)
    assert res[1] == ("ok", "left")
    status, out = res[0]
    assert status == "ok" and out[0] == "error" and out[2] < 30, out


def _dropped_p2p(rank, world):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    t = torch.zeros(8)
    if rank == 0:
        time.sleep(3.0)  # "drops" the message: never sends
        return "dropped"
    work = dist.irecv(t, src=0)
    t0 = time.monotonic()
    try:
        work.wait(timeout=timedelta(seconds=1.5))
    except Exception as e:
        return ("timeout", type(e).__name__, time.monotonic() - t0)
    return ("received",)


def test_dropped_p2p_message_times_out():
    res = run_ranks_raw(_dropped_p2p, 2, pg_timeout_s=30.0)
    status, out = res[1]
    assert status == "ok" and out[0] == "timeout" and out[2] < 10, out


def _trainer_rank_dies(rank, world):
    import heiretsu_b200.trainer as T
    from heiretsu_b200.utils.fault import PeerFailure

    orig = T.Engine.train_step
    calls = {"n": 0}

    def train_step(self, loader):
        calls["n"] += 1
        if rank == 1 and calls["n"] == 3:
            raise RuntimeError("injected: rank 1 fails at step 3")
        return orig(self, loader)

    T.Engine.train_step = train_step
    argv = ["--device", "cpu", "--dist_backend", "gloo", "--dp", "2", "--synthetic_data", "--n_layer", "1",
            "--n_head", "2", "--n_embed", "32", "--block_size", "16", "--batch_size", "2", "--max_iters", "50",
            "--eval_interval", "1000", "--eval_iters", "1", "--pg_timeout_s", "20", "--watchdog_s", "10",
            "--dropout", "0"]
    try:
        T.main(argv)
    except PeerFailure as e:
        return ("peer_failure", e.rank)
    except RuntimeError as e:
        return ("raised", "injected" in str(e))
    return ("finished",)


def test_trainer_stops_on_peer_failure():
    res = run_ranks_raw(_trainer_rank_dies, 2, init=False, timeout=180)
    assert res[1] == ("ok", ("raised", True)), res[1]
    status, out = res[0]
    # rank 0 either sees the announcement before its next step, or its
    # in-flight all-reduce errors when rank 1's connections close.
    assert status == "ok" and out[0] in ("peer_failure", "raised"), res[0]


def _nonfinite(rank, world, tp, clip_mode):
    import torch

    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser

    dp = world // tp
    topo = init_topology(dp=dp, tp=tp)
    args = build_argparser().parse_args([
        "--batch_size", "2", "--block_size", "16", "--n_layer", "2", "--n_head", "2", "--n_embed", "16",
        "--dp", str(dp), "--tp", str(tp), "--engine", "plain", "--device", "cpu", "--learning_rate", "1e-2",
        "--clip_mode", clip_mode])
    torch.manual_seed(0)
    eng = Engine(args, topo, torch.device("cpu"), GPTConfig(block_size=16, vocab_size=64, n_layer=2, n_head=2,
                                                            n_embed=16, dropout=0.0))
    poison = [False]
    w = eng.module.tr.h[0].mlp.c_fc.weight
    if rank == world - 1:  # one rank's gradient turns NaN (injected on the host)
        w.register_hook(lambda g: g * float("nan") if poison[0] else g)

    class Feed:
        B = 2

        def __init__(self):
            self.g = torch.Generator().manual_seed(5 + topo.dp_rank)

        def next_batch(self, device):
            return (torch.randint(0, 64, (2, 16), generator=self.g), torch.randint(0, 64, (2, 16), generator=self.g))

    feed = Feed()
    snap = lambda: [p.detach().clone() for p in eng.module.parameters()]
    same = lambda a, b: all(torch.equal(x, y) for x, y in zip(a, b))
    s0 = snap()
    eng.train_step(feed)
    s1 = snap()
    poison[0] = True
    eng.train_step(feed)
    s2 = snap()
    poison[0] = False
    eng.train_step(feed)
    s3 = snap()
    finite = all(bool(torch.isfinite(p).all()) for p in s3)
    return dict(moved1=not same(s0, s1), skipped2=same(s1, s2), moved3=not same(s2, s3), finite=finite,
                skipped=eng.skipped_steps)


@pytest.mark.parametrize("tp", [1, 2])
def test_nonfinite_gradient_skips_the_step_on_every_rank(tp):
    """A NaN in one rank's gradient reaches every rank through the DP average and
    the model-parallel norm; every rank skips that step and training continues."""
    res = run_ranks_raw(_nonfinite, 4, tp, "global")
    for status, out in res:
        assert status == "ok", out
        assert out == dict(moved1=True, skipped2=True, moved3=True, finite=True, skipped=1), out


def test_nonfinite_gradient_with_local_clip_follows_the_reference():
    """clip_mode local reproduces the reference (train.py:446): the NaN reaches the weights."""
    res = run_ranks_raw(_nonfinite, 2, 1, "local")
    for status, out in res:
        assert status == "ok", out
        assert out["skipped"] == 0 and not out["finite"]
