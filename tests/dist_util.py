"""Run a function on N CPU processes joined by a gloo process group (127.0.0.1)."""
from __future__ import annotations

import os
import socket
import traceback

import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _entry(rank, world, port, fn, args, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank))
    torch.set_num_threads(1)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
        out = fn(rank, world, *args)
        q.put((rank, "ok", out))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "err", traceback.format_exc()))


def run_ranks(fn, world: int, *args, timeout: float = 300.0):
    """Returns the list of per-rank results (ordered by rank); raises on any rank's error."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, out = q.get(timeout=timeout)
            if status != "ok":
                raise AssertionError(f"rank {rank} failed:\n{out}")
            results[rank] = out
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return [results[r] for r in range(world)]


def _entry_raw(rank, world, port, fn, args, q, init, pg_timeout_s):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK="0")
    torch.set_num_threads(1)
    try:
        if init:
            dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=pg_timeout_s))
        q.put((rank, "ok", fn(rank, world, *args)))
    except BaseException:
        q.put((rank, "err", traceback.format_exc()))


def run_ranks_raw(fn, world: int, *args, init: bool = True, pg_timeout_s: float = 30.0, timeout: float = 120.0):
    """Fault-injection runner: no closing barrier (a rank may leave early) and
    no raise on a rank's error. Returns [(status, result_or_traceback)] by rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry_raw, args=(r, world, port, fn, args, q, init, pg_timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, out = q.get(timeout=timeout)
            results[rank] = (status, out)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return [results[r] for r in range(world)]
