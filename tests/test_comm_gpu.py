"""Peer-memory collectives: fused DP all-reduce over NVLink and bounded waits.

The multi-rank test spawns one process per GPU (NCCL only bootstraps the
IPC handle exchange); it is skipped with fewer than two GPUs. The timeout
test runs on one GPU: a barrier whose peer slot nobody ever writes must come
back with a timeout status, leaving the context usable.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _dp_worker(rank, world, port, n, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from heiretsu_b200.ops._C import load
        from heiretsu_b200.parallel.symm import SymmetricBuffer, check_comm_status

        buf = SymmetricBuffer(dist.group.WORLD, n * 4, dev)
        t = buf.tensor(torch.float32, n)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        errs = []
        for it in range(3):  # repeated calls exercise the epoch counters
            data = torch.randn(n, device=dev, generator=g)
            t.copy_(data)
            allv = [torch.empty_like(data) for _ in range(world)]
            dist.all_gather(allv, data)
            ref = torch.stack(allv).sum(0) / world
            torch.cuda.synchronize()
            load().dp_allreduce(buf.ptrs, buf.signal_ptrs, buf.rank, n, 1.0 / world, buf.counter)
            torch.cuda.synchronize()
            check_comm_status(rank)
            errs.append((t - ref).abs().max().item())
        q.put((rank, max(errs)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_dp_allreduce_two_gpus():
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    n = 3 * 1024 * 1024 + 4 * 37  # not a multiple of world * 4 chunks
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err in res:
        assert not isinstance(err, str), (rank, err)
        assert err < 1e-5, (rank, err)


def _dp_stress_worker(rank, world, port, n, iters, q):
    """``iters`` fused all-reduces back to back on one stream, no host sync between
    them. Each is followed at once by a consumer (torch kernels on the same stream)
    that counts wrong elements of the whole buffer, then by the producer of the next
    call's input. Inputs are small integers, so every correct result is exact: any
    element a peer had not yet delivered when the kernel's closing barrier released
    this rank shows up as a miscount. The last call uses random data and is checked
    against NCCL's all-reduce of the same inputs."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from heiretsu_b200.ops._C import load
        from heiretsu_b200.parallel.symm import SymmetricBuffer, check_comm_status

        ext = load()
        buf = SymmetricBuffer(dist.group.WORLD, n * 4, dev)
        t = buf.tensor(torch.float32, n)
        pat = (torch.arange(n, device=dev) % 7).float()
        rank_sum = world * (world + 1) // 2  # sum over ranks of (r + 1)
        bad = torch.zeros(iters, dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        for i in range(iters):
            t.copy_(pat + float((rank + 1) * (i + 1)))
            ext.dp_allreduce(buf.ptrs, buf.signal_ptrs, buf.rank, n, 1.0 / world, buf.counter, 512)
            want = (pat * world + float(rank_sum * (i + 1))) * (1.0 / world)
            bad[i] = (t != want).sum()
        torch.cuda.synchronize()
        check_comm_status(rank)
        g = torch.Generator(device=dev).manual_seed(7 + rank)
        data = torch.randn(n, device=dev, generator=g)
        t.copy_(data)
        ref = data.clone()
        dist.all_reduce(ref)
        ref /= world
        ext.dp_allreduce(buf.ptrs, buf.signal_ptrs, buf.rank, n, 1.0 / world, buf.counter, 512)
        torch.cuda.synchronize()
        check_comm_status(rank)
        q.put((rank, (int(bad.sum().item()), (t - ref).abs().max().item())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_dp_allreduce_back_to_back_consumers():
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    n = 8 * 1024 * 1024 + 4 * 13
    procs = [ctx.Process(target=_dp_stress_worker, args=(r, world, port, n, 200, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, out in res:
        assert not isinstance(out, str), (rank, out)
        wrong, err = out
        assert wrong == 0, (rank, f"{wrong} elements wrong over 200 back-to-back calls")
        assert err < 1e-5, (rank, err)


def test_barrier_timeout_is_reported_not_hung():
    from heiretsu_b200.ops._C import load
    from heiretsu_b200.parallel.symm import CommTimeoutError, check_comm_status

    ext = load()
    dev = torch.cuda.current_device()
    check_comm_status(dev)
    # Two "ranks" whose pads are both local memory: rank 0 waits for a slot of
    # rank 1 that nothing writes.
    sig = [ext.raw_malloc(8 * 1024 * 4), ext.raw_malloc(8 * 1024 * 4)]
    data = [ext.raw_malloc(256), ext.raw_malloc(256)]
    counter = torch.zeros(1024, dtype=torch.int32, device="cuda")
    ext.group_barrier(data, sig, 0, counter)
    torch.cuda.synchronize()
    with pytest.raises(CommTimeoutError):
        check_comm_status(dev)
    # The context is still usable.
    x = torch.ones(1024, device="cuda")
    assert (x * 2).sum().item() == 2048
    for p in sig + data:
        ext.raw_free(p)
