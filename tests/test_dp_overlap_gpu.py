"""Data-parallel gradient reduction overlapped with backward (block by block
on a side stream, inside the captured CUDA graph) against the one-shot
reduction after backward. 2 GPUs.

Training is not bitwise reproducible run to run (the attention dQ, split-K
weight gradients and the embedding scatter add in a non-deterministic
order), so two one-shot runs set the noise floor; the overlapped run must
stay within a small multiple of it. A stale or partial gradient would be
orders of magnitude larger (one AdamW step moves weights by ~lr).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
        from heiretsu_b200.config import GPTConfig
        from heiretsu_b200.ops._C import check_status
        from heiretsu_b200.topo import init_topology
        from heiretsu_b200.trainer import Engine, build_argparser
        from heiretsu_b200.utils.data import SyntheticLoader

        topo = init_topology(dp=world, timeout=timedelta(seconds=120))
        cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=3, n_head=4, n_embed=256, dropout=0.0)
        out = {}
        for run, overlap in (("a", 0), ("b", 0), ("o", 1)):
            args = build_argparser().parse_args([
                "--batch_size", "2", "--block_size", "256", "--grad_accum_steps", "2", "--n_layer", "3",
                "--n_head", "4", "--n_embed", "256", "--dropout", "0", "--amp", "bf16", "--engine", "fused",
                "--dp", str(world), "--overlap_dp", str(overlap)])
            torch.manual_seed(0)
            eng = Engine(args, topo, dev, cfg)
            assert eng.use_graph and eng.overlap_dp == bool(overlap)
            loader = SyntheticLoader(2, 256, 1000, seed=3, rank=rank)
            losses = [float(eng.train_step(loader)[0].item()) for _ in range(5)]  # 2 eager + capture + 2 replays
            torch.cuda.synchronize()
            check_status()
            out[run] = (losses, eng.flat.data.clone())
            eng.close()
        noise = (out["a"][1] - out["b"][1]).abs().max().item()
        diff = (out["o"][1] - out["a"][1]).abs().max().item()
        q.put((rank, out["a"][0], out["o"][0], noise, diff))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), None, None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_overlapped_dp_reduction_is_exact():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, l0, l1, noise, diff in res:
        assert not isinstance(l0, str), l0
        assert all(abs(a - b) < 1e-3 for a, b in zip(l0, l1)), (rank, l0, l1)
        assert diff <= 20 * noise + 1e-6, (rank, diff, noise)
