"""Fused expert x tensor parallelism (ep2 x tp2 on 4 GPUs; the TP blocks run
sequence-sharded and each EP pair shares a token shard) against the same
weights with every expert on one GPU. One process per GPU; skipped with
fewer than four GPUs.
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


def _rel(a, b):
    return (a.float() - b.float()).norm().item() / (b.float().norm().item() + 1e-8)


def _worker(rank, world, port, q):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
        from heiretsu_b200.config import GPTConfig
        from heiretsu_b200.models.gpt import GPT
        from heiretsu_b200.ops._C import check_status
        from heiretsu_b200.parallel.flat import FlatParams
        from heiretsu_b200.parallel.symm import check_comm_status
        from heiretsu_b200.topo import init_topology
        from heiretsu_b200.trainer import mark_tp_sharded, replication_weight
        from heiretsu_b200.utils.ckpt import load_from_full, shard_from_full

        topo = init_topology(dp=1, ep=2, tp=2)
        cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=4, n_head=4, n_embed=256, dropout=0.0,
                        num_experts=8, top_k=2, moe_freq=2)
        torch.manual_seed(0)
        dense = GPT(cfg).to(dev)
        with torch.no_grad():
            for blk in dense.tr.h:
                if hasattr(blk, "moe"):
                    blk.moe.router.gate.weight.mul_(20.0)
        full = {k: v.detach().clone() for k, v in dense.state_dict().items()}
        FlatParams(dense, dev)
        dense.fused = True
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randint(0, 1000, (2, 256), device=dev, generator=g)
        y = torch.randint(0, 1000, (2, 256), device=dev, generator=g)
        _, loss_d, aux_d = dense(x, y, return_logits=False)
        (loss_d + aux_d).backward()
        dgrads = {n: p.main_grad.detach().clone() for n, p in dense.named_parameters()}

        model = GPT(cfg, topo=topo).to(dev)
        load_from_full(model, full, topo.tp_rank, topo.tp)
        mark_tp_sharded(model)
        flat = FlatParams(model, dev, weight_of=replication_weight(topo), tp_group=topo.tp_group,
                          tp_sum_of=lambda n, p: not getattr(p, "tp_sharded", False))
        model.fused = True
        for _ in range(2):  # the second pass reuses every buffer and barrier epoch
            flat.zero_grad()
            _, loss_s, aux_s = model(x, y, return_logits=False)
            (loss_s + aux_s).backward()
            for (start, end, _), tp_sum in zip(flat.ranges, flat.tp_sum):
                if tp_sum:
                    flat.grad_symm_tp.sum_range(start, end - start, 1.0)
            torch.cuda.synchronize()
            check_status()
            check_comm_status(rank)
        lt = loss_s.detach().clone()
        dist.all_reduce(lt, group=topo.tp_group)
        expect = shard_from_full(model, {**full, **dgrads}, topo.tp_rank, topo.tp)
        worst, worst_name = 0.0, ""
        for n, p in model.named_parameters():
            if "router" in n:
                continue  # the shard-local aux loss differs from the dense one (see below)
            r = _rel(p.main_grad, expect[n])
            if r > worst:
                worst, worst_name = r, n
        q.put((rank, abs(lt.item() - loss_d.item()), worst, worst_name))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_fused_ep2_tp2_matches_single_gpu():
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    for rank, dloss, worst, name in res:
        assert not isinstance(dloss, str), dloss
        assert dloss < 3e-2, (rank, dloss)
        assert worst < 6e-2, (rank, worst, name)
