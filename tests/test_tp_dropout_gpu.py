"""Fused tensor parallelism with dropout (the default; --fused_tp_dropout 0 turns it off) against the
single-GPU fused model with dropout. Both draw their masks from the same seed,
indexed by global head and token row, so the two runs drop the same elements:
loss and gradients must agree within the bf16 tolerance of the plain TP test.

One process per GPU; skipped with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

P_DROP = 0.1
SEED = 4321


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _set_dropout(blocks, dev):
    seed = torch.tensor([SEED], dtype=torch.int32, device=dev)
    for layer, blk in enumerate(blocks):
        blk._hb_dropout = (seed, layer, P_DROP)
    return seed


def _worker(rank, world, port, q):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
        from heiretsu_b200.config import GPTConfig
        from heiretsu_b200.models.fused import fused_supported
        from heiretsu_b200.models.gpt import GPT
        from heiretsu_b200.ops._C import check_status
        from heiretsu_b200.parallel.flat import FlatParams
        from heiretsu_b200.topo import init_topology
        from heiretsu_b200.trainer import mark_tp_sharded, replication_weight
        from heiretsu_b200.utils.ckpt import load_from_full, shard_from_full

        topo = init_topology(dp=1, tp=world)
        cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=2, n_head=4, n_embed=256, dropout=P_DROP)
        assert fused_supported(cfg, topo)[0] and not fused_supported(cfg, topo, tp_dropout=False)[0]
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randint(0, 1000, (2, 256), device=dev, generator=g)
        y = torch.randint(0, 1000, (2, 256), device=dev, generator=g)

        # single-GPU fused model with dropout (the oracle), same weights on every rank
        torch.manual_seed(0)
        one = GPT(cfg).to(dev)
        full = {k: v.detach().clone() for k, v in one.state_dict().items()}
        flat_1 = FlatParams(one, dev)  # kept alive: the bf16 shadows and gradients live in its buffers
        one.fused = True
        _set_dropout(one.tr.h, dev)
        _, loss_1, _ = one(x, y, return_logits=False)
        loss_1.backward()
        torch.cuda.synchronize()
        check_status()
        grads_1 = {n: p.main_grad.detach().clone() for n, p in one.named_parameters()}
        del flat_1

        model = GPT(cfg, topo=topo).to(dev)
        load_from_full(model, full, topo.tp_rank, topo.tp)
        mark_tp_sharded(model)
        flat = FlatParams(model, dev, weight_of=replication_weight(topo), tp_group=topo.tp_group,
                          tp_sum_of=lambda n, p: not getattr(p, "tp_sharded", False))
        model.fused = True
        _set_dropout(model.tr.h, dev)
        flat.zero_grad()
        _, loss_s, _ = model(x, y, return_logits=False)
        loss_s.backward()
        for (start, end, _), tp_sum in zip(flat.ranges, flat.tp_sum):
            if tp_sum:
                flat.grad_symm_tp.sum_range(start, end - start, 1.0)
        torch.cuda.synchronize()
        check_status()
        lt = loss_s.detach().clone()
        dist.all_reduce(lt)
        expect = shard_from_full(model, {**full, **grads_1}, topo.tp_rank, topo.tp)
        worst, worst_name = 0.0, ""
        for n, p in model.named_parameters():
            e = expect[n]
            rel = (p.main_grad - e).norm().item() / (e.norm().item() + 1e-8)
            if rel > worst:
                worst, worst_name = rel, n
        q.put((rank, abs(lt.item() - loss_1.item()), worst, worst_name))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_tp2_dropout_matches_single_gpu_fused():
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
    for rank, dloss, worst, name in res:
        assert not isinstance(dloss, str), dloss
        assert dloss < 3e-2, (rank, dloss)
        assert worst < 6e-2, (rank, worst, name)
