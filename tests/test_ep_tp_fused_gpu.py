"""Fused expert x tensor parallelism (ep2 x tp2 on 4 GPUs; the TP blocks run
sequence-sharded and each EP pair shares a token shard).

Oracle: the same 4 GPUs as dp2 x tp2 with all experts on every rank (fused
TP + MoE, same token shards, same TP partner, hence identical attention
numerics and identical routing). A dense single-GPU oracle is not exact
here: TP sums bf16 partial outputs, the difference flips top-k choices of a
few near-tie tokens, and one flipped token moves a whole per-token term of
an expert's gradient. The TP + MoE model is checked against the dense
loss only. One process per GPU; skipped with fewer than four GPUs.
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
        from heiretsu_b200.utils.ckpt import load_from_full

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
        _, loss_d, _ = dense(x, y, return_logits=False)

        def run(topo):
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
            return model, lt.item()

        topo_ep = init_topology(dp=1, ep=2, tp=2)
        model_ep, loss_ep = run(topo_ep)
        topo_tp = init_topology(dp=2, tp=2)  # same tp_rank and TP partner for every rank
        model_tp, loss_tp = run(topo_tp)
        tp_grads = {n: p.main_grad for n, p in model_tp.named_parameters()}
        E_l = cfg.num_experts // 2
        worst, worst_name = 0.0, ""
        for n, p in model_ep.named_parameters():
            ref_name = n
            if ".experts." in n:
                pre, rest = n.split(".experts.", 1)
                j, tail = rest.split(".", 1)
                ref_name = f"{pre}.experts.{topo_ep.ep_rank * E_l + int(j)}.{tail}"
            r = _rel(p.main_grad, tp_grads[ref_name])
            if r > worst:
                worst, worst_name = r, n
        q.put((rank, abs(loss_ep - loss_tp), abs(loss_tp - loss_d.item()), worst, worst_name))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), None, None, None))


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
    for rank, d_ep_tp, d_tp_dense, worst, name in res:
        assert not isinstance(d_ep_tp, str), d_ep_tp
        assert d_ep_tp < 1e-4, (rank, d_ep_tp)
        assert d_tp_dense < 3e-2, (rank, d_tp_dense)
        assert worst < 1e-2, (rank, worst, name)
