"""Fused expert parallelism (local-expert windows; the second expert GEMM pushes
each weighted output row into every EP rank's slot buffer over NVLink) against
the same model run with every expert on one GPU.

The slots hold 16-bit rows round16(w * round16(acc)), and the one-GPU combine
adds exactly those terms in the same order, so the forward is the same on
either side; backward sums the expert input gradients across EP ranks in a
different order (fp32). Each parameter's gradient must match the one-GPU run
within 1e-2, or else be as close to an fp32 oracle (the plain PyTorch engine in
fp32 on the same weights and tokens) as the one-GPU fused run is:
err(EP) <= 2 err(one GPU) + 5e-3. The routing of every MoE call is recorded on
both sides; at most two tokens per layer may choose differently.

One process per GPU; skipped with fewer than two GPUs.
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

        from heiretsu_b200.models import fused_moe

        routes = []  # top-k expert ids [N, k] of every MoE forward, in call order
        orig_route = fused_moe.moe_route_and_experts

        def recording_route(moe, xn2, flat=None):
            aux, state = orig_route(moe, xn2, flat)
            routes.append(state[1].detach().sort(dim=1).values.clone())
            return aux, state

        fused_moe.moe_route_and_experts = recording_route
        topo = init_topology(dp=1, ep=world)
        cfg = GPTConfig(block_size=256, vocab_size=1000, n_layer=4, n_head=4, n_embed=256, dropout=0.0,
                        num_experts=8, top_k=2, moe_freq=2)
        torch.manual_seed(0)
        dense = GPT(cfg).to(dev)  # all 8 experts on this GPU
        with torch.no_grad():  # sharper routing than the 0.02-std init
            for blk in dense.tr.h:
                if hasattr(blk, "moe"):
                    blk.moe.router.gate.weight.mul_(20.0)
        full = {k: v.detach().clone() for k, v in dense.state_dict().items()}
        fd = FlatParams(dense, dev)
        dense.fused = True
        g = torch.Generator(device=dev).manual_seed(5)
        x = torch.randint(0, 1000, (2, 256), device=dev, generator=g)
        y = torch.randint(0, 1000, (2, 256), device=dev, generator=g)
        _, loss_d, aux_d = dense(x, y, return_logits=False)
        (loss_d + aux_d).backward()
        dgrads = {n: p.main_grad.detach().clone() for n, p in dense.named_parameters()}
        moe_blocks = [i for i, blk in enumerate(dense.tr.h) if hasattr(blk, "moe")]
        dense_routes = routes[:len(moe_blocks)]

        oracle = GPT(cfg).to(dev)  # plain PyTorch engine, fp32
        oracle.load_state_dict(full)
        _, loss_o, aux_o = oracle(x, y, return_logits=False)
        (loss_o + aux_o).backward()
        ograds = {n: p.grad.detach().clone() for n, p in oracle.named_parameters()}
        del oracle

        model = GPT(cfg, topo=topo).to(dev)  # 4 experts per rank
        load_from_full(model, full)
        mark_tp_sharded(model)
        flat = FlatParams(model, dev, weight_of=replication_weight(topo))
        model.fused = True
        for _ in range(2):  # the second pass reuses every buffer and barrier epoch
            del routes[:]
            flat.zero_grad()
            _, loss_e, aux_e = model(x, y, return_logits=False)
            (loss_e + aux_e).backward()
            torch.cuda.synchronize()
            check_status()
            check_comm_status(rank)
        expect = shard_from_full(model, {**full, **dgrads})
        expect_o = shard_from_full(model, {**full, **ograds})
        flips = max(int((rd != re_).any(dim=1).sum().item()) for rd, re_ in zip(dense_routes, routes))
        bad = []  # (name, err vs one GPU, err vs oracle, one GPU's err vs oracle)
        for n, p in model.named_parameters():
            r = _rel(p.main_grad, expect[n])
            if r < 1e-2:
                continue
            r_ep, r_one = _rel(p.main_grad, expect_o[n]), _rel(expect[n], expect_o[n])
            if r_ep > 2 * r_one + 5e-3:
                bad.append((n, r, r_ep, r_one))
        q.put((rank, abs(loss_e.item() - loss_d.item()), abs(aux_e.item() - aux_d.item()), bad, flips))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc(), None, None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_ep2_matches_single_gpu_experts():
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
    for rank, dloss, daux, bad, flips in res:
        assert not isinstance(dloss, str), dloss
        assert dloss < 1e-3 and daux < 1e-4, (rank, dloss, daux)
        assert flips <= 2, (rank, "tokens routed differently in one layer", flips)
        assert not bad, (rank, bad)
