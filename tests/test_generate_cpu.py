"""Sampling (models/generate.py, sample.py): the KV-cache decoder against
re-running the whole context, on one process and on TP / EP gloo ranks."""
import os
import subprocess
import sys

import pytest
import torch

from dist_util import run_ranks

from heiretsu_b200.config import GPTConfig
from heiretsu_b200.models.generate import KVCache, _forward_cached, generate
from heiretsu_b200.models.gpt import GPT

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = dict(block_size=48, vocab_size=96, n_layer=3, n_head=4, n_embed=32, dropout=0.1)


def _model(moe=False, seed=3):
    kw = dict(CFG, **(dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}))
    torch.manual_seed(seed)
    return GPT(GPTConfig(**kw))


@pytest.mark.parametrize("moe", [False, True])
def test_cached_logits_match_full_forward(moe):
    m = _model(moe).eval()
    idx = torch.randint(0, 96, (2, 20), generator=torch.Generator().manual_seed(0))
    cache = KVCache(m, 2, idx.device, torch.float32)
    got = [_forward_cached(m, idx[:, :12], cache)]
    for t in range(12, 20):
        got.append(_forward_cached(m, idx[:, t:t + 1], cache))
    with torch.no_grad():
        full, _, _ = m(idx)
    for i, t in enumerate(range(11, 20)):
        assert torch.allclose(got[i], full[:, t], atol=1e-5, rtol=1e-5), t


@pytest.mark.parametrize("moe", [False, True])
def test_generate_cache_equals_recompute(moe):
    m = _model(moe)
    idx = torch.randint(0, 96, (3, 5), generator=torch.Generator().manual_seed(1))
    greedy_c = generate(m, idx, 30, temperature=0)
    greedy_r = generate(m, idx, 30, temperature=0, kv_cache=False)
    assert torch.equal(greedy_c, greedy_r)
    s1 = generate(m, idx, 30, temperature=0.9, top_k=10, generator=torch.Generator().manual_seed(7))
    s2 = generate(m, idx, 30, temperature=0.9, top_k=10, generator=torch.Generator().manual_seed(7), kv_cache=False)
    assert torch.equal(s1, s2)
    assert m.training  # mode restored
    with pytest.raises(ValueError, match="block_size"):
        generate(m, idx, 60, temperature=0)
    assert generate(m, idx, 60, temperature=0, kv_cache=False).shape == (3, 65)  # sliding window


def _worker_tp(rank, world, tp, ep, moe):
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.utils.ckpt import load_from_full

    topo = init_topology(dp=1, ep=ep, tp=tp)
    dense = _model(moe)
    full = dense.state_dict()
    kw = dict(CFG, **(dict(num_experts=4, top_k=2, moe_freq=2) if moe else {}))
    m = GPT(GPTConfig(**kw), topo=topo)
    load_from_full(m, full, topo.tp_rank, topo.tp)
    idx = torch.randint(0, 96, (2, 6), generator=torch.Generator().manual_seed(2))
    out = generate(m, idx, 20, temperature=0.8, top_k=20, generator=torch.Generator().manual_seed(9))
    ref = generate(dense, idx, 20, temperature=0.8, top_k=20, generator=torch.Generator().manual_seed(9))
    return out.tolist(), ref.tolist()


@pytest.mark.parametrize("tp,ep,moe", [(2, 1, False), (1, 2, True)])
def test_generate_on_parallel_ranks(tp, ep, moe):
    for out, ref in run_ranks(_worker_tp, tp * ep, tp, ep, moe):
        assert out == ref


def test_sample_script_on_a_sharded_checkpoint(tmp_path):
    """sample.py merges the shards of a tp2 checkpoint and samples the dense model."""
    from dataclasses import asdict

    from heiretsu_b200.topo import Topology
    from heiretsu_b200.utils.ckpt import shard_from_full

    m = _model()
    full = m.state_dict()
    for t in range(2):
        shard = GPT(GPTConfig(**CFG), topo=Topology(dp=1, ep=1, tp=2, pp=1, rank=t, world_size=2, dp_rank=0,
                                                    ep_rank=0, pp_rank=0, tp_rank=t, tp_group=None, pp_group=None,
                                                    ep_group=None, dp_group=None))
        sd = shard_from_full(shard, full, t, 2)
        torch.save({"model": sd, "cfg": asdict(m.cfg), "step": 7,
                    "topo": {"dp": 1, "ep": 1, "tp": 2, "pp": 1, "pp_rank": 0, "tp_rank": t, "ep_rank": 0}},
                   tmp_path / f"ckpt_0000007_pp0_ep0_tp{t}.pt")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "sample.py"), "--ckpt",
                        str(tmp_path / "ckpt_0000007_pp0_ep0_tp1.pt"), "--start", "1,2,3", "--max_new_tokens", "10",
                        "--temperature", "0", "--device", "cpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = [int(t) for t in r.stdout.strip().splitlines()[0].split(",")]
    want = generate(m, torch.tensor([[1, 2, 3]]), 10, temperature=0)[0].tolist()
    assert got == want
