"""Race detection by replay.

A kernel that reads a buffer before its producer finished (a missing wait, a
barrier that releases early) makes results depend on timing, so repeating the
same work must show it. Repeats are not bitwise equal even without a race:
the attention dQ reduce-adds, split-K partial sums and embedding scatter-adds
add fp32 values in whatever order they arrive, and an fp32 sum whose order
changes can flip a bf16 rounding further down. So the checks compare against
that noise, on quantities it leaves small:

* gradients of one fused forward/backward, repeated on the same weights and
  tokens, eagerly and as replays of one captured CUDA graph: every
  parameter's gradient must agree within 1e-2 of its norm (measured noise on
  a B200 is ~1e-3; a race corrupts whole tiles);
* the loss curve of a 5-step training run (AdamW, dropout) repeated from the
  same seed, eager and graph-replayed: within 1e-3 per step.

Weights after several AdamW steps are not compared: Adam turns a gradient
element that is pure rounding noise into a full +-lr update, and some are
exactly that (the key bias gets zero gradient in exact arithmetic, since a
constant added to every key of a query leaves its softmax unchanged).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _grads_of(model, flat):
    return {n: p.main_grad.detach().clone() for n, p in model.named_parameters()}


def _assert_close(ga, gb, what):
    bad = []
    for n in ga:
        rel = (ga[n] - gb[n]).norm().item() / (ga[n].norm().item() + 1e-12)
        if rel > 1e-2:
            bad.append((n, rel))
    assert not bad, (what, bad)


def test_fused_gradients_replay_eager_and_graph():
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.gpt import GPT
    from heiretsu_b200.ops._C import check_status
    from heiretsu_b200.parallel.flat import FlatParams

    cfg = GPTConfig(block_size=256, vocab_size=2048, n_layer=2, n_head=4, n_embed=256, dropout=0.1)
    torch.manual_seed(0)
    model = GPT(cfg).cuda()
    flat = FlatParams(model, torch.device("cuda"))
    model.fused = True
    seed = torch.tensor([7], dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randint(0, 2048, (4, 256), device="cuda", generator=g)
    y = torch.randint(0, 2048, (4, 256), device="cuda", generator=g)

    def step():
        # the same dropout masks every time: the device seed is reset before each forward
        seed.fill_(7)
        for layer, blk in enumerate(model.tr.h):
            blk._hb_dropout = (seed, layer, 0.1)
        flat.zero_grad()
        _, loss, _ = model(x, y, return_logits=False)
        loss.backward()
        return loss

    eager = []
    for _ in range(3):
        step()
        torch.cuda.synchronize()
        check_status()
        eager.append(_grads_of(model, flat))
    _assert_close(eager[0], eager[1], "eager repeat 1")
    _assert_close(eager[0], eager[2], "eager repeat 2")

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for i in range(3):
        graph.replay()
        torch.cuda.synchronize()
        check_status()
        _assert_close(eager[0], _grads_of(model, flat), f"graph replay {i}")
    del graph


def _run(graph: int):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.ops._C import check_status
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser
    from heiretsu_b200.utils.data import SyntheticLoader

    args = build_argparser().parse_args([
        "--batch_size", "4", "--block_size", "256", "--grad_accum_steps", "2", "--n_layer", "2", "--n_head", "4",
        "--n_embed", "256", "--dropout", "0.1", "--amp", "bf16", "--engine", "fused", "--learning_rate", "1e-3",
        "--cuda_graph", str(graph)])
    torch.manual_seed(0)
    cfg = GPTConfig(block_size=256, vocab_size=2048, n_layer=2, n_head=4, n_embed=256, dropout=0.1)
    eng = Engine(args, init_topology(dp=1), torch.device("cuda"), cfg)
    loader = SyntheticLoader(4, 256, 2048, seed=11)
    losses = [float(eng.train_step(loader)[0].item()) for _ in range(5)]
    torch.cuda.synchronize()
    check_status()
    eng.close()
    return losses


@pytest.mark.parametrize("graph", [0, 1])
def test_fused_training_losses_replay(graph):
    la = _run(graph)
    lb = _run(graph)
    assert all(abs(a - b) < 1e-3 for a, b in zip(la, lb)), (la, lb)
