"""The plain engine's AMP modes on the GPU (the reference's only precision
knob, train.py:353-357): bf16 autocast, and fp16 autocast with a GradScaler,
global-norm clipping and torch's fused AdamW. A learnable token pattern must be
learnt in both, with fp16 close to bf16."""
import pytest
import torch

pytestmark = pytest.mark.gpu


class _Pattern:
    B = 4

    def __init__(self):
        self.i = 0

    def next_batch(self, device):
        base = torch.arange(129)
        ids = torch.stack([(base * 7 + 3 * (self.i + r)) % 512 for r in range(4)]).to(device)
        self.i += 1
        return ids[:, :-1].contiguous(), ids[:, 1:].contiguous()


def _losses(amp):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser

    args = build_argparser().parse_args([
        "--batch_size", "4", "--block_size", "128", "--grad_accum_steps", "2", "--n_layer", "2", "--n_head", "2",
        "--n_embed", "64", "--dropout", "0", "--amp", amp, "--engine", "plain", "--learning_rate", "3e-3"])
    cfg = GPTConfig(block_size=128, vocab_size=512, n_layer=2, n_head=2, n_embed=64, dropout=0.0)
    torch.manual_seed(0)
    eng = Engine(args, init_topology(dp=1), torch.device("cuda"), cfg)
    assert not eng.fused and eng.use_amp
    loader = _Pattern()
    out = [float(eng.train_step(loader)[0]) for _ in range(12)]
    return out, eng


def test_plain_engine_bf16_and_fp16():
    bf, _ = _losses("bf16")
    fp, eng = _losses("fp16")
    assert eng.scaler is not None and eng.scaler.is_enabled()
    for losses in (bf, fp):
        assert all(torch.isfinite(torch.tensor(losses))), losses
        assert losses[-1] < losses[0] - 0.3, losses
    assert abs(fp[-1] - bf[-1]) < 0.5, (fp, bf)
