"""--amp fp16 on the fused engine: the kernels in their fp16 instantiations
against fp32 PyTorch, and the engine end to end with the device loss scale.

The reference's fp16 mode (train.py:197, :353-357, :436-452) is autocast in
fp16 plus torch.cuda.amp.GradScaler. Here activations and weight shadows are
fp16, the loss is multiplied by a device-resident scale before backward, the
optimizer unscales inside its clip coefficient, skips a step whose gradient
norm is not finite and halves the scale, and doubles it after a run of
finite steps (GradScaler's rule)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


def _check():
    from heiretsu_b200.ops._C import check_status
    check_status()


@pytest.mark.parametrize("M,N,K", [(8192, 2304, 768), (300, 200, 136), (1000, 3072, 768)])
def test_gemm_fp16_epilogues(M, N, K):
    from heiretsu_b200.ops import gemm as g

    torch.manual_seed(0)
    x = (0.5 * torch.randn(M, K, device="cuda")).half()
    w = (0.05 * torch.randn(N, K, device="cuda")).half()
    b = 0.1 * torch.randn(N, device="cuda")
    y = g.linear_fwd(x, w, b)
    _check()
    assert y.dtype == torch.float16
    ref = x.float() @ w.float().t() + b
    _close(y, ref, 1e-2)
    out, pre = g.linear_fwd_gelu(x, w, b)
    _check()
    _close(pre, ref, 1e-2)
    _close(out, F.gelu(pre.float(), approximate="tanh"), 1e-2)
    dy = torch.randn(M, N, device="cuda").half()
    wt = (0.05 * torch.randn(K, N, device="cuda")).half()  # a [K, N] weight: dgrad output is [M, N]
    dh = g.linear_dgrad(dy, w, f32=True)
    _check()
    _close(dh, dy.float() @ w.float(), 1e-2)
    dpre_in = torch.randn(M, K, device="cuda").half()
    dg = g.linear_dgrad(dpre_in, wt, gelu_pre=pre)
    _check()
    pre_f = pre.float().requires_grad_(True)
    F.gelu(pre_f, approximate="tanh").backward(dpre_in.float() @ wt.float())
    _close(dg, pre_f.grad, 3e-2)
    r = torch.randn(M, N, device="cuda")
    want = r + ref
    g.linear_fwd_resid(x, w, b, r, out=r)
    _check()
    _close(r, want, 1e-2)
    acc = torch.zeros(N, K, device="cuda")
    g.linear_wgrad(dy, x, out=acc, accumulate=True)
    _check()
    _close(acc, dy.float().t() @ x.float(), 1e-2)


@pytest.mark.parametrize("dh", [64, 128])
def test_attention_fp16(dh):
    from heiretsu_b200.ops import kernels as K

    torch.manual_seed(3)
    B, T, nh = 2, 384, 4
    H = nh * dh
    qkv = torch.randn(B * T, 3 * H, device="cuda").half()
    y, lse = K.attention_fwd(qkv, B, T, nh, head_dim=dh)
    _check()
    assert y.dtype == torch.float16
    q, k, v = (t.float().detach().requires_grad_(True) for t in
               qkv.view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4).unbind(0))
    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B * T, H)
    assert (y.float() - ref).abs().max().item() < 1e-2
    dy = torch.randn(B * T, H, device="cuda").half()
    ref.backward(dy.float())
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, T, nh, head_dim=dh)
    _check()
    d = dqkv.float().view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4)
    for i, g in enumerate((q.grad, k.grad, v.grad)):
        assert (d[i] - g).abs().max().item() <= 2e-2 * g.abs().max().item() + 1e-3


def test_layernorm_and_cross_entropy_fp16():
    from heiretsu_b200.ops import kernels as K

    torch.manual_seed(4)
    M, H, V = 512, 768, 1000
    x = torch.randn(M, H, device="cuda")
    w = torch.randn(H, device="cuda")
    b = torch.randn(H, device="cuda")
    y, mean, rstd = K.layernorm_fwd(x, w, b, dtype=torch.float16)
    _check()
    assert y.dtype == torch.float16
    _close(y, F.layer_norm(x, (H,), w, b), 2e-3)
    Vp = (V + 127) // 128 * 128
    logits = torch.zeros(M, Vp, device="cuda", dtype=torch.float16)
    logits[:, :V] = (3 * torch.randn(M, V, device="cuda")).half()
    t = torch.randint(0, V, (M,), device="cuda")
    loss, lse, _ = K.cross_entropy_fwd(logits, V, t)
    _check()
    want = F.cross_entropy(logits[:, :V].float(), t)
    assert abs(loss.item() - want.item()) < 1e-4 * max(1.0, want.item())
    g = logits.clone()
    K.cross_entropy_bwd_(g, V, t, lse, None, 1.0 / M)
    _check()
    lf = logits[:, :V].float().requires_grad_(True)
    F.cross_entropy(lf, t).backward()
    _close(g[:, :V], lf.grad, 1e-2)


def _engine(amp: str, extra=()):
    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.topo import init_topology
    from heiretsu_b200.trainer import Engine, build_argparser

    args = build_argparser().parse_args([
        "--batch_size", "4", "--block_size", "256", "--grad_accum_steps", "2", "--n_layer", "2", "--n_head", "4",
        "--n_embed", "256", "--dropout", "0.0", "--amp", amp, "--engine", "fused", "--learning_rate", "1e-3",
        "--grad_clip", "1.0", *extra])
    torch.manual_seed(0)
    cfg = GPTConfig(block_size=256, vocab_size=2048, n_layer=2, n_head=4, n_embed=256, dropout=0.0)
    return Engine(args, init_topology(dp=1), torch.device("cuda"), cfg)


def test_fused_engine_fp16_trains_and_matches_bf16_curve():
    """--amp fp16 runs the fused engine (fp16 shadows, device loss scale); on a fixed
    batch its loss curve follows the bf16 engine's."""
    from heiretsu_b200.utils.data import SyntheticLoader

    curves = {}
    for amp in ("fp16", "bf16"):
        eng = _engine(amp)
        assert eng.fused
        if amp == "fp16":
            assert eng.flat.data16.dtype == torch.float16 and eng.scaler is not None
        x, y = SyntheticLoader(4, 256, 2048, seed=3).next_batch_host()
        x, y = x.cuda(), y.cuda()

        class Fixed:
            B = 4

            def next_batch(self, device):
                return x, y

        curves[amp] = [float(eng.train_step(Fixed())[0].item()) for _ in range(8)]
        torch.cuda.synchronize()
        _check()
        if amp == "fp16":
            assert eng.scaler.get_scale() == 2.0 ** 16  # no overflow on this model: scale unchanged
        eng.close()
    a, b = curves["fp16"], curves["bf16"]
    assert a[-1] < a[0] - 0.5, a
    assert all(abs(p - q) < 5e-2 * max(1.0, q) for p, q in zip(a, b)), (a, b)


def test_fused_fp16_overflow_skips_the_step_and_backs_off():
    """A loss scale that overflows fp16 gradients: the step is skipped on the device
    (weights unchanged) and the scale halves, as GradScaler does."""
    from heiretsu_b200.utils.data import SyntheticLoader

    eng = _engine("fp16", ("--cuda_graph", "0"))
    eng.scaler.state[0] = 2.0 ** 40
    before = eng.flat.data.clone()
    loader = SyntheticLoader(4, 256, 2048, seed=5)
    eng.train_step(loader)
    torch.cuda.synchronize()
    _check()
    assert torch.equal(before, eng.flat.data)
    assert eng.scaler.get_scale() == 2.0 ** 39
    for _ in range(40):  # the scale keeps halving until the gradients fit, then steps resume
        eng.train_step(loader)
    torch.cuda.synchronize()
    assert eng.scaler.get_scale() < 2.0 ** 39
    assert not torch.equal(before, eng.flat.data)
    assert bool(torch.isfinite(eng.flat.data).all())
    eng.close()
