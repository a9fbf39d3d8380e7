"""Numerics of the tcgen05 GEMM against a plain PyTorch fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from heiretsu_b200.ops import gemm as g
    from heiretsu_b200.ops._C import check_status
    return g, check_status


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


SHAPES = [(256, 256, 128), (8192, 2304, 768), (300, 200, 136), (128, 50304, 768), (1000, 3072, 768)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("bn", [128, 192, 256])
def test_fwd_bias(M, N, K, bn):
    g, check = _ops()
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    b = torch.randn(N, device="cuda")
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    g.gemm(x, w, out, N, g.EPI_BF16, False, False, bias=b, block_n=bn)
    check()
    ref = x.float() @ w.float().t() + b
    _close(out, ref)


@pytest.mark.parametrize("M,N,K", [(8192, 768, 3072), (200, 136, 72), (512, 384, 256)])
def test_dgrad(M, N, K):
    g, check = _ops()
    torch.manual_seed(1)
    dy = torch.randn(M, N, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    out = g.linear_dgrad(dy, w, f32=True)
    check()
    _close(out, dy.float() @ w.float(), 1e-2)


@pytest.mark.parametrize("M,N,K", [(8192, 768, 3072), (200, 136, 72), (4096, 2304, 768)])
def test_wgrad_accumulate(M, N, K):
    g, check = _ops()
    torch.manual_seed(2)
    dy = torch.randn(M, N, device="cuda").bfloat16()
    x = torch.randn(M, K, device="cuda").bfloat16()
    acc = torch.randn(N, K, device="cuda")
    ref = acc + dy.float().t() @ x.float()
    g.linear_wgrad(dy, x, out=acc, accumulate=True)
    check()
    _close(acc, ref, 1e-2)


def test_gelu_and_dgelu():
    g, check = _ops()
    torch.manual_seed(3)
    M, N, K = 1024, 3072, 768
    x = (0.5 * torch.randn(M, K, device="cuda")).bfloat16()
    w = (0.05 * torch.randn(N, K, device="cuda")).bfloat16()
    b = 0.1 * torch.randn(N, device="cuda")
    out, pre = g.linear_fwd_gelu(x, w, b)
    check()
    pre_ref = x.float() @ w.float().t() + b
    _close(pre, pre_ref)
    _close(out, torch.nn.functional.gelu(pre.float(), approximate="tanh"))
    dy = torch.randn(M, K, device="cuda").bfloat16()
    # dgrad through w^T: dh = dy @ w^T (w^T: [K, N] as a [N', K'] = [K, N] weight)
    wt = w.t().contiguous()  # [K, N]
    dh = g.linear_dgrad(dy, wt, gelu_pre=pre)
    check()
    pre_f = pre.float().requires_grad_(True)
    gl = torch.nn.functional.gelu(pre_f, approximate="tanh")
    gl.backward(dy.float() @ wt.float())
    _close(dh, pre_f.grad, 3e-2)


def test_resid_epilogue():
    g, check = _ops()
    torch.manual_seed(4)
    M, N, K = 2048, 768, 768
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    b = torch.randn(N, device="cuda")
    r = torch.randn(M, N, device="cuda")
    ref = r + x.float() @ w.float().t() + b
    g.linear_fwd_resid(x, w, b, r, out=r)
    check()
    _close(r, ref, 1e-2)


@pytest.mark.parametrize("M,N,K", [(768, 768, 8192), (8192, 768, 50304), (2304, 768, 8192)])
def test_split_k_fp32_paths(M, N, K):
    """Shapes with few output tiles and long K take the split-K (atomic) epilogue."""
    g, check = _ops()
    torch.manual_seed(7)
    a = torch.randn(M, K, device="cuda").bfloat16()
    b = torch.randn(N, K, device="cuda").bfloat16()
    ref = a.float() @ b.float().t()
    out = torch.full((M, N), 3.0, device="cuda")
    g.gemm(a, b, out, N, g.EPI_F32, False, False)
    check()
    _close(out, ref, 1e-2)
    acc = torch.ones(M, N, device="cuda")
    g.gemm(a, b, acc, N, g.EPI_F32_ACC, False, False)
    check()
    _close(acc, ref + 1, 1e-2)
