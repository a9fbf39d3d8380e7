"""The allocation-free cross-entropy entry point, called through its C symbol.

It exists for callers that cannot allocate device memory (an allocator's
out-of-memory handler, a C/C++ host that owns every allocation). It must match
the regular entry point (the torch binding) and an fp32 PyTorch log-sum-exp on
two calls in a row; the second call reuses the file-scope scratch left by the
first. Collected last on purpose, so a failure here never hides another test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    import heiretsu_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.hb_cross_entropy_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _inputs(M, V, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    Vp = (V + 127) // 128 * 128
    logits = torch.zeros(M, Vp, device="cuda", dtype=torch.bfloat16)
    logits[:, :V] = (3 * torch.randn(M, V, device="cuda", generator=g)).bfloat16()
    t = torch.randint(0, V, (M,), device="cuda", generator=g)
    return logits, t


def test_noalloc_matches_regular_entry_point_twice():
    from heiretsu_b200.ops import kernels as K

    fn = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (M, V, seed) in enumerate([(1024, 50257, 0), (333, 1000, 1)]):
        logits, t = _inputs(M, V, seed)
        ref_loss, ref_lse, _ = K.cross_entropy_fwd(logits, V, t)
        lse = torch.full((M,), float("nan"), device="cuda")
        loss = torch.full((1,), float("nan"), device="cuda")
        rc = fn(logits.data_ptr(), logits.stride(0), M, V, t.data_ptr(), -100, lse.data_ptr(), loss.data_ptr(),
                stream)
        assert rc == 0, f"call {call}: return code {rc}"
        torch.cuda.synchronize()
        assert torch.allclose(lse, ref_lse, atol=1e-5, rtol=1e-5), call
        assert abs(loss.item() - ref_loss.item()) <= 1e-5 * max(1.0, abs(ref_loss.item())), call
        # fp32 PyTorch oracle of the same op on the same bf16 logits
        x = logits[:, :V].float()
        want_lse = torch.logsumexp(x, dim=1)
        want_loss = (want_lse - x.gather(1, t[:, None]).squeeze(1)).mean()
        assert torch.allclose(lse, want_lse, atol=1e-4, rtol=1e-5), (call, (lse - want_lse).abs().max().item())
        assert abs(loss.item() - want_loss.item()) <= 1e-4 * max(1.0, abs(want_loss.item())), call


def test_noalloc_rejects_too_many_rows():
    fn = _symbol()
    dummy = torch.zeros(8, device="cuda")
    rc = fn(dummy.data_ptr(), 128, 65537, 128, dummy.data_ptr(), -100, dummy.data_ptr(), dummy.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2


def test_noalloc_rejects_unaligned_logits_and_leaves_outputs_for_zero_rows():
    fn = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    logits, t = _inputs(16, 256, 2)
    lse = torch.full((16,), 7.0, device="cuda")
    loss = torch.full((1,), 7.0, device="cuda")
    # a row start 2 bytes into the buffer: rejected before any launch
    rc = fn(logits.data_ptr() + 2, logits.stride(0), 16, 256, t.data_ptr(), -100, lse.data_ptr(), loss.data_ptr(),
            stream)
    assert rc == 1
    rc = fn(logits.data_ptr(), logits.stride(0), 0, 256, t.data_ptr(), -100, lse.data_ptr(), loss.data_ptr(), stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert loss.item() == 7.0 and bool((lse == 7.0).all())
