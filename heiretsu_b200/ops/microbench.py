"""Kernel micro-benchmarks: the model's hot ops against their PyTorch/cuBLAS
counterparts on the GPT-2 shapes (M = 8 x 1024 tokens).

    python -m heiretsu_b200.ops.microbench [--only gemm] [--shape fc_gelu] [--reps 20 --warmup 5] [--json out.json]

Timing: CUDA events around CUDA-graph replays of the op (host launch work
excluded, as in the graph-replayed training step), warm-up first, L2
flushed before every timed replay by READING a 256 MB buffer (a flush that
writes leaves ~126 MB of dirty lines whose write-back the timed kernel would
pay, about 20 us on a B200), median of the
repeats. PyTorch / cuBLAS references are timed the same way.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch


class _Flush:
    """Evicts the timed op's data from L2 without dirtying it: a sum over 256 MB
    (written once here, only read afterwards) into a preallocated scalar."""

    def __init__(self):
        self.buf = torch.zeros(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
        self.out = torch.empty((), dtype=torch.float32, device="cuda")

    def __call__(self):
        torch.sum(self.buf, dim=0, out=self.out)


def _flush_buf():
    return _Flush()


REPS, WARMUP = 20, 5
SHAPE = None


def time_fn(fn, reps=None, warmup=None, flush=None, graph=True):
    """Median device time of fn. With graph=True (default) fn is captured in a
    CUDA graph and the replays are timed, so host-side launch work (argument
    checks, tensor-map encoding) is not counted -- the training step replays a
    graph too. Both our kernels and the PyTorch references are timed this way."""
    reps = REPS if reps is None else reps
    warmup = WARMUP if warmup is None else warmup
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    run = fn
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        run = g.replay
        run()
        torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        if flush is not None:
            flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        run()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


GEMM_SHAPES = [
    # name, M, N, K, layout
    ("qkv_fwd", 8192, 2304, 768, "fwd"),
    ("attnproj_fwd", 8192, 768, 768, "fwd"),
    ("fc_fwd", 8192, 3072, 768, "fwd"),
    ("mlpproj_fwd", 8192, 768, 3072, "fwd"),
    ("lmhead_fwd", 8192, 50304, 768, "fwd"),
    ("fc_dgrad", 8192, 768, 3072, "dgrad"),  # dx[M,K=768] = dy[M,N=3072] @ W[3072,768]
    ("fc_wgrad", 8192, 3072, 768, "wgrad"),  # dW[3072,768] = dy^T @ x
    ("lmhead_dgrad", 8192, 768, 50304, "dgrad"),
    ("lmhead_wgrad", 8192, 50304, 768, "wgrad"),
    ("square_8192", 8192, 8192, 8192, "fwd"),
    # fused epilogues as the model uses them (reference time: the plain cuBLAS GEMM)
    ("attnproj_resid", 8192, 768, 768, "resid"),     # x_new = x + y W^T + b   (fp32 out)
    ("mlpproj_resid", 8192, 768, 3072, "resid"),
    ("fc_gelu", 8192, 3072, 768, "gelu"),            # h = GELU(x W^T + b), pre-activation kept
    ("fc_dgrad_dgelu", 8192, 3072, 768, "dgelu"),    # dpre = (dy W) * GELU'(pre)
    ("qkv_dgrad_f32", 8192, 768, 2304, "dgrad32"),   # dx (fp32) = dqkv W
]


def bench_gemm(flush):
    from . import gemm as g
    from ._C import check_status

    rows = []
    for name, M, N, K, kind in GEMM_SHAPES:
        if SHAPE is not None and name != SHAPE:
            continue
        torch.manual_seed(0)
        if kind == "fwd":
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            ours = lambda: g.gemm(x, w, out, N, g.EPI_BF16, False, False)
            ref = lambda: torch.matmul(x, w.t())
            flops = 2.0 * M * N * K
        elif kind == "dgrad":
            # output [M, N] from dy [M, K] and W [K, N]
            dy = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            ours = lambda: g.gemm(dy, w, out, N, g.EPI_BF16, False, True)
            ref = lambda: torch.matmul(dy, w)
            flops = 2.0 * M * N * K
        elif kind == "wgrad":
            dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            out = torch.zeros(N, K, device="cuda", dtype=torch.float32)
            ours = lambda: g.gemm(dy, x, out, K, g.EPI_F32_ACC, True, True)
            ref = lambda: torch.matmul(dy.t(), x)
            flops = 2.0 * M * N * K
        elif kind in ("resid", "gelu"):
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
            bias = torch.randn(N, device="cuda")
            if kind == "resid":
                res = torch.randn(M, N, device="cuda")
                out = torch.empty(M, N, device="cuda")
                ours = lambda: g.gemm(x, w, out, N, g.EPI_F32_RESID, False, False, bias=bias, resid=res)
            else:
                out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                ours = lambda: g.gemm(x, w, out, N, g.EPI_BF16_GELU, False, False, bias=bias, aux=pre)
            ref = lambda: torch.matmul(x, w.t())
            flops = 2.0 * M * N * K
        else:  # dgelu / dgrad32: output [M, N] from dy [M, K] and W stored [K, N]
            dy = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            w = torch.randn(K, N, device="cuda", dtype=torch.bfloat16)
            if kind == "dgelu":
                pre = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
                out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                ours = lambda: g.gemm(dy, w, out, N, g.EPI_BF16_DGELU, False, True, aux=pre)
            else:
                out = torch.empty(M, N, device="cuda")
                ours = lambda: g.gemm(dy, w, out, N, g.EPI_F32, False, True)
            ref = lambda: torch.matmul(dy, w)
            flops = 2.0 * M * N * K
        t_ours = time_fn(ours, flush=flush)
        check_status()
        t_ref = time_fn(ref, flush=flush)
        rows.append(dict(op="gemm", name=name, M=M, N=N, K=K, kind=kind, ms=t_ours, ref_ms=t_ref,
                         tflops=flops / t_ours / 1e9, ref_tflops=flops / t_ref / 1e9))
    return rows


def bench_attention(flush):
    """Causal attention fwd / bwd vs torch SDPA on the same box: GPT-2 small's heads
    (B=8, T=1024, 12 heads of 64) and the reference's default model's (6 heads of 128)."""
    import torch.nn.functional as F

    from . import kernels as K
    from ._C import check_status

    rows = []
    for tag, B, T, nh, dh in (("", 8, 1024, 12, 64), ("_d128", 8, 1024, 6, 128)):
        H = nh * dh
        qkv = torch.randn(B * T, 3 * H, device="cuda", dtype=torch.bfloat16)
        y, lse = K.attention_fwd(qkv, B, T, nh, head_dim=dh)
        dy = torch.randn_like(y)
        q, k, v = qkv.view(B, T, 3, nh, dh).permute(2, 0, 3, 1, 4).unbind(0)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        fwd_flops = 4.0 * B * nh * T * T * dh / 2
        t = time_fn(lambda: K.attention_fwd(qkv, B, T, nh, out=y, head_dim=dh), flush=flush)
        tr = time_fn(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), flush=flush)
        rows.append(dict(op="attention", name="fwd" + tag, ms=t, ref_ms=tr, tflops=fwd_flops / t / 1e9,
                         ref_tflops=fwd_flops / tr / 1e9))
        t = time_fn(lambda: K.attention_bwd(qkv, y, dy, lse, B, T, nh, head_dim=dh), flush=flush)
        qg, kg, vg = (x.detach().requires_grad_(True) for x in (q, k, v))
        o = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True)
        g = torch.randn_like(o)
        # (autograd runs on its own threads and cannot be graph-captured; timed eagerly)
        tr = time_fn(lambda: torch.autograd.grad(o, (qg, kg, vg), g, retain_graph=True), flush=flush, graph=False)
        rows.append(dict(op="attention", name="bwd" + tag, ms=t, ref_ms=tr, tflops=2.5 * fwd_flops / t / 1e9,
                         ref_tflops=2.5 * fwd_flops / tr / 1e9))
    check_status()
    return rows


def bench_norm(flush):
    """LayerNorm fwd/bwd at [8192, 768] vs torch (bytes moved / time)."""
    import torch.nn.functional as F

    from . import kernels as K

    M, H = 8192, 768
    x = torch.randn(M, H, device="cuda")
    w = torch.randn(H, device="cuda")
    b = torch.randn(H, device="cuda")
    rows = []
    t = time_fn(lambda: K.layernorm_fwd(x, w, b), flush=flush)
    tr = time_fn(lambda: F.layer_norm(x, (H,), w, b), flush=flush)
    rows.append(dict(op="layernorm", name="fwd", ms=t, ref_ms=tr, gbs=(M * H * 6) / t / 1e6))
    y, mean, rstd = K.layernorm_fwd(x, w, b)
    dy = torch.randn(M, H, device="cuda")
    dres = torch.zeros(M, H, device="cuda")
    d16 = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
    dg = torch.zeros(H, device="cuda")
    db = torch.zeros(H, device="cuda")
    t = time_fn(lambda: K.layernorm_bwd(dy, x, mean, rstd, w, dres, dres, d16, dg, db), flush=flush)
    rows.append(dict(op="layernorm", name="bwd", ms=t, gbs=(M * H * 18) / t / 1e6))
    # bias gradients: column sums of the bf16 output gradients (dqkv width)
    g16 = torch.randn(M, 3 * H, device="cuda").bfloat16()
    acc = torch.zeros(3 * H, device="cuda")
    t = time_fn(lambda: K.colsum_bf16(g16, acc), flush=flush)
    tr = time_fn(lambda: g16.float().sum(0), flush=flush)
    rows.append(dict(op="colsum", name=f"{M}x{3 * H}", ms=t, ref_ms=tr, gbs=(M * 3 * H * 2) / t / 1e6))
    return rows


def bench_ce(flush):
    """Cross-entropy over [8192, 50304] bf16 logits: forward + in-place gradient as two
    kernels (ref_ms) against the single-pass kernel (ms). gbs counts the single pass's
    bytes (one read and one write of the logits)."""
    from . import kernels as K
    from ._C import check_status

    M, V, Vp = 8192, 50257, 50304
    logits = torch.zeros(M, Vp, device="cuda", dtype=torch.bfloat16)
    logits[:, :V] = torch.randn(M, V, device="cuda").bfloat16()
    t = torch.randint(0, V, (M,), device="cuda")
    scale = torch.full((1,), 1.0 / M, device="cuda")

    def two():
        _, lse, _ = K.cross_entropy_fwd(logits, V, t)
        K.cross_entropy_bwd_(logits, V, t, lse, scale, 1.0)

    tr = time_fn(two, flush=flush)
    ts = time_fn(lambda: K.cross_entropy_fused_(logits, V, t, scale), flush=flush)
    check_status()
    return [dict(op="cross_entropy", name=f"{M}x{Vp} single pass vs two kernels", ms=ts, ref_ms=tr,
                 gbs=2 * M * Vp * 2 / ts / 1e6)]


EXTRA_BENCHES = {"attention": bench_attention, "norm": bench_norm, "ce": bench_ce}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--json", default=None)
    ap.add_argument("--shape", default=None, help="run only this GEMM shape (by name)")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args(argv)
    global REPS, WARMUP, SHAPE
    REPS, WARMUP, SHAPE = args.reps, args.warmup, args.shape
    flush = _flush_buf()
    rows = []
    if args.only in (None, "gemm"):
        rows += bench_gemm(flush)
    extra = globals().get("EXTRA_BENCHES", {})
    for k, fn in extra.items():
        if args.only in (None, k):
            rows += fn(flush)
    for r in rows:
        print(json.dumps(r))
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
