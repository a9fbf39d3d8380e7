"""Fused compute + collective paths against their rooflines and against NCCL + cuBLAS.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m heiretsu_b200.parallel.commbench [--json out.json]

All N ranks form one group (dp = N for ``dp_reduce``, tp = N for the TP cases,
ep = N for ``ep_combine``). Each case is timed with CUDA events on the
launching stream after warm-up, with a barrier and a device synchronize on
both sides; the reported time is the maximum over ranks. The roofline target
of a case is the slower of its math at the bf16 GEMM peak and its NVLink
bytes (per GPU, per direction) at the measured peer bandwidth
(``heiretsu_b200.utils.roofline``).

Cases (shapes default to the benchmark models: GPT-2 small gradients, GPT-2
medium TP layers, the MoE model's combine):

* ``dp_reduce``: one kernel does reduce-scatter + 1/dp + all-gather of an
  fp32 gradient buffer of S bytes over peer memory (dp.py:13-26 made one
  kernel). Baseline: NCCL all_reduce + scale. NVLink bytes 2 (N-1)/N * S.
* ``tp_ag_gemm``: the column-parallel GEMM gathers the [M/tp, K] token
  shards of its input from the peers inside the kernel and multiplies by the
  local [N/tp, K] weight shard (tp_linear.py:135-155 with sequence-sharded
  input). Baseline: NCCL all_gather + cuBLAS. FLOPs 2 M (N/tp) K; NVLink
  bytes (tp-1)/tp * M K * 2.
* ``tp_gemm_rs``: the row-parallel GEMM [M, K/tp] x [N, K/tp]^T stores each
  partial tile into its token owner's receive slot, then the owner sums the
  slots with the residual (tp_linear.py:278-312, all-reduce turned into a
  reduce-scatter). Baseline: cuBLAS + NCCL reduce_scatter + residual add.
  FLOPs 2 M N K/tp; NVLink bytes (tp-1)/tp * M N * 2.
* ``ep_combine``: x + sum over the ep ranks of the partial expert outputs
  [T, H] fp32, every rank reading its peers' partials (ep_comm.py:83-135
  combine replaced by a partial-sum exchange). Baseline: NCCL all_reduce +
  add. NVLink bytes (ep-1) * T H * 4.
"""
from __future__ import annotations

import argparse
import json
import os
import types
from datetime import timedelta
from typing import Callable, Dict, List

import torch
import torch.distributed as dist

from ..utils.roofline import NVLINK_GBS, fused_target_ms, load_peaks

GPT2S_GRAD_ELEMS = 124_439_808  # GPT-2 small parameter count (fp32 gradients)


# -- work of each case (pure functions; unit-tested on CPU) -------------------
def dp_reduce_bytes(n_elem: int, world: int) -> float:
    """NVLink bytes per GPU and direction of a reduce-scatter + all-gather of n fp32 elements."""
    return 2.0 * (world - 1) / world * n_elem * 4


def tp_ag_gemm_work(M: int, N: int, K: int, tp: int):
    """(FLOPs, NVLink bytes) per rank of the gathered column-parallel GEMM (N = full width)."""
    return 2.0 * M * (N // tp) * K, (tp - 1) / tp * M * K * 2


def tp_gemm_rs_work(M: int, N: int, K: int, tp: int):
    """(FLOPs, NVLink bytes) per rank of the row-parallel GEMM with reduce-scatter (K = full depth)."""
    return 2.0 * M * N * (K // tp), (tp - 1) / tp * M * N * 2


def ep_combine_bytes(T: int, H: int, ep: int) -> float:
    return float(ep - 1) * T * H * 4


# -- timing --------------------------------------------------------------------
def _sync():
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()


def time_ms(fn: Callable[[], None], warmup: int, reps: int) -> float:
    """Mean ms per call (CUDA events on the current stream), maximum over ranks."""
    for _ in range(warmup):
        fn()
    _sync()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    _sync()
    t = torch.tensor([s.elapsed_time(e) / reps], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _check(dev: torch.device) -> None:
    from .symm import check_comm_status
    torch.cuda.synchronize()
    check_comm_status(dev.index)


# -- cases ---------------------------------------------------------------------
def case_dp_reduce(world, dev, n_elem, warmup, reps) -> Dict:
    from ..ops._C import load
    from .symm import SymmetricBuffer

    group = dist.group.WORLD
    symm = SymmetricBuffer(group, n_elem * 4, dev)
    buf = symm.tensor(torch.float32, n_elem)
    buf.fill_(1.0)
    ext = load()

    def fused():
        ext.dp_allreduce(symm.ptrs, symm.signal_ptrs, symm.rank, n_elem, 1.0 / world, symm.counter)

    ms = time_ms(fused, warmup, reps)
    _check(dev)
    ref_buf = torch.ones(n_elem, device=dev)

    def nccl():
        dist.all_reduce(ref_buf)
        ref_buf.mul_(1.0 / world)

    ref_ms = time_ms(nccl, warmup, reps)
    return dict(case="dp_reduce", shape=f"{n_elem} fp32", ms=ms, ref_ms=ref_ms, flops=0.0,
                nvlink_bytes=dp_reduce_bytes(n_elem, world))


def _tp_topo(world):
    return types.SimpleNamespace(tp=world, tp_rank=dist.get_rank(), tp_group=dist.group.WORLD)


def case_tp_ag_gemm(world, dev, M, N, K, warmup, reps) -> Dict:
    from ..models.fused_tp import TPComm
    from ..ops import gemm as G

    tp = world
    Ms, n_loc = M // tp, N // tp
    comm = TPComm(_tp_topo(world), Ms, K, dev)
    g = torch.Generator(device=dev).manual_seed(11 + comm.rank)
    comm.src_view(0).copy_(torch.randn(Ms, K, device=dev, generator=g).bfloat16())
    w = (0.02 * torch.randn(n_loc, K, device=dev, generator=g)).bfloat16()
    bias = torch.zeros(n_loc, device=dev)
    full = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
    out = torch.empty(M, n_loc, device=dev, dtype=torch.bfloat16)
    comm.barrier()

    def fused():
        G.gemm(full, w, out, n_loc, G.EPI_BF16, False, False, bias=bias, ag=comm.ag(0))

    ms = time_ms(fused, warmup, reps)
    _check(dev)
    shard = comm.src_view(0).clone()
    gath = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
    ref_out = torch.empty(M, n_loc, device=dev, dtype=torch.bfloat16)

    def baseline():
        dist.all_gather_into_tensor(gath, shard)
        torch.addmm(bias.bfloat16(), gath, w.t(), out=ref_out)

    ref_ms = time_ms(baseline, warmup, reps)
    flops, nbytes = tp_ag_gemm_work(M, N, K, tp)
    return dict(case="tp_ag_gemm", shape=f"M{M} N{N} K{K} tp{tp}", ms=ms, ref_ms=ref_ms, flops=flops,
                nvlink_bytes=nbytes)


def case_tp_gemm_rs(world, dev, M, N, K, warmup, reps) -> Dict:
    from ..models.fused_tp import TPComm
    from ..ops import gemm as G
    from ..ops import kernels as Kn

    tp = world
    Ms, k_loc = M // tp, K // tp
    comm = TPComm(_tp_topo(world), Ms, N, dev)
    g = torch.Generator(device=dev).manual_seed(23 + comm.rank)
    x = torch.randn(M, k_loc, device=dev, generator=g).bfloat16()
    w = (0.02 * torch.randn(N, k_loc, device=dev, generator=g)).bfloat16()
    bias = torch.zeros(N, device=dev)
    resid = torch.randn(Ms, N, device=dev, generator=g)
    out = torch.empty(Ms, N, device=dev)

    def fused():
        G.gemm(x, w, comm.recv16_all(), N, G.EPI_BF16, False, False, rs=comm.rs16())
        comm.barrier()  # partials delivered
        Kn.resid_sum_ln(resid, comm.recv16_all(), tp, bias, out)
        comm.barrier()  # slots consumed before the next GEMM overwrites them

    ms = time_ms(fused, warmup, reps)
    _check(dev)
    part = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    red = torch.empty(Ms, N, device=dev, dtype=torch.bfloat16)

    def baseline():
        torch.mm(x, w.t(), out=part)
        dist.reduce_scatter_tensor(red, part)
        torch.add(resid, red, out=out)

    ref_ms = time_ms(baseline, warmup, reps)
    flops, nbytes = tp_gemm_rs_work(M, N, K, tp)
    return dict(case="tp_gemm_rs", shape=f"M{M} N{N} K{K} tp{tp}", ms=ms, ref_ms=ref_ms, flops=flops,
                nvlink_bytes=nbytes)


def case_ep_combine(world, dev, T, H, warmup, reps) -> Dict:
    from ..ops._C import load
    from .symm import SymmetricBuffer

    symm = SymmetricBuffer(dist.group.WORLD, T * H * 4, dev)
    part = symm.tensor(torch.float32, T * H).view(T, H)
    part.normal_()
    x = torch.randn(T, H, device=dev)
    dst = torch.empty(T, H, device=dev)
    ext = load()

    def fused():
        ext.peer_sum(symm.ptrs, symm.signal_ptrs, symm.rank, x, dst, T * H, symm.counter)

    ms = time_ms(fused, warmup, reps)
    _check(dev)
    ref_part = part.clone()

    def nccl():
        red = ref_part.clone()
        dist.all_reduce(red)
        torch.add(x, red, out=dst)

    ref_ms = time_ms(nccl, warmup, reps)
    return dict(case="ep_combine", shape=f"T{T} H{H} ep{world}", ms=ms, ref_ms=ref_ms, flops=0.0,
                nvlink_bytes=ep_combine_bytes(T, H, world))


# -- report --------------------------------------------------------------------
def attach_roofline(rows: List[Dict], peaks=None) -> List[Dict]:
    peaks = peaks or load_peaks()
    for r in rows:
        tgt = fused_target_ms(r["flops"], r["nvlink_bytes"], peaks)
        r["target_ms"] = tgt
        r["frac"] = tgt / r["ms"] if r["ms"] > 0 else 0.0
        r["ref_frac"] = tgt / r["ref_ms"] if r["ref_ms"] > 0 else 0.0
        r["nvlink_gbs"] = r["nvlink_bytes"] / (r["ms"] * 1e-3) / 1e9 if r["ms"] > 0 else 0.0
        r["label"] = f"{peaks.label} (GEMM {peaks.bf16_tflops:.0f} TFLOP/s, NVLink {NVLINK_GBS:.0f} GB/s)"
    return rows


def table(rows: List[Dict]) -> str:
    out = ["| case | shape | fused ms | NCCL+cuBLAS ms | roofline ms | fused frac | baseline frac | NVLink GB/s |",
           "|---|---|---|---|---|---|---|---|"]
    for r in rows:
        out.append(f"| {r['case']} | {r['shape']} | {r['ms']:.3f} | {r['ref_ms']:.3f} | {r['target_ms']:.3f} | "
                   f"{r['frac']:.2f} | {r['ref_frac']:.2f} | {r['nvlink_gbs']:.0f} |")
    return "\n".join(out)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--cases", default="dp_reduce,tp_ag_gemm,tp_gemm_rs,ep_combine")
    ap.add_argument("--dp-elems", type=int, default=GPT2S_GRAD_ELEMS)
    ap.add_argument("--tokens", type=int, default=8192, help="M / T: tokens of one micro-batch (8 x 1024)")
    ap.add_argument("--hidden", type=int, default=1024, help="TP model width (GPT-2 medium)")
    ap.add_argument("--ep-hidden", type=int, default=768, help="MoE model width")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--json", default=None)
    args = ap.parse_args(argv)

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()
    rows: List[Dict] = []
    try:
        if world < 2:
            if rank == 0:
                print("commbench needs 2 or more ranks (torchrun --nproc-per-node N)")
            return
        M, H = args.tokens, args.hidden
        for c in args.cases.split(","):
            if c == "dp_reduce":
                rows.append(case_dp_reduce(world, dev, args.dp_elems, args.warmup, args.reps))
            elif c == "tp_ag_gemm":
                rows.append(case_tp_ag_gemm(world, dev, M, 3 * H, H, args.warmup, args.reps))  # QKV
                rows.append(case_tp_ag_gemm(world, dev, M, 4 * H, H, args.warmup, args.reps))  # MLP up
            elif c == "tp_gemm_rs":
                rows.append(case_tp_gemm_rs(world, dev, M, H, H, args.warmup, args.reps))  # attention out
                rows.append(case_tp_gemm_rs(world, dev, M, H, 4 * H, args.warmup, args.reps))  # MLP down
            elif c == "ep_combine":
                rows.append(case_ep_combine(world, dev, M, args.ep_hidden, args.warmup, args.reps))
            else:
                raise SystemExit(f"unknown case {c}")
        attach_roofline(rows)
        if rank == 0:
            for r in rows:
                print(json.dumps(r))
            print(table(rows))
            if args.json:
                with open(args.json, "w") as f:
                    json.dump(rows, f, indent=1)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
