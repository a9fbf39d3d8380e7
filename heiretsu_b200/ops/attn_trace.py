"""Phase traces of the head_dim-64 causal attention kernels.

With a trace buffer set (``attention_set_trace``), every CTA of the attention
kernels stamps ``%globaltimer`` (ns) at its pipeline hand-offs into its own
row of an int64 [grid, 80] array. This module captures one forward and one
backward launch on the GPT-2 small shape and reduces the stamps to per-tile
phase durations, which is how the softmax / tensor-core overlap of these
kernels is measured (an ncu capture gives totals, not the order of events).

Slots (csrc/attention.cu documents the same layout at the kernels):

forward, CTA = pair of query tiles; g = query tile of the pair, j = key tile (< 8)
    0 start, 1 Q tiles loaded (MMA warp), 2 end
    8 + 24g + j   S_j ready for the softmax warpgroup of tile g
    16 + 24g + j  softmax start
    56 + 8g + j   row max done
    24 + 24g + j  P_j stored (hand-over to the PV MMA)
backward, CTA = key tile; g = query half, i = query tile (< 8)
    0 start, 1 K/V and the first Q/dO loaded, 2 end
    8 + i / 16 + i  P^T / dS^T half 0 / half 1 taken by the MMA warp
    24 + 24g + i  S^T / dP^T half ready
    32 + 24g + i  previous tile's MMAs complete (P^T / dS^T smem free)
    40 + 24g + i  P^T / dS^T half stored

    python -m heiretsu_b200.ops.attn_trace [--json report.json] [--npy-dir DIR]
"""
from __future__ import annotations

import argparse
import json
from typing import Dict, List

import numpy as np

SLOTS = 80


def _mean(x: np.ndarray) -> float:
    return float(x.mean()) if x.size else float("nan")


def _span(t: np.ndarray) -> Dict[str, float]:
    live = t[t[:, 0] != 0]
    t0 = live[:, 0].min()
    return {"ctas": int(live.shape[0]), "span_us": float((live[:, 2].max() - t0) / 1e3),
            "mean_cta_us": float((live[:, 2] - live[:, 0]).mean() / 1e3),
            "first_load_ns": _mean((live[:, 1] - live[:, 0]).astype(np.float64))}


def forward_report(trace: np.ndarray) -> Dict[str, object]:
    """Per (query tile g, key tile j) means over the CTAs that reached the step:
    softmax = S ready -> P stored; max_pass = softmax start -> row max done;
    turnaround = P stored -> next S ready (the S MMA round trip)."""
    t = trace.astype(np.int64)
    t = t[t[:, 0] != 0]
    rows: List[Dict[str, float]] = []
    for g in (0, 1):
        for j in range(8):
            s_ready, start, p_done = t[:, 8 + 24 * g + j], t[:, 16 + 24 * g + j], t[:, 24 + 24 * g + j]
            mx = t[:, 56 + 8 * g + j]
            ok = (s_ready > 0) & (p_done > 0)
            if not ok.any():
                continue
            row = {"g": g, "j": j, "ctas": int(ok.sum()), "softmax_ns": _mean((p_done - s_ready)[ok])}
            okm = ok & (mx > 0) & (start > 0)
            row["max_pass_ns"] = _mean((mx - start)[okm])
            if j < 7:
                nxt = t[:, 8 + 24 * g + j + 1]
                okn = ok & (nxt > 0)
                row["turnaround_ns"] = _mean((nxt - p_done)[okn])
            rows.append(row)
    return {"kernel": "attn_fwd", **_span(t), "tiles": rows}


def backward_report(trace: np.ndarray) -> Dict[str, object]:
    """Per (query half g, query tile i): softmax = S^T/dP^T ready -> P^T/dS^T
    stored, of which wait_prev_mma = ready -> previous tile's MMAs complete;
    turnaround = stored -> next tile's half ready."""
    t = trace.astype(np.int64)
    t = t[t[:, 0] != 0]
    rows: List[Dict[str, float]] = []
    for g in (0, 1):
        for i in range(8):
            ready, prev, done = t[:, 24 + 24 * g + i], t[:, 32 + 24 * g + i], t[:, 40 + 24 * g + i]
            ok = (ready > 0) & (done > 0)
            if not ok.any():
                continue
            row = {"g": g, "i": i, "ctas": int(ok.sum()), "softmax_ns": _mean((done - ready)[ok])}
            okp = ok & (prev > 0)
            row["wait_prev_mma_ns"] = _mean((prev - ready)[okp])
            if i < 7:
                nxt = t[:, 24 + 24 * g + i + 1]
                okn = ok & (nxt > 0)
                row["turnaround_ns"] = _mean((nxt - done)[okn])
            rows.append(row)
    return {"kernel": "attn_bwd", **_span(t), "tiles": rows}


def _print(rep: Dict[str, object]) -> None:
    print(f"{rep['kernel']}: {rep['ctas']} CTAs, span {rep['span_us']:.1f} us, mean CTA {rep['mean_cta_us']:.2f} us, "
          f"first loads {rep['first_load_ns']:.0f} ns")
    for r in rep["tiles"]:
        idx = f"g{r['g']} {'j' if 'j' in r else 'i'}{r.get('j', r.get('i'))}"
        extra = "  ".join(f"{k[:-3]} {v:6.0f}" for k, v in r.items() if k.endswith("_ns") and k != "softmax_ns")
        print(f"  {idx}: {r['ctas']:4d} CTAs  softmax {r['softmax_ns']:6.0f}  {extra}  (ns)")


def capture(B: int = 8, T: int = 1024, nh: int = 12, dh: int = 64, seed: int = 0):
    """One traced forward and one traced backward launch; returns (fwd, bwd) int64 arrays."""
    import torch

    from . import kernels as K
    from ._C import load

    ext = load()
    torch.manual_seed(seed)
    qkv = (torch.randn(B * T, 3 * nh * dh, device="cuda") * 0.5).bfloat16()
    y, lse = K.attention_fwd(qkv, B, T, nh, head_dim=dh)
    dy = torch.randn_like(y)
    for _ in range(3):  # warm-up
        K.attention_fwd(qkv, B, T, nh, out=y, head_dim=dh)
        K.attention_bwd(qkv, y, dy, lse, B, T, nh, head_dim=dh)
    torch.cuda.synchronize()
    out = []
    for kind in ("fwd", "bwd"):
        tr = torch.zeros(4096, SLOTS, dtype=torch.int64, device="cuda")
        ext.attention_set_trace(tr)
        try:
            if kind == "fwd":
                K.attention_fwd(qkv, B, T, nh, out=y, head_dim=dh)
            else:
                K.attention_bwd(qkv, y, dy, lse, B, T, nh, head_dim=dh)
            torch.cuda.synchronize()
        finally:
            ext.attention_set_trace(None)
        out.append(tr.cpu().numpy())
    return out[0], out[1]


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--json", default=None, help="write both reports here")
    ap.add_argument("--npy-dir", default=None, help="also save the raw stamps (attn_trace_{fwd,bwd}.npy)")
    args = ap.parse_args(argv)
    fwd, bwd = capture()
    reps = [forward_report(fwd), backward_report(bwd)]
    for r in reps:
        _print(r)
    if args.npy_dir:
        np.save(f"{args.npy_dir}/attn_trace_fwd.npy", fwd)
        np.save(f"{args.npy_dir}/attn_trace_bwd.npy", bwd)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(reps, f, indent=1)


if __name__ == "__main__":
    main()
