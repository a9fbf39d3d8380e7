"""Roofline fractions of the measured hardware peaks.

    python -m heiretsu_b200.ops.microbench --json mb.json
    python -m heiretsu_b200.utils.roofline mb.json

Denominators come from ``MEASURED_PEAKS.json`` at the repository root when
it exists (a STREAM-style copy ``hbm_gbs`` and a cuBLAS bf16 GEMM,
``bf16_tflops`` as a burst and ``bf16_tflops_sustained`` under the power
cap), else from fallback figures measured earlier on the same kind of GPU.
The label ("of measured" / "of fallback") travels with every fraction.
A fused compute + collective path is bounded by the slower of its math and
its NVLink traffic: target = max(FLOPs / GEMM peak, bytes / link bandwidth).
"""
from __future__ import annotations

import argparse
import json
import os
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


@dataclass
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    label: str  # "of measured" | "of fallback"


def load_peaks(path: Optional[str] = None) -> Peaks:
    path = path or os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)

        def pick(key: str) -> float:
            v = d.get(key)
            if isinstance(v, dict):  # tolerate {"value": ...} entries
                v = v.get("value")
            return float(v) if v is not None else FALLBACK[key]

        return Peaks(pick("hbm_gbs"), pick("bf16_tflops"), pick("bf16_tflops_sustained"), "of measured")
    return Peaks(FALLBACK["hbm_gbs"], FALLBACK["bf16_tflops"], FALLBACK["bf16_tflops_sustained"], "of fallback")


def fused_target_ms(flops: float, nvlink_bytes: float, peaks: Peaks) -> float:
    """Roofline time of a fused compute + collective step (ms)."""
    return max(flops / (peaks.bf16_tflops * 1e12), nvlink_bytes / (NVLINK_GBS * 1e9)) * 1e3


def fractions(rows: Iterable[Dict], peaks: Peaks) -> List[Dict]:
    """Attach ``frac`` (achieved / peak) to microbench rows (GEMM / attention by
    TFLOP/s, memory-bound ops by GB/s)."""
    out = []
    for r in rows:
        r = dict(r)
        if "tflops" in r:
            r["frac"] = r["tflops"] / peaks.bf16_tflops
            if r.get("ref_tflops"):
                r["ref_frac"] = r["ref_tflops"] / peaks.bf16_tflops
        elif "gbs" in r:
            r["frac"] = r["gbs"] / peaks.hbm_gbs
        r["peak"] = peaks.label
        out.append(r)
    return out


def render(rows: List[Dict]) -> str:
    lines = ["| op | case | ms | achieved | fraction | torch / cuBLAS fraction |", "|---|---|---|---|---|---|"]
    for r in rows:
        ach = f"{r['tflops']:.0f} TFLOP/s" if "tflops" in r else (f"{r['gbs']:.0f} GB/s" if "gbs" in r else "")
        frac = f"{100 * r['frac']:.0f}% {r['peak']}" if "frac" in r else ""
        ref = f"{100 * r['ref_frac']:.0f}%" if "ref_frac" in r else ""
        lines.append(f"| {r.get('op', '')} | {r.get('name', '')} | {r.get('ms', 0):.4f} | {ach} | {frac} | {ref} |")
    return "\n".join(lines)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("microbench_json")
    ap.add_argument("--peaks", default=None)
    args = ap.parse_args(argv)
    with open(args.microbench_json) as f:
        rows = json.load(f)
    print(render(fractions(rows, load_peaks(args.peaks))))


if __name__ == "__main__":
    main()
