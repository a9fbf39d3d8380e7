"""The HB_DEBUG variant of the checked kernels compiles for sm_100a (nvcc
cross-compiles without a GPU)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "heiretsu_b200", "csrc")


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not available")
@pytest.mark.parametrize("src", ["moe.cu", "comm.cu"])
def test_debug_checks_compile(src, tmp_path):
    out = tmp_path / (src + ".o")
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O1", "--expt-relaxed-constexpr",
           "-DHB_DEBUG", "-I", CSRC, "-c", os.path.join(CSRC, src), "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    assert out.stat().st_size > 0
