"""LayerNorm backward with the residual-gradient loads batched ahead of the
stores (the default; HB_LN_BWD_HOIST=0 selects the plain order) gives
bit-identical outputs to the plain ordering, in place (dres aliasing dres_in) and out of place, at the model's
widths. The switch is read once per process, so each setting runs in a child
process that writes its outputs to a file."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from heiretsu_b200.ops import kernels as K
from heiretsu_b200.ops._C import check_status
out = {}
for M, H in ((8192, 768), (4096, 1024), (2048, 1280), (333, 256)):
    g = torch.Generator(device="cuda").manual_seed(M + H)
    x = torch.randn(M, H, device="cuda", generator=g) * 2 + 0.5
    w = torch.randn(H, device="cuda", generator=g)
    b = torch.randn(H, device="cuda", generator=g)
    _, mean, rstd = K.layernorm_fwd(x, w, b)
    dy = torch.randn(M, H, device="cuda", generator=g)
    dres_in = torch.randn(M, H, device="cuda", generator=g)
    for inplace in (False, True):
        dres = dres_in.clone() if inplace else torch.empty_like(dres_in)
        src = dres if inplace else dres_in
        d16 = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
        dg, db = torch.zeros(H, device="cuda"), torch.zeros(H, device="cuda")
        K.layernorm_bwd(dy, x, mean, rstd, w, src, dres, d16, dg, db)
        out[(M, H, inplace)] = (dres.cpu(), d16.cpu(), dg.cpu(), db.cpu())
torch.cuda.synchronize()
check_status()
torch.save(out, sys.argv[2])
"""


def test_hoisted_ln_backward_is_bit_identical(tmp_path):
    res = {}
    for flag in ("0", "1"):
        path = tmp_path / f"ln_{flag}.pt"
        r = subprocess.run([sys.executable, "-c", CHILD, ROOT, str(path)], capture_output=True, text=True,
                           timeout=300, env=dict(os.environ, HB_LN_BWD_HOIST=flag))
        assert r.returncode == 0, r.stderr[-3000:]
        res[flag] = torch.load(path)
    for key, ref in res["0"].items():
        for a, b in zip(ref, res["1"][key]):
            assert torch.equal(a, b), key
