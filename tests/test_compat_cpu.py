"""Drop-in compatibility: the reference's own test scripts, unmodified, run on this
framework's top-level modules (gpt_model, tp_linear, moe, ep_comm, dp, pipeline,
topo) and on the reference's, as gloo CPU ranks under torchrun. Their printed
results (logit and gradient differences against a single-model baseline, losses
of short training runs) must be the same lines; where they differ by design
(expert-parallel gradients, which the reference cuts: its ep_comm.py
all-to-alls are not differentiable) ours must be the ones that match the
baseline. The scripts are read from the reference checkout; absent that, the
tests skip."""
import os
import re
import shutil
import socket
import subprocess
import sys

import pytest

from oracle import ref_dir

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The reference's test scripts: copied next to the installed reference
# (baseline/_ref/reference_tests) when it was installed, or the tests/ folder of a
# checkout named by HB_REFERENCE_DIR.
_REF_TEST_DIRS = [os.path.join(ROOT, "baseline", "_ref", "reference_tests")]
if os.environ.get("HB_REFERENCE_DIR"):
    _REF_TEST_DIRS.append(os.path.join(os.environ["HB_REFERENCE_DIR"], "tests"))
REF_TESTS = next((d for d in _REF_TEST_DIRS if os.path.isdir(d)), "")

pytestmark = pytest.mark.skipif(not os.path.isdir(REF_TESTS) or ref_dir() is None,
                                reason="reference checkout not available")


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _launch(tmp, impl_dir, tag, script, nproc, args):
    """Start `script` (a copy under tmp/tag/tests/, so its own sys.path insert of the
    parent directory finds no modules) with `impl_dir` on PYTHONPATH."""
    d = os.path.join(tmp, tag, "tests")
    os.makedirs(d, exist_ok=True)
    dst = os.path.join(d, script)
    shutil.copy(os.path.join(REF_TESTS, script), dst)
    env = dict(os.environ, PYTHONPATH=impl_dir, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr", "127.0.0.1", f"--master-port={_port()}", dst] + list(args)
    return subprocess.Popen(cmd, cwd=tmp, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)


_NOISE = re.compile(r"^(\*+|Setting OMP_NUM_THREADS.*|.*[Ww]arning.*|\s*warnings\.warn.*|)$")


def _result(p):
    out, _ = p.communicate(timeout=600)
    assert p.returncode == 0, out[-3000:]
    return [l for l in out.splitlines() if not _NOISE.match(l)]


def _both(tmp_path, script, nproc, args):
    ours = _launch(str(tmp_path), ROOT, "ours", script, nproc, args)
    ref = _launch(str(tmp_path), ref_dir(), "ref", script, nproc, args)
    return _result(ours), _result(ref)


CASES = [
    ("tests_equiv.py", 2, ["--tp", "2"]),
    ("parallel_sanity.py", 2, ["--backend", "gloo", "--dp", "2"]),
    ("parallel_sanity.py", 2, ["--backend", "gloo", "--tp", "2"]),
    ("parallel_sanity.py", 2, ["--backend", "gloo", "--pp", "2"]),
    ("parallel_sanity.py", 2, ["--backend", "gloo", "--ep", "2", "--num_experts", "4"]),
    ("parallel_sanity.py", 4, ["--backend", "gloo", "--tp", "2", "--pp", "2"]),
    ("grad_parity.py", 2, ["--backend", "gloo", "--tp", "2"]),
    ("grad_parity.py", 2, ["--backend", "gloo", "--pp", "2"]),
    ("boundary_push.py", 4, ["--backend", "gloo", "--dp", "2", "--tp", "2", "--steps", "2", "--micro_batches", "2"]),
    ("boundary_push.py", 2, ["--backend", "gloo", "--pp", "2", "--steps", "2", "--micro_batches", "2"]),
    # the 4-rank dense layouts of the reference's own suite (tests/run_full_suite.sh:35-42)
    ("parallel_sanity.py", 4, ["--backend", "gloo", "--dp", "4"]),
    ("parallel_sanity.py", 4, ["--backend", "gloo", "--tp", "4"]),
    ("parallel_sanity.py", 4, ["--backend", "gloo", "--pp", "4"]),
    ("parallel_sanity.py", 4, ["--backend", "gloo", "--dp", "2", "--pp", "2"]),
    ("grad_parity.py", 4, ["--backend", "gloo", "--dp", "2", "--tp", "2"]),
]


@pytest.mark.parametrize("script,nproc,args", CASES, ids=[f"{c[0]}:{' '.join(c[2])}" for c in CASES])
def test_reference_script_prints_the_same(tmp_path, script, nproc, args):
    ours, ref = _both(tmp_path, script, nproc, args)
    assert ours, "no output"
    assert ours == ref


def test_reference_grad_parity_with_expert_parallelism(tmp_path):
    """grad_parity.py --ep 2: the reference's gradients miss the single-model baseline (its
    all-to-alls cut autograd through the experts); ours match it."""
    ours, ref = _both(tmp_path, "grad_parity.py", 2, ["--backend", "gloo", "--ep", "2", "--num_experts", "4"])

    def worst(lines):
        vals = [float(m.group(1)) for l in lines for m in [re.search(r"GRAD_DIFF \S+ max=(\S+)", l)] if m]
        assert vals, lines
        return max(vals)

    assert worst(ours) < 1e-3 < 1e-2 < worst(ref), (ours, ref)


def test_reference_moe_unit_tests_pass_on_our_modules(tmp_path):
    d = tmp_path / "tests"
    d.mkdir()
    shutil.copy(os.path.join(REF_TESTS, "test_moe.py"), d / "test_moe.py")
    env = dict(os.environ, PYTHONPATH=ROOT, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES="")
    p = subprocess.run([sys.executable, str(d / "test_moe.py")], cwd=str(tmp_path), env=env, capture_output=True,
                       text=True, timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert "All MoE tests passed" in p.stdout
