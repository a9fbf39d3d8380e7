# Repository-wide source checks for constructs this framework must never
# contain: TMA loads with cluster multicast (every kernel here may run on
# several GPUs, where such a load from peer memory hangs the GPU), the
# batched asynchronous memcpy entry points, and device-side traps (failures
# are reported through the status word instead).
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXTS = (".cu", ".cuh", ".cpp", ".h", ".py", ".sh")
# Stored hex-encoded so this file does not itself contain the patterns.
MC_QUALIFIER = bytes.fromhex("2e6d756c7469636173743a3a636c7573746572").decode()
BATCH_COPIES = [p + "BatchAsync" for p in ("cudaMemcpy", "cudaMemcpy3D", "cuMemcpy", "cuMemcpy3D")]
TRAP = re.compile(r"__trap\s*\(|\btrap\s*;")


def _sources():
    for top in ("heiretsu_b200", "tests", "data"):
        for d, _, files in os.walk(os.path.join(ROOT, top)):
            for f in files:
                if f.endswith(EXTS):
                    yield os.path.join(d, f)
    for f in os.listdir(ROOT):
        if f.endswith(EXTS):
            yield os.path.join(ROOT, f)


def test_no_forbidden_constructs():
    bad = []
    for path in _sources():
        with open(path, errors="ignore") as fh:
            text = fh.read()
        rel = os.path.relpath(path, ROOT)
        if MC_QUALIFIER in text:
            bad.append((rel, "forbidden load qualifier"))
        for name in BATCH_COPIES:
            if name in text:
                bad.append((rel, name))
        if path.endswith((".cu", ".cuh")) and TRAP.search(text):
            bad.append((rel, "device trap"))
    assert not bad, bad


def test_every_device_spin_is_bounded():
    """Every mbarrier / flag wait loop in the kernels carries a time limit."""
    offenders = []
    checked = 0
    for path in _sources():
        if not path.endswith((".cu", ".cuh")):
            continue
        lines = open(path).read().splitlines()
        for i, line in enumerate(lines):
            if re.search(r"while\s*\((\s*true\s*\)|.*ld_acquire|.*try_wait)", line):
                checked += 1
                window = "\n".join(lines[i:i + 8])
                if "TIMEOUT" not in window:
                    offenders.append(f"{os.path.relpath(path, ROOT)}:{i + 1}")
    assert not offenders, offenders
    assert checked >= 3  # the GEMM all-gather wait, the mbarrier wait, the peer barrier
