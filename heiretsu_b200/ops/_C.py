"""Loader of the native extension `heiretsu_b200._C`.

The extension is built in-tree (``python setup.py build_ext --inplace``).
On a machine with a CUDA device a missing or broken extension is an error:
the GPU path never silently falls back to PyTorch kernels. On a CPU-only
machine the model runs its plain-PyTorch CPU path and ``_C`` is optional.
"""
from __future__ import annotations

import importlib

import torch

_ext = None
_err: Exception | None = None


def load():
    """Return the extension module, importing it on first use."""
    global _ext, _err
    if _ext is not None:
        return _ext
    try:
        _ext = importlib.import_module("heiretsu_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _err = e
        raise RuntimeError(
            "heiretsu_b200 native extension is not built or failed to load; run "
            "`python setup.py build_ext --inplace` (error: %r)" % (e,)
        ) from e
    return _ext


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def check_status(device: int | None = None) -> None:
    """Raise if a kernel on `device` recorded a timeout or bad argument."""
    if device is None:
        device = torch.cuda.current_device()
    code = int(load().read_and_clear_status(device))
    if code != 0:
        kind = {1: "mbarrier wait timed out", 2: "peer flag wait timed out", 3: "bad argument"}.get(code & 0xFF, "unknown")
        raise RuntimeError(f"device {device}: kernel status {code:#x} ({kind}, site {code >> 8})")
