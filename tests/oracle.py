"""Load the unmodified reference implementation as a test oracle.

The reference modules use generic top-level names (topo, dp, moe, ...) and
import each other lazily by those names (e.g. ``from moe import Expert``
inside ``GPT._init_weights``), so they stay registered in ``sys.modules``
under their own names. heiretsu_b200 never imports those top-level names.
"""
from __future__ import annotations

import importlib
import os
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The installed reference (pip --target baseline/_ref), else a checkout named by
# HB_REFERENCE_DIR.
CANDIDATES = [os.path.join(ROOT, "baseline", "_ref")] + (
    [os.environ["HB_REFERENCE_DIR"]] if os.environ.get("HB_REFERENCE_DIR") else [])
NAMES = ["topo", "dp", "ep_comm", "tp_linear", "moe", "gpt_model", "pipeline"]

_cache = None


def ref_dir():
    for d in CANDIDATES:
        if os.path.exists(os.path.join(d, "gpt_model.py")):
            return d
    return None


def load_reference() -> types.SimpleNamespace:
    global _cache
    if _cache is not None:
        return _cache
    d = ref_dir()
    if d is None:
        raise ImportError("reference implementation not found")
    for n in NAMES:
        m = sys.modules.get(n)
        if m is not None and not os.path.abspath(getattr(m, "__file__", "")).startswith(os.path.abspath(d)):
            del sys.modules[n]
    sys.path.insert(0, d)
    try:
        mods = {n: importlib.import_module(n) for n in NAMES}
    finally:
        sys.path.remove(d)
    _cache = types.SimpleNamespace(**mods)
    return _cache


def have_reference() -> bool:
    try:
        load_reference()
        return True
    except Exception:
        return False
