"""Top-level alias of data-parallel gradient averaging (same import path as the reference's dp.py)."""
from heiretsu_b200.parallel.dp import average_gradients  # noqa: F401
