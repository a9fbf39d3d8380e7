"""Top-level alias of the expert-parallel token exchange (same import path as the
reference's ep_comm.py; here dispatch and combine are differentiable)."""
from heiretsu_b200.parallel.ep import all_to_all_combine, all_to_all_dispatch, compute_ep_send_counts  # noqa: F401
