"""Top-level alias of :mod:`heiretsu_b200.topo` (same import path as the reference's topo.py)."""
from heiretsu_b200.topo import (Topology, build_groups, cleanup, coords_from_rank, group_members,  # noqa: F401
                                init_topology, rank_from_coords)
