"""Top-level alias of the MoE layer (same import path as the reference's moe.py)."""
from heiretsu_b200.config import MoEConfig, make_moe_config  # noqa: F401
from heiretsu_b200.models.moe import Expert, ExpertGroup, MoELayer, Router, load_balancing_loss  # noqa: F401
