"""heiretsu_b200: a 4-D parallel (DP x EP x TP x PP) GPT training framework for NVIDIA B200.

PyTorch is the framework layer (tensors, autograd, torch.distributed
bootstrap); the hot ops are hand-written sm_100a kernels in the native
extension ``heiretsu_b200._C`` (built in-tree by ``python setup.py build_ext --inplace``).
"""
from .config import GPTConfig, MoEConfig, make_moe_config  # noqa: F401
from .topo import Topology, coords_from_rank, init_topology, rank_from_coords  # noqa: F401

__version__ = "0.1.0"
