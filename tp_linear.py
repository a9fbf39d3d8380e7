"""Top-level alias of the tensor-parallel linears (same import path and names as the
reference's tp_linear.py)."""
from heiretsu_b200.parallel.tp import (ColumnParallelLinear, ColumnParallelLinearQKV,  # noqa: F401
                                       RowParallelLinear, copy_to_model_parallel_region,
                                       reduce_from_model_parallel_region)
from heiretsu_b200.parallel.tp import _CopyToTP as _CopyToModelParallelRegion  # noqa: F401
from heiretsu_b200.parallel.tp import _ReduceFromTP as _ReduceFromModelParallelRegion  # noqa: F401
from heiretsu_b200.parallel.tp import _rk as _tp_rank  # noqa: F401
from heiretsu_b200.parallel.tp import _split_last_dim as _split
from heiretsu_b200.parallel.tp import _ws as _tp_world_size  # noqa: F401


def _split_last_dim(x, tp_size):
    """(..., tp_size*d) -> (tp_size, ..., d)."""
    return _split(x, tp_size)
