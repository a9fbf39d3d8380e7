"""Top-level alias of GPipe pipeline parallelism (same import path as the reference's pipeline.py)."""
from heiretsu_b200.parallel.pipeline import (GPipeEngine, PipelineState, StageModule,  # noqa: F401
                                             TiedEmbeddings, _partition_layers)
