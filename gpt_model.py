"""Top-level alias of the GPT model (same import path as the reference's gpt_model.py).

Scripts written against the reference (``from gpt_model import GPT, GPTConfig``)
get this framework's modules, with the same class names and state_dict keys."""
from heiretsu_b200.config import GPTConfig  # noqa: F401
from heiretsu_b200.models.gpt import GPT, AttentionTP, BlockMoE, BlockTP, MLPTP, make_block  # noqa: F401
