"""Model configuration dataclasses.

Field names, defaults and order match the reference so that checkpoints'
``cfg`` dicts round-trip (reference: gpt_model.py:18-30, moe.py:24-31,
moe.py:408-422).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class GPTConfig:
    block_size: int = 1024
    vocab_size: int = 50257  # GPT-2 vocabulary
    n_layer: int = 12
    n_head: int = 12
    n_embed: int = 768
    dropout: float = 0.0
    # MoE
    num_experts: int = 0  # 0 = dense model
    top_k: int = 2
    moe_freq: int = 2  # MoE every N-th block (0 = all dense)
    aux_loss_coef: float = 0.01

    def is_moe_layer(self, layer_idx: int) -> bool:
        """Block i is MoE iff (i + 1) % moe_freq == 0 (reference gpt_model.py:184-188)."""
        return self.num_experts > 0 and self.moe_freq > 0 and (layer_idx + 1) % self.moe_freq == 0


@dataclass
class MoEConfig:
    num_experts: int = 8
    top_k: int = 2
    hidden_size: int = 768
    intermediate_size: int = 3072
    aux_loss_coef: float = 0.01


def make_moe_config(hidden_size: int, num_experts: int = 8, top_k: int = 2, intermediate_mult: int = 4,
                    aux_loss_coef: float = 0.01) -> MoEConfig:
    return MoEConfig(num_experts=num_experts, top_k=top_k, hidden_size=hidden_size,
                     intermediate_size=hidden_size * intermediate_mult, aux_loss_coef=aux_loss_coef)
