"""Model definitions (GPT-2 with optional MoE blocks)."""
