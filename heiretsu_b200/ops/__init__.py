"""sm_100a kernels (GEMM, attention, LayerNorm, cross-entropy, embedding, AdamW, comm)."""
