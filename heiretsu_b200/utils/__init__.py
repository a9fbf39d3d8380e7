"""Data loading, checkpoints, timing and logging helpers."""
