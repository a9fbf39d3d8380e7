"""Parallelism: tensor (tp), data (dp), expert (ep) and pipeline (pp)."""
