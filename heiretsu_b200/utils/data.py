"""Token data loaders.

* ``RandomBatchLoader`` reads GPT-2 token shards (flat uint16 files
  ``fineweb_{split}_%06d.bin``) exactly like the reference (train.py:33-118):
  DP-sharded file list ``files[dp_rank::dp_size]``, file chosen with
  probability proportional to its number of valid start positions, random
  crop of T+1 tokens, x = crop[:-1], y = crop[1:], Python ``random.Random``
  seeded with ``seed + rank`` — so the same seed yields the same batches.
  Batches are assembled in pinned host memory and copied asynchronously.
* ``SyntheticLoader`` draws uniform token ids in [0, vocab) from a seeded
  generator into pinned host memory (benchmarks; no dataset needed).
* ``write_synthetic_bins`` writes uniform-random shards in the reference's
  on-disk format, so the reference trainer can run on the same data.
"""
from __future__ import annotations

import glob
import os
import random
from typing import List, Optional, Tuple

import numpy as np
import torch


def list_split_bins(data_dir: str, split: str, num_chunks: Optional[int]) -> List[str]:
    pattern = os.path.join(data_dir, f"fineweb_{split}_*.bin")
    files = sorted(glob.glob(pattern))
    if not files:
        raise FileNotFoundError(f"No {split} .bin files found under {data_dir} (looked for {pattern}).")
    return files[:num_chunks] if num_chunks is not None else files


class BinChunkSampler:
    """uint16 memmaps plus weighted file choice by available start positions."""

    def __init__(self, files: List[str], T: int):
        self.T = T
        self.arrs = [np.memmap(f, dtype=np.uint16, mode="r") for f in files]
        self.lengths = [int(a.shape[0]) for a in self.arrs]
        self.starts_cap = [max(0, L - (T + 1)) for L in self.lengths]
        self.total_cap = sum(self.starts_cap)
        if self.total_cap <= 0:
            raise ValueError("No valid start positions across files (increase T or use larger files).")
        self.cum_caps = np.cumsum(self.starts_cap)

    def _sample_file_index_with_rng(self, rng: random.Random) -> int:
        return int(np.searchsorted(self.cum_caps, rng.randrange(self.total_cap), side="right"))


class RandomBatchLoader:
    def __init__(self, data_dir, split, B, T, num_chunks, seed=1337, rank=0, dp_rank=0, dp_size=1, log_rank=None,
                 pin_memory: bool = True):
        files_all = list_split_bins(data_dir, split, num_chunks)
        files = files_all[dp_rank::dp_size] if dp_size > 1 else files_all
        if not files:
            raise FileNotFoundError(f"No {split} files assigned to dp_rank={dp_rank} out of {len(files_all)} total.")
        self.sampler = BinChunkSampler(files, T)
        self.B, self.T = B, T
        self.rng = random.Random(seed + rank)
        self.pin = pin_memory and torch.cuda.is_available()
        if (rank if log_rank is None else log_rank) == 0:
            print(f"[{split}] dp_shard={dp_rank}/{dp_size} files={len(files)} "
                  f"tokens={sum(self.sampler.lengths):,} T={T}")

    def next_batch_host(self) -> Tuple[torch.Tensor, torch.Tensor]:
        buf = np.empty((self.B, self.T + 1), dtype=np.int64)
        for i in range(self.B):
            fi = self.sampler._sample_file_index_with_rng(self.rng)
            L = self.sampler.lengths[fi]
            start = self.rng.randint(0, L - (self.T + 1))
            buf[i] = self.sampler.arrs[fi][start:start + self.T + 1]
        t = torch.from_numpy(buf)
        x, y = t[:, :-1].contiguous(), t[:, 1:].contiguous()
        if self.pin:
            x, y = x.pin_memory(), y.pin_memory()
        return x, y

    def next_batch(self, device):
        x, y = self.next_batch_host()
        nb = self.pin and torch.device(device).type == "cuda"
        return x.to(device, non_blocking=nb), y.to(device, non_blocking=nb)

    # data position for exact resume (the state of the sampling RNG)
    def state_dict(self) -> dict:
        return {"rng": self.rng.getstate()}

    def load_state_dict(self, sd: dict) -> None:
        self.rng.setstate(sd["rng"])


class SyntheticLoader:
    """Uniform-random token ids; y is x shifted by one within a (T+1)-token draw.

    Host batches are drawn into a small ring of preallocated pinned buffers and
    copied to the device asynchronously on the current stream; a slot is
    reused only after the event recorded behind its previous copy completed.
    """

    def __init__(self, B: int, T: int, vocab_size: int, seed: int = 1337, rank: int = 0, pin_memory: bool = True,
                 ring: int = 4):
        self.B, self.T, self.V = B, T, vocab_size
        self.gen = torch.Generator().manual_seed(seed + rank)
        self.pin = pin_memory and torch.cuda.is_available()
        self._ring = [torch.empty(2, B, T, dtype=torch.int64, pin_memory=self.pin) for _ in range(ring)]
        self._events = [None] * ring
        self._i = 0
        self.h2d_bytes = 2 * B * T * 8

    def next_batch_host(self):
        buf = torch.randint(0, self.V, (self.B, self.T + 1), generator=self.gen, dtype=torch.int64)
        return buf[:, :-1].contiguous(), buf[:, 1:].contiguous()

    def next_batch(self, device):
        dev = torch.device(device)
        buf = torch.randint(0, self.V, (self.B, self.T + 1), generator=self.gen, dtype=torch.int64)
        if dev.type != "cuda":
            return buf[:, :-1].contiguous(), buf[:, 1:].contiguous()
        slot = self._i % len(self._ring)
        self._i += 1
        if self._events[slot] is not None:
            self._events[slot].synchronize()
        host = self._ring[slot]
        host[0].copy_(buf[:, :-1])
        host[1].copy_(buf[:, 1:])
        dev_xy = host.to(dev, non_blocking=self.pin)
        ev = torch.cuda.Event()
        ev.record()
        self._events[slot] = ev
        return dev_xy[0], dev_xy[1]

    def state_dict(self) -> dict:
        return {"gen": self.gen.get_state()}

    def load_state_dict(self, sd: dict) -> None:
        self.gen.set_state(sd["gen"])


def write_synthetic_bins(data_dir: str, vocab_size: int = 50257, train_tokens: int = 8_000_000,
                         val_tokens: int = 2_000_000, seed: int = 0, num_train: int = 1) -> None:
    """Uniform-random uint16 shards in the reference's format (no header)."""
    os.makedirs(data_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    for i in range(1, num_train + 1):
        rng.integers(0, vocab_size, size=train_tokens, dtype=np.uint16).tofile(
            os.path.join(data_dir, f"fineweb_train_{i:06d}.bin"))
    rng.integers(0, vocab_size, size=val_tokens, dtype=np.uint16).tofile(
        os.path.join(data_dir, "fineweb_val_000000.bin"))
