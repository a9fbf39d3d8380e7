"""Token data loaders.

Both loaders hand out (x, y) batches of int64 token ids, y being x shifted by
one position, staged in a small ring of pinned host buffers and copied to the
device asynchronously on the current stream (``_PinnedStaging``).

* ``RandomBatchLoader`` serves random (T+1)-token windows of GPT-2 token shards
  (headerless uint16 files ``fineweb_{split}_NNNNNN.bin``). A DP rank owns every
  dp_size-th shard, starting at its own dp_rank. Each window is drawn in two
  steps from a ``random.Random(seed + rank)``: a shard, with probability
  proportional to its count of full windows, then a start offset inside it.
  That call sequence is what the reference trainer's loader does
  (reference train.py:33-118), so a given seed yields the reference's batches
  token for token; the checkpointed RNG state resumes it exactly.
* ``SyntheticLoader`` draws uniform token ids in [0, vocab) from a seeded
  generator (benchmarks; no dataset needed).
* ``write_synthetic_bins`` writes uniform-random shards in the same on-disk
  format, so either trainer can run on the same data.
"""
from __future__ import annotations

import bisect
import glob
import os
import random
from typing import List, Optional, Tuple

import numpy as np
import torch


def shard_paths(data_dir: str, split: str, limit: Optional[int] = None) -> List[str]:
    """Sorted shard files of one split, the first ``limit`` of them when given."""
    found = sorted(glob.glob(os.path.join(data_dir, f"fineweb_{split}_*.bin")))
    if not found:
        raise FileNotFoundError(f"{data_dir}: no token shards for split '{split}' "
                                f"(expected files named fineweb_{split}_NNNNNN.bin)")
    return found if limit is None else found[:limit]


class TokenShards:
    """Memory-mapped uint16 shards and the two-step window draw.

    ``windows[i]`` counts the window starts that shard i contributes to the shard
    draw (its length minus the window length, floored at 0); ``_ends`` holds
    their running totals, so a uniform index in [0, total) falls in shard i with
    probability windows[i] / total."""

    def __init__(self, paths: List[str], window: int):
        self.window = window
        self.maps = [np.memmap(p, dtype=np.uint16, mode="r") for p in paths]
        self.sizes = [len(m) for m in self.maps]
        self.windows = [max(0, n - window) for n in self.sizes]
        self._ends = np.cumsum(self.windows).tolist()
        self.total = self._ends[-1] if self._ends else 0
        if self.total <= 0:
            raise ValueError(f"every shard is shorter than one window of {window} tokens")

    def draw(self, rng: random.Random) -> np.ndarray:
        """One window of ``window`` tokens: shard index from rng.randrange(total),
        then a start in [0, size - window] from rng.randint."""
        shard = bisect.bisect_right(self._ends, rng.randrange(self.total))
        start = rng.randint(0, self.sizes[shard] - self.window)
        return self.maps[shard][start:start + self.window]


class _PinnedStaging:
    """A ring of pinned [2, B, T] int64 host buffers. A slot is refilled only after
    the event recorded behind its previous host->device copy has completed."""

    def __init__(self, B: int, T: int, pin: bool, ring: int = 4):
        self.pin = pin
        self._ring = [torch.empty(2, B, T, dtype=torch.int64, pin_memory=pin) for _ in range(ring)]
        self._events: List[Optional[torch.cuda.Event]] = [None] * ring
        self._i = 0
        self.h2d_bytes = 2 * B * T * 8

    def take(self) -> Tuple[int, torch.Tensor]:
        slot = self._i % len(self._ring)
        self._i += 1
        ev = self._events[slot]
        if ev is not None:
            ev.synchronize()
        return slot, self._ring[slot]

    def to_device(self, slot: int, dev: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
        xy = self._ring[slot].to(dev, non_blocking=self.pin)
        ev = torch.cuda.Event()
        ev.record()
        self._events[slot] = ev
        return xy[0], xy[1]


class RandomBatchLoader:
    """Random windows of the token shards assigned to one DP rank (see module doc)."""

    def __init__(self, data_dir, split, B, T, num_chunks, seed=1337, rank=0, dp_rank=0, dp_size=1, log_rank=None,
                 pin_memory: bool = True):
        every = shard_paths(data_dir, split, num_chunks)
        mine = every[dp_rank::dp_size] if dp_size > 1 else every
        if not mine:
            raise FileNotFoundError(f"{data_dir}: {len(every)} '{split}' shard(s) cannot cover dp rank {dp_rank} "
                                    f"of {dp_size}; each DP rank needs at least one shard")
        self.B, self.T = B, T
        self.shards = TokenShards(mine, T + 1)
        self.rng = random.Random(seed + rank)
        self.staging = _PinnedStaging(B, T, pin_memory and torch.cuda.is_available())
        if (rank if log_rank is None else log_rank) == 0:
            print(f"data {split}: dp rank {dp_rank}/{dp_size} reads {len(mine)} shard(s), "
                  f"{sum(self.shards.sizes):,} tokens, windows of {T + 1}")

    def _fill(self, out: torch.Tensor) -> None:
        """Draws B windows into out[0] (inputs) and out[1] (targets)."""
        xs, ys = out[0].numpy(), out[1].numpy()
        for b in range(self.B):
            w = self.shards.draw(self.rng)
            xs[b] = w[:-1]
            ys[b] = w[1:]

    def next_batch_host(self) -> Tuple[torch.Tensor, torch.Tensor]:
        buf = torch.empty(2, self.B, self.T, dtype=torch.int64)
        self._fill(buf)
        return buf[0], buf[1]

    def next_batch(self, device):
        dev = torch.device(device)
        if dev.type != "cuda":
            return self.next_batch_host()
        slot, host = self.staging.take()
        self._fill(host)
        return self.staging.to_device(slot, dev)

    # data position for exact resume (the state of the sampling RNG)
    def state_dict(self) -> dict:
        return {"rng": self.rng.getstate()}

    def load_state_dict(self, sd: dict) -> None:
        self.rng.setstate(sd["rng"])


class SyntheticLoader:
    """Uniform-random token ids; y is x shifted by one within a (T+1)-token draw."""

    def __init__(self, B: int, T: int, vocab_size: int, seed: int = 1337, rank: int = 0, pin_memory: bool = True,
                 ring: int = 4):
        self.B, self.T, self.V = B, T, vocab_size
        self.gen = torch.Generator().manual_seed(seed + rank)
        self.staging = _PinnedStaging(B, T, pin_memory and torch.cuda.is_available(), ring)
        self.h2d_bytes = self.staging.h2d_bytes

    def _draw(self) -> torch.Tensor:
        return torch.randint(0, self.V, (self.B, self.T + 1), generator=self.gen, dtype=torch.int64)

    def next_batch_host(self):
        buf = self._draw()
        return buf[:, :-1].contiguous(), buf[:, 1:].contiguous()

    def next_batch(self, device):
        dev = torch.device(device)
        buf = self._draw()
        if dev.type != "cuda":
            return buf[:, :-1].contiguous(), buf[:, 1:].contiguous()
        slot, host = self.staging.take()
        host[0].copy_(buf[:, :-1])
        host[1].copy_(buf[:, 1:])
        return self.staging.to_device(slot, dev)

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
