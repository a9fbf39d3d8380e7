"""Fetch the GPT-2-tokenised FineWeb10B shards (reference data/data_bins.py).

    python data/data_bins.py [num_chunks]          # val shard 0 + train shards 1..num_chunks (default 103)
    python data/data_bins.py 4 --synthetic          # offline: uniform-random shards of the same format

Shards land in data/fineweb10B/ as fineweb_{train,val}_NNNNNN.bin: raw uint16
token ids, the layout heiretsu_b200.utils.data memory-maps. Downloading needs
huggingface_hub and network access; files already present are skipped. With
--synthetic (or when the hub is unreachable and --fallback-synthetic is given)
the same file names are written with random ids, 100M tokens per train shard
unless --tokens-per-shard says otherwise.
"""
from __future__ import annotations

import argparse
import os
import sys

REPO_ID = "kjj0/fineweb10B-gpt2"
HERE = os.path.dirname(os.path.abspath(__file__))


def shard_names(num_chunks: int):
    return ["fineweb_val_%06d.bin" % 0] + ["fineweb_train_%06d.bin" % i for i in range(1, num_chunks + 1)]


def download(local_dir: str, num_chunks: int) -> None:
    from huggingface_hub import hf_hub_download  # optional dependency

    for fname in shard_names(num_chunks):
        if not os.path.exists(os.path.join(local_dir, fname)):
            hf_hub_download(repo_id=REPO_ID, filename=fname, repo_type="dataset", local_dir=local_dir)


def synthesize(local_dir: str, num_chunks: int, tokens_per_shard: int, seed: int = 0) -> None:
    sys.path.insert(0, os.path.dirname(HERE))
    from heiretsu_b200.utils.data import write_synthetic_bins

    write_synthetic_bins(local_dir, train_tokens=tokens_per_shard, val_tokens=tokens_per_shard,
                         seed=seed, num_train=num_chunks)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("num_chunks", nargs="?", type=int, default=103, help="train shards (100M tokens each)")
    ap.add_argument("--dir", default=os.path.join(HERE, "fineweb10B"))
    ap.add_argument("--synthetic", action="store_true")
    ap.add_argument("--fallback-synthetic", action="store_true")
    ap.add_argument("--tokens-per-shard", type=int, default=100_000_000)
    args = ap.parse_args(argv)
    os.makedirs(args.dir, exist_ok=True)
    if args.synthetic:
        synthesize(args.dir, args.num_chunks, args.tokens_per_shard)
        return
    try:
        download(args.dir, args.num_chunks)
    except Exception as e:  # no hub package or no network
        if not args.fallback_synthetic:
            raise SystemExit(f"download failed ({type(e).__name__}: {e}); rerun with --synthetic for offline shards")
        print(f"download failed ({type(e).__name__}); writing synthetic shards instead")
        synthesize(args.dir, args.num_chunks, args.tokens_per_shard)


if __name__ == "__main__":
    main()
