#!/usr/bin/env python3
"""Sample tokens from a trained checkpoint (one process).

    python sample.py --ckpt out/ckpt_0005000.pt --start 50256 --max_new_tokens 100 --temperature 0.8 --top_k 200

``--ckpt`` takes a dense checkpoint or any shard of a sharded step (the shards
of that step are merged into the dense model first). ``--start`` is a
comma-separated list of token ids (GPT-2 ids; 50256 is <|endoftext|>), or text
when the ``tiktoken`` package is installed. Output: one line of token ids per
sample, and the decoded text when ``tiktoken`` is installed.
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from heiretsu_b200.config import GPTConfig  # noqa: E402
from heiretsu_b200.models.generate import generate  # noqa: E402
from heiretsu_b200.models.gpt import GPT  # noqa: E402
from heiretsu_b200.utils.ckpt import merge_shards, step_files  # noqa: E402


def load_model(path: str, device) -> GPT:
    objs = [torch.load(f, map_location="cpu", weights_only=False) for f in step_files(path)]
    state = objs[0]["model"] if len(objs) == 1 and "topo" not in objs[0] else merge_shards(objs)
    cfg = GPTConfig(**objs[0]["cfg"])
    model = GPT(cfg)
    model.load_state_dict({k.removeprefix("_orig_mod."): v for k, v in state.items()})
    return model.to(device)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--start", default="50256", help="comma-separated token ids, or text with tiktoken installed")
    ap.add_argument("--num_samples", type=int, default=1)
    ap.add_argument("--max_new_tokens", type=int, default=64)
    ap.add_argument("--temperature", type=float, default=0.8, help="<= 0: always the most likely token")
    ap.add_argument("--top_k", type=int, default=200)
    ap.add_argument("--seed", type=int, default=1337)
    ap.add_argument("--device", default="auto")
    ap.add_argument("--no_kv_cache", action="store_true", help="re-run the whole context every token")
    a = ap.parse_args(argv)
    device = torch.device("cuda" if a.device == "auto" and torch.cuda.is_available() else
                          ("cpu" if a.device == "auto" else a.device))
    model = load_model(a.ckpt, device)
    try:
        import tiktoken
        enc = tiktoken.get_encoding("gpt2")
    except Exception:
        enc = None
    if all(p.strip().lstrip("-").isdigit() for p in a.start.split(",")):
        ids = [int(p) for p in a.start.split(",")]
    elif enc is not None:
        ids = enc.encode(a.start, allowed_special={"<|endoftext|>"})
    else:
        raise SystemExit("--start is text but tiktoken is not installed; pass token ids")
    g = torch.Generator(device=device).manual_seed(a.seed)
    idx = torch.tensor([ids] * a.num_samples, dtype=torch.long, device=device)
    out = generate(model, idx, a.max_new_tokens, temperature=a.temperature, top_k=a.top_k, generator=g,
                   kv_cache=not a.no_kv_cache)
    for row in out.tolist():
        print(",".join(str(t) for t in row))
        if enc is not None:
            print(enc.decode(row))


if __name__ == "__main__":
    main()
