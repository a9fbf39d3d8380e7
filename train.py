#!/usr/bin/env python3
"""GPT trainer entry point (same command line as the reference's train.py).

    torchrun --standalone --nproc_per_node=N train.py --dp ... --tp ... --pp ... --ep ...
"""
from heiretsu_b200.trainer import main

if __name__ == "__main__":
    main()
