#!/usr/bin/env bash
# Quick smoke run: 6L/6H/384d, 100 iterations on 4 GPUs (reference run_train_quick.sh).
set -euo pipefail
export N_LAYER=6 N_HEAD=6 N_EMBED=384
export BATCH_SIZE=8 BLOCK_SIZE=256 GRAD_ACCUM=2
export MAX_ITERS=100 EVAL_INTERVAL=50 SAVE_INTERVAL=0 DROPOUT=0.1 AMP=bf16
export RUN_NAME="heiretsu-quicktest-$(date +%H%M%S)"
export WANDB_PROJECT="heiretsu-test"
export DP=${DP:-4} TP=${TP:-1} PP=${PP:-1}
exec bash "$(dirname "$0")/run_train.sh"
