#!/usr/bin/env bash
# MoE 12L/768d, 8 experts top-2 every 2nd block, on 8 GPUs as dp2 x ep2 x tp2
# (reference run_moe_4d.sh).
set -euo pipefail
export DP=2 EP=2 TP=2 PP=1
export N_LAYER=12 N_HEAD=12 N_EMBED=768
export NUM_EXPERTS=8 TOP_K=2 MOE_FREQ=2
export BATCH_SIZE=8 GRAD_ACCUM=4 BLOCK_SIZE=1024
export MAX_ITERS=${MAX_ITERS:-5000} LEARNING_RATE=3e-4
export EVAL_INTERVAL=500 EVAL_ITERS=50 SAVE_INTERVAL=1000 AMP=bf16
export WANDB_PROJECT=heiretsu-moe RUN_NAME=${RUN_NAME:-"moe-8e-top2-4D-dp2ep2tp2-12L768D"}
exec bash "$(dirname "$0")/run_train.sh"
