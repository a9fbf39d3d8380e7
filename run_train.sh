#!/usr/bin/env bash
# Training launcher: one process per GPU via torchrun, every knob an env var.
# Presets mirror the reference's run_train.sh (GPT-2 medium, DP=4 by default,
# reference run_train.sh:28-72); flags map 1:1 onto train.py's argparse.
#   DP=8 bash run_train.sh
#   DP=2 TP=2 PP=2 N_LAYER=36 N_HEAD=20 N_EMBED=1280 bash run_train.sh
#   SYNTHETIC=1 MAX_ITERS=50 bash run_train.sh      # no dataset needed
set -euo pipefail

DP=${DP:-4}
TP=${TP:-1}
PP=${PP:-1}
EP=${EP:-1}

NUM_EXPERTS=${NUM_EXPERTS:-0}
TOP_K=${TOP_K:-2}
MOE_FREQ=${MOE_FREQ:-2}
AUX_LOSS_COEF=${AUX_LOSS_COEF:-0.01}

N_LAYER=${N_LAYER:-24}
N_HEAD=${N_HEAD:-16}
N_EMBED=${N_EMBED:-1024}
DROPOUT=${DROPOUT:-0.1}

BATCH_SIZE=${BATCH_SIZE:-8}
BLOCK_SIZE=${BLOCK_SIZE:-1024}
GRAD_ACCUM=${GRAD_ACCUM:-4}
MAX_ITERS=${MAX_ITERS:-50000}
LEARNING_RATE=${LEARNING_RATE:-3e-4}
WEIGHT_DECAY=${WEIGHT_DECAY:-0.1}
GRAD_CLIP=${GRAD_CLIP:-1.0}
AMP=${AMP:-bf16}
ENGINE=${ENGINE:-auto}
DEVICE=${DEVICE:-auto}
DIST_BACKEND=${DIST_BACKEND:-nccl}

EVAL_INTERVAL=${EVAL_INTERVAL:-500}
EVAL_ITERS=${EVAL_ITERS:-100}
SAVE_INTERVAL=${SAVE_INTERVAL:-5000}
SAVE_PATH=${SAVE_PATH:-./checkpoints}
DATA_DIR=${DATA_DIR:-data/fineweb10B}
SYNTHETIC=${SYNTHETIC:-0}
RESUME=${RESUME:-}

WANDB=${WANDB:-0}
WANDB_PROJECT=${WANDB_PROJECT:-heiretsu-fineweb}
WANDB_MODE=${WANDB_MODE:-online}
RUN_NAME=${RUN_NAME:-"heiretsu-$(date +%Y%m%d_%H%M%S)"}

MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29500}
# Upper bound on the whole job; process-group timeouts end a stuck collective long before.
JOB_TIMEOUT=${JOB_TIMEOUT:-0}

WORLD_SIZE=$((DP * TP * PP * EP))
echo "run ${RUN_NAME}: dp=${DP} tp=${TP} pp=${PP} ep=${EP} (world ${WORLD_SIZE}); ${N_LAYER}L ${N_HEAD}H ${N_EMBED}D;" \
     "micro-batch ${BATCH_SIZE} x ${BLOCK_SIZE}, accum ${GRAD_ACCUM}, global batch $((BATCH_SIZE * GRAD_ACCUM * DP))"

EXTRA=()
if [[ ${NUM_EXPERTS} -gt 0 ]]; then
  EXTRA+=(--num_experts "${NUM_EXPERTS}" --top_k "${TOP_K}" --moe_freq "${MOE_FREQ}" --aux_loss_coef "${AUX_LOSS_COEF}")
fi
[[ ${SYNTHETIC} != 0 ]] && EXTRA+=(--synthetic_data)
[[ -n ${RESUME} ]] && EXTRA+=(--resume "${RESUME}")
[[ ${WANDB} != 0 ]] && EXTRA+=(--wandb --wandb_project "${WANDB_PROJECT}" --wandb_mode "${WANDB_MODE}")

mkdir -p "${SAVE_PATH}"
cd "$(dirname "$0")"
LAUNCH=(python -m torch.distributed.run --nnodes=1 --nproc-per-node="${WORLD_SIZE}"
        --master-addr "${MASTER_ADDR}" --master-port "${MASTER_PORT}")
if [[ ${JOB_TIMEOUT} -gt 0 ]]; then LAUNCH=(timeout -k 60 "${JOB_TIMEOUT}" "${LAUNCH[@]}"); fi
exec "${LAUNCH[@]}" train.py \
  --data_dir "${DATA_DIR}" \
  --batch_size "${BATCH_SIZE}" --block_size "${BLOCK_SIZE}" \
  --n_layer "${N_LAYER}" --n_head "${N_HEAD}" --n_embed "${N_EMBED}" --dropout "${DROPOUT}" \
  --max_iters "${MAX_ITERS}" --learning_rate "${LEARNING_RATE}" --weight_decay "${WEIGHT_DECAY}" \
  --grad_clip "${GRAD_CLIP}" --grad_accum_steps "${GRAD_ACCUM}" --amp "${AMP}" --engine "${ENGINE}" \
  --dp "${DP}" --tp "${TP}" --pp "${PP}" --ep "${EP}" --device "${DEVICE}" --dist_backend "${DIST_BACKEND}" \
  --eval_interval "${EVAL_INTERVAL}" --eval_iters "${EVAL_ITERS}" \
  --save_interval "${SAVE_INTERVAL}" --out_dir "${SAVE_PATH}" \
  --run_name "${RUN_NAME}" --seed 1337 \
  "${EXTRA[@]}"
