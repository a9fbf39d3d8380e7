#!/usr/bin/env bash
# Training launcher: one process per GPU via torchrun, every knob an env var.
# Presets mirror the reference's run_train.sh (GPT-2 medium, DP=4 by default,
# reference run_train.sh:28-72); flags map 1:1 onto train.py's argparse.
#   DP=8 bash run_train.sh
#   DP=2 TP=2 PP=2 N_LAYER=36 N_HEAD=20 N_EMBED=1280 bash run_train.sh
#   SYNTHETIC=1 MAX_ITERS=50 bash run_train.sh      # no dataset needed
#   CONFIG_FILE=run.yaml bash run_train.sh          # flag values from a YAML/TOML/JSON file
# Multi-node: run the same command on every node with NNODES, NODE_RANK and a
# MASTER_ADDR that all nodes reach (node 0's address), e.g. on two 8-GPU nodes
#   NNODES=2 NODE_RANK=0 MASTER_ADDR=10.0.0.1 DP=16 bash run_train.sh   # node 0
#   NNODES=2 NODE_RANK=1 MASTER_ADDR=10.0.0.1 DP=16 bash run_train.sh   # node 1
# Ranks are numbered node by node, so TP (innermost), then PP and EP groups
# stay inside a node when tp*pp*ep divides the GPUs per node; the fused TP/EP
# collectives use NVLink peer memory and need that. DP groups may span nodes:
# their gradient reduction then runs as NCCL all-reduces (over the inter-node
# network, e.g. InfiniBand with GPUDirect RDMA when NCCL finds it).
set -euo pipefail

# Topology and launch (always from the environment: the launcher needs the world size).
DP=${DP:-4}
TP=${TP:-1}
PP=${PP:-1}
EP=${EP:-1}
MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29500}
NNODES=${NNODES:-1}
NODE_RANK=${NODE_RANK:-0}
CONFIG_FILE=${CONFIG_FILE:-}
# Restarts of the whole worker group after a rank fails (torchrun --max-restarts);
# with restarts the job resumes from its newest complete checkpoint (RESUME=auto).
MAX_RESTARTS=${MAX_RESTARTS:-0}
# Upper bound on the whole job; process-group timeouts end a stuck collective long before.
JOB_TIMEOUT=${JOB_TIMEOUT:-0}
SAVE_PATH=${SAVE_PATH:-./checkpoints}
SYNTHETIC=${SYNTHETIC:-0}
RESUME=${RESUME:-}
if [[ ${MAX_RESTARTS} -gt 0 && -z ${RESUME} ]]; then RESUME=auto; fi
NUM_EXPERTS=${NUM_EXPERTS:-0}
WANDB=${WANDB:-0}

# Run settings: "flag ENV_VAR default". Without CONFIG_FILE every flag is passed
# (the env var or its preset default); with CONFIG_FILE only the env vars that
# are set are passed, so everything else comes from the file.
SPEC=(
  "--data_dir DATA_DIR data/fineweb10B"
  "--batch_size BATCH_SIZE 8"
  "--block_size BLOCK_SIZE 1024"
  "--n_layer N_LAYER 24"
  "--n_head N_HEAD 16"
  "--n_embed N_EMBED 1024"
  "--dropout DROPOUT 0.1"
  "--max_iters MAX_ITERS 50000"
  "--learning_rate LEARNING_RATE 3e-4"
  "--weight_decay WEIGHT_DECAY 0.1"
  "--grad_clip GRAD_CLIP 1.0"
  "--grad_accum_steps GRAD_ACCUM 4"
  "--amp AMP bf16"
  "--engine ENGINE auto"
  "--device DEVICE auto"
  "--dist_backend DIST_BACKEND nccl"
  "--eval_interval EVAL_INTERVAL 500"
  "--eval_iters EVAL_ITERS 100"
  "--save_interval SAVE_INTERVAL 5000"
  "--run_name RUN_NAME heiretsu-$(date +%Y%m%d_%H%M%S)"
  "--seed SEED 1337"
)
ARGS=(--dp "${DP}" --tp "${TP}" --pp "${PP}" --ep "${EP}" --out_dir "${SAVE_PATH}")
for row in "${SPEC[@]}"; do
  read -r flag var def <<< "${row}"
  if [[ -n "${!var:-}" ]]; then
    ARGS+=("${flag}" "${!var}")
  elif [[ -z ${CONFIG_FILE} ]]; then
    ARGS+=("${flag}" "${def}")
  fi
done
if [[ ${NUM_EXPERTS} -gt 0 ]]; then
  ARGS+=(--num_experts "${NUM_EXPERTS}" --top_k "${TOP_K:-2}" --moe_freq "${MOE_FREQ:-2}"
         --aux_loss_coef "${AUX_LOSS_COEF:-0.01}")
fi
[[ ${SYNTHETIC} != 0 ]] && ARGS+=(--synthetic_data)
[[ -n ${RESUME} ]] && ARGS+=(--resume "${RESUME}")
[[ -n ${CONFIG_FILE} ]] && ARGS+=(--config_file "${CONFIG_FILE}")
[[ ${WANDB} != 0 ]] && ARGS+=(--wandb --wandb_project "${WANDB_PROJECT:-heiretsu-fineweb}"
                              --wandb_mode "${WANDB_MODE:-online}")

WORLD_SIZE=$((DP * TP * PP * EP))
if (( WORLD_SIZE % NNODES != 0 )); then
  echo "world size ${WORLD_SIZE} (dp*tp*pp*ep) is not a multiple of NNODES=${NNODES}" >&2; exit 2
fi
NPROC_PER_NODE=$((WORLD_SIZE / NNODES))
echo "launch: dp=${DP} tp=${TP} pp=${PP} ep=${EP} (world ${WORLD_SIZE}, ${NNODES} node(s) x ${NPROC_PER_NODE});" \
     "train.py ${ARGS[*]}"

mkdir -p "${SAVE_PATH}"
cd "$(dirname "$0")"
if [[ ${MAX_RESTARTS} -gt 0 ]]; then
  # Elastic rendezvous: every restart gets a fresh store, so no rank of a new attempt
  # reads addresses that ranks of the failed attempt published.
  RDZV=(--rdzv-backend=c10d --rdzv-endpoint="${MASTER_ADDR}:${MASTER_PORT}" --rdzv-id="${RUN_NAME:-heiretsu}"
        --max-restarts="${MAX_RESTARTS}")
else
  RDZV=(--node-rank="${NODE_RANK}" --master-addr "${MASTER_ADDR}" --master-port "${MASTER_PORT}")
fi
LAUNCH=(python -m torch.distributed.run --nnodes="${NNODES}" --nproc-per-node="${NPROC_PER_NODE}" "${RDZV[@]}")
if [[ ${JOB_TIMEOUT} -gt 0 ]]; then LAUNCH=(timeout -k 60 "${JOB_TIMEOUT}" "${LAUNCH[@]}"); fi
exec "${LAUNCH[@]}" train.py "${ARGS[@]}"
