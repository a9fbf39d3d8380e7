#!/usr/bin/env bash
# Full test suite (the counterpart of the reference's tests/run_full_suite.sh):
# the CPU suite (gloo multi-process parity of every DP/TP/PP/EP layout against
# the dense model and the reference modules, the reference's own test scripts,
# checkpoints, faults, launcher), then the GPU suite when GPUs are present
# (every kernel against an fp32 PyTorch oracle, the fused model, and the
# 2- and 4-GPU fused collectives, which skip when fewer GPUs are visible).
#   bash tests/run_full_suite.sh                 # everything this machine can run
#   CPU_ONLY=1 bash tests/run_full_suite.sh
#   PYTEST_ARGS="-k parallel" bash tests/run_full_suite.sh
set -euo pipefail
cd "$(dirname "$0")/.."
LOG_DIR=${LOG_DIR:-tests/logs/full_suite_$(date +%Y%m%d_%H%M%S)}
mkdir -p "${LOG_DIR}"
read -r -a EXTRA <<< "${PYTEST_ARGS:-}"

num_gpus=0
if command -v nvidia-smi &> /dev/null; then
  num_gpus=$(nvidia-smi --list-gpus 2>/dev/null | wc -l || echo 0)
fi
echo "Detected ${num_gpus} GPUs; logs in ${LOG_DIR}"

status=0
echo "=== CPU suite ==="
python -m pytest tests -q -m "not gpu" "${EXTRA[@]}" 2>&1 | tee "${LOG_DIR}/cpu.log" || status=1
if [[ ${CPU_ONLY:-0} == 0 && ${num_gpus} -gt 0 ]]; then
  echo "=== GPU suite ==="
  python -m pytest tests -q -m gpu "${EXTRA[@]}" 2>&1 | tee "${LOG_DIR}/gpu.log" || status=1
fi
[[ ${status} == 0 ]] && echo "FULL SUITE: PASS" || echo "FULL SUITE: FAIL"
exit ${status}
