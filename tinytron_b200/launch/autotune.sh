#!/bin/bash
# Throughput auto-tuner launcher with the reference's scripts/autotune.sh knobs
# (SEP_SIZES BATCH_SIZES TARGET_STEPS WARMUP_STEPS DEBUG, plus MODEL_SIZE NUM_GPUS of the
# pretraining launcher); flags after the script name override them.
set -euo pipefail
SCRIPT_DIR=$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)
cd "$SCRIPT_DIR/../.."
exec python -m tinytron_b200.launch.autotune "$@"
