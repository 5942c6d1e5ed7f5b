#!/bin/bash
# Environment-driven pretraining launcher with the same knobs as the reference's
# scripts/debug/pretrain.sh (NUM_NODES NUM_GPUS NODE_RANK MASTER_ADDR MASTER_PORT
# LR_WARMUP_STEPS MAX_LR MIN_LR SEED BATCH_SIZE SEQ_LEN GBS SEP_SIZE DEBUG DETER_MODE
# MODEL_SIZE MOE_BALANCE_LOSS_WEIGHT LOG_DIR) and those of its streaming example
# (STREAMING_DATA_DIR BATCH_SIZE_SCALE_WITH_SEP PRECISION MAX_STEPS MAX_EPOCHS LOG_EVERY
# DO_SAVE SAVE_EVERY_STEPS USE_DISTRIBUTED_OPTIMIZER).  Model sizes come from the Python
# preset table (tinytron_b200/models/presets.py) instead of a shell case block.
# USE_COMPILE is accepted and ignored: the hot paths are hand-written kernels.
# MAX_STEPS, when set, replaces the epoch budget (the trainer rejects a step budget and
# an epoch budget that disagree).
set -euo pipefail

SCRIPT_DIR=$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)
REPO_ROOT=$(cd "$SCRIPT_DIR/../.." && pwd)
cd "$REPO_ROOT"
export CUBLAS_WORKSPACE_CONFIG=${CUBLAS_WORKSPACE_CONFIG:-:4096:8}

NUM_NODES=${NUM_NODES:-1}
NUM_GPUS=${NUM_GPUS:-8}
NODE_RANK=${NODE_RANK:-0}
MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29500}
LR_WARMUP_STEPS=${LR_WARMUP_STEPS:-2}
MAX_LR=${MAX_LR:-6e-4}
MIN_LR=${MIN_LR:-6e-5}
SEED=${SEED:-1337}
BATCH_SIZE=${BATCH_SIZE:-8}
SEQ_LEN=${SEQ_LEN:-4096}
GBS=${GBS:-1024}
TOTAL_BATCH_SIZE=$((GBS * SEQ_LEN))
SEP_SIZE=${SEP_SIZE:-1}
BATCH_SIZE_SCALE_WITH_SEP=${BATCH_SIZE_SCALE_WITH_SEP:-1}
if [ "$BATCH_SIZE_SCALE_WITH_SEP" -eq 1 ]; then
  BATCH_SIZE_PER_DP_RANK=$((BATCH_SIZE * SEP_SIZE))
else
  BATCH_SIZE_PER_DP_RANK=$BATCH_SIZE
fi
PRECISION=${PRECISION:-bf16}
STREAMING_DATA_DIR=${STREAMING_DATA_DIR:-}
DEBUG=${DEBUG:-1}
DETER_MODE=${DETER_MODE:-1}
MODEL_SIZE=${MODEL_SIZE:-0.25B}
MOE_BALANCE_LOSS_WEIGHT=${MOE_BALANCE_LOSS_WEIGHT:-}
MAX_STEPS=${MAX_STEPS:-}
MAX_EPOCHS=${MAX_EPOCHS:-1}
LOG_EVERY=${LOG_EVERY:-10}
DO_SAVE=${DO_SAVE:-1}
SAVE_EVERY_STEPS=${SAVE_EVERY_STEPS:-500}
USE_DISTRIBUTED_OPTIMIZER=${USE_DISTRIBUTED_OPTIMIZER:-1}
LOG_DIR=${LOG_DIR:-"$REPO_ROOT/logs/debug_gpt_${MODEL_SIZE}"}

ARGS=(--preset "$MODEL_SIZE" --seed "$SEED" --precision "$PRECISION" --log_dir "$LOG_DIR"
      --total_batch_size "$TOTAL_BATCH_SIZE" --batch_size "$BATCH_SIZE_PER_DP_RANK" --seq_len "$SEQ_LEN"
      --block_size "$SEQ_LEN" --max_lr "$MAX_LR" --min_lr "$MIN_LR" --weight_decay 0.1 --grad_clip_value 1.0
      --warmup_steps "$LR_WARMUP_STEPS" --log_every "$LOG_EVERY" --save_every_steps "$SAVE_EVERY_STEPS"
      --sep_size "$SEP_SIZE")
if [ -n "$STREAMING_DATA_DIR" ]; then
  ARGS+=(--streaming_data_dir "$STREAMING_DATA_DIR")
else
  ARGS+=(--use_mock_data --mock_data_num_samples 12800)
fi
[ "$DEBUG" -eq 1 ] && ARGS+=(--debug)
[ "$DETER_MODE" -eq 1 ] && ARGS+=(--deterministic)
[ -n "$MOE_BALANCE_LOSS_WEIGHT" ] && ARGS+=(--moe_balance_loss_weight "$MOE_BALANCE_LOSS_WEIGHT")
if [ -n "$MAX_STEPS" ]; then
  ARGS+=(--max_steps "$MAX_STEPS")
else
  ARGS+=(--max_epochs "$MAX_EPOCHS")
fi
[ "$DO_SAVE" -eq 1 ] && ARGS+=(--do_save)
[ "$USE_DISTRIBUTED_OPTIMIZER" -eq 1 ] && ARGS+=(--use_distributed_optimizer)

exec python -m torch.distributed.run --nnodes="$NUM_NODES" --nproc_per_node="$NUM_GPUS" --node_rank="$NODE_RANK" \
  --master_addr="$MASTER_ADDR" --master_port="$MASTER_PORT" -m tinytron_b200.launch.pretrain "${ARGS[@]}" "$@"
