#!/bin/bash
# Environment-driven synchronous RL (GRPO) launcher with the knobs of the reference's
# scripts/debug/rl.sh (NUM_NODES NUM_GPUS NODE_RANK MASTER_ADDR MASTER_PORT MODEL_SIZE SEED
# SEP_SIZE BATCH_SIZE PROMPT_LEN GBS WARMUP_STEPS MAX_LR MIN_LR LOG_DIR and the RL_* group).
# The same ranks train the actor and run the rollouts; every step the bridge reshards the
# actor into the inference layout.  Model sizes come from the Python preset table.
# The actor recomputes prompt_len + max_new_tokens - 1 positions, which must split evenly
# over the SEP group: RL_MAX_NEW_TOKENS is raised to the next length that does.
set -euo pipefail

SCRIPT_DIR=$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)
REPO_ROOT=$(cd "$SCRIPT_DIR/../.." && pwd)
cd "$REPO_ROOT"

NUM_NODES=${NUM_NODES:-1}
NUM_GPUS=${NUM_GPUS:-8}
NODE_RANK=${NODE_RANK:-0}
MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29501}
MODEL_SIZE=${MODEL_SIZE:-0.03B}
SEED=${SEED:-1337}
SEP_SIZE=${SEP_SIZE:-1}
BATCH_SIZE=${BATCH_SIZE:-2}
PROMPT_LEN=${PROMPT_LEN:-17}
SEQ_LEN=$(( (PROMPT_LEN + SEP_SIZE - 1) / SEP_SIZE * SEP_SIZE ))
GBS=${GBS:-64}
TOTAL_BATCH_SIZE=$((GBS * SEQ_LEN))
WARMUP_STEPS=${WARMUP_STEPS:-1}
MAX_LR=${MAX_LR:-6e-5}
MIN_LR=${MIN_LR:-6e-6}
LOG_DIR=${LOG_DIR:-"$REPO_ROOT/logs/debug_rl_${MODEL_SIZE}"}

RL_MAX_NEW_TOKENS=${RL_MAX_NEW_TOKENS:-8}
RL_GROUP_SIZE=${RL_GROUP_SIZE:-2}
RL_TEMPERATURE=${RL_TEMPERATURE:-1.0}
RL_TOP_K=${RL_TOP_K:-0}
RL_TOP_P=${RL_TOP_P:-0.0}
RL_REWARD_TARGET_TOKEN_ID=${RL_REWARD_TARGET_TOKEN_ID:-0}
RL_CLIP_RANGE=${RL_CLIP_RANGE:-0.2}
RL_KL_COEF=${RL_KL_COEF:-0.0}
RL_ROLLOUT_SHARD_QKV=${RL_ROLLOUT_SHARD_QKV:-1}

RECOMPUTE=$((SEQ_LEN + RL_MAX_NEW_TOKENS - 1))
if [ $((RECOMPUTE % SEP_SIZE)) -ne 0 ]; then
  RECOMPUTE=$(( (RECOMPUTE + SEP_SIZE - 1) / SEP_SIZE * SEP_SIZE ))
  RL_MAX_NEW_TOKENS=$((RECOMPUTE - SEQ_LEN + 1))
fi

ARGS=(--preset "$MODEL_SIZE" --seed "$SEED" --use_mock_data --mock_data_num_samples 1280 --log_dir "$LOG_DIR"
      --total_batch_size "$TOTAL_BATCH_SIZE" --batch_size "$BATCH_SIZE" --seq_len "$SEQ_LEN" --max_epochs 1
      --max_lr "$MAX_LR" --min_lr "$MIN_LR" --warmup_steps "$WARMUP_STEPS" --weight_decay 0.0
      --grad_clip_value 1.0 --debug --deterministic --sep_size "$SEP_SIZE" --backend nccl --block_size 4096
      --rl_max_new_tokens "$RL_MAX_NEW_TOKENS" --rl_group_size "$RL_GROUP_SIZE" --rl_temperature "$RL_TEMPERATURE"
      --rl_top_k "$RL_TOP_K" --rl_top_p "$RL_TOP_P" --rl_reward_target_token_id "$RL_REWARD_TARGET_TOKEN_ID"
      --rl_clip_range "$RL_CLIP_RANGE" --rl_kl_coef "$RL_KL_COEF")
[ "$RL_ROLLOUT_SHARD_QKV" -eq 1 ] && ARGS+=(--rl_rollout_shard_qkv)

echo "[rl] PROMPT_LEN=$PROMPT_LEN SEQ_LEN=$SEQ_LEN RL_MAX_NEW_TOKENS=$RL_MAX_NEW_TOKENS RECOMPUTE=$RECOMPUTE SEP_SIZE=$SEP_SIZE"
exec python -m torch.distributed.run --nnodes="$NUM_NODES" --nproc_per_node="$NUM_GPUS" --node_rank="$NODE_RANK" \
  --master_addr="$MASTER_ADDR" --master_port="$MASTER_PORT" -m tinytron_b200.launch.rl "${ARGS[@]}" "$@"
