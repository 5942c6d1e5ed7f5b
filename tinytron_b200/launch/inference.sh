#!/bin/bash
# Environment-driven inference launcher with the knobs of the reference's
# scripts/debug/inference.sh (MODEL_SIZE CKPT_PATH PROMPT_TOKEN_IDS MAX_NEW_TOKENS TEMPERATURE
# TOP_K TOP_P EOS_TOKEN_ID DEVICE DTYPE SEP_SIZE NPROC_PER_NODE BACKEND INIT_METHOD MASTER_ADDR
# MASTER_PORT).  Model sizes come from the Python preset table
# (tinytron_b200/models/presets.py).  Extra knobs: BATCH_SIZE and PROMPT_LEN run a seeded
# synthetic prompt batch and report prefill/decode tokens per second; PAGE_SIZE sets the KV
# page size (0 = contiguous cache).
#
#   bash tinytron_b200/launch/inference.sh                                   # random-init smoke test
#   MODEL_SIZE=0.1B CKPT_PATH=/path/00500_model.pt bash tinytron_b200/launch/inference.sh
#   MODEL_SIZE=2.7B-A1B SEP_SIZE=8 BATCH_SIZE=32 PROMPT_LEN=1024 MAX_NEW_TOKENS=512 \
#       bash tinytron_b200/launch/inference.sh                             # expert-parallel decode
set -euo pipefail

SCRIPT_DIR=$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)
REPO_ROOT=$(cd "$SCRIPT_DIR/../.." && pwd)
cd "$REPO_ROOT"

MODEL_SIZE=${MODEL_SIZE:-0.25B}
CKPT_PATH=${CKPT_PATH:-}
PROMPT_TOKEN_IDS=${PROMPT_TOKEN_IDS:-1,2,3,4}
MAX_NEW_TOKENS=${MAX_NEW_TOKENS:-16}
TEMPERATURE=${TEMPERATURE:-1.0}
TOP_K=${TOP_K:-50}
TOP_P=${TOP_P:-}
EOS_TOKEN_ID=${EOS_TOKEN_ID:-}
DEVICE=${DEVICE:-cuda}
DTYPE=${DTYPE:-bf16}
SEP_SIZE=${SEP_SIZE:-1}
NPROC_PER_NODE=${NPROC_PER_NODE:-$SEP_SIZE}
BACKEND=${BACKEND:-nccl}
INIT_METHOD=${INIT_METHOD:-env://}
MASTER_ADDR=${MASTER_ADDR:-127.0.0.1}
MASTER_PORT=${MASTER_PORT:-29500}
BATCH_SIZE=${BATCH_SIZE:-0}
PROMPT_LEN=${PROMPT_LEN:-0}
PAGE_SIZE=${PAGE_SIZE:-}

ARGS=(--preset "$MODEL_SIZE" --max_new_tokens "$MAX_NEW_TOKENS" --temperature "$TEMPERATURE" --top_k "$TOP_K"
      --device "$DEVICE" --dtype "$DTYPE" --backend "$BACKEND" --init_method "$INIT_METHOD"
      --sep_size "$SEP_SIZE" --tied_lm_head)
if [ "$BATCH_SIZE" -gt 0 ] && [ "$PROMPT_LEN" -gt 0 ]; then
  ARGS+=(--batch_size "$BATCH_SIZE" --prompt_len "$PROMPT_LEN")
else
  ARGS+=(--prompt_token_ids "$PROMPT_TOKEN_IDS")
fi
[ -n "$TOP_P" ] && ARGS+=(--top_p "$TOP_P")
[ -n "$EOS_TOKEN_ID" ] && ARGS+=(--eos_token_id "$EOS_TOKEN_ID")
if [ -n "$PAGE_SIZE" ]; then
  if [ "$PAGE_SIZE" -eq 0 ]; then ARGS+=(--no-paged_kv_cache); else ARGS+=(--kv_cache_page_size "$PAGE_SIZE"); fi
fi
if [ -n "$CKPT_PATH" ]; then ARGS+=(--checkpoint_path "$CKPT_PATH"); else ARGS+=(--init_from_scratch); fi

echo "Running inference with MODEL_SIZE=$MODEL_SIZE, DEVICE=$DEVICE, DTYPE=$DTYPE, SEP_SIZE=$SEP_SIZE"
if [ "$SEP_SIZE" -gt 1 ]; then
  exec python -m torch.distributed.run --nproc_per_node "$NPROC_PER_NODE" --master_addr "$MASTER_ADDR" \
    --master_port "$MASTER_PORT" -m tinytron_b200.launch.inference "${ARGS[@]}" "$@"
fi
exec python -m tinytron_b200.launch.inference "${ARGS[@]}" "$@"
