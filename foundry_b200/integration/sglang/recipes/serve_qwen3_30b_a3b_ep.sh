#!/usr/bin/env bash
# Qwen3-30B-A3B-FP8 with expert parallelism and DP attention (2 GPUs) under SGLang, SAVE then LOAD.
# Usage: serve_qwen3_30b_a3b_ep.sh save|load [MODEL_DIR]
set -euo pipefail
MODE=${1:-save}
MODEL=${2:-Qwen/Qwen3-30B-A3B-FP8}
HERE=$(cd "$(dirname "$0")" && pwd)
exec python -m foundry_b200.integration.sglang.serve --foundry-config "$HERE/foundry_${MODE}.toml" -- \
  --model-path "$MODEL" --tp-size 2 --dp-size 2 --enable-dp-attention --ep-size 2 \
  --cuda-graph-max-bs 256 --load-format dummy --port 30000
