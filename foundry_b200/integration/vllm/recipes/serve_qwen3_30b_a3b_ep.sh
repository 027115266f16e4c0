#!/usr/bin/env bash
# Qwen3-30B-A3B with expert parallelism (EP=2) under vLLM, SAVE then LOAD.
# Usage: serve_qwen3_30b_a3b_ep.sh save|load [MODEL_DIR]
set -euo pipefail
MODE=${1:-save}
MODEL=${2:-Qwen/Qwen3-30B-A3B-FP8}
HERE=$(cd "$(dirname "$0")" && pwd)
exec python -m foundry_b200.integration.vllm.serve --foundry-config "$HERE/foundry_${MODE}.toml" -- \
  "$MODEL" --tensor-parallel-size 1 --data-parallel-size 2 --enable-expert-parallel \
  --compilation-config '{"cudagraph_mode": "FULL_DECODE_ONLY", "cudagraph_capture_sizes": [1,2,4,8,16,32,64,128,256]}' \
  --max-model-len 4096 --load-format dummy --port 8000
