"""TensorRT-LLM integration: not provided (the reference ships a placeholder
too, python/foundry/integration/trtllm/__init__.py:1-4). Use the engine-
agnostic pieces in foundry_b200.integration (config, runtime, graph_ops) to
wire another engine's graph capture to foundry."""
