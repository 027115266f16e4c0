"""The vLLM baseline's local model folder (foundry_b200/runner/vllm_baseline.py)
parses as a Hugging Face config of the same shapes as this package's models,
so vLLM builds the same architecture from it with dummy weights."""

import pytest

from foundry_b200.models import config_by_name
from foundry_b200.runner.vllm_baseline import write_model_dir


@pytest.mark.parametrize("model", ["llama-3-8b", "llama-3-70b", "qwen3-30b-a3b"])
def test_model_dir_matches_shapes(model, tmp_path):
    transformers = pytest.importorskip("transformers")
    cfg = config_by_name(model)
    path = write_model_dir(model, str(tmp_path / "m"))
    hf = transformers.AutoConfig.from_pretrained(path)
    assert hf.hidden_size == cfg.hidden and hf.num_hidden_layers == cfg.layers
    assert hf.num_attention_heads == cfg.n_q and hf.num_key_value_heads == cfg.n_kv
    assert hf.vocab_size == cfg.vocab and hf.head_dim == cfg.head_dim
    if cfg.arch == "qwen3_moe":
        assert hf.num_experts == cfg.num_experts and hf.num_experts_per_tok == cfg.topk
        assert hf.moe_intermediate_size == cfg.moe_inter
        assert hf.quantization_config["weight_block_size"] == [128, 128]
    else:
        assert hf.intermediate_size == cfg.inter
