"""Same-box vLLM baseline of a decode benchmark (``bench.py --impl vllm``).

The reference persists vLLM's and SGLang's CUDA graphs. Its steady-state
decode is the engine's own, so upstream vLLM on the same box, model shape and
batch is the closest stand-in for the reference's decode throughput.

Nothing is downloaded. ``write_model_dir`` writes a Hugging Face
``config.json`` of the named shape (Llama-3 or Qwen3-MoE architecture) into
a local folder. vLLM loads it with ``load_format="dummy"`` (random weights)
and ``skip_tokenizer_init=True``, and the prompts are token ids. Decode
throughput is taken from two greedy generations of the same prompts:
``gen`` tokens and one token. The difference is the decode time of
``gen - 1`` steps of the whole batch, timed on the host around the blocking
``generate`` call with a device synchronize on both sides.
"""

from __future__ import annotations

import json
import os
import time


def hf_config(cfg) -> dict:
    """Hugging Face config of one of this package's model configs."""
    common = {
        "hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.n_q,
        "num_key_value_heads": cfg.n_kv, "head_dim": cfg.head_dim, "vocab_size": cfg.vocab,
        "rms_norm_eps": cfg.eps, "rope_theta": cfg.rope_theta, "max_position_embeddings": 8192,
        "torch_dtype": "bfloat16", "tie_word_embeddings": False, "bos_token_id": 1, "eos_token_id": 2,
        "hidden_act": "silu", "attention_bias": False, "initializer_range": cfg.init_std,
    }
    if getattr(cfg, "arch", "llama") == "qwen3_moe":
        return {**common, "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
                "num_experts": cfg.num_experts, "num_experts_per_tok": cfg.topk,
                "moe_intermediate_size": cfg.moe_inter, "intermediate_size": 6144,
                "norm_topk_prob": cfg.norm_topk_prob, "decoder_sparse_step": 1, "mlp_only_layers": [],
                # block-scaled e4m3 like the checkpoint this package's MoE path serves
                "quantization_config": {"quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic",
                                        "weight_block_size": [128, 128]}}
    return {**common, "architectures": ["LlamaForCausalLM"], "model_type": "llama", "intermediate_size": cfg.inter,
            "mlp_bias": False, "rope_scaling": None}


def write_model_dir(model: str, path: str) -> str:
    """Writes ``config.json`` (+ ``generation_config.json``) of ``model`` into ``path``."""
    from ..models import config_by_name

    cfg = config_by_name(model)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config(cfg), f, indent=1)
    with open(os.path.join(path, "generation_config.json"), "w") as f:
        json.dump({"bos_token_id": 1, "eos_token_id": 2}, f)
    return path


def run(model: str, batch: int, prompt_len: int, gen: int, graph_sizes: list[int], workdir: str,
        seed: int = 1234) -> dict:
    import torch
    from vllm import LLM, SamplingParams

    from ..models import config_by_name

    cfg = config_by_name(model)
    path = write_model_dir(model, os.path.join(workdir, f"vllm_{model.replace('@', '_')}"))
    t0 = time.perf_counter()
    llm = LLM(model=path, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16", seed=seed,
              max_model_len=prompt_len + gen + 8, max_num_seqs=max(batch, max(graph_sizes)),
              max_num_batched_tokens=max(8192, batch), gpu_memory_utilization=0.85,
              compilation_config={"cudagraph_mode": "FULL_DECODE_ONLY",
                                  "cudagraph_capture_sizes": sorted(s for s in graph_sizes if s <= 512)})
    startup_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(seed)
    prompts = [{"prompt_token_ids": torch.randint(3, cfg.vocab, (prompt_len,), generator=g).tolist()}
               for _ in range(batch)]

    def timed(n_tokens: int) -> tuple[float, int]:
        sp = SamplingParams(max_tokens=n_tokens, temperature=0.0, ignore_eos=True, detokenize=False)
        torch.cuda.synchronize()
        t = time.perf_counter()
        outs = llm.generate(prompts, sp, use_tqdm=False)
        torch.cuda.synchronize()
        return time.perf_counter() - t, sum(len(o.outputs[0].token_ids) for o in outs)

    timed(2)  # warm-up (lazy initialisation, first graph replays)
    t_prefill, _ = timed(1)
    t_full, n_full = timed(gen)
    decode_tokens = n_full - batch
    decode_s = max(t_full - t_prefill, 1e-9)
    return {"startup_s": startup_s, "prefill_s": t_prefill, "decode_s": decode_s, "decode_tokens": decode_tokens,
            "decode_tok_s": decode_tokens / decode_s, "ms_per_step": decode_s * 1e3 / max(gen - 1, 1)}


__all__ = ["hf_config", "run", "write_model_dir"]
