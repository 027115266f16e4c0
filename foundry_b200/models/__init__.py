"""Model families of the serving runner.

``llama``      dense Llama-3 decoder (bf16), tensor-parallel capable
``qwen3_moe``  Qwen3-MoE decoder with block-scaled fp8 weights, expert-parallel capable
"""

from __future__ import annotations

from . import llama, qwen3_moe
from .llama import LlamaConfig, LlamaModel, LlamaWeights
from .qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel, Qwen3MoeWeights

CONFIGS = {**llama.CONFIGS, **qwen3_moe.CONFIGS}

_FAMILIES = {
    "llama": (LlamaConfig, LlamaWeights, LlamaModel),
    "qwen3_moe": (Qwen3MoeConfig, Qwen3MoeWeights, Qwen3MoeModel),
}


def family(cfg):
    """(config class, weights class, model class) of a config."""
    return _FAMILIES[getattr(cfg, "arch", "llama")]


def config_from_dict(d: dict):
    d = dict(d)
    cls = _FAMILIES[d.get("arch", "llama")][0]
    return cls(**d)


def config_by_name(name: str):
    """A named config; ``<name>@<N>l`` (or the older ``llama-3-8b-<N>l``) keeps
    the per-layer shapes and sets the layer count (tests, quick runs)."""
    layers = None
    if "@" in name:
        name, suffix = name.split("@", 1)
        layers = int(suffix.rstrip("l"))
    elif name.startswith("llama-3-8b-") and name.endswith("l"):
        name, layers = "llama-3-8b", int(name[len("llama-3-8b-"):-1])
    if name not in CONFIGS:
        raise KeyError(f"unknown model {name!r}; known: {sorted(CONFIGS)}")
    cfg = CONFIGS[name]()
    if layers:
        cfg.layers = layers
        cfg.name = f"{cfg.name}-{layers}l"
    return cfg


__all__ = ["CONFIGS", "LlamaConfig", "LlamaModel", "LlamaWeights", "Qwen3MoeConfig", "Qwen3MoeModel",
           "Qwen3MoeWeights", "config_by_name", "config_from_dict", "family"]
