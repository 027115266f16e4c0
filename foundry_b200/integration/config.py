"""Graph-extension configuration shared by the engine integrations.

A TOML file selects the mode and the deterministic region:

    mode = "save"                 # "none" | "save" | "load"
    base_addr = "0x600000000000"  # region base (same in SAVE and LOAD)
    region_size = "64GB"
    workspace_root = "foundry_archive"
    scratch_space_size = "64MB"   # skipped after the communicator init
    # hook_library_path = ".../libfoundry_hook.so"   (auto-detected)

Keys and defaults follow the reference's TOML (reference
python/foundry/integration/vllm/config.py:26-80) so existing config files work;
a per-rank workspace ``<workspace_root>/rank_<global rank>`` holds each
process's archive.
"""

from __future__ import annotations

import enum
import os
import tomllib
from dataclasses import dataclass, field
from pathlib import Path

from ..allocation_region import parse_size


class GraphExtensionMode(str, enum.Enum):
    NONE = "none"
    SAVE = "save"
    LOAD = "load"


def hook_library_path() -> str | None:
    from .._native import HOOK_LIB

    return str(HOOK_LIB) if Path(HOOK_LIB).exists() else None


@dataclass
class GraphExtensionConfig:
    mode: GraphExtensionMode = GraphExtensionMode.NONE
    base_addr: int = 0x600000000000
    region_size: str = "64GB"
    workspace_root: str = "foundry_archive"
    scratch_space_size: str = "64MB"
    hook_library_path: str | None = field(default_factory=hook_library_path)
    workspace_dir: str | None = None  # set per rank by the runtime

    @classmethod
    def from_toml(cls, path: str | os.PathLike) -> "GraphExtensionConfig":
        with open(path, "rb") as f:
            data = tomllib.load(f)
        return cls.from_dict(data)

    @classmethod
    def from_dict(cls, data: dict) -> "GraphExtensionConfig":
        known = {"mode", "base_addr", "region_size", "workspace_root", "scratch_space_size", "hook_library_path",
                 "nvshmem_host_path"}
        unknown = set(data) - known
        if unknown:
            raise ValueError(f"unknown graph-extension keys: {sorted(unknown)}")
        base = data.get("base_addr", cls.base_addr)
        base = int(base, 0) if isinstance(base, str) else int(base)
        cfg = cls(
            mode=GraphExtensionMode(str(data.get("mode", "none")).lower()),
            base_addr=base,
            region_size=str(data.get("region_size", cls.region_size)),
            workspace_root=str(data.get("workspace_root", cls.workspace_root)),
            scratch_space_size=str(data.get("scratch_space_size", cls.scratch_space_size)),
        )
        if data.get("hook_library_path"):
            cfg.hook_library_path = str(data["hook_library_path"])
        parse_size(cfg.region_size)
        if parse_size(cfg.scratch_space_size) >= parse_size(cfg.region_size):
            raise ValueError("scratch_space_size must be smaller than region_size")
        return cfg

    def workspace_for(self, global_rank: int) -> str:
        return os.path.join(self.workspace_root, f"rank_{global_rank}")


def global_rank(rank: int, world_size: int, dp_rank: int = 0) -> int:
    """Rank used for the workspace folder: data-parallel replicas are stacked
    after each other (dp_rank * world_size + rank), as in the reference
    (python/foundry/integration/vllm/config.py:130-142)."""
    return dp_rank * world_size + rank


__all__ = ["GraphExtensionConfig", "GraphExtensionMode", "global_rank", "hook_library_path"]
