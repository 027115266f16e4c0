"""vLLM integration (SAVE/LOAD of the engine's CUDA graphs); see hooks.py."""

from .hooks import install_hooks, installed, uninstall_hooks

__all__ = ["install_hooks", "installed", "uninstall_hooks"]
