"""SGLang integration (SAVE/LOAD of CudaGraphRunner graphs); see hooks.py."""

from .hooks import install_hooks, uninstall_hooks

__all__ = ["install_hooks", "uninstall_hooks"]
