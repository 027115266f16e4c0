"""SGLang integration (SAVE/LOAD of CudaGraphRunner graphs); see hooks.py."""

from .hooks import install_hooks, installed, uninstall_hooks, workspace_rank

__all__ = ["install_hooks", "installed", "uninstall_hooks", "workspace_rank"]
