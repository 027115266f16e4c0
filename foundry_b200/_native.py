"""Loads the native core module (``foundry_b200._C``).

The module is built in-tree by ``foundry_b200._build`` (``__graft_entry__.build()``
or ``python -m foundry_b200._build``). Importing it never triggers a build: a
missing extension raises with the command to run, so a GPU run can never fall
back silently to a non-native path.
"""

from __future__ import annotations

import importlib
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "lib"
KERNEL_DIR = PKG_DIR / "kernels"
HOOK_LIB = LIB_DIR / "libfoundry_hook.so"
MOCK_DRIVER = LIB_DIR / "libfoundry_mockcuda.so"

_C = None


def core():
    """Returns the native module, importing it on first use."""
    global _C
    if _C is None:
        try:
            _C = importlib.import_module("foundry_b200._C")
        except ImportError as e:  # pragma: no cover - exercised only on a broken install
            raise ImportError(
                "foundry_b200 native core is not built; run `python -m foundry_b200._build` "
                f"(or __graft_entry__.build()): {e}"
            ) from e
    return _C


def use_mock_driver() -> None:
    """Points the native layer at the CPU mock driver (tests on a box without a GPU).

    Must run before the first driver call of the process.
    """
    os.environ["FOUNDRY_CUDA_DRIVER"] = str(MOCK_DRIVER)


def hook_library_path() -> str:
    """Path of the LD_PRELOAD interposer library."""
    return str(HOOK_LIB)
