"""Loader for the in-tree native extension (``_ashqk_torch.so`` + ``libashqk_b200.so``).

There is no fallback: if the extension is missing, every kernel entry point
raises. Build it with ``python ash-quant-kernels_b200/build.py``.
"""

from __future__ import annotations

import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
TORCH_BINDING = os.path.join(_HERE, "_ashqk_torch.so")
C_LIBRARY = os.path.join(_HERE, "libashqk_b200.so")

_lock = threading.Lock()
_loaded = False


class ExtensionMissing(ImportError):
    """The sm_100a extension has not been built into the package directory."""


def ops():
    """Return ``torch.ops.ashqk``, loading the native binding on first use."""
    global _loaded
    if not _loaded:
        with _lock:
            if not _loaded:
                if not os.path.exists(TORCH_BINDING):
                    raise ExtensionMissing(
                        f"ashqk: native extension not found at {TORCH_BINDING}; "
                        "build it with `python ash-quant-kernels_b200/build.py`")
                torch.ops.load_library(TORCH_BINDING)
                _loaded = True
    return torch.ops.ashqk
