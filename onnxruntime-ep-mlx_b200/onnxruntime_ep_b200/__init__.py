"""B200-native paged-KV attention path of an ONNX Runtime plugin execution provider.

Mirrors the reference package's helper surface (python/src/onnxruntime_ep_mlx/__init__.py:43-167):
``EP_NAME``, ``library_path()`` and ``register_execution_provider_library()``, plus direct
operator entry points (``paged_attention``, ``kv_append``) over the C ABI in
``include/b200_paged.h``.
"""

from __future__ import annotations

import os

from ._capi import LIB, B200Error, library_file
from .paged import kv_append, paged_attention

EP_NAME = "B200ExecutionProvider"
EP_SHELL_NAME = "libonnxruntime_ep_b200.so"

__all__ = [
    "EP_NAME",
    "B200Error",
    "kv_append",
    "library_path",
    "kernel_library_path",
    "paged_attention",
    "register_execution_provider_library",
]


def kernel_library_path() -> str:
    """Path of the kernel library (C ABI of include/b200_paged.h)."""
    return library_file()


def library_path() -> str:
    """Path of the ORT plugin-EP shell library (exports ``CreateEpFactories``).

    The shell is built only where ONNX Runtime's plugin-EP headers are available
    (``ORT_INCLUDE_DIR``); without it this raises, as the reference helper does for a missing
    dylib (__init__.py:77-94).
    """
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), EP_SHELL_NAME)
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} not found: build the EP shell with ORT_INCLUDE_DIR pointing at ONNX Runtime "
            ">= 1.31 headers")
    return path


def register_execution_provider_library(name: str = EP_NAME, path: str | None = None):
    """Register the plugin EP with ONNX Runtime (reference __init__.py:108-133)."""
    import onnxruntime as ort  # deferred: the kernels themselves need no ORT

    ort.register_execution_provider_library(name, path or library_path())
    return name
