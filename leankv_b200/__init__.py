"""leankv_b200 — B200-native (sm_100a) TurboQuant KV-cache hot path.

Drop-in for LeanKV's src/ggml-tq.c quantize / dequantize / Hadamard API (C ABI
in include/leankv_tq.h, library in leankv_b200/_lib/) plus the fused decode
attention that reads packed TQ blocks.  Torch tensors go through
``leankv_b200.ops``.
"""
from . import _lib
from ._lib import TQError

__all__ = ["TQError", "ops", "load_library"]


def load_library():
    """Load libleankv_tq.so (raises if it has not been built)."""
    return _lib.load()


def __getattr__(name):
    # torch-backed submodules load on first use so the C-ABI layer imports without torch
    if name in ("ops", "attention", "distributed", "turboquant"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
