"""raya_b200 — B200-native (sm_100a) block-local attention for raya.

The hot path of raya's encoder (crates/raya-kernels, the tiled block-local
attention kernel) as hand-written CUDA behind raya's own AttentionKernel
contract.  ``libraya_attn.so`` (C ABI: include/raya_attn.h) is the product;
this package is its host-side mirror of the reference interface.

The library is loaded on first use of any name below (PEP 562), not by
``import raya_b200`` itself: ``raya_b200.workloads`` (the benchmark
configurations) is plain numpy and imports without it.  There is still no
fallback: the first attribute that needs the library raises ImportError when
``raya_b200/_lib/libraya_attn.so`` has not been built.
"""
from __future__ import annotations

import importlib

_FROM_ATTENTION = (
    "BLOCK", "WINDOW", "AttentionKernel", "AttnParams", "AttnShape", "Cuda", "CudaConfig", "CudaError",
    "DeviceTimeout", "KernelError", "LengthError", "Mask", "ShapeError", "UnsupportedError", "ErrorInfo",
    "fill_normal", "ffma_peak", "kernel_for", "last_error_info", "make_desc", "multi_gpu", "shard", "stage_times",
    "sync_status", "validate", "work",
)
_FROM_LIB = (
    "KERNEL_AUTO", "KERNEL_ROWWISE", "KERNEL_TC16_WS", "KERNEL_TC16_WS2", "KERNEL_TC32_WS", "KERNEL_TC32_WS2",
    "KERNEL_TILED64",
    "LIB_PATH",
)

__all__ = [*_FROM_ATTENTION, *_FROM_LIB]


def __getattr__(name: str):
    if name in _FROM_ATTENTION:
        value = getattr(importlib.import_module(".attention", __name__), name)
    elif name in _FROM_LIB:
        value = getattr(importlib.import_module("._lib", __name__), name)
    else:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(__all__))
