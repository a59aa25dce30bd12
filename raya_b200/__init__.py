"""raya_b200 — B200-native (sm_100a) block-local attention for raya.

The hot path of raya's encoder (crates/raya-kernels, the tiled block-local
attention kernel) as hand-written CUDA behind raya's own AttentionKernel
contract.  ``libraya_attn.so`` (C ABI: include/raya_attn.h) is the product;
this package is its host-side mirror of the reference interface.
"""
from .attention import (BLOCK, WINDOW, AttentionKernel, AttnParams, AttnShape, Cuda, CudaConfig,
                        CudaError, DeviceTimeout, KernelError, LengthError, Mask, ShapeError,
                        UnsupportedError, fill_normal, ffma_peak, kernel_for, make_desc, shard,
                        stage_times, sync_status, validate, work)
from ._lib import (KERNEL_AUTO, KERNEL_ROWWISE, KERNEL_TC32, KERNEL_TC32_PIPE, KERNEL_TC32_STREAM, KERNEL_TC32_WS,
                   KERNEL_TC32_WS2, KERNEL_TILED64, LIB_PATH)

__all__ = [
    "BLOCK", "WINDOW", "AttentionKernel", "AttnParams", "AttnShape", "Cuda", "CudaConfig",
    "CudaError", "DeviceTimeout", "KernelError", "LengthError", "Mask", "ShapeError",
    "UnsupportedError", "fill_normal", "ffma_peak", "kernel_for", "make_desc", "shard", "stage_times", "sync_status",
    "validate", "work", "KERNEL_AUTO", "KERNEL_ROWWISE", "KERNEL_TC32", "KERNEL_TC32_PIPE", "KERNEL_TC32_STREAM",
    "KERNEL_TC32_WS", "KERNEL_TC32_WS2", "KERNEL_TILED64", "LIB_PATH",
]
