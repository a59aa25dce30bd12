"""ctypes binding of libraya_attn.so (the C ABI in include/raya_attn.h).

The library is built in-tree by ``python -m raya_b200.build`` (or
``__graft_entry__.build()``).  There is no fallback: if the shared object is
missing, importing this module raises ImportError.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libraya_attn.so")

OK, ERR_SHAPE, ERR_LENGTH, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT = range(6)
MASK_BLOCK, MASK_WINDOW, MASK_FULL = 0, 1, 2
KERNEL_AUTO, KERNEL_TILED64, KERNEL_ROWWISE = 0, 1, 2
KERNEL_TC32_WS = 34
KERNEL_TC32_WS2 = 37
KERNEL_TC16_WS = 40
KERNEL_TC16_WS2 = 41
KERNEL_TILED64_VARIANTS = {"w4r32": 16, "w4r16": 19, "w4r16p2": 20, "w4r32p2": 21}

# Every symbol include/raya_attn.h declares (checked by the ABI test).
EXPORTS = (
    "raya_attn_validate", "raya_attn_forward_host", "raya_attn_forward",
    "raya_attn_forward_ex", "raya_attn_sync_status", "raya_attn_last_error",
    "raya_attn_work", "raya_attn_shard", "raya_attn_fill_normal",
    "raya_attn_ffma_peak", "raya_attn_version", "raya_attn_forward_timed",
    "raya_attn_probe_timeout", "raya_attn_forward_packed", "raya_attn_packed_workspace",
    "raya_attn_forward_packed_noalloc", "raya_attn_kernel_for", "raya_attn_last_error_info",
    "raya_attn_forward_multi_gpu",
)


class Desc(ctypes.Structure):
    """raya_attn_desc."""

    _fields_ = [
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seq", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("block", ctypes.c_int64),
        ("mask", ctypes.c_int32),
        ("halo", ctypes.c_int32),
        ("window", ctypes.c_int64),
        ("scale", ctypes.c_float),
    ]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built; run `python raya_b200/build.py` (the CUDA path has no fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    fp = ctypes.POINTER(ctypes.c_float)
    ip = ctypes.POINTER(ctypes.c_int32)
    dp = ctypes.POINTER(Desc)
    sz = ctypes.c_size_t
    vp = ctypes.c_void_p
    st = ctypes.c_int
    lib.raya_attn_validate.argtypes = [dp, ip, sz, sz, sz, sz]
    lib.raya_attn_validate.restype = st
    lib.raya_attn_forward_host.argtypes = [dp, fp, sz, fp, sz, fp, sz, fp, sz, ip, ctypes.c_int]
    lib.raya_attn_forward_host.restype = st
    lib.raya_attn_forward.argtypes = [dp, vp, vp, vp, vp, vp, vp]
    lib.raya_attn_forward.restype = st
    lib.raya_attn_forward_ex.argtypes = [dp, vp, vp, vp, vp, vp, vp, ctypes.c_int]
    lib.raya_attn_forward_ex.restype = st
    lib.raya_attn_forward_timed.argtypes = [dp, vp, vp, vp, vp, vp, vp, ctypes.c_int, vp]
    lib.raya_attn_forward_timed.restype = st
    lib.raya_attn_forward_packed.argtypes = [dp, vp, vp, vp, ctypes.c_float, vp, sz, vp]
    lib.raya_attn_forward_packed.restype = st
    lib.raya_attn_packed_workspace.argtypes = [dp, ctypes.c_float, ctypes.POINTER(ctypes.c_size_t)]
    lib.raya_attn_packed_workspace.restype = st
    lib.raya_attn_forward_packed_noalloc.argtypes = [dp, vp, vp, vp, ctypes.c_float, vp]
    lib.raya_attn_forward_packed_noalloc.restype = st
    lib.raya_attn_probe_timeout.argtypes = [ctypes.c_int64, vp]
    lib.raya_attn_probe_timeout.restype = st
    lib.raya_attn_sync_status.argtypes = [vp]
    lib.raya_attn_sync_status.restype = st
    lib.raya_attn_last_error.argtypes = []
    lib.raya_attn_last_error.restype = ctypes.c_char_p
    lib.raya_attn_last_error_info.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_char_p),
                                              ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]
    lib.raya_attn_last_error_info.restype = st
    lib.raya_attn_forward_multi_gpu.argtypes = [dp, fp, sz, fp, sz, fp, sz, fp, sz, ip,
                                                ctypes.POINTER(ctypes.c_int), ctypes.c_int, vp]
    lib.raya_attn_forward_multi_gpu.restype = st
    lib.raya_attn_work.argtypes = [dp, ip, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
    lib.raya_attn_work.restype = st
    lib.raya_attn_shard.argtypes = [dp, ip, ctypes.c_int, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]
    lib.raya_attn_shard.restype = st
    lib.raya_attn_fill_normal.argtypes = [vp, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32,
                                          ctypes.c_int64, ctypes.c_float, vp]
    lib.raya_attn_fill_normal.restype = st
    lib.raya_attn_ffma_peak.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
    lib.raya_attn_ffma_peak.restype = st
    lib.raya_attn_kernel_for.argtypes = [dp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.raya_attn_kernel_for.restype = st
    lib.raya_attn_version.argtypes = []
    lib.raya_attn_version.restype = ctypes.c_int
    return lib


lib = _load()


def last_error() -> str:
    return lib.raya_attn_last_error().decode("utf-8", "replace")
