"""raya's attention contract, mirrored over the B200 library.

Python restatement of crates/raya-kernels/src/attention.rs (paths relative to
the raya project root) so that callers and tests read like the reference's:

* ``BLOCK`` / ``WINDOW``                       attention.rs:3-6
* ``KernelError`` and its three kinds          attention.rs:8-20 (plus device errors)
* ``Mask`` with ``key_range`` / ``allows``     attention.rs:22-70 (generalised:
  ``Mask.block(halo)``, ``Mask.sliding(w)``; ``BLOCK3`` = halo 1,
  ``WINDOW64`` = sliding(64))
* ``AttnShape`` / ``AttnParams``               attention.rs:72-106 (a ``batch``
  dimension and per-sequence ``valid_len``)
* ``AttentionKernel``                          attention.rs:108-125
* ``validate``                                 attention.rs:127-170

``Cuda`` is the drop-in kernel: ``attend`` takes host buffers like the Rust
trait (``raya_attn_forward_host``); ``attend_device`` takes CUDA tensors that
already live in HBM (``raya_attn_forward``).  Every compute call goes to the
CUDA library; there is no CPU path.
"""
from __future__ import annotations

import abc
import ctypes
from dataclasses import dataclass, field
from typing import Sequence, Union

import numpy as np

from . import _lib
from ._lib import Desc, lib

BLOCK = 128   # attention.rs:4 — Laya's block_local block size
WINDOW = 64   # attention.rs:6 — half width of the exact local window


class KernelError(Exception):
    """attention.rs:8-20.  ``str(err)`` is the reference's Display text."""


class ShapeError(KernelError):
    """KernelError::Shape"""


class LengthError(KernelError):
    """KernelError::Length { name, got, expected }"""

    def __init__(self, message: str, name: str = "", got: int = 0, expected: int = 0):
        super().__init__(message)
        self.name, self.got, self.expected = name, got, expected


class UnsupportedError(KernelError):
    """KernelError::Unsupported"""


class CudaError(KernelError):
    """A CUDA runtime call failed (no reference counterpart)."""


class DeviceTimeout(KernelError):
    """A bounded device-side wait gave up (no reference counterpart)."""


_ERRORS = {
    _lib.ERR_SHAPE: ShapeError,
    _lib.ERR_LENGTH: LengthError,
    _lib.ERR_UNSUPPORTED: UnsupportedError,
    _lib.ERR_CUDA: CudaError,
    _lib.ERR_TIMEOUT: DeviceTimeout,
}


@dataclass(frozen=True)
class ErrorInfo:
    """The calling thread's last library error as data
    (``raya_attn_last_error_info``): ``kind`` is the status code; ``name``,
    ``got`` and ``expected`` are KernelError::Length's fields
    (attention.rs:13-18) for length errors, else "", 0, 0."""

    kind: int
    name: str
    got: int
    expected: int


def last_error_info() -> ErrorInfo:
    kind, name = ctypes.c_int(), ctypes.c_char_p()
    got, expected = ctypes.c_size_t(), ctypes.c_size_t()
    lib.raya_attn_last_error_info(ctypes.byref(kind), ctypes.byref(name), ctypes.byref(got), ctypes.byref(expected))
    return ErrorInfo(kind.value, (name.value or b"").decode(), got.value, expected.value)


def _check(status: int) -> None:
    if status == _lib.OK:
        return
    msg = _lib.last_error()
    cls = _ERRORS.get(status, KernelError)
    if cls is LengthError:
        info = last_error_info()
        raise LengthError(msg, name=info.name, got=info.got, expected=info.expected)
    raise cls(msg)


@dataclass(frozen=True)
class Mask:
    """Which keys a query may attend (besides ``j < valid_len``)."""

    kind: int
    param: int = 0  # halo for BLOCK masks, half width for WINDOW masks

    @staticmethod
    def block(halo: int) -> "Mask":
        """Query block b sees key blocks b-halo ..= b+halo (halo 1 = Block3)."""
        return Mask(_lib.MASK_BLOCK, halo)

    @staticmethod
    def sliding(w: int) -> "Mask":
        """Exact window |i - j| <= w (w = 64 is Window64)."""
        return Mask(_lib.MASK_WINDOW, w)

    def name(self) -> str:  # attention.rs:38-45
        if self.kind == _lib.MASK_BLOCK:
            return "block3" if self.param == 1 else f"block{2 * self.param + 1}"
        if self.kind == _lib.MASK_WINDOW:
            return "window64" if self.param == WINDOW else "sliding"
        return "full"

    def key_range(self, i: int, valid_len: int, block: int = BLOCK) -> range:
        """attention.rs:48-59 with BLOCK -> block and 1 -> halo."""
        if self.kind == _lib.MASK_BLOCK:
            b = i // block
            lo, hi = max(b - self.param, 0) * block, (b + self.param + 1) * block
        elif self.kind == _lib.MASK_WINDOW:
            lo, hi = max(i - self.param, 0), i + self.param + 1
        else:
            lo, hi = 0, valid_len
        return range(min(lo, valid_len), min(hi, valid_len))

    def allows(self, i: int, j: int, block: int = BLOCK) -> bool:
        """attention.rs:62-69, ignoring valid_len."""
        if self.kind == _lib.MASK_BLOCK:
            return abs(i // block - j // block) <= self.param
        if self.kind == _lib.MASK_WINDOW:
            return abs(i - j) <= self.param
        return True


Mask.BLOCK3 = Mask.block(1)
Mask.WINDOW64 = Mask.sliding(WINDOW)
Mask.FULL = Mask(_lib.MASK_FULL, 0)


@dataclass(frozen=True)
class AttnShape:
    """Buffers are ``[batch][heads][seq][head_dim]`` row-major fp32
    (attention.rs:72-84 is batch = 1)."""

    heads: int
    seq: int
    head_dim: int
    batch: int = 1

    def numel(self) -> int:
        return self.batch * self.heads * self.seq * self.head_dim


ValidLen = Union[int, Sequence[int], np.ndarray]


@dataclass(frozen=True)
class AttnParams:
    """attention.rs:86-106.  ``valid_len`` is one length for every batch
    entry or one per batch entry."""

    mask: Mask
    block: int
    valid_len: ValidLen
    scale: float

    @staticmethod
    def new(mask: Mask, valid_len: ValidLen, head_dim: int, block: int = BLOCK) -> "AttnParams":
        # attention.rs:103: 1.0 / (head_dim as f32).sqrt(), computed in f32
        scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
        return AttnParams(mask=mask, block=block, valid_len=valid_len, scale=scale)

    def valid_array(self, batch: int) -> np.ndarray:
        v = np.asarray(self.valid_len, dtype=np.int64)
        if v.ndim == 0:
            v = np.full(batch, int(v), dtype=np.int64)
        if v.shape != (batch,):
            raise ShapeError(f"invalid shape: {v.size} valid lengths for batch {batch}")
        if (v < -2**31).any() or (v > 2**31 - 1).any():
            raise ShapeError("invalid shape: valid_len out of int32 range")
        return np.ascontiguousarray(v.astype(np.int32))


def make_desc(shape: AttnShape, params: AttnParams) -> Desc:
    m = params.mask
    return Desc(batch=shape.batch, heads=shape.heads, seq=shape.seq, head_dim=shape.head_dim,
                block=params.block, mask=m.kind,
                halo=m.param if m.kind == _lib.MASK_BLOCK else 0,
                window=m.param if m.kind == _lib.MASK_WINDOW else 0,
                scale=params.scale)


def _i32p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def _f32p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _host_f32(name: str, a, writable: bool = False) -> np.ndarray:
    arr = np.asarray(a)
    if arr.dtype != np.float32:
        raise TypeError(f"buffer `{name}` must be float32, got {arr.dtype}")
    if writable:
        if not arr.flags["C_CONTIGUOUS"] or not arr.flags["WRITEABLE"]:
            raise TypeError(f"buffer `{name}` must be a writable C-contiguous array")
        return arr
    return np.ascontiguousarray(arr)


def validate(shape: AttnShape, params: AttnParams, q, k, v, out) -> None:
    """attention.rs:128-170 over the batch layout; raises KernelError."""
    valid = params.valid_array(shape.batch)
    lens = {n: int(np.asarray(b).size) for n, b in (("q", q), ("k", k), ("v", v), ("out", out))}
    d = make_desc(shape, params)
    _check(lib.raya_attn_validate(ctypes.byref(d), _i32p(valid), lens["q"], lens["k"], lens["v"],
                                  lens["out"]))


def work(shape: AttnShape, params: AttnParams) -> tuple[int, int]:
    """Exact (allowed pairs, valid query rows); FLOPs = 4 * head_dim * pairs."""
    valid = params.valid_array(shape.batch)
    d = make_desc(shape, params)
    pairs, rows = ctypes.c_uint64(), ctypes.c_uint64()
    _check(lib.raya_attn_work(ctypes.byref(d), _i32p(valid), ctypes.byref(pairs), ctypes.byref(rows)))
    return pairs.value, rows.value


def multi_gpu(shape: AttnShape, params: AttnParams, q, k, v, out=None, devices: Sequence[int] = (0,),
              out_device0=None) -> None:
    """The host-buffer call over several GPUs of this process
    (``raya_attn_forward_multi_gpu``): batch x heads slices split by
    allowed-pair count, one range per device, all devices at once.  ``out``
    is a host float32 array or None; ``out_device0`` (a CUDA float32 tensor
    of the whole output on ``devices[0]``, or None) also receives every
    device's part by peer copies.  Synchronous."""
    valid = params.valid_array(shape.batch)
    qh, kh, vh = _host_f32("q", q), _host_f32("k", k), _host_f32("v", v)
    oh = _host_f32("out", out, writable=True) if out is not None else None
    devs = (ctypes.c_int * len(devices))(*devices)
    d0 = None
    if out_device0 is not None:
        if not out_device0.is_cuda or not out_device0.is_contiguous() or out_device0.device.index != devices[0]:
            raise TypeError("out_device0 must be a contiguous CUDA tensor on devices[0]")
        d0 = out_device0.data_ptr()
    d = make_desc(shape, params)
    _check(lib.raya_attn_forward_multi_gpu(ctypes.byref(d), _f32p(qh), qh.size, _f32p(kh), kh.size, _f32p(vh),
                                           vh.size, _f32p(oh) if oh is not None else None,
                                           oh.size if oh is not None else 0, _i32p(valid), devs, len(devices), d0))


def kernel_for(shape: AttnShape, params: AttnParams, packed: bool = False, rope: bool = False) -> int:
    """The kernel id the automatic choice launches for this call, in the
    head-major or (``packed``) the caller's packed layout, there with or
    without the rotation (``rope``) (host-only)."""
    d = make_desc(shape, params)
    kid = ctypes.c_int()
    _check(lib.raya_attn_kernel_for(ctypes.byref(d), (2 if rope else 1) if packed else 0, ctypes.byref(kid)))
    return kid.value


def shard(shape: AttnShape, params: AttnParams, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of flattened batch*heads slices owned by ``rank``."""
    valid = params.valid_array(shape.batch)
    d = make_desc(shape, params)
    b, e = ctypes.c_int64(), ctypes.c_int64()
    _check(lib.raya_attn_shard(ctypes.byref(d), _i32p(valid), world, rank, ctypes.byref(b),
                               ctypes.byref(e)))
    return b.value, e.value


class AttentionKernel(abc.ABC):
    """attention.rs:108-125: the single entry point for attention."""

    @abc.abstractmethod
    def name(self) -> str: ...

    @abc.abstractmethod
    def attend(self, shape: AttnShape, params: AttnParams, q, k, v, out) -> None: ...


@dataclass
class CudaConfig:
    """Counterpart of TiledConfig (tiled/mod.rs:14-19): which GPU runs it."""

    device: int = 0
    kernel: int = field(default=_lib.KERNEL_AUTO)


class Cuda(AttentionKernel):
    """The B200 block-local attention kernel behind the reference's trait."""

    def __init__(self, config: CudaConfig | None = None):
        self.config = config or CudaConfig()

    def name(self) -> str:
        return "cuda-b200"

    def attend(self, shape: AttnShape, params: AttnParams, q, k, v, out) -> None:
        """Host buffers in, host buffer out, synchronous (attention.rs:116-124)."""
        valid = params.valid_array(shape.batch)
        qh, kh, vh = _host_f32("q", q), _host_f32("k", k), _host_f32("v", v)
        oh = _host_f32("out", out, writable=True)
        d = make_desc(shape, params)
        _check(lib.raya_attn_forward_host(ctypes.byref(d), _f32p(qh), qh.size, _f32p(kh), kh.size,
                                          _f32p(vh), vh.size, _f32p(oh), oh.size, _i32p(valid),
                                          self.config.device))

    def attend_device(self, shape: AttnShape, params: AttnParams, q, k, v, out,
                      valid_len=None, stream=None, kernel: int | None = None) -> None:
        """Device tensors (torch CUDA tensors or raw pointers) on ``stream``,
        asynchronous.  ``valid_len`` is a device int32 tensor / pointer, or
        None to upload ``params.valid_len`` here (a synchronous copy)."""
        import torch

        def ptr(x):
            if isinstance(x, torch.Tensor):
                if not x.is_cuda or x.dtype not in (torch.float32, torch.int32) or not x.is_contiguous():
                    raise TypeError("device buffers must be contiguous CUDA float32/int32 tensors")
                return x.data_ptr()
            return int(x) if x is not None else None

        keep = None
        if valid_len is None:
            keep = torch.from_numpy(params.valid_array(shape.batch)).to(
                q.device if isinstance(q, torch.Tensor) else "cuda")
            valid_len = keep
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream
        elif isinstance(stream, torch.cuda.Stream):
            stream = stream.cuda_stream
        d = make_desc(shape, params)
        kid = self.config.kernel if kernel is None else kernel
        _check(lib.raya_attn_forward_ex(ctypes.byref(d), ptr(q), ptr(k), ptr(v), ptr(out),
                                        ptr(valid_len), stream, kid))
        if keep is not None:  # keep the uploaded lengths alive until the kernel has run
            _sync(stream)

    def attend_packed(self, shape: AttnShape, params: AttnParams, qkv, ctx, valid_len=None,
                      rope_theta: float | None = None, workspace=None, stream=None) -> None:
        """The encoder's attention step in its own layout (encoder.rs:57-92):
        qkv is the packed projection [batch][seq][3][heads][64] and ctx the
        context [batch][seq][heads][64], both CUDA float32 tensors; with
        rope_theta, q and k get raya's rotary embedding (ops.rs:110-141)
        first.  Asynchronous on ``stream``, except that uploading
        ``params.valid_len`` (``valid_len`` None) waits for the call, as in
        attend_device.  A caller's ``workspace`` must stay allocated until
        the call has run; one allocated here is held for the stream by
        torch's caching allocator."""
        import torch

        d = make_desc(shape, params)
        theta = float(rope_theta or 0.0)
        need = ctypes.c_size_t()
        _check(lib.raya_attn_packed_workspace(ctypes.byref(d), theta, ctypes.byref(need)))
        own_workspace = workspace is None and need.value > 0
        if own_workspace:
            workspace = torch.empty(need.value // 4, dtype=torch.float32, device=qkv.device)
        keep = valid_len
        if keep is None:
            keep = torch.from_numpy(params.valid_array(shape.batch)).to(qkv.device)
        if stream is None:
            stream = torch.cuda.current_stream(qkv.device).cuda_stream
        elif isinstance(stream, torch.cuda.Stream):
            stream = stream.cuda_stream
        ws_ptr = workspace.data_ptr() if workspace is not None else None
        ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
        _check(lib.raya_attn_forward_packed(ctypes.byref(d), qkv.data_ptr(), ctx.data_ptr(), keep.data_ptr(),
                                            theta, ws_ptr, ws_bytes, stream))
        if own_workspace:  # not reused by the allocator before the work queued on `stream` has run
            workspace.record_stream(torch.cuda.ExternalStream(stream, device=qkv.device))
        if valid_len is None:  # keep the uploaded lengths alive until the kernel has run
            _sync(stream)


STAGE_NAMES = ("qk", "softmax", "pv", "k_wait", "v_wait", "refill", "tiles", "total")


def stage_times(shape: AttnShape, params: AttnParams, q, k, v, out, valid_len=None,
                kernel: int = _lib.KERNEL_TILED64, stream=None) -> dict:
    """Runs a kernel once with per-stage clocks (the counterpart of
    Tiled::attend_with_stages, tiled/mod.rs:60-126) and returns the cycles
    per stage plus qk/softmax/pv percentages of their total
    (StageTimes::percentages, tiled/stages.rs:19-31).  ``kernel``: a tiled
    kernel (warp cycles per stage), or KERNEL_TC32_WS / KERNEL_TC32_WS2 /
    KERNEL_TC16_WS / KERNEL_TC16_WS2 / KERNEL_AUTO for the tensor-core kernels (per-CTA cycles of QK^T and PV
    products in flight and of one softmax warp; these overlap in time)."""
    import torch

    dev = q.device
    counters = torch.zeros(len(STAGE_NAMES), dtype=torch.int64, device=dev)
    keep = valid_len
    if keep is None:
        keep = torch.from_numpy(params.valid_array(shape.batch)).to(dev)
    if stream is None:
        stream = torch.cuda.current_stream(dev).cuda_stream
    d = make_desc(shape, params)
    _check(lib.raya_attn_forward_timed(ctypes.byref(d), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                       out.data_ptr(), keep.data_ptr(), stream, kernel,
                                       counters.data_ptr()))
    _sync(stream)
    c = dict(zip(STAGE_NAMES, (int(x) for x in counters.cpu().tolist())))
    work_cycles = c["qk"] + c["softmax"] + c["pv"]
    if work_cycles:
        c["qk_pct"] = 100.0 * c["qk"] / work_cycles
        c["softmax_pct"] = 100.0 * c["softmax"] / work_cycles
        c["pv_pct"] = 100.0 * c["pv"] / work_cycles
    if c["total"]:
        for name in ("qk", "softmax", "pv", "k_wait", "v_wait", "refill"):
            c[name + "_of_total_pct"] = 100.0 * c[name] / c["total"]
    return c


def _sync(stream) -> None:
    _check(lib.raya_attn_sync_status(ctypes.c_void_p(stream)))


def sync_status(stream=None) -> None:
    """Synchronise ``stream`` and raise DeviceTimeout if a device-side wait
    gave up since the last check."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    elif isinstance(stream, torch.cuda.Stream):
        stream = stream.cuda_stream
    _sync(stream)


def fill_normal(tensor, seed: int, stream_id: int, first_index: int = 0, stddev: float = 1.0,
                stream=None) -> None:
    """Seeded N(0, stddev^2) values into a CUDA float32 tensor (device-side)."""
    import torch

    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    _check(lib.raya_attn_fill_normal(tensor.data_ptr(), tensor.numel(), seed, stream_id, first_index,
                                     stddev, stream))


def ffma_peak(reps: int = 5) -> float:
    """Measured FP32 FFMA throughput of the current GPU, TFLOP/s."""
    out = ctypes.c_double()
    _check(lib.raya_attn_ffma_peak(reps, ctypes.byref(out)))
    return out.value
