"""The C ABI on a host without a GPU: the library loads, exports every entry
point include/raya_attn.h declares, and its host-side logic (argument
validation, work counts, the shard partition) behaves like the reference's
(crates/raya-kernels/src/attention.rs:128-170, tests/oracle.rs:35-78)."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import oracle
import raya_b200 as rb
from raya_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "raya_attn.h")).read()
    return sorted(set(re.findall(r"\b(raya_attn_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    declared = header_symbols()
    assert declared, "no declarations found"
    assert sorted(_lib.EXPORTS) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (raya_attn_\w+)", out.stdout))
    missing = [s for s in declared if s not in exported]
    assert not missing, f"not exported: {missing}"
    for s in declared:
        assert hasattr(_lib.lib, s)
    assert _lib.lib.raya_attn_version() == 1


def _shape(heads=1, seq=4, d=8, batch=1):
    return rb.AttnShape(heads=heads, seq=seq, head_dim=d, batch=batch)


def test_bad_arguments_are_errors_not_panics():
    """tests/oracle.rs:35-78, through the library's validate."""
    shape = _shape()
    ok = np.zeros(shape.numel(), dtype=np.float32)
    p = rb.AttnParams.new(rb.Mask.BLOCK3, 4, 8)
    with pytest.raises(rb.LengthError) as e:
        rb.validate(shape, p, np.zeros(3, np.float32), ok, ok, ok)
    assert e.value.name == "q" and e.value.got == 3 and e.value.expected == 32
    assert str(e.value) == "buffer `q` has length 3, expected 32"
    with pytest.raises(rb.LengthError) as e:
        rb.validate(shape, p, ok, ok, ok, np.zeros(3, np.float32))
    assert e.value.name == "out"
    bad = _shape(d=12)
    buf = np.zeros(bad.numel(), np.float32)
    with pytest.raises(rb.ShapeError, match="not a multiple of 8"):
        rb.validate(bad, p, buf, buf, buf, buf)
    with pytest.raises(rb.ShapeError, match="exceeds seq"):
        rb.validate(shape, rb.AttnParams.new(rb.Mask.BLOCK3, 5, 8), ok, ok, ok, ok)
    with pytest.raises(rb.ShapeError, match="at least 1"):
        z = _shape(heads=0)
        rb.validate(z, p, ok[:0], ok[:0], ok[:0], ok[:0])
    # The reference rejects block != 128; this library accepts any block >= 1
    # and rejects block 0 with the same error kind.
    with pytest.raises(rb.UnsupportedError):
        rb.validate(shape, rb.AttnParams(rb.Mask.BLOCK3, 0, 4, p.scale), ok, ok, ok, ok)
    rb.validate(shape, rb.AttnParams(rb.Mask.BLOCK3, 64, 4, p.scale), ok, ok, ok, ok)
    with pytest.raises(rb.UnsupportedError, match="head_dim"):
        big = _shape(d=264)
        b = np.zeros(big.numel(), np.float32)
        rb.validate(big, p, b, b, b, b)


def test_host_call_validates_before_touching_the_gpu():
    """The host-buffer entry point raises the reference's errors without a
    device (validation runs first)."""
    shape = _shape()
    ok = np.zeros(shape.numel(), dtype=np.float32)
    p = rb.AttnParams.new(rb.Mask.BLOCK3, 4, 8)
    with pytest.raises(rb.LengthError):
        rb.Cuda().attend(shape, p, ok[:3], ok, ok, ok.copy())
    with pytest.raises(rb.ShapeError):
        rb.Cuda().attend(shape, rb.AttnParams.new(rb.Mask.BLOCK3, 9, 8), ok, ok, ok, ok.copy())


def test_per_sequence_valid_lengths_are_validated():
    shape = _shape(batch=3)
    buf = np.zeros(shape.numel(), np.float32)
    with pytest.raises(rb.ShapeError, match="exceeds seq"):
        rb.validate(shape, rb.AttnParams.new(rb.Mask.BLOCK3, [4, 5, 1], 8), buf, buf, buf, buf)
    with pytest.raises(rb.ShapeError, match="negative"):
        rb.validate(shape, rb.AttnParams.new(rb.Mask.BLOCK3, [4, -1, 1], 8), buf, buf, buf, buf)
    with pytest.raises(rb.ShapeError):
        rb.validate(shape, rb.AttnParams.new(rb.Mask.BLOCK3, [4, 4], 8), buf, buf, buf, buf)
    rb.validate(shape, rb.AttnParams.new(rb.Mask.BLOCK3, [4, 0, 1], 8), buf, buf, buf, buf)


@pytest.mark.parametrize("mask,block", [(rb.Mask.BLOCK3, 128), (rb.Mask.block(0), 64), (rb.Mask.block(2), 7),
                                        (rb.Mask.WINDOW64, 128), (rb.Mask.sliding(3), 128), (rb.Mask.FULL, 128)])
def test_work_counts_match_the_oracle(mask, block):
    shape = _shape(heads=3, seq=333, d=64, batch=4)
    valid = [333, 200, 1, 0]
    pairs, rows = rb.work(shape, rb.AttnParams.new(mask, valid, 64, block=block))
    kind = {rb.Mask.WINDOW64.kind: oracle.MASK_WINDOW, rb.Mask.FULL.kind: oracle.MASK_FULL}.get(mask.kind, oracle.MASK_BLOCK)
    p = oracle.Problem(4, 3, 333, 64, mask=kind, block=block, halo=mask.param, window=mask.param)
    assert (pairs, rows) == oracle.count(p, valid)


def test_mask_mirror_matches_the_oracle_key_range():
    for mask, kw in ((rb.Mask.BLOCK3, dict(mask=oracle.MASK_BLOCK, block=128, halo=1)),
                     (rb.Mask.block(0), dict(mask=oracle.MASK_BLOCK, block=128, halo=0)),
                     (rb.Mask.WINDOW64, dict(mask=oracle.MASK_WINDOW, window=64)),
                     (rb.Mask.FULL, dict(mask=oracle.MASK_FULL))):
        p = oracle.Problem(1, 1, 500, 8, **kw)
        for valid in (500, 333, 0):
            for i in range(0, 500, 7):
                r = mask.key_range(i, valid)
                assert (r.start, r.stop) == oracle.key_range(p, i, valid)
    assert rb.Mask.BLOCK3.allows(127, 255) and not rb.Mask.BLOCK3.allows(127, 256)
    assert rb.Mask.WINDOW64.allows(100, 164) and not rb.Mask.WINDOW64.allows(100, 165)
    assert rb.Mask.BLOCK3.name() == "block3" and rb.Mask.WINDOW64.name() == "window64"


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_tile_the_batch_and_balance_work(world):
    shape = _shape(heads=12, seq=1024, d=64, batch=32)
    valid = list(np.random.default_rng(0).integers(512, 1025, 32))
    params = rb.AttnParams.new(rb.Mask.BLOCK3, valid, 64, block=64)
    ranges = [rb.shard(shape, params, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == 32 * 12
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 <= a1
    # balance: per-slice pair counts
    per = np.repeat([oracle.count(oracle.Problem(1, 1, 1024, 64, mask=0, block=64, halo=1), [v])[0] for v in valid], 12)
    loads = [per[a:b].sum() for a, b in ranges]
    assert max(loads) <= per.sum() / world + per.max()


def test_shard_rejects_bad_ranks():
    shape = _shape(batch=2)
    params = rb.AttnParams.new(rb.Mask.BLOCK3, 4, 8)
    for world, rank in ((0, 0), (2, 2), (2, -1)):
        with pytest.raises(rb.ShapeError):
            rb.shard(shape, params, world, rank)


def test_packed_call_validates_on_the_host():
    import ctypes

    shape = _shape(heads=2, seq=128, d=64, batch=1)
    d = rb.make_desc(shape, rb.AttnParams.new(rb.Mask.BLOCK3, 128, 64))
    need = ctypes.c_size_t()
    assert _lib.lib.raya_attn_packed_workspace(ctypes.byref(d), ctypes.c_float(10000.0), ctypes.byref(need)) == 0
    assert need.value == 128 * 32 * 2 * 4
    assert _lib.lib.raya_attn_packed_workspace(ctypes.byref(d), ctypes.c_float(0.0), ctypes.byref(need)) == 0
    assert need.value == 0
    # rotation without a workspace: the reference's Length error kind
    st = _lib.lib.raya_attn_forward_packed(ctypes.byref(d), 16, 16, None, ctypes.c_float(10000.0), None, 0, None)
    assert st == _lib.ERR_LENGTH and "workspace" in _lib.last_error()
    bad = rb.make_desc(_shape(heads=2, seq=128, d=32, batch=1), rb.AttnParams.new(rb.Mask.BLOCK3, 128, 32))
    assert _lib.lib.raya_attn_forward_packed(ctypes.byref(bad), 16, 16, None, ctypes.c_float(0.0), None, 0,
                                             None) == _lib.ERR_UNSUPPORTED


def test_two_tile_form_for_short_blocks_with_many_tiles():
    """Blocks below 128 with a halo and >= 1024 128-row tiles (c2: 32 x 12 x 8) run the two-tile
    form of the tensor-core kernel, in the packed layout too unless it rotates; with fewer tiles,
    the one-tile form."""
    params = rb.AttnParams.new(rb.Mask.block(1), [1024] * 32, 64, block=64)
    c2 = _shape(heads=12, seq=1024, d=64, batch=32)
    assert rb.kernel_for(c2, params) == rb._lib.KERNEL_TC32_WS2
    assert rb.kernel_for(c2, params, packed=True) == rb._lib.KERNEL_TC32_WS2
    assert rb.kernel_for(c2, params, packed=True, rope=True) == rb._lib.KERNEL_TC32_WS
    assert rb.kernel_for(c2, params, rope=True) == rb._lib.KERNEL_TC32_WS2  # head-major: no rotation
    small = rb.AttnParams.new(rb.Mask.block(1), [1024] * 2, 64, block=64)
    assert rb.kernel_for(_shape(heads=12, seq=1024, d=64, batch=2), small) == rb._lib.KERNEL_TC32_WS
    # blocks of 128: the two-tile form from 2048 tiles on (here 3072), the one-tile form below
    b128 = rb.AttnParams.new(rb.Mask.block(1), [1024] * 32, 64, block=128)
    assert rb.kernel_for(_shape(heads=12, seq=1024, d=64, batch=32), b128) == rb._lib.KERNEL_TC32_WS2
    b128s = rb.AttnParams.new(rb.Mask.block(1), [1024] * 4, 64, block=128)
    assert rb.kernel_for(_shape(heads=12, seq=1024, d=64, batch=4), b128s) == rb._lib.KERNEL_TC32_WS


@pytest.mark.parametrize("mask,block,expect_tc", [
    (rb.Mask.block(1), 128, True),    # Block3: every allowed key of a 128-row span
    (rb.Mask.block(0), 256, True),    # halo 0, 2-4 key tiles per 128-row tile (the persistent kernel: on request)
    (rb.Mask.block(0), 128, True),
    (rb.Mask.block(0), 512, True),
    (rb.Mask.block(0), 192, True),
    (rb.Mask.block(2), 64, True),     # 320 of 384 span keys allowed per row
    (rb.Mask.block(1), 64, True),     # 192 of 256
    (rb.Mask.block(1), 32, True),     # 96 of 192
    (rb.Mask.block(0), 64, False),    # halo 0 below 128: the 64-row FFMA tiles
    (rb.Mask.block(2), 32, True),
    (rb.Mask.block(1), 7, False),     # 21 of 192
    (rb.Mask.WINDOW64, 128, True),
    (rb.Mask.sliding(31), 128, False),
    (rb.Mask.FULL, 128, True),
])
def test_automatic_kernel_choice(mask, block, expect_tc):
    """The host-side rule behind RAYA_KERNEL_AUTO: the tensor-core kernel
    (RAYA_KERNEL_TC32_WS) where enough of a 128-row CTA's key span is allowed, the tuned FFMA
    kernel else, rowwise for head_dim != 64 (no device work involved)."""
    shape = _shape(heads=2, seq=1024, d=64)
    params = rb.AttnParams.new(mask, 1024, 64, block=block)
    kid = rb.kernel_for(shape, params)
    if expect_tc:
        assert kid == rb._lib.KERNEL_TC32_WS
    else:
        assert kid in _lib.KERNEL_TILED64_VARIANTS.values()
    assert rb.kernel_for(_shape(heads=2, seq=1024, d=32), rb.AttnParams.new(mask, 1024, 32, block=block)) \
        == rb.KERNEL_ROWWISE
    # the caller's packed layout: the two-issuer tensor-core kernel where a tensor-core kernel is
    # chosen (the persistent variant has no packed form), else the tuned tiled kernel
    for rope in (False, True):
        if expect_tc:
            assert rb.kernel_for(shape, params, packed=True, rope=rope) == rb._lib.KERNEL_TC32_WS
        else:
            assert rb.kernel_for(shape, params, packed=True, rope=rope) in _lib.KERNEL_TILED64_VARIANTS.values()


def test_length_errors_carry_their_fields_as_data():
    """KernelError::Length { name, got, expected } (attention.rs:13-18) comes
    back from raya_attn_last_error_info, not from parsing the message."""
    shape = _shape()
    ok = np.zeros(shape.numel(), dtype=np.float32)
    p = rb.AttnParams.new(rb.Mask.BLOCK3, 4, 8)
    with pytest.raises(rb.LengthError):
        rb.validate(shape, p, ok, ok, np.zeros(5, np.float32), ok)
    info = rb.last_error_info()
    assert (info.kind, info.name, info.got, info.expected) == (_lib.ERR_LENGTH, "v", 5, 32)
    with pytest.raises(rb.ShapeError):
        rb.validate(_shape(d=12), p, ok, ok, ok, ok)
    info = rb.last_error_info()
    assert (info.kind, info.name, info.got, info.expected) == (_lib.ERR_SHAPE, "", 0, 0)
    # NULL outputs are allowed
    assert _lib.lib.raya_attn_last_error_info(None, None, None, None) == _lib.OK


def test_multi_gpu_call_validates_before_touching_a_gpu():
    """raya_attn_forward_multi_gpu rejects bad arguments with the reference's
    error kinds before any device work."""
    shape = _shape(batch=2)
    ok = np.zeros(shape.numel(), dtype=np.float32)
    p = rb.AttnParams.new(rb.Mask.BLOCK3, 4, 8)
    with pytest.raises(rb.LengthError) as e:
        rb.multi_gpu(shape, p, ok[:7], ok, ok, ok.copy(), devices=[0, 1])
    assert (e.value.name, e.value.got, e.value.expected) == ("q", 7, 64)
    with pytest.raises(rb.ShapeError, match="listed twice"):
        rb.multi_gpu(shape, p, ok, ok, ok, ok.copy(), devices=[1, 1])
    with pytest.raises(rb.ShapeError, match="devices"):
        rb.multi_gpu(shape, p, ok, ok, ok, ok.copy(), devices=[])
    with pytest.raises(rb.ShapeError, match="no output"):
        rb.multi_gpu(shape, p, ok, ok, ok, None, devices=[0])
    with pytest.raises(rb.ShapeError, match="exceeds seq"):
        rb.multi_gpu(shape, rb.AttnParams.new(rb.Mask.BLOCK3, [4, 5], 8), ok, ok, ok, ok.copy(), devices=[0])


def test_no_cpu_fallback_when_the_library_is_missing(tmp_path):
    """The package imports without loading the library (its workloads module
    is plain numpy), but the first name that needs the CUDA library raises
    ImportError when it is missing: there is no CPU path."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import raya_b200, raya_b200.workloads\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'libraya_attn' not in maps, 'library mapped by a plain import'\n"
        "from raya_b200 import _lib\n"
        "_lib.LIB_PATH = %r\n"
        "try:\n"
        "    _lib._load()\n"
        "except ImportError as e:\n"
        "    print('raised:', e)\n"
    ) % (ROOT, str(tmp_path / "missing.so"))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert "raised:" in out.stdout and "no fallback" in out.stdout


def test_automatic_choice_two_tile_form_for_many_long_block_tiles():
    """Blocks of 128 or more with a halo take the two-tile form (kernel 37)
    when there are >= 2048 row tiles and the span is at most 2048 keys (c5's
    shape), the single-tile form otherwise."""
    params = lambda b: rb.AttnParams.new(rb.Mask.block(1), 8192, 64, block=b)
    c5 = _shape(heads=16, seq=8192, d=64, batch=256)
    assert rb.kernel_for(c5, params(128)) == rb.KERNEL_TC32_WS2
    one = _shape(heads=16, seq=8192, d=64, batch=1)  # 1024 tiles
    assert rb.kernel_for(one, params(128)) == rb.KERNEL_TC32_WS
    assert rb.kernel_for(c5, params(1024)) == rb.KERNEL_TC32_WS  # 3072 keys per span


def test_rust_binding_matches_the_header():
    """The FFI crate crates/raya-kernels-cuda (no cargo in this image, so it
    is checked as text): every function its extern block declares is
    exported by the library, and its #[repr(C)] descriptor has the fields of
    raya_attn_desc in the header's order with the same widths."""
    src = open(os.path.join(ROOT, "crates", "raya-kernels-cuda", "src", "lib.rs")).read()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    declared = set(re.findall(r"fn (raya_attn_\w+)\(", block))
    assert declared and declared <= set(_lib.EXPORTS), declared - set(_lib.EXPORTS)
    rust = re.findall(r"^\s+(\w+): (i64|i32|f32),$", src[src.index("struct RayaAttnDesc"):src.index("// raya_attn_status")],
                      flags=re.M)
    header = open(os.path.join(ROOT, "include", "raya_attn.h")).read()
    body = header[header.index("typedef struct {"):header.index("} raya_attn_desc;")]
    c = re.findall(r"(int64_t|int32_t|float) (\w+);", body)
    width = {"i64": "int64_t", "i32": "int32_t", "f32": "float"}
    assert [(n, width[t]) for n, t in rust] == [(n, t) for t, n in c]
