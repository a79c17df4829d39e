"""The C-ABI library loads, exports every symbol include/mtl_b200.h
declares, and validates arguments on the host (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mtl_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(mtl_\w+)\s*\(", src, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "mtl_w4a16_linear" in names and "mtl_w4_pack_ref" in names
    assert len(names) >= 8


def test_library_exports_every_declared_symbol():
    from moss_tts_lite_b200 import _lib
    for name in _declared():
        assert hasattr(_lib.lib, name), f"{name} declared in include/mtl_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version():
    from moss_tts_lite_b200 import _lib
    assert _lib.lib.mtl_abi_version() == _lib.ABI_VERSION


@pytest.mark.parametrize("K,N,g,fmt,tiles", [
    (4096, 12288, 128, 1, 26148864),       # == qweight + qzeros + scales bytes (AutoGPTQ)
    (4096, 12288, 128, 0, 26738688),       # == codes/2 + qsz bytes (reference format)
    (12288, 4096, 128, 0, 26738688),
])
def test_plan_sizes(K, N, g, fmt, tiles):
    from moss_tts_lite_b200 import _lib
    tb, sb = _lib.w4_plan(1, K, N, g, fmt)
    assert tb == tiles
    assert sb > 0 and sb % 256 == 0


@pytest.mark.parametrize("args,frag", [
    ((1, 4096, 12288, 16, 0), "group_size"),
    ((1, 4100, 12288, 128, 0), "multiple of group_size"),
    ((1, 4096, 12290, 128, 0), "multiple of 64"),
    ((1, 4096, 12288, 128, 7), "param_fmt"),
    ((0, 4096, 12288, 128, 0), "M=0"),
])
def test_plan_rejects_bad_shapes(args, frag):
    from moss_tts_lite_b200 import _lib
    with pytest.raises(_lib.MtlError) as ei:
        _lib.w4_plan(*args)
    assert ei.value.code == -1
    assert frag in str(ei.value)


def test_linear_rejects_null_and_small_scratch():
    """Validation happens before any device work, so it runs without a GPU."""
    from moss_tts_lite_b200 import _lib
    rc = _lib.lib.mtl_w4a16_linear(None, 4096, 1, 4096, 4096, 128, 0, None, 0, None, None,
                                   ctypes.c_float(1e-6), 0, None, None, 4096, None, 0, None)
    assert rc == -1 and "NULL" in _lib.last_error()
    fake = ctypes.c_void_p(0x1000)   # never dereferenced: validation fails first
    rc = _lib.lib.mtl_w4a16_linear(fake, 4096, 1, 4096, 4096, 128, 0, fake, 0, None, None,
                                   ctypes.c_float(1e-6), 0, None, fake, 4096, fake, 16, None)
    assert rc == -3 and "scratch" in _lib.last_error()
    rc = _lib.lib.mtl_w4a16_linear(fake, 4096, 1, 4096, 4096, 128, 0, fake, 0, None, None,
                                   ctypes.c_float(1e-6), 9, None, fake, 4096, fake, 1 << 30, None)
    assert rc == -1 and "epilogue" in _lib.last_error()


@pytest.mark.parametrize("cols,rows,top_k,slices", [
    (151936, 1, 50, 148),     # the text head at the reference's text top-k: 148 slices of 1027
    (151936, 1, 2048, 72),    # the largest candidate set: every slice (the last included) >= 2048
    (151936, 3, 1, 148),
    (20000, 2, 1000, 19),
    (16384, 1, 16, 16),
    (1025, 32, 50, 0),        # audio rows: one CTA per row, no scratch
    (151936, 1, 0, 0),        # no top-k: no slicing
    (151936, 1, 151936, 0),
])
def test_sample_scratch_bytes(cols, rows, top_k, slices):
    """mtl_sample_scratch_bytes (host only): (value, id) per candidate of
    every slice; slices of equal length with the last one at least top_k."""
    from moss_tts_lite_b200 import _lib
    got = _lib.lib.mtl_sample_scratch_bytes(cols, rows, top_k)
    assert got == rows * slices * top_k * 8
    if slices:
        sl = -(-cols // slices)
        assert cols - (slices - 1) * sl >= top_k and sl <= 8192


def test_plan_rejects_tile_counts_past_32_bit_owner_math():
    """The stream-K owner arithmetic is 32-bit: T x CTAs < 2^32 or the plan fails."""
    from moss_tts_lite_b200 import _lib
    with pytest.raises(_lib.MtlError):
        _lib.w4_plan(1, 16384 * 128, 64 * 8192, 32, 0)


def test_sampling_limits_rejected_up_front():
    """A sampled decision the fused sampler does not serve is refused before
    any device work: top-p alone (or a top-k beyond 2048) over the text head."""
    from moss_tts_lite_b200.sampling import SAMPLE_MAX_CANDIDATES, check_top_k
    check_top_k(50, 151936, "text")                 # the reference text default
    check_top_k(SAMPLE_MAX_CANDIDATES, 151936, "text")
    check_top_k(None, 1025, "audio")                # no top-k over an audio row
    check_top_k(0, 2, "two-way")
    for k in (None, 0, -1, SAMPLE_MAX_CANDIDATES + 1, 151936):
        with pytest.raises(NotImplementedError, match="not supported"):
            check_top_k(k, 151936, "text")
