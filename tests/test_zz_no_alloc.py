"""mtl_w4a16_linear_noalloc: the W4A16 linear for callers that cannot
allocate device memory (a host that owns all device memory and gives the
library no allocator, or a step recorded under stream capture, where
cudaMalloc is not permitted).  Its split-K scratch is a fixed device array
inside the library, so these calls pass no scratch.

Called through the C ABI (ctypes) and checked against the existing entry
point mtl_w4a16_linear, which takes caller scratch: both run the same launch
plan and kernel, so the outputs must be equal bit for bit; they must also be
within the tolerance of the other W4 tests of the exact product.  Each case
makes two calls in a row (the second reuses the array the first one left
behind).  The cases cover the register-MMA tiles at one and four rows (with
the residual epilogue) and the tensor-core tiles at one row (RMSNorm
prologue) and four rows (the batched tensor-core kernel).  This file sorts
last so that a run stopping at the first failure has already run every other
test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu

ARRAY_BYTES = 1 << 20   # the library's fixed scratch array


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(dev)


def _bits(t):
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _gptq_weight(dev, K, N, g, seed):
    """AutoGPTQ tensors packed into register-MMA tiles; returns (tiles, W [K, N] f64-able)."""
    from moss_tts_lite_b200 import _lib
    d = ow.synth_gptq_linear(K, N, g, seed=seed)
    tb, _ = _lib.w4_plan(1, K, N, g, _lib.MTL_FMT_GPTQ)
    tiles = torch.empty(tb, dtype=torch.uint8, device=dev)
    qw, qz, sc = _t(d["qweight"], dev), _t(d["qzeros"], dev), _t(d["scales"], dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.mtl_w4_pack_gptq(qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), None, K, N, g,
                                     tiles.data_ptr(), stream) == 0, _lib.last_error()
    return tiles, ow.gptq_dequant(d["qweight"], d["qzeros"], d["scales"], d["g_idx"])


def _tc_weight(dev, K, N, g, seed):
    """RTN codes + (scale, zero) of a random bf16 weight packed into tensor-core tiles."""
    from moss_tts_lite_b200 import _lib
    rng = np.random.default_rng(seed)
    w = f32_to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    q, s, mn = ow.rtn_quantize(w, g)
    qsz = ow.pack_qsz(s, mn)
    tb, _ = _lib.w4_plan(1, K, N, g, _lib.MTL_FMT_TC)
    tiles = torch.empty(tb, dtype=torch.uint8, device=dev)
    qt, qszt = _t(q, dev), _t(qsz, dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.mtl_w4_pack_tc(qt.data_ptr(), qszt.data_ptr(), K, N, g, tiles.data_ptr(), stream) == 0, \
        _lib.last_error()
    return tiles, ow.ref_operand_weight(q, qsz, g).T


# (name, param format, M, K, N, fused RMSNorm prologue, residual epilogue)
CASES = [
    ("gptq-1row", "GPTQ", 1, 4096, 12288, False, False),
    ("gptq-4rows-residual", "GPTQ", 4, 4096, 4096, False, True),
    ("tc-1row-norm", "TC", 1, 4096, 4096, True, False),
    ("tc-4rows-batched", "TC", 4, 2048, 1024, False, False),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_noalloc_linear_matches_scratch_linear_twice(case):
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    lib = _lib.lib
    name, fmt_name, M, K, N, norm, res = case
    g = 128
    fmt = _lib.MTL_FMT_GPTQ if fmt_name == "GPTQ" else _lib.MTL_FMT_TC
    _, sb = _lib.w4_plan(M, K, N, g, fmt)
    assert sb <= ARRAY_BYTES, (name, sb)
    tiles, W = (_gptq_weight if fmt_name == "GPTQ" else _tc_weight)(dev, K, N, g, seed=4 + M)
    scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(9 + M)
    nw = f32_to_bf16((1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)) if norm else None
    nwt = _t(nw, dev, torch.bfloat16) if norm else None
    epi = _lib.MTL_EPI_RESIDUAL if res else _lib.MTL_EPI_STORE
    for call in range(2):
        x = f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
        r = f32_to_bf16(rng.standard_normal((M, N)).astype(np.float32)) if res else None
        xt = _t(x, dev, torch.bfloat16)
        rt = _t(r, dev, torch.bfloat16) if res else None
        y_ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        y_new = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        common = (xt.data_ptr(), K, M, K, N, g, fmt, tiles.data_ptr(), 0, None,
                  nwt.data_ptr() if norm else None, ctypes.c_float(1e-6), epi, rt.data_ptr() if res else None)
        rc = lib.mtl_w4a16_linear(*common, y_ref.data_ptr(), N, scratch.data_ptr(), sb, stream)
        assert rc == 0, _lib.last_error()
        rc = lib.mtl_w4a16_linear_noalloc(*common, y_new.data_ptr(), N, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        a, b = _bits(y_new), _bits(y_ref)
        # same plan, same kernel: bitwise equal to the existing entry point
        assert np.array_equal(a, b), (name, call, int((a != b).sum()))
        # and within the W4 tests' tolerance of the exact product
        xin = x
        if norm:
            from oracle.step import rms_norm
            xin = rms_norm(x, nw)
        want = ow.linear_f64(xin, W)
        if res:
            # residual + bf16(x . W^T): compare the linear part
            want = bf16_to_f32(r).astype(np.float64) + bf16_to_f32(f32_to_bf16(want.astype(np.float32)))
        ok, dmax = ow.close_enough(a, want)
        assert ok, (name, call, dmax)
    assert _lib.device_status() == 0


def test_noalloc_rejects_shapes_beyond_the_array():
    require_cuda()
    from moss_tts_lite_b200 import _lib
    _, need = _lib.w4_plan(8, 4096, 24576, 128, 0)
    assert need > ARRAY_BYTES                   # a batch-8 fused gate|up needs more than the array
    fake = ctypes.c_void_p(0x1000)   # rejected before any device access
    rc = _lib.lib.mtl_w4a16_linear_noalloc(fake, 4096, 8, 4096, 24576, 128, 0, fake, 0, None, None,
                                           ctypes.c_float(1e-6), 0, None, fake, 24576, None)
    assert rc == -3 and "fixed device array" in _lib.last_error()


def test_noalloc_checks_arguments_first():
    """Argument errors other than the scratch size come back as such (the
    checks run before the counter clear is enqueued): a misaligned tile
    pointer gives MTL_E_ALIGN, an unknown epilogue MTL_E_INVALID."""
    require_cuda()
    from moss_tts_lite_b200 import _lib
    fake = ctypes.c_void_p(0x1000)
    odd = ctypes.c_void_p(0x1008)    # not 16-byte aligned
    rc = _lib.lib.mtl_w4a16_linear_noalloc(fake, 4096, 1, 4096, 4096, 128, 0, odd, 0, None, None,
                                           ctypes.c_float(1e-6), 0, None, fake, 4096, None)
    assert rc == _lib.MTL_E_ALIGN, _lib.last_error()
    rc = _lib.lib.mtl_w4a16_linear_noalloc(fake, 4096, 1, 4096, 4096, 128, 0, fake, 0, None, None,
                                           ctypes.c_float(1e-6), 7, None, fake, 4096, None)
    assert rc == _lib.MTL_E_INVALID, _lib.last_error()
