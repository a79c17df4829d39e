"""mtl_w4a16_linear_noalloc: the W4A16 linear for callers that cannot
allocate device memory (a host that owns all device memory and gives the
library no allocator, or a step recorded under stream capture, where
cudaMalloc is not permitted).  Its split-K scratch is a fixed device array
inside the library, so these calls pass no scratch.

Called through the C ABI (ctypes) and checked against the existing entry
point mtl_w4a16_linear, which takes caller scratch, with the tolerance of
the other W4 tests, on two calls in a row (the second call reuses the array
the first one left behind).  This file sorts last so that a run stopping at
the first failure has already run every other test; it also passes alone in
a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(dev)


def test_noalloc_linear_matches_scratch_linear_twice():
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    lib = _lib.lib
    K, N, g, M = 4096, 12288, 128, 1
    d = ow.synth_gptq_linear(K, N, g, seed=4)
    tb, sb = _lib.w4_plan(M, K, N, g, _lib.MTL_FMT_GPTQ)
    assert sb <= 1 << 20
    tiles = torch.empty(tb, dtype=torch.uint8, device=dev)
    qw, qz = _t(d["qweight"], dev), _t(d["qzeros"], dev)
    sc = _t(d["scales"], dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.mtl_w4_pack_gptq(qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), None, K, N, g,
                                tiles.data_ptr(), stream) == 0
    scratch = torch.zeros(sb, dtype=torch.uint8, device=dev)
    W = ow.gptq_dequant(d["qweight"], d["qzeros"], d["scales"], d["g_idx"])
    rng = np.random.default_rng(9)
    for call in range(2):
        x = f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
        xt = _t(x, dev, torch.bfloat16)
        y_ref = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        y_new = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        rc = lib.mtl_w4a16_linear(xt.data_ptr(), K, M, K, N, g, _lib.MTL_FMT_GPTQ, tiles.data_ptr(), 0, None,
                                  None, ctypes.c_float(1e-6), _lib.MTL_EPI_STORE, None, y_ref.data_ptr(), N,
                                  scratch.data_ptr(), sb, stream)
        assert rc == 0, _lib.last_error()
        rc = lib.mtl_w4a16_linear_noalloc(xt.data_ptr(), K, M, K, N, g, _lib.MTL_FMT_GPTQ, tiles.data_ptr(), 0,
                                          None, None, ctypes.c_float(1e-6), _lib.MTL_EPI_STORE, None,
                                          y_new.data_ptr(), N, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        a = y_new.cpu().view(torch.int16).numpy().view(np.uint16)
        b = y_ref.cpu().view(torch.int16).numpy().view(np.uint16)
        # same tolerance as the other W4 tests, against the existing entry point
        # and against the exact product
        ok, dmax = ow.close_enough(a, bf16_to_f32(b).astype(np.float64))
        assert ok, (call, dmax)
        assert ow.close_enough(a, ow.linear_f64(x, W))[0], call
    assert _lib.device_status() == 0


def test_noalloc_rejects_shapes_beyond_the_array():
    require_cuda()
    from moss_tts_lite_b200 import _lib
    _, need = _lib.w4_plan(8, 4096, 24576, 128, 0)
    assert need > 1 << 20                       # a batch-8 fused gate|up needs more than the array
    fake = ctypes.c_void_p(0x1000)   # rejected before any device access
    rc = _lib.lib.mtl_w4a16_linear_noalloc(fake, 4096, 8, 4096, 24576, 128, 0, fake, 0, None, None,
                                           ctypes.c_float(1e-6), 0, None, fake, 24576, None)
    assert rc == -3 and "fixed device array" in _lib.last_error()
