"""Tensor-core (tcgen05) W4A16 GEMV, tile format MTL_FMT_TC, on the B200:
bit-exact code round trips, outputs against the oracle's effective-weight
product at the configuration shapes (max-abs 2e-2 or
rel 1e-2 per bf16 element, plus a relative-norm bound), the fused epilogues,
agreement with the register-MMA kernel on the same codes, determinism and
graph capture."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import step as ost
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16
from test_w4_gpu import _bits, _check, _ref_case, _t

pytestmark = pytest.mark.gpu


def _tc(q, qsz, g, dev):
    from moss_tts_lite_b200 import _lib
    from moss_tts_lite_b200.quant import W4Weight
    return W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g, fmt=_lib.MTL_FMT_TC)


@pytest.mark.parametrize("K,N,g", [(256, 128, 32), (1024, 384, 64), (4096, 1024, 128)])
def test_tc_codes_roundtrip_bit_exact(K, N, g):
    dev = require_cuda()
    q, qsz, _ = _ref_case(K, N, g, seed=K + g)
    w = _tc(q, qsz, g, dev)
    assert np.array_equal(w.unpack_codes().cpu().numpy(), q)


@pytest.mark.parametrize("K,N,g", [(4096, 6144, 128), (4096, 4096, 128), (4096, 24576, 128),
                                   (12288, 4096, 128), (1024, 256, 32), (2048, 640, 64)])
def test_tc_linear_vs_oracle(K, N, g):
    dev = require_cuda()
    q, qsz, Wnk = _ref_case(K, N, g, seed=N + g)
    w = _tc(q, qsz, g, dev)
    rng = np.random.default_rng(K)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    y = w.linear(_t(x, dev, torch.bfloat16))
    _check(_bits(y), ow.linear_f64(x, Wnk.T))
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def test_tc_batch_rows_and_agreement_with_register_mma():
    """Three rows (one launch per row) equal row-by-row calls; and the same
    codes through the register-MMA tiles agree within bf16 rounding."""
    dev = require_cuda()
    from moss_tts_lite_b200.quant import W4Weight
    K, N, g = 4096, 2048, 128
    q, qsz, Wnk = _ref_case(K, N, g, seed=5)
    w = _tc(q, qsz, g, dev)
    wr = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    rng = np.random.default_rng(3)
    x = f32_to_bf16(rng.standard_normal((3, K)).astype(np.float32))
    xt = _t(x, dev, torch.bfloat16)
    y3 = w.linear(xt)
    for r in range(3):
        assert torch.equal(y3[r:r + 1], w.linear(xt[r:r + 1]))
    _check(_bits(y3), ow.linear_f64(x, Wnk.T))
    d = np.abs(bf16_to_f32(_bits(y3)) - bf16_to_f32(_bits(wr.linear(xt))))
    ref = np.abs(ow.linear_f64(x, Wnk.T))
    assert (d <= 2e-2 + 1e-2 * ref).all()


def test_tc_epilogues_residual_norm_swiglu():
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    from moss_tts_lite_b200.quant import W4Weight
    K, I, g = 4096, 1024, 128
    rng = np.random.default_rng(21)
    q, qsz, Wnk = _ref_case(K, K, g, seed=1)
    w = _tc(q, qsz, g, dev)
    h = f32_to_bf16((rng.standard_normal((1, K)) * 3).astype(np.float32))
    nw = f32_to_bf16((1 + 0.1 * rng.standard_normal(K)).astype(np.float32))
    ht = _t(h, dev, torch.bfloat16)
    y = w.linear(ht, norm_weight=_t(nw, dev, torch.bfloat16), residual=ht.clone())
    xn = ost.rms_norm(h, nw)
    lin = ow.linear_bf16(xn, Wnk.T)
    ref = f32_to_bf16(bf16_to_f32(h) + bf16_to_f32(lin))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95
    # in place (residual aliases the output), as the decode step uses it
    h2 = ht.clone()
    w.linear(h2, norm_weight=_t(nw, dev, torch.bfloat16), residual=h2, out=h2)
    assert torch.equal(h2, y)
    # SwiGLU: gate and up rows interleaved one by one
    qg, qszg, Wg = _ref_case(K, I, g, seed=2)
    qu, qszu, Wu = _ref_case(K, I, g, seed=3)
    qf = np.stack([qg, qu], 1).reshape(2 * I, K)
    qszf = np.stack([qszg, qszu], 2).reshape(K // g, 2 * I, 2)
    wf = W4Weight.from_ref(_t(qf, dev), _t(qszf, dev, torch.bfloat16), g, fmt=_lib.MTL_FMT_TC)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    y = wf.linear(_t(x, dev, torch.bfloat16), swiglu=True)
    ref = ost.silu_mul(ow.linear_bf16(x, Wg.T), ow.linear_bf16(x, Wu.T))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95
    assert _lib.device_status() == 0


def test_tc_deterministic_and_graph_capture():
    dev = require_cuda()
    K, N, g = 12288, 4096, 128
    q, qsz, _ = _ref_case(K, N, g, seed=9)
    w = _tc(q, qsz, g, dev)
    x = _t(f32_to_bf16(np.random.default_rng(1).standard_normal((1, K)).astype(np.float32)), dev, torch.bfloat16)
    y1 = w.linear(x).clone()
    assert torch.equal(y1, w.linear(x))
    out = torch.empty_like(y1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        w.linear(x, out=out)
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(3):
            w.linear(x, out=out)
    out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y1)


@pytest.mark.parametrize("M,K,N,g", [(2, 4096, 6144, 128), (5, 12288, 4096, 128), (16, 4096, 24576, 128),
                                     (21, 1024, 384, 64), (16, 2048, 640, 32), (9, 4096, 4096, 128)])
def test_tc_batched_rows(M, K, N, g):
    """2..16 rows per launch (the batch is the N dimension of the tcgen05
    MMAs, activations staged per tile): every row equals its own one-row
    call bit for bit and the oracle within tolerance; 21 rows run as 16 + 5."""
    dev = require_cuda()
    q, qsz, Wnk = _ref_case(K, N, g, seed=M + K + N)
    w = _tc(q, qsz, g, dev)
    rng = np.random.default_rng(M)
    x = f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    xt = _t(x, dev, torch.bfloat16)
    y = w.linear(xt)
    torch.cuda.synchronize()
    _check(_bits(y), ow.linear_f64(x, Wnk.T))
    for r in range(M):
        assert torch.equal(y[r:r + 1], w.linear(xt[r:r + 1])), r
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def test_tc_batched_epilogues_norm_residual_swiglu():
    """The fused RMSNorm prologue, the in-place residual and the SwiGLU
    epilogue with 5 rows per launch, against the oracle."""
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    from moss_tts_lite_b200.quant import W4Weight
    K, I, g, M = 4096, 1024, 128, 5
    rng = np.random.default_rng(31)
    q, qsz, Wnk = _ref_case(K, K, g, seed=11)
    w = _tc(q, qsz, g, dev)
    h = f32_to_bf16((rng.standard_normal((M, K)) * 3).astype(np.float32))
    nw = f32_to_bf16((1 + 0.1 * rng.standard_normal(K)).astype(np.float32))
    ht = _t(h, dev, torch.bfloat16)
    y = w.linear(ht, norm_weight=_t(nw, dev, torch.bfloat16), residual=ht.clone())
    xn = ost.rms_norm(h, nw)
    ref = f32_to_bf16(bf16_to_f32(h) + bf16_to_f32(ow.linear_bf16(xn, Wnk.T)))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95
    h2 = ht.clone()
    w.linear(h2, norm_weight=_t(nw, dev, torch.bfloat16), residual=h2, out=h2)
    assert torch.equal(h2, y)
    qg, qszg, Wg = _ref_case(K, I, g, seed=12)
    qu, qszu, Wu = _ref_case(K, I, g, seed=13)
    qf = np.stack([qg, qu], 1).reshape(2 * I, K)
    qszf = np.stack([qszg, qszu], 2).reshape(K // g, 2 * I, 2)
    wf = W4Weight.from_ref(_t(qf, dev), _t(qszf, dev, torch.bfloat16), g, fmt=_lib.MTL_FMT_TC)
    x = f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    y = wf.linear(_t(x, dev, torch.bfloat16), swiglu=True)
    ref = ost.silu_mul(ow.linear_bf16(x, Wg.T), ow.linear_bf16(x, Wu.T))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95
    assert _lib.device_status() == 0
