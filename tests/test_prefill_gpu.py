"""The tcgen05 W4 prefill GEMM (mtl_w4a16_gemm) on the B200.

It multiplies the same bf16 operand as the reference's int4 GEMM
(bf16((q - 8) * scale + zero), oracle.w4.ref_operand_weight) with fp32
accumulation, so against the oracle's product it differs only by the fp32
summation order: within the north-star tolerance everywhere and bitwise
equal for almost every output.  Shapes cover partial prompt-row tiles (64,
128 and 256-row tiles), every epilogue, group sizes 64-256 and the
configuration-2 projection shapes; the reference's own kernel
(torch._weight_int4pack_mm at M = prompt rows, as fast.py:218-270 prefills)
is compared where the reference package is importable."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import step as ost
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16
from test_w4_gpu import _bits, _check, _ref_case, _t

pytestmark = pytest.mark.gpu


def _x(M, K, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return f32_to_bf16((rng.standard_normal((M, K)) * scale).astype(np.float32))


@pytest.mark.parametrize("M,K,N,g", [(128, 4096, 6144, 128), (300, 4096, 4096, 128), (40, 1024, 256, 64),
                                     (520, 2048, 512, 256), (4096, 1024, 384, 128), (33, 12288, 256, 128)])
def test_gemm_vs_oracle(M, K, N, g):
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    from moss_tts_lite_b200.quant import W4Weight
    q, qsz, Wnk = _ref_case(K, N, g, seed=M + K + N)
    w = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    x = _x(M, K, seed=M)
    y = w.gemm(_t(x, dev, torch.bfloat16))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    got = _bits(y)
    _check(got, ow.linear_f64(x, Wnk.T))
    want = ow.linear_bf16(x, Wnk.T)
    assert (got == want).mean() > 0.99


def test_gemm_epilogues_residual_and_swiglu():
    dev = require_cuda()
    from moss_tts_lite_b200.quant import W4Weight
    K, I, g, M = 1024, 256, 128, 200
    rng = np.random.default_rng(5)
    # residual, written in place (out aliases the residual)
    q, qsz, Wnk = _ref_case(K, K, g, seed=1)
    w = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    x = _x(M, K, seed=2)
    h = f32_to_bf16((rng.standard_normal((M, K)) * 3).astype(np.float32))
    ht = _t(h, dev, torch.bfloat16)
    w.gemm(_t(x, dev, torch.bfloat16), residual=ht, out=ht)
    ref = f32_to_bf16(bf16_to_f32(h) + bf16_to_f32(ow.linear_bf16(x, Wnk.T)))
    d = np.abs(bf16_to_f32(_bits(ht)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.99
    # SwiGLU: gate/up interleaved in 32-row blocks, as the fused layer weight
    qg, qszg, Wg = _ref_case(K, I, g, seed=3)
    qu, qszu, Wu = _ref_case(K, I, g, seed=4)
    blocks, qsb = [], []
    for b in range(I // 32):
        blocks += [qg[32 * b:32 * b + 32], qu[32 * b:32 * b + 32]]
        qsb += [qszg[:, 32 * b:32 * b + 32], qszu[:, 32 * b:32 * b + 32]]
    wf = W4Weight.from_ref(_t(np.concatenate(blocks, 0), dev), _t(np.concatenate(qsb, 1), dev, torch.bfloat16), g)
    y = wf.gemm(_t(x, dev, torch.bfloat16), swiglu=True)
    ref = ost.silu_mul(ow.linear_bf16(x, Wg.T), ow.linear_bf16(x, Wu.T))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.98


def test_gemm_equals_register_kernel_rows():
    """The prefill GEMM and the decode GEMV take the same operand: row by row
    they agree within the fp32 summation order (one bf16 ulp at most)."""
    dev = require_cuda()
    from moss_tts_lite_b200.quant import W4Weight
    K, N, g, M = 4096, 1024, 128, 96
    q, qsz, _ = _ref_case(K, N, g, seed=8)
    w = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    xt = _t(_x(M, K, seed=9), dev, torch.bfloat16)
    a = w.gemm(xt).float()
    b = w.linear(xt).float()
    # one bf16 ulp, or the fp32 summation noise where the output cancels to ~0
    tol = torch.clamp(b.abs() * 2.0 ** -7, min=1e-4)
    assert bool(((a - b).abs() <= tol * 1.001).all()), float((a - b).abs().max())
    assert (a == b).float().mean().item() > 0.99


def test_gemm_vs_reference_tinygemm():
    """The reference's prefill kernel on the same codes (torch._weight_int4pack_mm
    with M = prompt rows): bitwise equal for almost every output, never more
    than one bf16 ulp apart."""
    dev = require_cuda()
    ref = pytest.importorskip("moss_tts_lite.gptq")
    from moss_tts_lite_b200.quant import W4Weight
    K, N, g, M = 4096, 4096, 128, 256
    wt = (torch.randn(N, K, generator=torch.Generator().manual_seed(0)) * 0.02).to(torch.bfloat16).to(dev)
    q, s, mn = ref.rtn_quantize(wt, g)
    packed, qsz = ref.pack_fast(q, s, mn, 8)
    x = torch.randn(M, K, dtype=torch.bfloat16, device=dev)
    y_ref = torch._weight_int4pack_mm(x, packed, g, qsz)
    y = W4Weight.from_ref(q, qsz, g).gemm(x)
    same = (y.view(torch.int16) == y_ref.view(torch.int16)).float().mean().item()
    tol = torch.clamp(y_ref.float().abs() * 2.0 ** -7, min=1e-4)
    assert same > 0.99, same
    assert bool(((y.float() - y_ref.float()).abs() <= tol * 1.001).all())


def test_gemm_rejects_unserved_shapes():
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    from moss_tts_lite_b200.quant import W4Weight, gemm_supported
    q, qsz, _ = _ref_case(256, 128, 32, seed=1)
    w = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), 32)
    assert not gemm_supported(w)
    x = torch.zeros(8, 256, dtype=torch.bfloat16, device=dev)
    y = torch.empty(8, 128, dtype=torch.bfloat16, device=dev)
    rc = _lib.lib.mtl_w4a16_gemm(x.data_ptr(), 256, 8, 256, 128, 32, w.tiles.data_ptr(), 0, None, 0, y.data_ptr(),
                                 128, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MTL_E_UNSUPPORTED


@pytest.mark.parametrize("L,rep,streams,p0", [(128, 4, 1, 0), (300, 4, 1, 0), (77, 2, 3, 0), (64, 8, 2, 0),
                                              (40, 4, 1, 150), (1, 1, 1, 0)])
def test_attn_prefill_vs_oracle(L, rep, streams, p0):
    """mtl_attn_prefill against the oracle's causal attention (the
    flash-style rounding points) for every row and head, with partial query
    blocks, several streams over separate caches and a prompt chunk that
    starts at position p0 > 0 (rows beyond the chunk hold NaN and are never
    read)."""
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib, kernels
    rng = np.random.default_rng(L + rep + streams + p0)
    nkv, D, max_seq = 2, 128, 512
    nh = nkv * rep
    q = f32_to_bf16(rng.standard_normal((streams * L, nh, D)).astype(np.float32))
    kc = f32_to_bf16(rng.standard_normal((streams, nkv, max_seq, D)).astype(np.float32))
    vc = f32_to_bf16((rng.standard_normal((streams, nkv, max_seq, D)) * 1.5).astype(np.float32))
    kc[:, :, p0 + L:] = 0x7FC0
    vc[:, :, p0 + L:] = 0x7FC0
    out = torch.empty(streams * L, nh * D, dtype=torch.bfloat16, device=dev)
    kernels.attn_prefill(_t(q, dev, torch.bfloat16), _t(kc, dev, torch.bfloat16), _t(vc, dev, torch.bfloat16),
                         nh, nkv, out, rows_per_stream=L, streams=streams, p0=p0,
                         cache_stream_stride=nkv * max_seq * D)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    got = bf16_to_f32(_bits(out)).reshape(streams, L, nh, D)
    qf = bf16_to_f32(q).astype(np.float64).reshape(streams, L, nh, D)
    kf, vf = bf16_to_f32(kc).astype(np.float64), bf16_to_f32(vc).astype(np.float64)
    scale = 1.0 / np.sqrt(D)
    worst = 0.0
    for s in range(streams):
        for h in range(nh):
            kv = h // rep
            keys, vals = kf[s, kv, :p0 + L], vf[s, kv, :p0 + L]
            want = ost.attend(qf[s, :, h], keys, vals, scale, causal=True)
            d = np.abs(got[s, :, h] - want)
            assert np.isfinite(got[s, :, h]).all()
            # bf16 output rounding (2^-8 relative) plus fp32 summation order
            assert (d <= 1e-2 + 8e-3 * np.abs(want)).all(), (s, h, float(d.max()))
            worst = max(worst, float(d.max()))
