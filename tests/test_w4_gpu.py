"""W4A16 linear on the B200 vs the CPU oracle (bit-exact codes, tolerance
outputs).  Mirrors the reference's G2 kernel-semantics test
(tests/test_quant.py:96-119 of moss-tts-lite): the kernel against the
product with its weight operand, here with the north-star tolerance
(max-abs 2e-2 or rel 1e-2 per element on bf16 outputs) plus a tight
relative-norm bound.  Reference format: the operand is the effective weight
rounded once to bf16, as torch's int4 GEMM forms it (oracle.w4.
ref_operand_weight), and the outputs equal that kernel's up to the fp32
summation order; AutoGPTQ format: the exact (q - z) s."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu


def _lib():
    from moss_tts_lite_b200 import _lib
    return _lib


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(dev)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _gptq_case(K, N, g, seed, M=1, zero_offset=0):
    d = ow.synth_gptq_linear(K, N, g, seed)
    rng = np.random.default_rng(seed + 1000)
    x = f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    W = ow.gptq_dequant(d["qweight"], d["qzeros"], d["scales"], d["g_idx"], zero_offset)
    return d, x, W


def _check(y_bits, ref):
    ok, dmax = ow.close_enough(y_bits, ref)
    y = bf16_to_f32(y_bits).astype(np.float64)
    rel = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
    assert ok, f"max|d|={dmax}"
    assert rel < 4e-3, f"rel-norm {rel}"   # bf16 output rounding alone is ~2e-3
    return rel


def _quantlinear(d, g, dev, zero_offset=0):
    from moss_tts_lite_b200.quant import QuantLinear
    return QuantLinear.from_tensors(_t(d["qweight"], dev), _t(d["qzeros"], dev),
                                    _t(d["scales"], dev, torch.float16), _t(d["g_idx"], dev),
                                    group_size=g, zero_offset=zero_offset)


def test_codes_roundtrip_bit_exact():
    dev = require_cuda()
    for (K, N, g) in ((256, 64, 32), (4096, 1024, 128), (512, 192, 256), (1024, 128, 64)):
        d = ow.synth_gptq_linear(K, N, g, seed=K + N + g)
        ql = _quantlinear(d, g, dev)
        codes = ql.w.unpack_codes().cpu().numpy()             # [N, K]
        assert np.array_equal(codes, d["codes"].T), (K, N, g)


@pytest.mark.parametrize("K,N,g", [(4096, 12288, 128), (4096, 4096, 128), (12288, 4096, 128),
                                   (4096, 1024, 128), (256, 64, 32), (1024, 192, 64), (2048, 320, 256)])
def test_gptq_gemv_vs_oracle(K, N, g):
    dev = require_cuda()
    d, x, W = _gptq_case(K, N, g, seed=0)
    ql = _quantlinear(d, g, dev)
    y = ql(_t(x, dev, torch.bfloat16))
    torch.cuda.synchronize()
    _check(_bits(y), ow.linear_f64(x, W))
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


@pytest.mark.parametrize("M,K,N", [(1, 1024, 512), (2, 1024, 512), (3, 1024, 512), (5, 1024, 512), (8, 1024, 512),
                                   (9, 1024, 512), (13, 1024, 512), (16, 1024, 512), (21, 1024, 512),
                                   (16, 4096, 4096), (16, 4096, 6144), (16, 4096, 24576), (12, 12288, 4096)])
def test_batch_rows(M, K, N):
    """Batches of 1..21 rows: one launch per 8 rows (the n8 MMA tile), at
    small shapes and at the decode step's qkv / o / gate|up / down shapes."""
    dev = require_cuda()
    d, x, W = _gptq_case(K, N, 128, seed=3, M=M)
    ql = _quantlinear(d, 128, dev)
    y = ql(_t(x, dev, torch.bfloat16))
    _check(_bits(y), ow.linear_f64(x, W))


def test_zero_offset_one():
    dev = require_cuda()
    d, x, W = _gptq_case(1024, 256, 128, seed=5, zero_offset=1)
    ql = _quantlinear(d, 128, dev, zero_offset=1)
    _check(_bits(ql(_t(x, dev, torch.bfloat16))), ow.linear_f64(x, W))


def test_act_order_perm():
    dev = require_cuda()
    K, N, g = 1024, 256, 128
    rng = np.random.default_rng(11)
    d = ow.synth_gptq_linear(K, N, g, seed=11)
    g_idx = (rng.permutation(K) // g).astype(np.int32)     # each group gets exactly g rows
    d["g_idx"] = g_idx
    x = f32_to_bf16(rng.standard_normal((2, K)).astype(np.float32))
    W = ow.gptq_dequant(d["qweight"], d["qzeros"], d["scales"], g_idx)
    ql = _quantlinear(d, g, dev)
    _check(_bits(ql(_t(x, dev, torch.bfloat16))), ow.linear_f64(x, W))


def _ref_case(K, N, g, seed):
    rng = np.random.default_rng(seed)
    w = f32_to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    q, s, mn = ow.rtn_quantize(w, g)
    qsz = ow.pack_qsz(s, mn)
    Wnk = ow.ref_operand_weight(q, qsz, g)
    return q, qsz, Wnk


@pytest.mark.parametrize("K,N,g", [(4096, 6144, 128), (4096, 1024, 32), (12288, 4096, 128)])
def test_ref_face_vs_oracle(K, N, g):
    dev = require_cuda()
    from moss_tts_lite_b200.quant import RefW4Linear
    q, qsz, Wnk = _ref_case(K, N, g, seed=K + N)
    lin = RefW4Linear(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    rng = np.random.default_rng(7)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    y = lin(_t(x, dev, torch.bfloat16))
    _check(_bits(y), ow.linear_f64(x, Wnk.T))
    codes = lin.w.unpack_codes().cpu().numpy()
    assert np.array_equal(codes, q)


def test_epilogues_residual_swiglu_norm():
    dev = require_cuda()
    from moss_tts_lite_b200.quant import W4Weight
    from oracle import step as os_
    K, I, g = 1024, 256, 128
    rng = np.random.default_rng(21)
    # residual + norm prologue
    q, qsz, Wnk = _ref_case(K, K, g, seed=1)
    w = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    h = f32_to_bf16((rng.standard_normal((1, K)) * 3).astype(np.float32))
    nw = f32_to_bf16((1 + 0.1 * rng.standard_normal(K)).astype(np.float32))
    ht = _t(h, dev, torch.bfloat16)
    y = w.linear(ht, norm_weight=_t(nw, dev, torch.bfloat16), residual=ht.clone())
    xn = os_.rms_norm(h, nw)
    lin = ow.linear_bf16(xn, Wnk.T)
    ref = f32_to_bf16(bf16_to_f32(h) + bf16_to_f32(lin))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95          # identical except rare 1-ulp roundings
    # SwiGLU: gate/up interleaved in 32-column blocks
    qg, qszg, Wg = _ref_case(K, I, g, seed=2)
    qu, qszu, Wu = _ref_case(K, I, g, seed=3)
    blocks = []
    qsb = []
    for b in range(I // 32):
        blocks += [qg[32 * b:32 * b + 32], qu[32 * b:32 * b + 32]]
        qsb += [qszg[:, 32 * b:32 * b + 32], qszu[:, 32 * b:32 * b + 32]]
    qf = np.concatenate(blocks, 0)
    qszf = np.concatenate(qsb, 1)
    wf = W4Weight.from_ref(_t(qf, dev), _t(qszf, dev, torch.bfloat16), g)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    y = wf.linear(_t(x, dev, torch.bfloat16), swiglu=True)
    ref = os_.silu_mul(ow.linear_bf16(x, Wg.T), ow.linear_bf16(x, Wu.T))
    d = np.abs(bf16_to_f32(_bits(y)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95


def test_deterministic_and_graph_capture():
    dev = require_cuda()
    d, x, W = _gptq_case(4096, 4096, 128, seed=9)
    ql = _quantlinear(d, 128, dev)
    xt = _t(x, dev, torch.bfloat16)
    y1 = ql(xt).clone()
    y2 = ql(xt).clone()
    assert torch.equal(y1, y2)
    out = torch.empty_like(y1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ql.w.linear(xt, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ql.w.linear(xt, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y1)


def test_vs_reference_tinygemm():
    """Same codes through the reference's own kernel (torch._weight_int4pack_mm,
    tinygemm) when the reference package is importable on this box: the same
    bf16 operand, so the outputs agree up to the fp32 summation order (bitwise
    for almost every element, never more than one bf16 ulp apart)."""
    dev = require_cuda()
    ref = pytest.importorskip("moss_tts_lite.gptq")
    from moss_tts_lite_b200.quant import RefW4Linear
    K, N, g = 4096, 4096, 128
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(0)) * 0.02).to(torch.bfloat16).to(dev)
    q, s, mn = ref.rtn_quantize(w, g)
    packed, qsz = ref.pack_fast(q, s, mn, 8)
    for M in (1, 8):
        x = torch.randn(M, K, dtype=torch.bfloat16, device=dev)
        y_ref = torch._weight_int4pack_mm(x, packed, g, qsz)
        y = RefW4Linear(q, qsz, g)(x)
        same = (y.view(torch.int16) == y_ref.view(torch.int16)).float().mean().item()
        # one bf16 ulp, or the fp32 summation noise where an output cancels to ~0
        tol = torch.clamp(y_ref.float().abs() * 2.0 ** -7, min=1e-4)
        assert same > 0.99, (M, same)
        assert bool(((y.float() - y_ref.float()).abs() <= tol * 1.001).all()), M
        w_eff = ref.effective_weight(q, qsz, g)
        exact = x.float() @ w_eff.t()
        rel_mine = ((y.float() - exact).norm() / exact.norm()).item()
        assert rel_mine < 5e-3, rel_mine
@pytest.mark.parametrize("K,N,M", [(4096, 4096, 1), (12288, 4096, 1), (4096, 24576, 1), (1024, 128, 2),
                                   (4096, 1024, 3)])
def test_back_to_back_same_scratch(K, N, M):
    """64 launches of one linear (one scratch) queued back to back, with
    programmatic dependent launch overlapping neighbours: every output equals
    the same input's output from a launch run alone (bitwise), and the
    scratch's split-K counters are re-armed to zero afterwards."""
    dev = require_cuda()
    from moss_tts_lite_b200.quant import RefW4Linear
    q, qsz, Wnk = _ref_case(K, N, 128, seed=K + N + M)
    lin = RefW4Linear(_t(q, dev), _t(qsz, dev, torch.bfloat16), 128)
    rng = np.random.default_rng(M)
    xs = [_t(f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32)), dev, torch.bfloat16) for _ in range(4)]
    alone = []
    for x in xs:
        alone.append(lin(x).clone())
        torch.cuda.synchronize()
    outs = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(64)]
    for i in range(64):
        lin.w.linear(xs[i % 4], out=outs[i])
    torch.cuda.synchronize()
    for i in range(64):
        assert torch.equal(outs[i], alone[i % 4]), i
    _check(_bits(alone[0]), ow.linear_f64(_bits(xs[0]), Wnk.T))
    from moss_tts_lite_b200 import _lib
    zb = (N // 64 * 4 + 255) // 256 * 256   # split-K counters
    assert int(lin.w.scratch[:zb].count_nonzero()) == 0
    assert _lib.device_status() == 0


@pytest.mark.parametrize("K,N,g", [(4096, 1024, 128), (1024, 192, 64), (512, 128, 32)])
def test_dequant_effective_weights(K, N, g):
    """mtl_w4_dequant: the reference's effective_weight (q - 8) * scale + zero
    (gptq.py:87-97) rounded to bf16, for every element (one fp32 FMA: equal to
    the oracle's multiply-then-add except rare 1-ulp bf16 roundings)."""
    dev = require_cuda()
    from moss_tts_lite_b200.quant import RefW4Linear
    q, qsz, Wnk = _ref_case(K, N, g, seed=K + N + g)
    lin = RefW4Linear(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    got = _bits(lin.w.dequant())
    want = f32_to_bf16(Wnk.astype(np.float32))
    diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.999


@pytest.mark.parametrize("M", [1, 3])
def test_activation_range_beyond_fp16(M):
    """Activation groups with |x| up to 1e6 (past fp16's 65504) and down to
    1e-8 (below fp16's normal range) meet the same tolerance against the fp64
    product as ordinary ones (bf16 staging covers the range; an fp16-staged
    variant with per-group power-of-two scaling failed this case)."""
    dev = require_cuda()
    from moss_tts_lite_b200.quant import RefW4Linear
    K, N, g = 4096, 1024, 128
    q, qsz, Wnk = _ref_case(K, N, g, seed=77)
    lin = RefW4Linear(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)
    rng = np.random.default_rng(78)
    mags = np.array([1e6, 3e4, 1.0, 1e-3, 1e-8, 7e4, 0.01, 200.0])
    xf = rng.standard_normal((M, K)) * np.repeat(np.resize(mags, K // g), g)[None, :]
    x = f32_to_bf16(xf.astype(np.float32))
    y = lin(_t(x, dev, torch.bfloat16))
    torch.cuda.synchronize()
    assert np.isfinite(bf16_to_f32(_bits(y))).all()
    _check(_bits(y), ow.linear_f64(x, Wnk.T))
