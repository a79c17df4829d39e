"""Persistent W4 chain (mtl_w4_chain: one launch for o -> gate|up -> down ->
next q|k|v) on the B200 against the CPU oracle and against the one-launch-
per-linear GEMV.  Same gates as the GEMV's own tests (tests/test_w4_gpu.py,
after the reference's kernel-semantics test tests/test_quant.py:96-119):
each phase's output equals the product with the reference's W4 operand
(oracle.w4.ref_operand_weight) within the north-star tolerance, checked
phase by phase on the chain's own inputs; the chain's results are bitwise
reproducible (graph replay = eager, in-place = separate buffers) and the
barrier word is re-armed after every launch."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import step as ost
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16
from test_w4_gpu import _bits, _check, _ref_case, _t

pytestmark = pytest.mark.gpu


def _strip(q, qsz, g, dev):
    from moss_tts_lite_b200.quant import StripWeight
    return StripWeight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g)


def _run(phases, g, dev, bar=None):
    from moss_tts_lite_b200 import _lib, kernels
    if bar is None:
        bar = torch.zeros(32, dtype=torch.int32, device=dev)
    kernels.w4_chain(phases, g, bar[0])
    torch.cuda.synchronize()
    assert int(bar[0]) == 0, "barrier word not re-armed"
    assert _lib.device_status() == 0


def _close_to_gemv(a_bits, b_bits):
    """Chain vs one-launch GEMV: the same products summed in another fp32
    order, each rounded once to bf16 - equal or a rounding step apart."""
    a, b = bf16_to_f32(a_bits).astype(np.float64), bf16_to_f32(b_bits).astype(np.float64)
    d = np.abs(a - b)
    assert (d <= np.maximum(1e-4, np.abs(b) * 2.0 ** -7)).all(), d.max()
    assert (d == 0).mean() > 0.9, (d == 0).mean()


@pytest.mark.parametrize("K,N,g", [(4096, 6144, 128), (4096, 16, 128), (1024, 4112, 64), (2048, 320, 256),
                                   (12288, 4096, 128), (4096, 24576, 128)])
def test_single_phase_vs_oracle_and_gemv(K, N, g):
    dev = require_cuda()
    from moss_tts_lite_b200.quant import W4Weight
    q, qsz, Wnk = _ref_case(K, N, g, seed=K + N + g)
    rng = np.random.default_rng(5)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    xt = _t(x, dev, torch.bfloat16).view(-1)
    y = torch.empty(N, dtype=torch.bfloat16, device=dev)
    _run([{"w": _strip(q, qsz, g, dev), "x": xt, "y": y}], g, dev)
    _check(_bits(y).reshape(1, N), ow.linear_f64(x, Wnk.T))
    if N % 64 == 0:   # the GEMV's 64-column tiles
        yg = W4Weight.from_ref(_t(q, dev), _t(qsz, dev, torch.bfloat16), g).linear(xt.view(1, K))
        _close_to_gemv(_bits(y), _bits(yg).reshape(-1))


def test_epilogues_norm_residual_swiglu_vs_oracle():
    dev = require_cuda()
    from moss_tts_lite_b200.quant import W4Weight
    K, I, g = 1024, 512, 128
    rng = np.random.default_rng(21)
    # RMSNorm prologue + residual epilogue, y aliasing the residual
    q, qsz, Wnk = _ref_case(K, K, g, seed=1)
    h = f32_to_bf16((rng.standard_normal((1, K)) * 3).astype(np.float32))
    nw = f32_to_bf16((1 + 0.1 * rng.standard_normal(K)).astype(np.float32))
    ht = _t(h, dev, torch.bfloat16).view(-1).clone()
    xt = ht.clone()              # a phase's y must not overlap its own x
    nwt = _t(nw, dev, torch.bfloat16)
    _run([{"w": _strip(q, qsz, g, dev), "x": xt, "y": ht, "norm_w": nwt, "residual": ht}], g, dev)
    ref = f32_to_bf16(bf16_to_f32(h) + bf16_to_f32(ow.linear_bf16(ost.rms_norm(h, nw), Wnk.T)))
    d = np.abs(bf16_to_f32(_bits(ht)) - bf16_to_f32(ref.reshape(-1)))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95
    # SwiGLU: a gate|up weight packed for the GEMV (32-row blocks) re-packed as strips
    qg, qszg, Wg = _ref_case(K, I, g, seed=2)
    qu, qszu, Wu = _ref_case(K, I, g, seed=3)
    qf = np.concatenate([np.stack([qg[i:i + 32], qu[i:i + 32]]) for i in range(0, I, 32)]).reshape(2 * I, K)
    qszf = np.concatenate([np.stack([qszg[:, i:i + 32], qszu[:, i:i + 32]], 1) for i in range(0, I, 32)],
                          1).reshape(K // g, 2 * I, 2)
    wf = W4Weight.from_ref(_t(qf, dev), _t(qszf, dev, torch.bfloat16), g)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    xt = _t(x, dev, torch.bfloat16).view(-1)
    act = torch.empty(I, dtype=torch.bfloat16, device=dev)
    _run([{"w": wf.to_strip(swiglu_block=32), "x": xt, "y": act, "swiglu": True}], g, dev)
    ref = ost.silu_mul(ow.linear_bf16(x, Wg.T), ow.linear_bf16(x, Wu.T)).reshape(-1)
    d = np.abs(bf16_to_f32(_bits(act)) - bf16_to_f32(ref))
    assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max()
    assert (d == 0).mean() > 0.95
    _close_to_gemv(_bits(act), _bits(wf.linear(xt.view(1, K), swiglu=True)).reshape(-1))


def _layer(H, I, NQKV, g, seed, dev):
    """One layer's four fused W4 weights (oracle operands + strips)."""
    from moss_tts_lite_b200.quant import W4Weight
    qo, zo, Wo = _ref_case(H, H, g, seed)
    qg, zg, Wg = _ref_case(H, I, g, seed + 1)
    qu, zu, Wu = _ref_case(H, I, g, seed + 2)
    qd, zd, Wd = _ref_case(I, H, g, seed + 3)
    qq, zq, Wq = _ref_case(H, NQKV, g, seed + 4)
    qf = np.concatenate([np.stack([qg[i:i + 32], qu[i:i + 32]]) for i in range(0, I, 32)]).reshape(2 * I, H)
    zf = np.concatenate([np.stack([zg[:, i:i + 32], zu[:, i:i + 32]], 1) for i in range(0, I, 32)],
                        1).reshape(H // g, 2 * I, 2)
    gu = W4Weight.from_ref(_t(qf, dev), _t(zf, dev, torch.bfloat16), g).to_strip(swiglu_block=32)
    return {"o": (_strip(qo, zo, g, dev), Wo), "gu": (gu, Wg, Wu), "down": (_strip(qd, zd, g, dev), Wd),
            "qkv": (_strip(qq, zq, g, dev), Wq)}


@pytest.mark.parametrize("H,I,NQKV", [(4096, 12288, 6144), (1024, 2816, 1536)])
def test_four_phase_chain_phase_by_phase(H, I, NQKV):
    """o -> gate|up -> down -> q|k|v at the benchmark configuration's shapes
    (and a small model's), every intermediate in its own buffer and checked
    against the oracle on the chain's own input to that phase; then the
    engine's in-place form (h updated in place) gives the same bits, and a
    captured graph replays them."""
    dev = require_cuda()
    g = 128
    L = _layer(H, I, NQKV, g, seed=40, dev=dev)
    rng = np.random.default_rng(9)
    h0 = f32_to_bf16((rng.standard_normal(H) * 2).astype(np.float32))
    attn = f32_to_bf16(rng.standard_normal(H).astype(np.float32))
    n1 = f32_to_bf16((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    n2 = f32_to_bf16((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    T = lambda a: _t(a, dev, torch.bfloat16)
    h0t, at, n1t, n2t = T(h0), T(attn), T(n1), T(n2)
    h1 = torch.empty(H, dtype=torch.bfloat16, device=dev)
    act = torch.empty(I, dtype=torch.bfloat16, device=dev)
    h2 = torch.empty(H, dtype=torch.bfloat16, device=dev)
    qkv = torch.empty(NQKV, dtype=torch.bfloat16, device=dev)
    phases = [{"w": L["o"][0], "x": at, "y": h1, "residual": h0t},
              {"w": L["gu"][0], "x": h1, "y": act, "norm_w": n1t, "swiglu": True},
              {"w": L["down"][0], "x": act, "y": h2, "residual": h1},
              {"w": L["qkv"][0], "x": h2, "y": qkv, "norm_w": n2t}]
    _run(phases, g, dev)
    tol = lambda got, ref: (np.abs(bf16_to_f32(got) - bf16_to_f32(ref)),
                            2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max())
    h1b, actb, h2b, qkvb = _bits(h1), _bits(act), _bits(h2), _bits(qkv)
    ref1 = ost.add_bf16(h0, ow.linear_bf16(attn[None], L["o"][1].T)[0])
    ref2 = ost.silu_mul(ow.linear_bf16(ost.rms_norm(h1b[None], n1), L["gu"][1].T),
                        ow.linear_bf16(ost.rms_norm(h1b[None], n1), L["gu"][2].T))[0]
    ref3 = ost.add_bf16(h1b, ow.linear_bf16(actb[None], L["down"][1].T)[0])
    ref4 = ow.linear_bf16(ost.rms_norm(h2b[None], n2), L["qkv"][1].T)[0]
    for name, got, ref in (("o", h1b, ref1), ("gu", actb, ref2), ("down", h2b, ref3), ("qkv", qkvb, ref4)):
        d, bound = tol(got, ref)
        assert d.max() <= bound, (name, d.max())
        assert (d == 0).mean() > 0.9, (name, (d == 0).mean())
    # in place, as the decode step runs it: h updated by o and by down
    h = h0t.clone()
    act2 = torch.empty_like(act)
    qkv2 = torch.empty_like(qkv)
    inplace = [{"w": L["o"][0], "x": at, "y": h, "residual": h},
               {"w": L["gu"][0], "x": h, "y": act2, "norm_w": n1t, "swiglu": True},
               {"w": L["down"][0], "x": act2, "y": h, "residual": h},
               {"w": L["qkv"][0], "x": h, "y": qkv2, "norm_w": n2t}]
    _run(inplace, g, dev)
    assert np.array_equal(_bits(h), h2b) and np.array_equal(_bits(qkv2), qkvb)
    # graph capture + replays: bitwise the eager result, barrier re-armed each time
    from moss_tts_lite_b200 import _lib, kernels
    bar = torch.zeros(32, dtype=torch.int32, device=dev)
    gph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.graph(gph, stream=s):
        kernels.w4_chain(inplace, g, bar[0])
    for _ in range(3):
        h.copy_(h0t)
        gph.replay()
        torch.cuda.synchronize()
        assert int(bar[0]) == 0
        assert np.array_equal(_bits(h), h2b) and np.array_equal(_bits(qkv2), qkvb)
    assert _lib.device_status() == 0


def test_chain_rejects_bad_arguments():
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib, kernels
    from moss_tts_lite_b200.quant import StripWeight
    q, qsz, _ = _ref_case(1024, 64, 128, seed=3)
    w = _strip(q, qsz, 128, dev)
    x = torch.zeros(1024, dtype=torch.bfloat16, device=dev)
    y = torch.zeros(64, dtype=torch.bfloat16, device=dev)
    bar = torch.zeros(32, dtype=torch.int32, device=dev)
    with pytest.raises(_lib.MtlError):
        kernels.w4_chain([{"w": w, "x": x, "y": y}] * 5, 128, bar[0])          # > 4 phases
    with pytest.raises(_lib.MtlError):
        kernels.w4_chain([{"w": w, "x": x, "y": y}], 32, bar[0])               # group size not served
    with pytest.raises(_lib.MtlError):
        kernels.w4_chain([{"w": w, "x": x[1:], "y": y}], 128, bar[0])          # x misaligned
    bad = StripWeight(w.tiles, 1024, 72, 128)                                   # N % 16 != 0
    with pytest.raises(_lib.MtlError):
        kernels.w4_chain([{"w": bad, "x": x, "y": y}], 128, bar[0])
    with pytest.raises(_lib.MtlError):                                          # y overlaps its own x
        kernels.w4_chain([{"w": w, "x": x, "y": x[:64]}], 128, bar[0])
    torch.cuda.synchronize()
    assert int(bar[0]) == 0 and _lib.device_status() == 0


def test_engine_chain_matches_per_linear_launches():
    """FastMossTTS with the chain (default) vs one launch per linear on the
    same W4 weights: decode steps agree to the two kernels' fp32 summation
    orders, and the chained step graph replays bitwise like its eager pass."""
    dev = require_cuda()
    from moss_tts_lite_b200.fast import FastMossTTS
    from moss_tts_lite_b200.model import MossTTSModel
    from test_step_gpu import _prompt, _torch_weights, _weights
    w = _weights(seed=31)
    outs = {}
    for chain in (True, False):
        m = MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=256)
        fast = FastMossTTS(m, quant="w4", w4_group_size=128, chain=chain)
        assert fast.chain == chain
        ids = _prompt(6, seed=4)
        fast.prefill(_t(ids, dev).view(1, 6, 33))
        fast.capture()
        rng = np.random.default_rng(2)
        res = []
        for t in range(6):
            row = np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
            lt, la, h, two = fast.step(_t(row, dev).view(1, 33), 6 + t, audio2=True)
            res.append((bf16_to_f32(_bits(h)), bf16_to_f32(_bits(la))))
        if chain:   # eager pass of the chained step = its graph replay
            fast.prefill(_t(ids, dev).view(1, 6, 33))
            rng = np.random.default_rng(2)
            for t in range(6):
                row = np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
                fast.ids_row.view(-1).copy_(_t(row, dev))
                fast.pos_dev.fill_(6 + t)
                fast._run_eager(True)
                assert np.array_equal(bf16_to_f32(_bits(fast.h_final)), res[t][0])
        outs[chain] = res
        del fast, m
        torch.cuda.empty_cache()
    for (ha, la), (hb, lb) in zip(outs[True], outs[False]):
        rel = np.linalg.norm(ha - hb) / np.linalg.norm(hb)
        assert rel < 2e-2, rel
        fin = np.isfinite(lb)                  # the masked pad column is -inf in both
        assert np.array_equal(fin, np.isfinite(la))
        assert np.abs(la[fin] - lb[fin]).max() < 0.1
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def _run_rows(phases, g):
    from moss_tts_lite_b200 import _lib, kernels
    bar = torch.zeros(32, dtype=torch.int32, device=phases[0]["x"].device)
    kernels.w4_chain_rows(phases, g, bar[0])
    torch.cuda.synchronize()
    assert int(bar[0]) == 0, "barrier word not re-armed"
    assert _lib.device_status() == 0


@pytest.mark.parametrize("M,K,N,g", [(2, 4096, 6144, 128), (9, 12288, 4096, 128), (16, 4096, 1536, 128),
                                     (16, 1024, 4112, 64), (5, 2048, 320, 256)])
def test_rows_single_phase_vs_oracle(M, K, N, g):
    """mtl_w4_chain_rows: every row against the product with the reference's
    operand (K = 12288 runs three x slices)."""
    dev = require_cuda()
    q, qsz, Wnk = _ref_case(K, N, g, seed=K + N + M)
    rng = np.random.default_rng(M)
    x = f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    xt = _t(x, dev, torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    _run_rows([{"w": _strip(q, qsz, g, dev), "x": xt, "y": y}], g)
    _check(_bits(y), ow.linear_f64(x, Wnk.T))


def test_rows_four_phases_phase_by_phase_and_replay():
    """o -> gate|up -> down -> q|k|v for 16 rows at the benchmark
    configuration's shapes, each phase against the oracle on the chain's own
    input to it, then in place as the batched step runs it (same bits) and
    as a replayed graph (same bits)."""
    dev = require_cuda()
    H, I, NQKV, g, M = 4096, 12288, 6144, 128, 16
    L = _layer(H, I, NQKV, g, seed=70, dev=dev)
    rng = np.random.default_rng(19)
    h0 = f32_to_bf16((rng.standard_normal((M, H)) * 2).astype(np.float32))
    attn = f32_to_bf16(rng.standard_normal((M, H)).astype(np.float32))
    n1 = f32_to_bf16((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    n2 = f32_to_bf16((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    T = lambda a: _t(a, dev, torch.bfloat16)
    h0t, at, n1t, n2t = T(h0), T(attn), T(n1), T(n2)
    h1 = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    act = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
    h2 = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    qkv = torch.empty(M, NQKV, dtype=torch.bfloat16, device=dev)
    _run_rows([{"w": L["o"][0], "x": at, "y": h1, "residual": h0t},
               {"w": L["gu"][0], "x": h1, "y": act, "norm_w": n1t, "swiglu": True},
               {"w": L["down"][0], "x": act, "y": h2, "residual": h1},
               {"w": L["qkv"][0], "x": h2, "y": qkv, "norm_w": n2t}], g)
    h1b, actb, h2b, qkvb = _bits(h1), _bits(act), _bits(h2), _bits(qkv)
    ref1 = ost.add_bf16(h0, ow.linear_bf16(attn, L["o"][1].T))
    ref2 = ost.silu_mul(ow.linear_bf16(ost.rms_norm(h1b, n1), L["gu"][1].T),
                        ow.linear_bf16(ost.rms_norm(h1b, n1), L["gu"][2].T))
    ref3 = ost.add_bf16(h1b, ow.linear_bf16(actb, L["down"][1].T))
    ref4 = ow.linear_bf16(ost.rms_norm(h2b, n2), L["qkv"][1].T)
    for name, got, ref in (("o", h1b, ref1), ("gu", actb, ref2), ("down", h2b, ref3), ("qkv", qkvb, ref4)):
        d = np.abs(bf16_to_f32(got) - bf16_to_f32(ref))
        assert d.max() <= 2e-2 + 1e-2 * np.abs(bf16_to_f32(ref)).max(), (name, d.max())
        assert (d == 0).mean() > 0.9, (name, (d == 0).mean())
    h = h0t.clone()
    act2, qkv2 = torch.empty_like(act), torch.empty_like(qkv)
    inplace = [{"w": L["o"][0], "x": at, "y": h, "residual": h},
               {"w": L["gu"][0], "x": h, "y": act2, "norm_w": n1t, "swiglu": True},
               {"w": L["down"][0], "x": act2, "y": h, "residual": h},
               {"w": L["qkv"][0], "x": h, "y": qkv2, "norm_w": n2t}]
    _run_rows(inplace, g)
    assert np.array_equal(_bits(h), h2b) and np.array_equal(_bits(qkv2), qkvb)
    from moss_tts_lite_b200 import _lib, kernels
    bar = torch.zeros(32, dtype=torch.int32, device=dev)
    gph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(gph, stream=s):
        kernels.w4_chain_rows(inplace, g, bar[0])
    for _ in range(2):
        h.copy_(h0t)
        gph.replay()
        torch.cuda.synchronize()
        assert int(bar[0]) == 0
        assert np.array_equal(_bits(h), h2b) and np.array_equal(_bits(qkv2), qkvb)
    assert _lib.device_status() == 0


def test_rows_reject_bad_arguments():
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib, kernels
    q, qsz, _ = _ref_case(8192, 64, 128, seed=5)
    w = _strip(q, qsz, 128, dev)
    x = torch.zeros(4, 8192, dtype=torch.bfloat16, device=dev)
    y = torch.zeros(4, 64, dtype=torch.bfloat16, device=dev)
    nw = torch.ones(8192, dtype=torch.bfloat16, device=dev)
    bar = torch.zeros(32, dtype=torch.int32, device=dev)
    with pytest.raises(_lib.MtlError):          # RMSNorm needs K <= 4096 (one x slice)
        kernels.w4_chain_rows([{"w": w, "x": x, "y": y, "norm_w": nw}], 128, bar[0])
    x17 = torch.zeros(17, 8192, dtype=torch.bfloat16, device=dev)
    y17 = torch.zeros(17, 64, dtype=torch.bfloat16, device=dev)
    with pytest.raises(_lib.MtlError):          # more than 16 rows
        kernels.w4_chain_rows([{"w": w, "x": x17, "y": y17}], 128, bar[0])
    torch.cuda.synchronize()
    assert int(bar[0]) == 0 and _lib.device_status() == 0
