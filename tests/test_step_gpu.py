"""Decoder-step kernels and the whole-step engine on the B200 against the
numpy oracle (pinned bit-exact to the reference model in test_oracle_cpu)
and, where the reference package is importable, against the reference
itself.  Mirrors the reference's own gates: bitwise graph replay vs eager
(tests/test_fast.py:57-93), kernel-vs-dequant semantics (tests/test_quant.py
:96-119), and teacher-forced text argmax / audio top-25 cover
(tests/test_quant.py:492-542)."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import step as ost
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu

SMALL = dict(hidden=1024, n_layers=3, n_heads=8, n_kv=2, head_dim=128, inter=2816, vocab=151936)


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.to(dev)


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _weights(seed=0, std=0.02, norm_ones=False):
    return ost.synth_weights(SMALL["hidden"], SMALL["n_layers"], SMALL["n_heads"], SMALL["n_kv"],
                             SMALL["head_dim"], SMALL["inter"], vocab=SMALL["vocab"], seed=seed, std=std,
                             norm_ones=norm_ones)


def _torch_weights(w, dev):
    return {k: _t(v, dev, torch.bfloat16) for k, v in w.items()}


def _prompt(L, seed=3, audio_start=True):
    rng = np.random.default_rng(seed)
    ids = np.zeros((L, 33), np.int64)
    ids[:, 0] = rng.integers(0, 151643, L)
    ids[:, 1:] = rng.integers(0, 1024, (L, 32))
    if audio_start:
        ids[-1, 0] = ost.AUDIO_START_TOKEN_ID
    return ids


# ------------------------------------------------------------------ kernels
def test_rtn_quantize_bit_exact():
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(0)
    for g in (32, 128):
        w = f32_to_bf16((rng.standard_normal((192, 1024)) * 0.02).astype(np.float32))
        w[0, :g] = 0
        q, qsz = kernels.rtn_quantize(_t(w, dev, torch.bfloat16), g)
        qo, so, mno = ow.rtn_quantize(w, g)
        assert np.array_equal(q.cpu().numpy(), qo)
        assert np.array_equal(_bits(qsz), ow.pack_qsz(so, mno))


def test_rtn_matches_reference_fast_quantize():
    dev = require_cuda()
    ref = pytest.importorskip("moss_tts_lite.gptq")
    from moss_tts_lite_b200 import kernels
    w = (torch.randn(512, 4096, generator=torch.Generator().manual_seed(1)) * 0.05).to(torch.bfloat16).to(dev)
    q_ref, s_ref, mn_ref = ref.rtn_quantize(w, 128)
    _, qsz_ref = ref.pack_fast(q_ref, s_ref, mn_ref, 8)
    q, qsz = kernels.rtn_quantize(w, 128)
    assert torch.equal(q, q_ref) and torch.equal(qsz, qsz_ref)


def test_embed_sum_bit_exact():
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(2)
    H, V = 512, 5000
    et = f32_to_bf16((rng.standard_normal((V, H)) * 0.02).astype(np.float32))
    ea = f32_to_bf16((rng.standard_normal((32 * 1025, H)) * 0.02).astype(np.float32))
    ids = np.zeros((3, 33), np.int64)
    ids[:, 0] = rng.integers(0, V, 3)
    ids[:, 1:] = rng.integers(0, 1025, (3, 32))
    out = torch.empty(3, H, dtype=torch.bfloat16, device=dev)
    kernels.embed_sum(_t(ids, dev), _t(et, dev, torch.bfloat16), _t(ea, dev, torch.bfloat16), out)
    h = et[ids[:, 0]]
    for i in range(32):
        h = ost.add_bf16(h, ea.reshape(32, 1025, H)[i][ids[:, i + 1]])
    assert np.array_equal(_bits(out), h)


def test_rmsnorm_and_argmax():
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(4)
    x = f32_to_bf16((rng.standard_normal((4, 4096)) * 3).astype(np.float32))
    w = f32_to_bf16((1 + 0.1 * rng.standard_normal(4096)).astype(np.float32))
    out = torch.empty(4, 4096, dtype=torch.bfloat16, device=dev)
    kernels.rmsnorm(_t(x, dev, torch.bfloat16), _t(w, dev, torch.bfloat16), out)
    ref = ost.rms_norm(x, w)
    d = np.abs(bf16_to_f32(_bits(out)) - bf16_to_f32(ref))
    assert (d == 0).mean() > 0.99 and d.max() <= 2 ** -6 * np.abs(bf16_to_f32(ref)).max()
    # argmax: ties -> first index, -inf pads never win
    lg = f32_to_bf16(rng.standard_normal((32, 1025)).astype(np.float32))
    lg[3, [7, 900]] = f32_to_bf16(np.float32(9.0))
    lg[:, 1024] = 0xFF80
    o = torch.empty(32, dtype=torch.long, device=dev)
    kernels.argmax_rows(_t(lg, dev, torch.bfloat16), o)
    assert np.array_equal(o.cpu().numpy(), np.argmax(bf16_to_f32(lg), -1))
    assert int(o[3]) == 7
    o1 = torch.empty(1, dtype=torch.long, device=dev)
    row = _t(lg[3], dev, torch.bfloat16)
    kernels.argmax_masked(row, o1, (7,))
    assert int(o1[0]) == 900


@pytest.mark.parametrize("cols", [4096, 155648, 151937])
def test_argmax_masked_grid_matches_one_cta(cols):
    """The GPU-wide text argmax (scratch given) equals the one-CTA kernel and
    numpy's first-index argmax over the non-excluded, non-NaN values, with
    planted ties, excluded maxima, -0/+0 and NaN, and re-arms its scratch."""
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(cols)
    sc = kernels.argmax_scratch(dev)
    for trial in range(6):
        x = f32_to_bf16(rng.standard_normal(cols).astype(np.float32))
        top = int(rng.integers(0, cols))
        excl = tuple(int(v) for v in rng.choice(cols, size=trial + 1, replace=False))
        x[top] = f32_to_bf16(np.array([9.0], np.float32))[0]
        if trial == 1:
            x[list(excl)] = 0x7F80                        # excluded +inf never wins
        if trial == 2:
            x[cols - 1] = x[top]                           # tie: first index wins
        if trial == 3:
            x[:] = 0x8000                                  # all -0 except one +0
            x[cols // 2] = 0x0000
        if trial == 4:
            x[top] = 0x7FC0                                # NaN is skipped
        ref = bf16_to_f32(x).astype(np.float64)
        ref[np.isnan(ref)] = -np.inf
        ref[list(excl)] = -np.inf
        want = int(np.argmax(ref))
        xt = _t(x, dev, torch.bfloat16)
        o1 = torch.empty(1, dtype=torch.long, device=dev)
        o2 = torch.empty(1, dtype=torch.long, device=dev)
        kernels.argmax_masked(xt, o1, excl)
        kernels.argmax_masked(xt, o2, excl, scratch=sc)
        assert int(o1[0]) == want and int(o2[0]) == want, (trial, int(o1[0]), int(o2[0]), want)
    torch.cuda.synchronize()
    assert int(sc.count_nonzero()) == 0


@pytest.mark.parametrize("s1,rep,streams,stable,splits",
                         [(1, 4, 1, False, 16), (7, 4, 1, True, 16), (64, 4, 1, False, 16), (65, 8, 1, True, 16),
                          (130, 4, 1, False, 16), (641, 4, 2, True, 16), (2000, 4, 1, True, 16),
                          (4096, 2, 1, False, 16), (3000, 8, 2, False, 16),
                          (641, 4, 3, True, 1), (2000, 4, 2, True, 1), (3000, 8, 2, False, 3), (300, 4, 4, False, 1)])
def test_attention_decode_vs_oracle(s1, rep, streams, stable, splits):
    """Fused q/k-norm + RoPE + append + split-KV attention against the oracle,
    at cache lengths around the 64-position tiles, GQA ratios 2-8, up to four
    streams, 16 / 3 / 1 splits per head (one split: a CTA streams its whole
    cache, as the batched step does), with the cache rows past pos poisoned
    with NaN (masked rows must contribute exactly nothing)."""
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib, kernels
    rng = np.random.default_rng(s1 + rep)
    nkv, D, max_seq = 2, 128, 4096
    nh = nkv * rep
    pos = s1 - 1
    kc = f32_to_bf16(rng.standard_normal((streams, nkv, max_seq, D)).astype(np.float32))
    vc = f32_to_bf16(rng.standard_normal((streams, nkv, max_seq, D)).astype(np.float32))
    kc[:, :, s1:] = 0x7FC0   # NaN past the decoded position
    vc[:, :, s1:] = 0x7FC0
    qkv = f32_to_bf16((rng.standard_normal((streams, (nh + 2 * nkv) * D)) * 2).astype(np.float32))
    qn = f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32))
    kn = f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32))
    cos, sin = ost.rope_tables(max_seq, D)
    scratch = torch.zeros(_lib.attn_scratch_bytes(streams, nh, nkv, splits), dtype=torch.uint8, device=dev)
    kct, vct = _t(kc, dev, torch.bfloat16), _t(vc, dev, torch.bfloat16)
    out = torch.empty(streams, nh * D, dtype=torch.bfloat16, device=dev)
    kernels.attn_decode(_t(qkv, dev, torch.bfloat16), _t(qn, dev, torch.bfloat16), _t(kn, dev, torch.bfloat16),
                        _t(cos, dev, torch.bfloat16), _t(sin, dev, torch.bfloat16), kct, vct,
                        torch.full((streams,), pos, device=dev), nh, nkv, splits, out, scratch, streams=streams,
                        cache_stream_stride=nkv * max_seq * D, kv_stable=stable)
    torch.cuda.synchronize()
    y_all = bf16_to_f32(_bits(out)).reshape(streams, nh, D)
    for st in range(streams):
        # oracle: norm + rope + append + attention
        q = ost.apply_rope(ost.rms_norm(qkv[st, :nh * D].reshape(nh, D), qn), cos[pos], sin[pos])
        k = ost.apply_rope(ost.rms_norm(qkv[st, nh * D:(nh + nkv) * D].reshape(nkv, D), kn), cos[pos], sin[pos])
        v = qkv[st, (nh + nkv) * D:].reshape(nkv, D)
        kc[st, :, pos], vc[st, :, pos] = k, v
        assert np.array_equal(_bits(kct)[st, :, pos], k) and np.array_equal(_bits(vct)[st, :, pos], v)
        ref = np.empty((nh, D))
        for h in range(nh):
            g = h // rep
            ref[h] = ost.attend(bf16_to_f32(q[h:h + 1]).astype(np.float64),
                                bf16_to_f32(kc[st, g, :s1]).astype(np.float64),
                                bf16_to_f32(vc[st, g, :s1]).astype(np.float64), 1 / np.sqrt(D))[0]
        y = y_all[st]
        assert np.isfinite(y).all()
        # split-KV rounds exp(s - running max of its slice) instead of
        # exp(s - row max) before P.V: a few bf16 ulps
        assert np.abs(y - ref).max() <= 2e-2 * max(1.0, np.abs(ref).max()), (st, np.abs(y - ref).max())
    from moss_tts_lite_b200 import _lib as L
    assert L.device_status() == 0


@pytest.mark.parametrize("p0,R,rep", [(0, 8, 4), (60, 8, 4), (125, 5, 8), (1021, 8, 2), (3000, 3, 4)])
def test_attention_prefill_chunk_matches_row_by_row(p0, R, rep):
    """Prefill chunk: K/V append of R rows, then one attention launch with the
    rows as streams over the shared cache, must equal R single-row decode
    attentions run in position order (outputs and cache bit for bit)."""
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib, kernels
    rng = np.random.default_rng(p0 + R)
    nkv, D, max_seq, splits = 2, 128, 4096, 16
    nh = nkv * rep
    kc = f32_to_bf16(rng.standard_normal((nkv, max_seq, D)).astype(np.float32))
    vc = f32_to_bf16(rng.standard_normal((nkv, max_seq, D)).astype(np.float32))
    kc[:, p0:] = 0x7FC0  # rows from the chunk on are not yet written
    vc[:, p0:] = 0x7FC0
    qkv = _t(f32_to_bf16((rng.standard_normal((R, (nh + 2 * nkv) * D)) * 2).astype(np.float32)), dev,
             torch.bfloat16)
    qn = _t(f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)), dev, torch.bfloat16)
    kn = _t(f32_to_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)), dev, torch.bfloat16)
    cos, sin = (_t(x, dev, torch.bfloat16) for x in ost.rope_tables(max_seq, D))
    pos = torch.arange(p0, p0 + R, device=dev)
    # row by row
    k1, v1 = _t(kc, dev, torch.bfloat16), _t(vc, dev, torch.bfloat16)
    s1 = torch.zeros(_lib.attn_scratch_bytes(1, nh, nkv, splits), dtype=torch.uint8, device=dev)
    o1 = torch.empty(R, nh * D, dtype=torch.bfloat16, device=dev)
    for i in range(R):
        kernels.attn_decode(qkv[i:i + 1], qn, kn, cos, sin, k1, v1, pos[i:i + 1], nh, nkv, splits, o1[i:i + 1], s1)
    # chunked
    k2, v2 = _t(kc, dev, torch.bfloat16), _t(vc, dev, torch.bfloat16)
    s2 = torch.zeros(_lib.attn_scratch_bytes(R, nh, nkv, splits), dtype=torch.uint8, device=dev)
    o2 = torch.empty(R, nh * D, dtype=torch.bfloat16, device=dev)
    kernels.attn_append(qkv, kn, cos, sin, k2, v2, pos, nh, nkv, streams=R)
    kernels.attn_decode(qkv, qn, kn, cos, sin, k2, v2, pos, nh, nkv, splits, o2, s2, streams=R)
    torch.cuda.synchronize()
    assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))
    assert torch.equal(v1.view(torch.int16), v2.view(torch.int16))
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert _lib.device_status() == 0


def test_bf16_linear_pad_and_epilogues():
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(5)
    K, N = 1024, 2050
    W = f32_to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    x = f32_to_bf16(rng.standard_normal((2, K)).astype(np.float32))
    y = torch.empty(2, N, dtype=torch.bfloat16, device=dev)
    kernels.bf16_linear(_t(x, dev, torch.bfloat16), _t(W, dev, torch.bfloat16), y, pad_period=1025, pad_col=1024)
    ref = bf16_to_f32(x).astype(np.float64) @ bf16_to_f32(W).astype(np.float64).T
    yy = bf16_to_f32(_bits(y))
    assert np.isneginf(yy[:, 1024]).all() and np.isneginf(yy[:, 2049]).all()
    mask = np.ones(N, bool)
    mask[[1024, 2049]] = False
    assert ow.close_enough(_bits(y)[:, mask], ref[:, mask])[0]


@pytest.mark.parametrize("M,N", [(16, 32800), (9, 4112), (5, 2), (3, 2050)])
def test_bf16_rows_tensor_core_heads(M, N):
    """The bf16 head kernels for several rows (5..16: the tensor-core kernel
    of the batched heads; 3: the CUDA-core kernel): final
    RMSNorm fused, pad column -inf, normed rows returned; against a torch fp32
    reference on the oracle's normed rows, and the normed rows bit-exact to
    the oracle's RMSNorm."""
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(M + N)
    K = 4096
    W = f32_to_bf16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    h = f32_to_bf16((rng.standard_normal((M, K)) * 3).astype(np.float32))
    nw = f32_to_bf16((1 + 0.1 * rng.standard_normal(K)).astype(np.float32))
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    xn = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    pad = 1025 if N % 1025 == 0 else 0
    kernels.bf16_linear(_t(h, dev, torch.bfloat16), _t(W, dev, torch.bfloat16), y, norm_weight=_t(nw, dev, torch.bfloat16),
                        x_normed=xn, pad_period=pad, pad_col=1024)
    torch.cuda.synchronize()
    xo = ost.rms_norm(h, nw)
    assert np.array_equal(_bits(xn), xo)
    ref = torch.from_numpy(bf16_to_f32(xo)).float() @ torch.from_numpy(bf16_to_f32(W)).float().T
    yy = bf16_to_f32(_bits(y))
    mask = np.ones(N, bool)
    if pad:
        mask[1024::1025] = False
        assert np.isneginf(yy[:, ~mask]).all()
    d = np.abs(yy[:, mask] - ref.numpy()[:, mask])
    assert (d <= 2e-2 + 1e-2 * np.abs(ref.numpy()[:, mask])).all(), d.max()
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


# ------------------------------------------------------------- whole model
def _oracle_model(w, max_seq):
    return ost.OracleModel(w, max_seq_len=max_seq)


def test_bf16_model_step_vs_oracle():
    dev = require_cuda()
    from moss_tts_lite_b200.model import MossTTSModel
    w = _weights(seed=11, norm_ones=False)
    m = MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=256)
    om = _oracle_model(w, 256)
    ids = _prompt(8)
    hp = m.prefill(_t(ids, dev).view(1, 8, 33)).last_hidden
    hp_o = om.prefill(ids)
    d = np.abs(bf16_to_f32(_bits(hp[0])) - bf16_to_f32(hp_o))
    # fp32-accumulated GEMVs vs the fp64 oracle differ in rare last bits, which
    # spread through the residual stream: a few ulps, most elements exact
    assert d.max() < 0.1 and (d == 0).mean() > 0.5, (d.max(), (d == 0).mean())
    rng = np.random.default_rng(7)
    agree = []
    for t in range(4):
        row = np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
        h = m.step(_t(row, dev).view(1, 1, 33)).last_hidden
        ho = om.step(row)
        d = np.abs(bf16_to_f32(_bits(h.view(-1))) - bf16_to_f32(ho.reshape(-1)))
        assert d.max() < 0.1, d.max()
        la = bf16_to_f32(_bits(m.audio_logits(h)))
        lo = bf16_to_f32(om.audio_logits(ho))
        am = np.argmax(la, -1)
        # tie-robust: the oracle's value at my argmax is within noise of its max
        agree.append((lo[np.arange(32), am] >= lo.max(-1) - 0.05).mean())
    assert np.mean(agree) > 0.97, agree


def _w4_setup(dev, seed=13, max_seq=256, chain=None):
    from moss_tts_lite_b200.fast import FastMossTTS
    from moss_tts_lite_b200.model import MossTTSModel
    w = _weights(seed=seed)
    m = MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=max_seq)
    fast = FastMossTTS(m, quant="w4", w4_group_size=128, chain=chain)
    om = _oracle_model(w, max_seq)
    recs = {}
    names = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
             "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
    for li in range(SMALL["n_layers"]):
        for n, key in names.items():
            q, s, mn = ow.rtn_quantize(w[f"language_model.layers.{li}.{key}.weight"], 128)
            recs[(li, n)] = (q, ow.pack_qsz(s, mn), 128)
    om.quantize_w4(recs)
    return fast, m, om


def test_w4_fast_step_graph_vs_eager_and_oracle():
    dev = require_cuda()
    fast, m, om = _w4_setup(dev)
    ids = _prompt(6, seed=21)
    fast.prefill(_t(ids, dev).view(1, 6, 33))
    om.prefill(ids)
    fast.capture()
    rng = np.random.default_rng(8)
    rows = [np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
            for _ in range(5)]
    # graph replay
    outs = []
    for t, row in enumerate(rows):
        lt, la, h, two = fast.step(_t(row, dev).view(1, 33), 6 + t, audio2=True)
        outs.append((_bits(la), _bits(h), _bits(two)))
    # eager re-run of the same rows from the same prefill state must be bitwise equal
    fast.prefill(_t(ids, dev).view(1, 6, 33))
    for t, row in enumerate(rows):
        fast.ids_row.view(-1).copy_(_t(row, dev))
        fast.pos_dev.fill_(6 + t)
        fast._run_eager(True)
        assert np.array_equal(_bits(fast.la_static), outs[t][0])
        assert np.array_equal(_bits(fast.h_final), outs[t][1])
        assert np.array_equal(_bits(fast.two_static), outs[t][2])
    # oracle (W4 effective weights, fp64 accumulation)
    cover = []
    for t, row in enumerate(rows):
        ho = om.step(row)
        d = np.abs(bf16_to_f32(outs[t][1].reshape(-1)) - bf16_to_f32(ho.reshape(-1)))
        assert d.max() < 0.1, (t, d.max())
        lo = bf16_to_f32(om.audio_logits(ho))
        la = bf16_to_f32(outs[t][0])
        am = np.argmax(la, -1)
        cover.append((lo[np.arange(32), am] >= lo.max(-1) - 0.05).mean())
        two_o = bf16_to_f32(om.text_logits_2way(ho))
        assert np.abs(bf16_to_f32(outs[t][2]) - two_o).max() < 0.05
    assert np.mean(cover) > 0.97, cover
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def test_w4_prefill_gemm_vs_chunked_and_oracle():
    """A 40-row prompt prefills through dequantised bf16 GEMMs (all rows per
    projection); the final hidden rows and the K/V cache agree with the
    chunked W4 prefill and with the oracle to within bf16 noise, and the
    decode steps that follow match the oracle (teacher-forced cover)."""
    dev = require_cuda()
    import moss_tts_lite_b200.fast as fm
    fast, m, om = _w4_setup(dev, seed=29, max_seq=128)
    ids = _prompt(40, seed=31)
    h_gemm = fast.prefill(_t(ids, dev).view(1, 40, 33)).last_hidden[0].clone()
    kc_gemm = m.k_cache[:, :, :40].clone()
    saved = fm._GEMM_PREFILL_ROWS
    fm._GEMM_PREFILL_ROWS = 10 ** 9
    try:
        h_chunk = fast.prefill(_t(ids, dev).view(1, 40, 33)).last_hidden[0].clone()
        kc_chunk = m.k_cache[:, :, :40].clone()
    finally:
        fm._GEMM_PREFILL_ROWS = saved
    ho = om.prefill(ids)
    a, b, o = bf16_to_f32(_bits(h_gemm)), bf16_to_f32(_bits(h_chunk)), bf16_to_f32(ho.reshape(40, -1))
    scale = np.abs(o).max()
    assert np.abs(a - b).max() < 0.05 * scale, np.abs(a - b).max()
    assert np.abs(a - o).max() < 0.05 * scale, np.abs(a - o).max()
    kg, kk = bf16_to_f32(_bits(kc_gemm)), bf16_to_f32(_bits(kc_chunk))
    kd = np.abs(kg - kk)
    # bf16 noise: normed + rotated keys differ by about one ulp in part of the elements
    assert kd.max() < 0.1 * np.abs(kk).max() and kd.mean() < 0.02 * np.abs(kk).mean()
    # decode after the GEMM prefill
    fast.prefill(_t(ids, dev).view(1, 40, 33))
    fast.capture()
    rng = np.random.default_rng(6)
    cover = []
    for t in range(3):
        row = np.concatenate([[ost.AUDIO_GEN_SLOT_TOKEN_ID], rng.integers(0, 1024, 32)]).astype(np.int64)
        lt, la, hh, two = fast.step(_t(row, dev).view(1, 33), 40 + t, audio2=True)
        hs = om.step(row)
        lo = bf16_to_f32(om.audio_logits(hs))
        am = np.argmax(bf16_to_f32(_bits(la)), -1)
        cover.append((lo[np.arange(32), am] >= lo.max(-1) - 0.05).mean())
    assert np.mean(cover) > 0.95, cover
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def test_w4_format_matches_reference_codes():
    """G1-style: the W4 codes this package packs are the reference's RTN codes."""
    dev = require_cuda()
    ref = pytest.importorskip("moss_tts_lite.gptq")
    fast, m, om = _w4_setup(dev)
    w = _weights(seed=13)
    wq = torch.from_numpy(w["language_model.layers.1.self_attn.o_proj.weight"].view(np.int16)).view(torch.bfloat16).to(dev)
    q_ref, _, _ = ref.rtn_quantize(wq, 128)
    codes = fast._lins[1]["o"].w.unpack_codes()
    assert torch.equal(codes, q_ref)


def test_generate_fast_greedy_matches_reference_loop():
    """Trajectory identity of the generation loop: the reference's own
    generate_fast (its host FSM and torch argmax) driving this package's
    FastMossTTS must produce exactly the tokens of this package's
    generate_fast (device argmax) for 48 greedy steps."""
    dev = require_cuda()
    ref_fast = pytest.importorskip("moss_tts_lite.fast")
    from moss_tts_lite_b200.fast import generate_fast
    fast, m, om = _w4_setup(dev, seed=17, max_seq=128)
    ids = _t(_prompt(16, seed=5), dev).view(1, 16, 33)
    mine = generate_fast(fast, {"input_ids": ids}, max_new_tokens=48, greedy=True, watchdog=False)
    theirs = ref_fast.generate_fast(fast, {"input_ids": ids}, max_new_tokens=48, greedy=True, watchdog=False)
    assert mine.n_steps == theirs.n_steps
    assert torch.equal(mine.text_ids, theirs.text_ids.cpu())
    assert torch.equal(mine.audio_frames, theirs.audio_frames.cpu())
