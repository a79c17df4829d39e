"""The numpy oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  Integer outputs are bit-exact; float
outputs are compared exactly where the reference's arithmetic is
order-independent and within tolerance where it is a reduction."""
import os

import numpy as np
import pytest

from oracle import sampling as osmp
from oracle import step as ost
from oracle import w4 as ow
from oracle.bf16 import bf16_to_f32, f32_to_bf16

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("g", [32, 64, 128, 256])
def test_rtn_quantize_pack_and_dequant_bit_exact(g):
    z = _load("w4_ref.npz")          # reference run on CPU
    q, s, mn = ow.rtn_quantize(z[f"g{g}_w"], g, device="cpu")
    assert np.array_equal(q, z[f"g{g}_q"])
    assert np.array_equal(s.view(np.uint32), z[f"g{g}_s"].view(np.uint32))
    assert np.array_equal(mn.view(np.uint32), z[f"g{g}_mn"].view(np.uint32))
    qsz = ow.pack_qsz(s, mn)
    assert np.array_equal(qsz, z[f"g{g}_qsz"])
    weff = ow.ref_effective_weight(q, qsz, g)
    assert np.array_equal(weff.view(np.uint32), z[f"g{g}_weff"].view(np.uint32))


@pytest.mark.parametrize("g", [32, 64, 128, 256])
def test_rtn_quantize_cuda_semantics_bit_exact(g):
    """The reference's real W4 path runs on CUDA (tests/golden/make_golden_cuda.py)."""
    z = _load("w4_ref_cuda.npz")
    q, s, mn = ow.rtn_quantize(z[f"g{g}_w"], g, device="cuda")
    assert np.array_equal(q, z[f"g{g}_q"])
    assert np.array_equal(s.view(np.uint32), z[f"g{g}_s"].view(np.uint32))
    assert np.array_equal(ow.pack_qsz(s, mn), z[f"g{g}_qsz"])


def test_autogptq_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, (256, 96), dtype=np.uint8)
    assert np.array_equal(ow.unpack_qweight(ow.pack_qweight(codes)), codes)
    zeros = rng.integers(0, 16, (2, 96), dtype=np.uint8)
    assert np.array_equal(ow.unpack_qzeros(ow.pack_qzeros(zeros)), zeros)
    # LSB-first: code k=1 of column 0 sits in bits 4..7 of qweight[0, 0]
    c = np.zeros((8, 8), np.uint8)
    c[1, 0] = 0xA
    assert int(ow.pack_qweight(c)[0, 0]) == 0xA0


def test_autogptq_semantics_equal_reference_dequant():
    """(q - z) * s equals the reference (q - 8) * scale + zero with
    scale = s and zero = (8 - z) * s whenever both are bf16-exact."""
    rng = np.random.default_rng(1)
    K, N, g = 256, 64, 128
    codes = rng.integers(0, 16, (K, N), dtype=np.uint8)
    zeros = rng.integers(0, 16, (K // g, N), dtype=np.uint8)
    s = (2.0 ** rng.integers(-8, -4, (K // g, N))).astype(np.float16)   # exact in bf16
    W = ow.gptq_dequant(ow.pack_qweight(codes), ow.pack_qzeros(zeros), s.view(np.uint16),
                        np.arange(K) // g)
    sf = s.astype(np.float32)
    qsz = np.stack([f32_to_bf16(sf), f32_to_bf16((8.0 - zeros) * sf)], -1)
    Wref = ow.ref_effective_weight(codes.T.copy(), qsz, g)
    assert np.array_equal(W.T, Wref)


def test_close_enough_tolerance():
    ref = np.array([[1.0, 100.0, -3.0]])
    y = f32_to_bf16(np.array([[1.019, 100.9, -3.0]], np.float32))
    assert ow.close_enough(y, ref)[0]
    y = f32_to_bf16(np.array([[1.05, 100.0, -3.0]], np.float32))
    assert not ow.close_enough(y, ref)[0]


def test_sampling_ops_vs_golden():
    z = _load("sampling.npz")
    x = z["x"]
    for k in (1, 7, 25, 50):
        mine, gold = osmp.apply_top_k(x, k), z[f"topk{k}"]
        for r in range(x.shape[0]):      # tie-robust: the kept values agree
            assert np.array_equal(np.sort(mine[r][np.isfinite(mine[r])]), np.sort(gold[r][np.isfinite(gold[r])]))
        assert np.array_equal(mine[1:], gold[1:])      # rows 1.. have no ties
    for p in (0.5, 0.8, 0.95):
        mine, gold = osmp.apply_top_p(x, p), z[f"topp{p}"]
        assert np.array_equal(np.isfinite(mine), np.isfinite(gold))
    assert np.array_equal(osmp.argmax_first(x), z["argmax"])
    out = osmp.apply_repetition_penalty(z["rep_lg"], z["rep_pv"], 1.2)
    assert np.array_equal(out.view(np.uint32), z["rep_out"].view(np.uint32))
    out = osmp.apply_repetition_penalty(z["rep2_lg"], z["rep2_pv"], 1.3)
    assert np.array_equal(out.view(np.uint32), z["rep2_out"].view(np.uint32))
    t = np.array([5, 3, 7, 3, 9])
    assert [osmp.find_last_equal(t, c) for c in (3, 9, 42)] == list(z["flc"])


def test_fsm_tables_vs_golden():
    z = _load("fsm.npz")
    for dl, wd, stop, aud, nt, ia, st, forced in z["text"]:
        dl = osmp.INT64_MAX if dl == 2**31 - 1 else int(dl)
        got = osmp.text_decision(dl, 32, bool(wd), bool(stop), bool(aud))
        assert (got[0], int(got[1]), int(got[2]), int(got[3])) == (nt, ia, st, forced)
    for row in z["mask"]:
        al, dl = int(row[0]), int(row[1])
        dl = osmp.INT64_MAX if dl == 2**31 - 1 else dl
        assert [int(v) for v in osmp.audio_sampling_mask(al, dl, 32)] == list(row[2:])


def test_mini_model_step_vs_reference():
    """The oracle decoder (the bf16 rounding points of model.py, flash-style
    SDPA rounding of the probabilities) against the reference MossTTSModel
    run on CPU: hidden states bit-exact for a 6-row prefill and 4 decode
    steps; logits exact up to the reference's own summation order (at most
    1 bf16 ulp on a handful of elements)."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden import MINI, MINI_STEPS, mini_prompt
    z = _load("mini_step.npz")
    w = ost.synth_weights(MINI["hidden"], MINI["n_layers"], MINI["n_heads"], MINI["n_kv"], MINI["head_dim"],
                          MINI["inter"], vocab=MINI["vocab"], seed=MINI["seed"], std=0.2, norm_ones=False)
    m = ost.OracleModel(w, max_seq_len=64)
    ids, steps = mini_prompt()
    assert np.array_equal(m.prefill(ids), z["prefill_h"])
    for t in range(MINI_STEPS):
        h = m.step(steps[t])
        assert np.array_equal(h.reshape(-1), z[f"h{t}"]), t
        la, ga = m.audio_logits(h), z[f"audio{t}"]
        assert (la == ga).mean() > 0.999
        d = np.abs(bf16_to_f32(la) - bf16_to_f32(ga))
        fin = np.isfinite(bf16_to_f32(ga))
        ulp = np.abs(bf16_to_f32(ga)) * 2.0 ** -7
        assert (d[fin] <= ulp[fin] + 1e-30).all()
        assert np.array_equal(m.text_logits_2way(h), z[f"two{t}"])
        lt = bf16_to_f32(m.text_logits(h))
        assert np.array_equal(lt[z[f"text_top_idx{t}"]], z[f"text_top_val{t}"])
        assert np.array_equal(np.sort(lt)[::-1][:16], z[f"text_top_val{t}"])
