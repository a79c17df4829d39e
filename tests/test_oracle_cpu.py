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


def test_philox4x32_10_known_answers():
    """Published known-answer vectors of Philox4x32-10 (Salmon et al. 2011,
    Random123 kat_vectors): the generator behind the sampling draws."""
    assert osmp.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert osmp.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6,
                                                                        0x6D5451FD]
    assert osmp.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_oracle_sample_row_candidates_follow_reference_ops():
    """The oracle's candidate set (top-k then top-p) equals the reference's
    apply_top_k / apply_top_p_optimized on the same bf16 logits (CPU torch,
    so with the CPU cumsum; tests/test_sampling_gpu.py checks CUDA)."""
    import torch
    import sys
    sys.path.insert(0, "/nonexistent")
    from oracle.bf16 import f32_to_bf16
    rng = np.random.default_rng(3)
    for trial in range(20):
        x = f32_to_bf16(rng.standard_normal(1025).astype(np.float32) * 2)
        k, p = [(25, 0.8), (50, 0.95), (0, 0.8), (25, 1.0)][trial % 4]
        cand, probs = osmp.sample_row(x, top_k=k, top_p=p, return_probs=True, device="cpu")
        mine = set(int(c) for c, pr in zip(cand, probs) if pr > 0)
        t = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).view(1, -1)
        ref = t.clone()
        if k:
            ref = torch.full_like(t, float("-inf")).scatter(1, torch.topk(t, k).indices, torch.topk(t, k).values)
        if p < 1:
            probs_t = torch.softmax(ref, -1)
            sp, si = torch.sort(probs_t, descending=True)
            cum = torch.cumsum(sp, -1)
            rem = cum > p
            rem[..., 1:] = rem[..., :-1].clone()
            rem[..., 0] = False
            mask = torch.zeros_like(ref, dtype=torch.bool).scatter(1, si, rem)
            ref = ref.masked_fill(mask, float("-inf"))
        theirs = set(torch.nonzero(torch.isfinite(ref[0])).view(-1).tolist())
        # tie-robust: torch.topk breaks ties at the cut-off in an unspecified
        # order, the oracle keeps the lowest ids; the kept values must agree
        vals = bf16_to_f32(x)
        assert sorted(vals[list(mine)]) == sorted(vals[list(theirs)]), (trial, sorted(mine ^ theirs))


def test_cuda_cumsum_grouping_vs_golden():
    """oracle.sampling.cumsum_bf16_cuda reproduces torch.cumsum of bf16 on a
    B200 bit for bit, for one-row tensors (device-wide scan, up to 8000
    items: several scan tiles) and multi-row tensors (per-row shared-memory
    scan with 2..31 rows); fixtures from tests/golden/make_golden_cumsum_cuda.py."""
    import sys
    sys.path.insert(0, GOLD)
    from make_golden_cumsum_cuda import SHAPES
    z = _load("cumsum_bf16_cuda.npz")
    for i, (r, n) in enumerate(SHAPES):
        p = bf16_to_f32(z[f"in{i}"]).reshape(r, n)
        want = bf16_to_f32(z[f"out{i}"]).reshape(r, n)
        got = np.stack([osmp.cumsum_bf16_cuda(p[j], r, n) for j in range(r)])
        assert np.array_equal(got, want), (i, r, n, int((got != want).sum()))
    # the plain bf16 running sum is not what the device computes past 30 items
    p = bf16_to_f32(z["in2"]).reshape(-1)
    run, seq = np.float32(0), []
    for v in p:
        run = np.float32(osmp._bf(np.float32(run + v)).item())
        seq.append(run)
    assert not np.array_equal(np.asarray(seq, np.float32), bf16_to_f32(z["out2"]).reshape(-1))


def test_inner_scan_thread_split():
    """get_log_num_threads_x_inner_scan for the audio row shapes the
    reference scans: [R, 1025] for R = 2..31 sampled channels."""
    assert [osmp.inner_scan_log_threads_x(r, 1025) for r in (2, 4, 5, 8, 9, 16, 17, 31)] == [9, 9, 8, 8, 8, 8, 7, 7]
    assert osmp.inner_scan_log_threads_x(1024, 16) == 4


def test_operand_weight_pinned_to_tinygemm():
    """The reference's W4 linear (torch._weight_int4pack_mm on the reference's
    own RTN codes, run on a B200 by tests/golden/make_golden_tinygemm.py)
    multiplies with the effective weight rounded once to bf16: the oracle
    with ref_operand_weight reproduces its outputs up to the fp32 summation
    order (almost all bitwise, the rest within one bf16 ulp), while the
    unrounded fp32 effective weight does not."""
    path = os.path.join(GOLD, "tinygemm.npz")
    if not os.path.exists(path):
        pytest.skip("tinygemm fixture not generated yet")
    z = np.load(path)
    n_cases = len([k for k in z.files if k.endswith("_shape")])
    for ci in range(n_cases):
        M, K, N, g = (int(v) for v in z[f"c{ci}_shape"])
        q, qsz, x, y = z[f"c{ci}_q"], z[f"c{ci}_qsz"], z[f"c{ci}_x"], z[f"c{ci}_y"]
        yo = ow.linear_bf16(x, ow.ref_operand_weight(q, qsz, g).T)
        ye = ow.linear_bf16(x, ow.ref_effective_weight(q, qsz, g).T)
        same = (yo == y).mean()
        ulp = np.abs(bf16_to_f32(y)) * 2.0 ** -7 + 1e-30
        assert same > 0.98, (ci, same)
        assert (np.abs(bf16_to_f32(yo) - bf16_to_f32(y)) <= ulp * 1.001).all(), ci
        assert (ye == y).mean() < same, ci
