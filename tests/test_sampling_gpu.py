"""Fused sampling kernel (mtl_sample_rows) on the B200.

* Every draw equals the oracle's restatement (oracle/sampling.py:sample_row:
  the same bf16 arithmetic and the same Philox4x32-10 stream).
* The candidate set (top-k then top-p) equals the reference's own torch ops
  run on CUDA (moss_tts_lite/sampling.py apply_top_k / apply_top_p_optimized
  after the temperature division), tie-robustly - the check of the reference
  tests/test_core.py:185-246, where the exact RNG stream cannot match.
* Draw frequencies follow the probabilities (distributional parity).
* generate_fast with sampling runs through the public API and is
  reproducible for a seed."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from oracle import sampling as osmp
from oracle.bf16 import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu

CASES = [
    dict(temperature=1.7, top_k=25, top_p=0.8),          # reference audio defaults
    dict(temperature=1.5, top_k=50, top_p=1.0),          # reference text defaults
    dict(temperature=0.8, top_k=50, top_p=0.95),         # benchmark config 3
    dict(temperature=1.0, top_k=0, top_p=0.9),
    dict(temperature=1.0, top_k=5, top_p=1.0, penalty=1.2),
    dict(temperature=1.3, top_k=0, top_p=1.0, excluded=(3, 1024)),
]


def _rows(n, cols, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, cols)).astype(np.float32) * 3
    x[:, 1024 % cols] = -np.inf
    if n > 1:
        x[1, 100:110] = x[1].max() + 0.5       # ties at the top
    return f32_to_bf16(x)


@pytest.mark.parametrize("ci", range(len(CASES)))
def test_sample_rows_equals_oracle(ci):
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    c = CASES[ci]
    x = _rows(8, 1025, 100 + ci)
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
    seen = {7, 100, 101, 500}
    bits = torch.zeros(1, 33, dtype=torch.int64)
    for t in seen:
        bits[0, t >> 5] |= 1 << (t & 31)
    seen_dev = bits.to(torch.int32).to(dev)
    out = torch.empty(8, dtype=torch.long, device=dev)
    mism = 0
    total = 0
    # one-row scans (device-wide cumsum) for even cases, a [8, V] scan for odd
    scan = [1 if ci % 2 == 0 else 8] * 8
    for off in range(1, 26):
        kernels.sample_rows(xt, list(range(8)), temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"],
                            penalty=c.get("penalty", 1.0), seen_bits=seen_dev, seen_set=[0] * 8,
                            excluded=c.get("excluded", ()), seed=1234, offset=off, out=out, scan_rows=scan)
        got = out.cpu().tolist()
        for r in range(8):
            want = osmp.sample_row(x[r], temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"],
                                   penalty=c.get("penalty", 1.0), seen=seen, excluded=c.get("excluded", ()),
                                   seed=1234, offset=off, row=r, scan_rows=scan[r])
            total += 1
            mism += int(got[r] != want)
    # identical arithmetic except the fp32 order of the softmax sums
    assert mism <= total // 100, (mism, total)


@pytest.mark.parametrize("n_rows", [1, 4, 31])
def test_candidates_match_reference_torch_ops_on_cuda(n_rows):
    """The reference's apply_top_k / apply_top_p_optimized on a CUDA tensor of
    n_rows rows (one row: channel 0 and text; several: the other audio
    channels) keep the same values as the oracle restatement for that shape."""
    dev = require_cuda()
    ref = pytest.importorskip("moss_tts_lite.sampling")
    for trial in range(9):
        x = _rows(n_rows, 1025, 7 + trial + 100 * n_rows)
        t, k, p = [(1.7, 25, 0.8), (0.8, 50, 0.95), (1.0, 0, 0.8)][trial % 3]
        lg = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev).view(n_rows, -1) / t
        if k:
            lg = ref.apply_top_k(lg, k)
        if p < 1:
            lg = ref.apply_top_p_optimized(lg, p)
        fin = torch.isfinite(lg).cpu().numpy()
        for r in range(n_rows):
            cand, probs = osmp.sample_row(x[r], temperature=t, top_k=k, top_p=p, return_probs=True,
                                          scan_rows=n_rows)
            mine = set(int(c_) for c_, pr in zip(cand, probs) if pr > 0)
            theirs = set(np.nonzero(fin[r])[0].tolist())
            vals = bf16_to_f32(x[r])
            assert sorted(vals[list(mine)]) == sorted(vals[list(theirs)]), (trial, r, sorted(mine ^ theirs))


LONG_CASES = [
    dict(cols=151936, n=1, top_k=50, top_p=1.0, temperature=1.5),               # text head, reference text defaults
    dict(cols=151936, n=1, top_k=1, top_p=1.0, temperature=1.0),
    dict(cols=151936, n=1, top_k=2048, top_p=0.9, temperature=0.8),             # the largest candidate set
    dict(cols=151936, n=3, top_k=50, top_p=0.95, temperature=1.0, penalty=1.3, excluded=(151643, 151652, 7)),
    dict(cols=20000, n=2, top_k=1000, top_p=1.0, temperature=1.0),              # few slices, long ones
    dict(cols=65537, n=1, top_k=25, top_p=0.8, temperature=1.7, ties=True),     # ties across slice boundaries
]


@pytest.mark.parametrize("ci", range(len(LONG_CASES)))
def test_sliced_long_rows(ci):
    """Rows of >= 16384 columns with a top-k (the text head): one CTA per
    slice selects the slice's top-k, then the candidates are sampled.  The
    draw equals the one-CTA-per-row path bit for bit, and the oracle's."""
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib, kernels
    c = LONG_CASES[ci]
    V, n = c["cols"], c["n"]
    assert _lib.lib.mtl_sample_scratch_bytes(V, n, c["top_k"]) > 0
    rng = np.random.default_rng(500 + ci)
    x = (rng.standard_normal((n, V)) * 2).astype(np.float32)
    x[:, rng.integers(0, V, 300)] = -np.inf
    if c.get("ties"):
        # 200 copies of the row maximum spread over every slice: the top-k
        # keeps the lowest ids among them
        x[:, np.sort(rng.choice(V, 200, replace=False))] = x.max() + 1.0
    xb = f32_to_bf16(x)
    xt = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
    seen = set(rng.integers(0, V, 400).tolist()) | {7}
    words = (V + 31) // 32
    bits = np.zeros((1, words), np.int64)
    for t in seen:
        bits[0, t >> 5] |= 1 << (t & 31)
    seen_dev = torch.from_numpy(bits.astype(np.uint32).view(np.int32)).to(dev)
    pen = c.get("penalty", 1.0)
    outs = {}
    for sliced in (True, False):
        out = torch.empty(n, dtype=torch.long, device=dev)
        got = []
        for off in range(1, 9):
            kernels.sample_rows(xt, list(range(n)), temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"],
                                penalty=pen, seen_bits=seen_dev if pen != 1.0 else None, seen_set=[0] * n,
                                excluded=c.get("excluded", ()), seed=77, offset=off, out=out, sliced=sliced)
            got.append(out.cpu().tolist())
        outs[sliced] = got
    assert outs[True] == outs[False]
    mism = 0
    for oi, off in enumerate(range(1, 9)):
        for r in range(n):
            want = osmp.sample_row(xb[r], temperature=c["temperature"], top_k=c["top_k"], top_p=c["top_p"],
                                   penalty=pen, seen=seen, excluded=c.get("excluded", ()), seed=77, offset=off,
                                   row=r)
            mism += int(outs[True][oi][r] != want)
    assert mism <= 1, mism
    assert _lib.device_status() == 0


def test_sliced_scratch_too_small_is_an_error():
    dev = require_cuda()
    from moss_tts_lite_b200 import _lib
    x = torch.zeros(1, 151936, dtype=torch.bfloat16, device=dev)
    out = torch.empty(1, dtype=torch.long, device=dev)
    need = _lib.lib.mtl_sample_scratch_bytes(151936, 1, 50)
    buf = torch.empty(need, dtype=torch.uint8, device=dev)
    import ctypes
    zero, one = (ctypes.c_int32 * 1)(0), (ctypes.c_int32 * 1)(1)
    args = (x.data_ptr(), 151936, 151936, 1, zero, ctypes.c_float(1.0), 50, ctypes.c_float(1.0), ctypes.c_float(1.0),
            None, 0, zero, zero, 0, one, 1, 1, 0, out.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.mtl_sample_rows(*args, buf.data_ptr(), need - 8, stream) == _lib.MTL_E_SCRATCH
    assert _lib.lib.mtl_sample_rows(*args, buf.data_ptr(), need, stream) == _lib.MTL_OK
    assert _lib.lib.mtl_sample_rows(*args, None, 0, stream) == _lib.MTL_OK
    torch.cuda.synchronize()


def test_draw_frequencies_follow_probabilities():
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    x = _rows(1, 1025, 55)
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
    cand, probs = osmp.sample_row(x[0], temperature=1.0, top_k=25, top_p=0.9, return_probs=True)
    p = probs / probs.sum()
    n = 4000
    out = torch.empty(40, dtype=torch.long, device=dev)
    counts = {}
    for off in range(n // 40):
        kernels.sample_rows(xt, [0] * 40, temperature=1.0, top_k=25, top_p=0.9, seed=99, offset=off + 1, out=out)
        for v in out.cpu().tolist():
            counts[v] = counts.get(v, 0) + 1
    assert set(counts) <= set(int(c) for c, pr in zip(cand, p) if pr > 0)
    emp = np.array([counts.get(int(c), 0) for c in cand], np.float64) / n
    # binomial standard error on n = 4000 draws
    assert np.all(np.abs(emp - p) <= 4.5 * np.sqrt(p * (1 - p) / n) + 2e-3), (emp, p)


def test_generate_fast_sampled_reproducible():
    dev = require_cuda()
    from test_step_gpu import _prompt, _t, _w4_setup
    from moss_tts_lite_b200.fast import generate_fast
    fast, m, om = _w4_setup(dev, seed=19, max_seq=128)
    ids = _t(_prompt(12, seed=6), dev).view(1, 12, 33)
    a = generate_fast(fast, {"input_ids": ids}, max_new_tokens=40, seed=5, watchdog=False)
    b = generate_fast(fast, {"input_ids": ids}, max_new_tokens=40, seed=5, watchdog=False)
    c = generate_fast(fast, {"input_ids": ids}, max_new_tokens=40, seed=6, watchdog=False,
                      audio_repetition_penalty=1.2)
    assert torch.equal(a.text_ids, b.text_ids) and torch.equal(a.audio_frames, b.audio_frames)
    assert a.n_steps > 0 and c.n_steps > 0
    assert int(a.audio_frames.max()) <= 1024 and int(a.audio_frames.min()) >= 0
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


@pytest.mark.parametrize("mode,compact", [(0, False), (1, False), (1, True), (2, True), (2, False)])
def test_feed_row_kernel(mode, compact):
    """mtl_feed_row against its definition: text by mode, audio by mask
    (per-channel or compact decisions), pos, and the history bit sets."""
    dev = require_cuda()
    from moss_tts_lite_b200 import kernels
    rng = np.random.default_rng(mode * 2 + compact)
    for trial in range(4):
        dec = rng.integers(0, 1025, 33)
        dec[0] = trial % 2 if mode == 1 else rng.integers(0, 151000)
        mask = int(rng.integers(0, 1 << 32)) if trial else 0xFFFFFFFF
        seen0 = rng.integers(0, 1 << 31, (2, 33)).astype(np.int32)
        ids = torch.zeros(33, dtype=torch.long, device=dev)
        pos = torch.zeros(1, dtype=torch.long, device=dev)
        seen = torch.from_numpy(seen0.copy()).to(dev)
        d = torch.from_numpy(dec).to(dev)
        for _ in range(2):  # a second identical feed changes nothing
            kernels.feed_row(d, ids, pos, 77 + trial, text_mode=mode, text_const=151662, gen_slot=151656,
                             delay_slot=151662, audio_mask=mask, audio_compact=compact, pad_code=1024,
                             seen_bits=seen)
        torch.cuda.synchronize()
        want = [151662 if mode == 0 else ((151656 if dec[0] == 0 else 151662) if mode == 1 else int(dec[0]))]
        k = 0
        for j in range(32):
            if mask >> j & 1:
                want.append(int(dec[1 + (k if compact else j)]))
                k += 1
            else:
                want.append(1024)
        assert ids.cpu().tolist() == want
        assert int(pos[0]) == 77 + trial
        exp = seen0.view(np.uint32).copy()
        for j in range(32):
            t = want[1 + j]
            exp[0 if j == 0 else 1, t >> 5] |= np.uint32(1 << (t & 31))
        assert np.array_equal(seen.cpu().numpy().view(np.uint32), exp)


def test_generate_fast_pipelined_matches_serial():
    """Speculative next-step launches (the default) give exactly the tokens of
    the loop that waits for every step, greedy and sampled, with a repetition
    penalty (device history bit sets) and a watchdog that fires."""
    dev = require_cuda()
    from test_step_gpu import _prompt, _t, _w4_setup
    from moss_tts_lite_b200.fast import generate_fast
    fast, m, om = _w4_setup(dev, seed=23, max_seq=160)
    ids = _t(_prompt(12, seed=8), dev).view(1, 12, 33)
    for kw in (dict(greedy=True, watchdog=False), dict(seed=5, watchdog=False),
               dict(seed=6, audio_repetition_penalty=1.3, watchdog_silence_frames=2),
               dict(seed=7, greedy=True, watchdog_silence_frames=1)):
        st = {}
        a = generate_fast(fast, {"input_ids": ids}, max_new_tokens=60, pipelined=True, stats=st, **kw)
        b = generate_fast(fast, {"input_ids": ids}, max_new_tokens=60, pipelined=False, **kw)
        assert a.n_steps == b.n_steps, kw
        assert torch.equal(a.text_ids, b.text_ids) and torch.equal(a.audio_frames, b.audio_frames), kw
        assert a.watchdog_stats == b.watchdog_stats
        assert st["launches"] >= a.n_steps and len(st["step_ms"]) == a.n_steps - 1
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0
