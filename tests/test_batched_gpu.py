"""Batched multi-stream decode (moss_tts_lite_b200.batched) on the B200.

With the register-MMA tiles every stream of a batched step must give exactly
what a batch-1 decode of that stream gives with the same kernels (one launch
per linear): the W4 rows, attention streams and head rows are computed
independently, so logits, final hidden states and the greedily fed next rows
are compared bit for bit, over several steps, eager and as a replayed CUDA
graph.  The tensor-core tiles and the batched persistent chain (the default)
sum in other fp32 orders and are compared within bf16 noise."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from test_step_gpu import _prompt, _t, _w4_setup

pytestmark = pytest.mark.gpu

GEN, DELAY = 151656, 151662


def _batch1_trajectory(fast, prompt, first_row, steps):
    """Greedy audio-phase steps of one stream through the batch-1 engine."""
    from moss_tts_lite_b200.model import AUDIO_PAD_CODE
    L = prompt.shape[0]
    fast.prefill(prompt.view(1, L, 33))
    row = first_row.clone()
    out = []
    for t in range(steps):
        fast.ids_row.view(-1).copy_(row)
        fast.pos_dev.fill_(L + t)
        fast._run_eager(True)
        la, two = fast.la_static.clone(), fast.two_static.clone()
        h = fast.h_final.clone()
        lf = la.float()
        assert torch.isinf(lf[:, AUDIO_PAD_CODE]).all()
        nxt = torch.empty(33, dtype=torch.long, device=la.device)
        nxt[1:] = torch.argmax(lf, -1)                 # first index on ties, as the kernel
        nxt[0] = DELAY if float(two[1]) > float(two[0]) else GEN
        out.append((la, two, h, nxt.clone()))
        row = nxt
    return out


@pytest.mark.parametrize("graph", [False, True])
def test_batched_streams_equal_batch1(graph):
    dev = require_cuda()
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    fast, m, om = _w4_setup(dev, seed=31, max_seq=128, chain=False)
    B, steps = 5, 4
    prompts = [_t(_prompt(6 + 3 * s, seed=40 + s), dev) for s in range(B)]
    rng = np.random.default_rng(9)
    firsts = [_t(np.concatenate([[GEN], rng.integers(0, 1024, 32)]).astype(np.int64), dev) for _ in range(B)]
    ref = [_batch1_trajectory(fast, prompts[s], firsts[s], steps) for s in range(B)]
    bt = BatchedFastMossTTS(fast, B, max_seq=128, tc=False, chain=False)
    for s in range(B):
        bt.prefill(s, prompts[s])
        bt.start(s, firsts[s], prompts[s].shape[0])
    if graph:
        bt.capture()
    for t in range(steps):
        bt.step()
        torch.cuda.synchronize()
        for s in range(B):
            la, two, h, nxt = ref[s][t]
            assert torch.equal(bt.la[s].view(torch.int16), la.view(torch.int16)), (s, t)
            assert torch.equal(bt.two[s].view(torch.int16), two.view(torch.int16)), (s, t)
            assert torch.equal(bt.h_final[s].view(torch.int16), h.view(-1).view(torch.int16)), (s, t)
            assert torch.equal(bt.ids[s], nxt), (s, t)
            assert int(bt.pos[s]) == prompts[s].shape[0] + t + 1
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def test_batched_tensor_core_tiles_agree():
    """The tensor-core tiles (tcgen05, the batch as the MMA N dimension)
    against the register-MMA batched step: every stream's logits agree to
    within bf16 noise and >= 95% of the greedy audio codes coincide."""
    dev = require_cuda()
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    fast, m, om = _w4_setup(dev, seed=33, max_seq=128, chain=False)
    B = 6
    prompts = [_t(_prompt(5 + 2 * s, seed=60 + s), dev) for s in range(B)]
    rng = np.random.default_rng(19)
    firsts = [_t(np.concatenate([[GEN], rng.integers(0, 1024, 32)]).astype(np.int64), dev) for _ in range(B)]
    outs = {}
    for tc in (False, True):
        bt = BatchedFastMossTTS(fast, B, max_seq=128, tc=tc, chain=False)
        assert bt.tc == tc
        for s in range(B):
            bt.prefill(s, prompts[s])
            bt.start(s, firsts[s], prompts[s].shape[0])
        bt.step()
        torch.cuda.synchronize()
        outs[tc] = (bt.la.float().cpu().numpy(), bt.h_final.float().cpu().numpy())
    la0, h0 = outs[False]
    la1, h1 = outs[True]
    assert np.abs(h0 - h1).max() < 0.05 * np.abs(h0).max()
    fin = np.isfinite(la0)
    assert np.array_equal(fin, np.isfinite(la1))
    assert np.abs(la0[fin] - la1[fin]).max() < 0.05 * np.abs(la0[fin]).max()
    agree = (np.argmax(la0, -1) == np.argmax(la1, -1)).mean()
    assert agree >= 0.95, agree
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


def test_prefill_all_equals_per_stream_prefill():
    """All streams' prompts prefilled together (tcgen05 GEMMs over M = streams
    x L rows, one attention launch over every stream's cache) equal the
    streams prefilled one at a time, bit for bit: hidden states and caches."""
    dev = require_cuda()
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    fast, m, om = _w4_setup(dev, seed=35, max_seq=160)
    B, L = 3, 40
    prompts = [_t(_prompt(L, seed=80 + s), dev) for s in range(B)]
    together = BatchedFastMossTTS(fast, B, max_seq=128)
    h_all = together.prefill_all(prompts)
    apart = BatchedFastMossTTS(fast, B, max_seq=128)
    h_each = torch.cat([apart.prefill(s, prompts[s]) for s in range(B)], 0)
    torch.cuda.synchronize()
    assert torch.equal(h_all.view(torch.int16), h_each.view(torch.int16))
    assert torch.equal(together.k_cache[:, :, :, :L].view(torch.int16), apart.k_cache[:, :, :, :L].view(torch.int16))
    assert torch.equal(together.v_cache[:, :, :, :L].view(torch.int16), apart.v_cache[:, :, :, :L].view(torch.int16))
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0


@pytest.mark.parametrize("B", [3, 12])
def test_batched_chain_agrees_with_batch1_chain(B):
    """The batched persistent chain (mtl_w4_chain_rows, the default) against
    batch-1 decodes of each stream with the batch-1 chain: per stream and
    step the logits and hidden states agree within bf16 noise and >= 95% of
    the greedy audio codes coincide; the batched step's graph replay equals
    its eager pass bit for bit (warp partials summed in fixed order)."""
    dev = require_cuda()
    from moss_tts_lite_b200.batched import BatchedFastMossTTS
    fast, m, om = _w4_setup(dev, seed=37, max_seq=128)
    assert fast.chain
    steps = 3
    prompts = [_t(_prompt(6 + s, seed=90 + s), dev) for s in range(B)]
    rng = np.random.default_rng(29)
    firsts = [_t(np.concatenate([[GEN], rng.integers(0, 1024, 32)]).astype(np.int64), dev) for _ in range(B)]
    ref = [_batch1_trajectory(fast, prompts[s], firsts[s], steps) for s in range(B)]
    runs = []
    for graph in (False, True):
        bt = BatchedFastMossTTS(fast, B, max_seq=128, chain=True)
        assert bt.chain and not bt.tc
        for s in range(B):
            bt.prefill(s, prompts[s])
            bt.start(s, firsts[s], prompts[s].shape[0])
        if graph:
            bt.capture()
        out = []
        for t in range(steps):
            bt.step()
            torch.cuda.synchronize()
            out.append((bt.la.clone(), bt.h_final.clone(), bt.ids.clone()))
        runs.append(out)
    agree = []
    for t in range(steps):
        la_e, h_e, ids_e = runs[0][t]
        la_g, h_g, ids_g = runs[1][t]
        assert torch.equal(la_e.view(torch.int16), la_g.view(torch.int16)), t
        assert torch.equal(h_e.view(torch.int16), h_g.view(torch.int16)), t
        assert torch.equal(ids_e, ids_g), t
        for s in range(B):
            la_r, two_r, h_r, nxt_r = ref[s][t]
            if t > 0 and not torch.equal(runs[0][t - 1][2][s], ref[s][t - 1][3]):
                break   # the streams fed different rows: no longer comparable
            h0, h1 = h_r.float().view(-1).cpu().numpy(), h_e[s].float().cpu().numpy()
            assert np.abs(h0 - h1).max() < 0.05 * np.abs(h0).max(), (s, t)
            l0, l1 = la_r.float().cpu().numpy(), la_e[s].float().cpu().numpy()
            fin = np.isfinite(l0)
            assert np.array_equal(fin, np.isfinite(l1))
            assert np.abs(l0[fin] - l1[fin]).max() < 0.05 * np.abs(l0[fin]).max(), (s, t)
            agree.append((np.argmax(l0, -1) == np.argmax(l1, -1)).mean())
    assert np.mean(agree) >= 0.95, agree
    from moss_tts_lite_b200 import _lib
    assert _lib.device_status() == 0
