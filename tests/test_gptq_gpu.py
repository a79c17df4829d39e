"""GptqMossTTS (the reference's GPTQ tier, moss_tts_lite/gptq.py:637-714) on
the B200 kernels, fed states packed by the reference's own tinygemm packer
(gptq.pack_fast on CUDA):

* a uniform g128 state holding exactly the RTN codes FastMossTTS makes
  decodes bit for bit like FastMossTTS (the packed codes are read back
  exactly and land in the same tiles);
* a mixed state (a g64 projection, a gate with another group size than its
  up, a projection and a whole layer kept in bf16) against the reference's
  own GptqMossTTS on the same state: hidden states and argmaxes agree to
  within bf16 noise over teacher-forced steps;
* kernel_linear against torch._weight_int4pack_mm on the same (packed, qsz)."""
import numpy as np
import pytest
import torch

from conftest import require_cuda
from test_step_gpu import SMALL, _prompt, _t, _torch_weights, _weights

pytestmark = pytest.mark.gpu

NAMES = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
         "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}


def _state(tw, ref_gptq, gmap, skip):
    state = {}
    for li in range(SMALL["n_layers"]):
        state[li] = {}
        for n, key in NAMES.items():
            if (li, n) in skip or li in skip:
                continue
            g = gmap.get((li, n), 128)
            q, s, mn = ref_gptq.rtn_quantize(tw[f"language_model.layers.{li}.{key}.weight"], g)
            packed, qsz = ref_gptq.pack_fast(q, s, mn, 8)
            state[li][n] = {"packed": packed.cpu(), "qsz": qsz.cpu()}
    return state


def test_uniform_state_equals_fast_rtn():
    dev = require_cuda()
    ref_gptq = pytest.importorskip("moss_tts_lite.gptq")
    from moss_tts_lite_b200.fast import FastMossTTS
    from moss_tts_lite_b200.gptq import GptqMossTTS
    from moss_tts_lite_b200.model import MossTTSModel
    w = _weights(seed=51)
    tw = _torch_weights(w, dev)
    state = _state(tw, ref_gptq, {}, set())
    a = FastMossTTS(MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=64), quant="w4")
    b = GptqMossTTS(MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=64), state)
    ids = _t(_prompt(8, seed=52), dev).view(1, 8, 33)
    a.prefill(ids)
    b.prefill(ids)
    a.capture()
    b.capture()
    rng = np.random.default_rng(53)
    for t in range(3):
        row = _t(np.concatenate([[151656], rng.integers(0, 1024, 32)]).astype(np.int64), dev).view(1, 33)
        la, lb = a.step(row, 8 + t, audio2=True), b.step(row, 8 + t, audio2=True)
        torch.cuda.synchronize()
        for x, y in zip(la[1:], lb[1:]):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16)), t


def test_mixed_state_vs_reference_gptq():
    dev = require_cuda()
    ref_gptq = pytest.importorskip("moss_tts_lite.gptq")
    ref_model = pytest.importorskip("moss_tts_lite.model")
    from moss_tts_lite_b200.gptq import GptqMossTTS
    from moss_tts_lite_b200.model import MossTTSModel
    w = _weights(seed=61)
    tw = _torch_weights(w, dev)
    gmap = {(0, "o"): 64, (1, "gate"): 64, (0, "down"): 256}
    keep = [(1, "down"), 2]
    state = _state(tw, ref_gptq, gmap, {(1, "down"), 2})
    ref = ref_gptq.GptqMossTTS(ref_model.MossTTSModel(_torch_weights(w, dev), device=dev, dtype=torch.bfloat16,
                                                      max_seq_len=64), state, bf16_keep=keep, group_size_map=gmap)
    mine = GptqMossTTS(MossTTSModel(_torch_weights(w, dev), device=dev, max_seq_len=64), state, bf16_keep=keep,
                       group_size_map=gmap)
    assert mine.mixed_groups() == ref.mixed_groups()
    assert mine.bf16_keep_layers == ref.bf16_keep_layers and mine.bf16_keep_linears == ref.bf16_keep_linears
    ids = _t(_prompt(8, seed=62), dev).view(1, 8, 33)
    ref.prefill(ids)
    mine.prefill(ids)
    ref.capture()
    mine.capture()
    rng = np.random.default_rng(63)
    agree, total = 0, 0
    for t in range(6):
        row = _t(np.concatenate([[151656], rng.integers(0, 1024, 32)]).astype(np.int64), dev).view(1, 33)
        _, la_r, h_r, _ = ref.step(row, 8 + t, audio2=True)
        h_r, la_r = h_r.float().clone(), la_r.float().clone()
        _, la_m, h_m, _ = mine.step(row, 8 + t, audio2=True)
        rel = float((h_m.float() - h_r).norm() / h_r.norm())
        assert rel < 2e-2, (t, rel)
        agree += int((la_m.float().argmax(-1) == la_r.argmax(-1)).sum())
        total += 32
    assert agree >= 0.9 * total, (agree, total)


def test_kernel_linear_vs_tinygemm():
    dev = require_cuda()
    ref_gptq = pytest.importorskip("moss_tts_lite.gptq")
    from moss_tts_lite_b200.gptq import kernel_linear
    wt = (torch.randn(1024, 2048, generator=torch.Generator().manual_seed(7)) * 0.02).to(torch.bfloat16).to(dev)
    for g in (64, 128):
        q, s, mn = ref_gptq.rtn_quantize(wt, g)
        packed, qsz = ref_gptq.pack_fast(q, s, mn, 8)
        x = torch.randn(3, 5, 2048, dtype=torch.bfloat16, device=dev)
        y = kernel_linear(x, packed, g, qsz, torch.bfloat16)
        y_ref = ref_gptq.kernel_linear(x, packed, g, qsz, torch.bfloat16)
        assert y.shape == y_ref.shape
        same = (y.view(torch.int16) == y_ref.view(torch.int16)).float().mean().item()
        assert same > 0.99, (g, same)
