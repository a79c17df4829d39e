"""Generate the golden vectors under tests/golden/ by running the REFERENCE
package (moss-tts-lite) on seeded synthetic inputs.

Run in a container where the reference source is available:

    python tests/golden/make_golden.py /path/to/moss-tts-lite

Every input is regenerated from numpy PCG64 seeds (stable across
platforms); the files hold the reference's outputs.  Nothing in the tests,
``smoke()`` or ``bench.py`` runs this script or needs the reference.

Files:
  w4_ref.npz        rtn_quantize / pack_qsz_only / effective_weight
                    (moss_tts_lite/gptq.py:35-97) on bf16 weights, g in
                    {32, 64, 128, 256}
  sampling.npz      apply_top_k / apply_top_p_optimized /
                    apply_repetition_penalty_delay_pattern / argmax /
                    find_last_equal_C (moss_tts_lite/sampling.py)
  fsm.npz           text_decision / audio_sampling_mask tables
                    (moss_tts_lite/fast_native.py:51-67, the isolated form of
                    fast.py:465-520)
  mini_step.npz     MossTTSModel (model.py) on CPU: a 2-layer, head_dim-128
                    synthetic checkpoint; prefill + 4 decode steps: hidden
                    states, audio logits, 2-way logits, text-logit argmax/top
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

MINI = dict(hidden=256, n_layers=2, n_heads=2, n_kv=1, head_dim=128, inter=512, vocab=151700, seed=5)
MINI_PROMPT_SEED = 9
MINI_L = 6
MINI_STEPS = 4


def _bits(t):
    import torch
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def mini_prompt():
    rng = np.random.default_rng(MINI_PROMPT_SEED)
    ids = np.zeros((MINI_L, 33), np.int64)
    ids[:, 0] = rng.integers(0, 151643, MINI_L)
    ids[:, 1:] = rng.integers(0, 1024, (MINI_L, 32))
    ids[-1, 0] = 151652
    rows = np.zeros((MINI_STEPS, 33), np.int64)
    rows[:, 0] = np.where(np.arange(MINI_STEPS) % 2 == 0, 151656, 151662)
    rows[:, 1:] = rng.integers(0, 1025, (MINI_STEPS, 32))
    return ids, rows


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    from moss_tts_lite import gptq, sampling, fast_native
    from moss_tts_lite.model import MossTTSModel
    from oracle.step import synth_weights

    torch.set_num_threads(8)
    out = {}
    # ---------------------------------------------------------------- W4
    rng = np.random.default_rng(123)
    for g in (32, 64, 128, 256):
        w = (rng.standard_normal((96, 512)) * 0.05).astype(np.float32)
        w[0, :g] = 0.0                      # degenerate group -> clamp(min=1e-6)
        w[1, :g] = 0.25                     # constant group
        wt = torch.from_numpy(w).to(torch.bfloat16)
        q, s, mn = gptq.rtn_quantize(wt, g)
        qsz = gptq.pack_qsz_only(s, mn, g)
        weff = gptq.effective_weight(q, qsz, g)
        out[f"g{g}_w"] = _bits(wt)
        out[f"g{g}_q"] = q.numpy()
        out[f"g{g}_s"] = s.numpy()
        out[f"g{g}_mn"] = mn.numpy()
        out[f"g{g}_qsz"] = _bits(qsz)
        out[f"g{g}_weff"] = weff.numpy()
    np.savez_compressed(os.path.join(HERE, "w4_ref.npz"), **out)

    # ---------------------------------------------------------- sampling
    out = {}
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, 1025)).astype(np.float32)
    x[0, 100:110] = x[0].max() + 1.0        # ties at the top
    xt = torch.from_numpy(x)
    out["x"] = x
    for k in (1, 7, 25, 50):
        out[f"topk{k}"] = sampling.apply_top_k(xt.clone(), k).numpy()
    for p in (0.5, 0.8, 0.95):
        out[f"topp{p}"] = sampling.apply_top_p_optimized(xt.clone(), p).numpy()
    out["argmax"] = torch.argmax(xt, dim=-1).numpy()
    lg = rng.standard_normal((1, 8, 50)).astype(np.float32)
    pv = rng.integers(0, 50, (1, 20, 8))
    out["rep_lg"] = lg
    out["rep_pv"] = pv
    out["rep_out"] = sampling.apply_repetition_penalty_delay_pattern(
        torch.from_numpy(lg).clone(), torch.from_numpy(pv), 1.2).numpy()
    lg2 = rng.standard_normal((1, 200)).astype(np.float32)
    pv2 = rng.integers(0, 200, (1, 30))
    out["rep2_lg"] = lg2
    out["rep2_pv"] = pv2
    out["rep2_out"] = sampling.apply_repetition_penalty_delay_pattern(
        torch.from_numpy(lg2).clone(), torch.from_numpy(pv2), 1.3).numpy()
    t = torch.tensor([[5, 3, 7, 3, 9]])
    out["flc"] = np.array([int(sampling.find_last_equal_C(t, c)) for c in (3, 9, 42)])
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), **out)

    # --------------------------------------------------------------- FSM
    INT64_MAX = 9223372036854775807
    rows = []
    for dl in (INT64_MAX, 0, 1, 5, 31, 32, 33):
        for wd in (False, True):
            for stop in (False, True):
                for aud in (False, True):
                    nt, ia, st, forced = fast_native.text_decision(dl, 32, wd, stop, aud)
                    rows.append([min(dl, 2**31 - 1), wd, stop, aud, nt, ia, st, forced])
    masks = []
    for al in (0, 1, 5, 32, 40):
        for dl in (INT64_MAX, 0, 1, 7, 31, 32):
            masks.append([al, min(dl, 2**31 - 1)] + [int(v) for v in fast_native.audio_sampling_mask(al, dl, 32)])
    np.savez_compressed(os.path.join(HERE, "fsm.npz"), text=np.array(rows, np.int64), mask=np.array(masks, np.int64))

    # ---------------------------------------------------------- mini step
    w = synth_weights(MINI["hidden"], MINI["n_layers"], MINI["n_heads"], MINI["n_kv"], MINI["head_dim"],
                      MINI["inter"], vocab=MINI["vocab"], seed=MINI["seed"], std=0.2, norm_ones=False)
    wt = {k: _bf16(v) for k, v in w.items()}
    model = MossTTSModel(wt, device="cpu", dtype=torch.bfloat16, max_seq_len=64)
    ids, steps = mini_prompt()
    out = {}
    with torch.inference_mode():
        hs = model.prefill(torch.from_numpy(ids).view(1, MINI_L, 33))
        out["prefill_h"] = _bits(hs.last_hidden[0])
        for t_ in range(MINI_STEPS):
            h = model.step(torch.from_numpy(steps[t_]).view(1, 1, 33)).last_hidden
            out[f"h{t_}"] = _bits(h.view(-1))
            out[f"audio{t_}"] = _bits(model.audio_logits(h))
            out[f"two{t_}"] = _bits(model.text_logits_2way(h))
            lt = model.text_logits(h).float()
            top = torch.topk(lt, 16)
            out[f"text_top_idx{t_}"] = top.indices.numpy()
            out[f"text_top_val{t_}"] = top.values.numpy()
    np.savez_compressed(os.path.join(HERE, "mini_step.npz"), **out)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference source tree>")
    main(sys.argv[1])
