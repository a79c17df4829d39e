"""Golden vectors of the reference's CUDA-only W4 path (run on a GPU box
with the reference package importable, e.g. from baseline/_ref):

    python tests/golden/make_golden_cuda.py [path-to-reference]

``FastMossTTS._quantize`` (moss_tts_lite/fast.py:85-96) only runs on CUDA
(the tinygemm packer has no CPU kernel), and PyTorch's CUDA division by a
Python scalar multiplies by the float reciprocal, so the RTN scales of the
real W4 path differ in the last bit from a CPU run of gptq.rtn_quantize.
This file records the CUDA codes and qsz for seeded bf16 weights.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str | None) -> None:
    if ref_root:
        sys.path.insert(0, ref_root)
    import torch
    from moss_tts_lite import gptq

    out = {}
    rng = np.random.default_rng(321)
    for g in (32, 64, 128, 256):
        w = (rng.standard_normal((96, 1024)) * 0.05).astype(np.float32)
        w[0, :g] = 0.0
        w[1, :g] = 0.25
        wt = torch.from_numpy(w).to(torch.bfloat16)
        q, s, mn = gptq.rtn_quantize(wt.cuda(), g)
        _, qsz = gptq.pack_fast(q, s, mn, 8)
        out[f"g{g}_w"] = wt.view(torch.int16).numpy().view(np.uint16)
        out[f"g{g}_q"] = q.cpu().numpy()
        out[f"g{g}_s"] = s.cpu().numpy()
        out[f"g{g}_qsz"] = qsz.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    dst = sys.argv[2] if len(sys.argv) > 2 else os.path.join(HERE, "w4_ref_cuda.npz")
    np.savez_compressed(dst, **out)
    print("written", dst)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
