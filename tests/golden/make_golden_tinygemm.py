"""Golden vectors of the reference's W4 linear kernel itself: torch's int4
GEMM ``torch._weight_int4pack_mm`` as the reference calls it
(moss_tts_lite/fast.py:118, gptq.py:582), on RTN codes from the reference's
own ``rtn_quantize`` / ``pack_fast`` (gptq.py:54-85).  CUDA only (the
tinygemm packer has no CPU kernel); run on a GPU box with the reference
package importable:

    python tests/golden/make_golden_tinygemm.py [path-to-reference] [out.npz]

Records, per case, the bf16 weight, codes, qsz, activations x [M, K] and the
kernel's bf16 output y [M, N], so that the numpy oracle's operand
(oracle.w4.ref_operand_weight) can be checked against the kernel on CPU.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = [(1, 1024, 256, 32), (1, 1024, 256, 64), (1, 2048, 256, 128), (4, 2048, 256, 128), (1, 2048, 256, 256)]


def main(ref_root: str | None) -> None:
    if ref_root:
        sys.path.insert(0, ref_root)
    import torch
    from moss_tts_lite import gptq

    out = {}
    g_ = torch.Generator().manual_seed(77)
    for ci, (M, K, N, g) in enumerate(CASES):
        w = (torch.randn(N, K, generator=g_) * 0.02).to(torch.bfloat16)
        x = torch.randn(M, K, generator=g_).to(torch.bfloat16)
        q, s, mn = gptq.rtn_quantize(w.cuda(), g)
        packed, qsz = gptq.pack_fast(q, s, mn, 8)
        y = torch._weight_int4pack_mm(x.cuda(), packed, g, qsz)
        out[f"c{ci}_shape"] = np.array([M, K, N, g], np.int64)
        out[f"c{ci}_q"] = q.cpu().numpy()
        out[f"c{ci}_qsz"] = qsz.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
        out[f"c{ci}_x"] = x.view(torch.int16).numpy().view(np.uint16)
        out[f"c{ci}_y"] = y.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    dst = sys.argv[2] if len(sys.argv) > 2 else os.path.join(HERE, "tinygemm.npz")
    np.savez_compressed(dst, **out)
    print("written", dst)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
