"""Golden vectors of torch.cumsum over bf16 probabilities on CUDA (the top-p
step of the reference, moss_tts_lite/sampling.py:101-113, runs it on the
decode device).  Run on a GPU box:

    python tests/golden/make_golden_cumsum_cuda.py [out.npz]

Each case is a [rows, n] block of bf16 softmax probabilities sorted
descending per row (the exact inputs the reference scans) and torch's
output.  One-row blocks go through PyTorch's device-wide scan, blocks of
several rows through its per-row shared-memory scan (the two structures
round bf16 partial sums at different points), so both shapes are recorded:
the reference scans channel 0 and the text row as [1, V] and the other
sampled audio channels as [R, 1025].
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

SHAPES = [(1, 50), (1, 50), (1, 1025), (1, 1025), (1, 2048), (1, 300), (1, 8000),
          (2, 1025), (3, 1025), (4, 1025), (7, 1025), (16, 1025), (31, 1025), (3, 300), (5, 50), (2, 2048)]


def main(dst):
    rng = np.random.default_rng(2024)
    out = {}
    for i, (r, n) in enumerate(SHAPES):
        x = torch.from_numpy((rng.standard_normal((r, n)) * (1 + i % 6)).astype(np.float32)).to(torch.bfloat16).cuda()
        p = torch.softmax(x, -1)
        sp, _ = torch.sort(p, descending=True, dim=-1)
        c = torch.cumsum(sp, -1)
        out[f"in{i}"] = sp.cpu().view(torch.int16).numpy().view(np.uint16)
        out[f"out{i}"] = c.cpu().view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(dst, **out)
    print("written", dst, torch.__version__)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "cumsum_bf16_cuda.npz"))
