"""Known-answer vectors of torch's tinygemm packer as the reference calls it
(torch.ops.aten._convert_weight_to_int4pack((q[:, 1::2] | q[:, 0::2] << 4),
inner_k_tiles=8), moss_tts_lite/gptq.py:75-76, fast.py:97-99): the layout of
the ``packed`` tensors a reference GPTQ state carries.  CUDA only (no CPU
kernel for this packer); run on a GPU box:

    python tests/golden/make_golden_int4pack.py [out.npz]

Records (a) three patterned 16 x 512 code matrices (codes = n % 16,
k % 16, (k // 16) % 16) whose packed words reveal, nibble by nibble, which
(n, k) each packed nibble holds, and (b) random code matrices of larger
shapes with their packed words, to check a layout restated from (a).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def pack(q):
    import torch
    q = q.to(torch.uint8).cuda()
    return torch.ops.aten._convert_weight_to_int4pack((q[:, 1::2] | (q[:, 0::2] << 4)).contiguous(), 8).cpu()


def main() -> None:
    import torch
    out = {}
    N, K = 16, 512
    n = torch.arange(N).view(N, 1).expand(N, K)
    k = torch.arange(K).view(1, K).expand(N, K)
    for name, codes in (("n", n % 16), ("k0", k % 16), ("k1", (k // 16) % 16), ("k2", (k // 256) % 16)):
        p = pack(codes)
        out[f"pat_{name}"] = p.numpy()
    g = torch.Generator().manual_seed(5)
    for (N, K) in ((64, 1024), (256, 4096), (48, 768)):
        q = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
        out[f"rand_{N}x{K}_q"] = q.numpy()
        out[f"rand_{N}x{K}_packed"] = pack(q).numpy()
    dst = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "int4pack.npz")
    np.savez_compressed(dst, **out)
    print("written", dst, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
