"""Host side of the GPTQ tier: the tinygemm packed layout read back into
codes (known-answer vectors of torch's packer, tests/golden/int4pack.npz)
and the state file with its side file (moss_tts_lite/gptq.py:610-628)."""
import json
import os

import numpy as np
import pytest
import torch

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_int4pack_to_codes_known_answers():
    from moss_tts_lite_b200.gptq import int4pack_to_codes
    z = np.load(os.path.join(GOLD, "int4pack.npz"))
    for N, K in ((64, 1024), (256, 4096), (48, 768)):
        packed = torch.from_numpy(z[f"rand_{N}x{K}_packed"])
        codes = int4pack_to_codes(packed, N, K)
        assert np.array_equal(codes.numpy(), z[f"rand_{N}x{K}_q"]), (N, K)
    # the patterned vectors: every nibble lands where the layout says
    codes = int4pack_to_codes(torch.from_numpy(z["pat_k0"]), 16, 512).numpy()
    assert np.array_equal(codes, np.tile(np.arange(512) % 16, (16, 1)))
    codes = int4pack_to_codes(torch.from_numpy(z["pat_n"]), 16, 512).numpy()
    assert np.array_equal(codes, np.tile((np.arange(16) % 16)[:, None], (1, 512)))


def test_int4pack_to_codes_rejects_other_layouts():
    from moss_tts_lite_b200.gptq import int4pack_to_codes
    with pytest.raises(ValueError):
        int4pack_to_codes(torch.zeros(8, 8, 32, 2, dtype=torch.int32), 64, 1024)   # inner_k_tiles 4


def test_load_gptq_state_and_side_file(tmp_path):
    from moss_tts_lite_b200.gptq import load_gptq_state
    state = {0: {"q": {"packed": torch.zeros(2, 2, 32, 4, dtype=torch.int32),
                       "qsz": torch.zeros(2, 16, 2, dtype=torch.bfloat16)}}}
    path = str(tmp_path / "w1p.pt")
    torch.save(state, path)
    with pytest.raises(FileNotFoundError):
        load_gptq_state(path)
    with open(path + ".meta.json", "w") as f:
        json.dump({"group_size_map": {"0:q": 64, "3:down": 256}, "bf16_linears": ["1:o"], "bf16_layers": [5]}, f)
    st, gmap, keep = load_gptq_state(path)
    assert torch.equal(st[0]["q"]["packed"], state[0]["q"]["packed"])
    assert gmap == {(0, "q"): 64, (3, "down"): 256}
    assert keep == [(1, "o"), 5]
