"""Standalone quantized exports (moss_tts_lite/export.py:639-770): this
package's reader (its own safetensors parser) against the reference's
read_standalone on the same directory, written here in the export format
(meta.json + quantized.safetensors with layers.<i>.<proj>.q / .qsz
payloads and bf16 weights under their checkpoint keys)."""
import json
import os
import struct

import numpy as np
import pytest
import torch

_TAGS = {torch.bfloat16: "BF16", torch.int32: "I32", torch.float32: "F32", torch.uint8: "U8"}


def write_safetensors(path, tensors: dict) -> None:
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.contiguous()
        raw = (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        header[name] = {"dtype": _TAGS[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def make_standalone(dirpath, weights: dict, state: dict, gmap: dict, keep: list, cfg: dict) -> None:
    tensors = dict(weights)
    for li, projs in state.items():
        for proj, rec in projs.items():
            tensors[f"layers.{li}.{proj}.q"] = rec["packed"]
            tensors[f"layers.{li}.{proj}.qsz"] = rec["qsz"]
    write_safetensors(os.path.join(dirpath, "quantized.safetensors"), tensors)
    meta = {"format": "moss_tts_lite.standalone-gptq", "preset_name": "w1",
            "quantization": {"method": "gptq", "inner_k_tiles": 8}, "model_config": cfg,
            "presets": {"w1": {"group_size_default": 128,
                               "group_size_map": {f"{a}:{b}": g for (a, b), g in gmap.items()},
                               "bf16_linears": [f"{a}:{b}" for a, b in (k for k in keep if not isinstance(k, int))],
                               "bf16_layers": [k for k in keep if isinstance(k, int)]}}}
    with open(os.path.join(dirpath, "meta.json"), "w") as f:
        json.dump(meta, f)


def test_reader_matches_reference_reader(tmp_path):
    from moss_tts_lite_b200 import export
    ref_export = pytest.importorskip("moss_tts_lite.export")
    g = torch.Generator().manual_seed(0)
    weights = {"language_model.norm.weight": torch.randn(64, generator=g).to(torch.bfloat16),
               "language_model.layers.1.self_attn.o_proj.weight": torch.randn(64, 64, generator=g).to(torch.bfloat16)}
    state = {0: {p: {"packed": torch.randint(-2 ** 31, 2 ** 31 - 1, (8, 1, 32, 4), generator=g, dtype=torch.int32),
                     "qsz": torch.randn(2, 64, 2, generator=g).to(torch.bfloat16)} for p in ("q", "k", "down")}}
    make_standalone(str(tmp_path), weights, state, {(0, "down"): 64}, [(1, "o"), 2],
                    {"layer0_q_proj_shape": [64, 128], "layer0_k_proj_shape": [16, 128]})
    assert export.is_standalone_dir(str(tmp_path)) and ref_export.is_standalone_dir(str(tmp_path))
    mine = export.read_standalone(str(tmp_path))
    ref = ref_export.read_standalone(str(tmp_path))
    assert mine[0] == ref[0]
    assert set(mine[1]) == set(ref[1])
    for k in mine[1]:
        assert torch.equal(mine[1][k].view(torch.int16), ref[1][k].view(torch.int16)), k
    for li in ref[2]:
        for p in ref[2][li]:
            assert torch.equal(mine[2][li][p]["packed"], ref[2][li][p]["packed"])
            assert torch.equal(mine[2][li][p]["qsz"].view(torch.int16), ref[2][li][p]["qsz"].view(torch.int16))
    assert mine[3] == ref[3] and sorted(map(str, mine[4])) == sorted(map(str, ref[4]))
    with pytest.raises(ValueError):
        export.read_standalone(str(tmp_path), expected_preset="w2")
