"""Standalone quantized exports on the B200 kernels (moss_tts_lite/export.py:639-770).

A standalone export is a directory holding ``meta.json`` (format tag
"moss_tts_lite.standalone-gptq", the model config, the quantization method
and the preset: per-linear group sizes, projections kept in bf16) and one
safetensors file with the GPTQ payload - ``layers.<i>.<proj>.q`` (the codes
in torch's tinygemm packed layout) and ``layers.<i>.<proj>.qsz`` (bf16
scale, zero) - next to every weight that stays bf16 under its checkpoint key.
``load_standalone_model`` reads it (the safetensors reader is this module's
own) and assembles this package's ``MossTTSModel`` + ``GptqMossTTS``: the
packed codes are read back by ``gptq.int4pack_to_codes`` and re-packed into
the tile layout of the W4 kernels.
"""
from __future__ import annotations

import json
import os
import re
import struct

import numpy as np
import torch

from .gptq import GptqMossTTS
from .model import LIN_NAMES, MossTTSModel

FORMAT_TAG = "moss_tts_lite.standalone-gptq"
META_FILE = "meta.json"
Q_FILE = "quantized.safetensors"
_PROJ_KEYS = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
              "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
_PAYLOAD = re.compile(r"^layers\.(\d+)\.(" + "|".join(LIN_NAMES) + r")\.(q|qsz)$")
# safetensors dtype tag -> (numpy dtype of the raw bytes, torch dtype)
_ST_DTYPES = {"BF16": (np.int16, torch.bfloat16), "F16": (np.float16, torch.float16),
              "F32": (np.float32, torch.float32), "I32": (np.int32, torch.int32), "I64": (np.int64, torch.int64),
              "U8": (np.uint8, torch.uint8), "I8": (np.int8, torch.int8), "I16": (np.int16, torch.int16)}


def checkpoint_key(li: int, proj: str) -> str:
    """The base checkpoint key of projection ``proj`` of layer ``li``."""
    return f"language_model.layers.{int(li)}.{_PROJ_KEYS[proj]}.weight"


def read_safetensors_file(path: str) -> dict:
    """All tensors of one safetensors file (8-byte little-endian header
    length, JSON header of dtype / shape / byte range, raw little-endian
    data) as CPU torch tensors."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        base = 8 + hlen
        out = {}
        for name, rec in header.items():
            if name == "__metadata__":
                continue
            if rec["dtype"] not in _ST_DTYPES:
                raise ValueError(f"{path}: tensor {name} has unsupported dtype {rec['dtype']}")
            npd, td = _ST_DTYPES[rec["dtype"]]
            a, b = rec["data_offsets"]
            f.seek(base + a)
            arr = np.frombuffer(f.read(b - a), dtype=npd).copy()
            t = torch.from_numpy(arr)
            if td == torch.bfloat16:
                t = t.view(torch.bfloat16)
            out[name] = t.reshape(rec["shape"])
    return out


def is_standalone_dir(path: str) -> bool:
    """Whether ``path`` holds a standalone export (its meta.json has the format tag)."""
    p = os.path.join(path, META_FILE)
    try:
        with open(p, encoding="utf-8") as f:
            return json.load(f).get("format") == FORMAT_TAG
    except (OSError, ValueError):
        return False


def read_standalone(model_dir: str, expected_preset: str | None = None):
    """(meta, bf16 weights {key: tensor}, GPTQ state {layer: {proj:
    {"packed", "qsz"}}}, group sizes {(layer, proj): g}, bf16 keeps) of a
    standalone export directory."""
    with open(os.path.join(model_dir, META_FILE), encoding="utf-8") as f:
        meta = json.load(f)
    if meta.get("format") != FORMAT_TAG:
        raise ValueError(f"{model_dir}/{META_FILE} is not a {FORMAT_TAG} directory")
    preset = meta.get("preset_name")
    if expected_preset and expected_preset != preset:
        raise ValueError(f"{model_dir} holds preset {preset!r}, not {expected_preset!r}")
    wf = meta.get("weight_file")
    qfile = os.path.join(model_dir, wf["name"] if isinstance(wf, dict) else Q_FILE)
    if not os.path.isfile(qfile):
        raise FileNotFoundError(f"{qfile} is missing")
    weights, state = {}, {}
    for key, t in read_safetensors_file(qfile).items():
        m = _PAYLOAD.match(key)
        if m is None:
            weights[key] = t
            continue
        li, proj, kind = int(m.group(1)), m.group(2), m.group(3)
        state.setdefault(li, {}).setdefault(proj, {})["packed" if kind == "q" else "qsz"] = t
    for li, projs in state.items():
        for proj, rec in projs.items():
            if set(rec) != {"packed", "qsz"}:
                raise ValueError(f"layer {li} {proj}: payload has {sorted(rec)}, needs packed codes and qsz")
    pm = (meta.get("presets") or {}).get(preset, {})
    gmap = {(int(k.split(":")[0]), k.split(":")[1]): int(v) for k, v in (pm.get("group_size_map") or {}).items()}
    keep = [(int(k.split(":")[0]), k.split(":")[1]) for k in (pm.get("bf16_linears") or [])]
    keep += [int(x) for x in (pm.get("bf16_layers") or [])]
    return meta, weights, state, gmap, keep


def load_standalone_model(model_dir: str, device="cuda", dtype=torch.bfloat16, max_seq_len: int = 8192,
                          expected_preset: str | None = None):
    """(MossTTSModel, GptqMossTTS) of a standalone export, on this package's kernels."""
    meta, weights, state, gmap, keep = read_standalone(model_dir, expected_preset)
    q = meta.get("quantization", {})
    if q.get("method") != "gptq":
        raise ValueError(f"{model_dir}: quantization {q.get('method')!r} is not served (only 'gptq')")
    cfg = meta["model_config"]
    dev = torch.device(device)
    # projections carried only as W4 payload get stand-ins; the model reads
    # the architecture from layer 0's q / k shapes, so those two are sized
    for li, projs in state.items():
        for proj in projs:
            key = checkpoint_key(li, proj)
            if key in weights:
                continue
            if li == 0 and proj in ("q", "k"):
                weights[key] = torch.zeros(tuple(cfg[f"layer0_{proj}_proj_shape"]), dtype=dtype)
            else:
                weights[key] = torch.zeros(0, dtype=dtype)
    model = MossTTSModel(weights, device=dev, dtype=dtype, max_seq_len=max_seq_len)
    preset = (meta.get("presets") or {}).get(meta.get("preset_name"), {})
    fast = GptqMossTTS(model, state, bf16_keep=keep, group_size_map=gmap,
                       inner_k_tiles=int(q.get("inner_k_tiles", 8)),
                       w4_group_size=int(preset.get("group_size_default", 128)))
    del weights, state
    return model, fast
