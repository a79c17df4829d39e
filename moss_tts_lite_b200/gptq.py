"""The reference's GPTQ tier on the B200 kernels (moss_tts_lite/gptq.py:577-714).

A reference GPTQ state holds, per layer and projection, ``{"packed", "qsz"}``:
the codes in torch's tinygemm layout (``_convert_weight_to_int4pack`` with
inner_k_tiles 8, gptq.py:75-76) and bf16 (scale, zero) per group, plus a
side file naming per-linear group sizes and projections kept in bf16
(gptq.py:610-628).  Here the packed codes are unpacked once at load and
re-packed into this package's tile layout; the decode then runs on the same
sm_100a kernels as ``FastMossTTS``.

* ``int4pack_to_codes`` - the inverse of the tinygemm packer.  Its layout
  was read off known-answer vectors of the packer itself
  (tests/golden/int4pack.npz, tests/golden/make_golden_int4pack.py):
  ``packed[nt, kt, lane, w]`` (int32 [N/8, K/128, 32, 4]) holds in nibble
  i the code of row n = 8 nt + lane / 4 and column
  k = 128 kt + 32 w + 8 (i % 4) + i / 4 + 2 (lane % 4).
* ``kernel_linear`` - drop-in for gptq.py:577-585 (x through a packed W4
  weight, any group size).
* ``load_gptq_state`` / ``load_gptq_fast`` - the state file and its side
  file (``<path>.meta.json``: ``group_size_map`` {"layer:name": g},
  ``bf16_linears`` ["layer:name"], ``bf16_layers`` [layer]).
* ``GptqMossTTS`` - ``FastMossTTS`` fed a GPTQ state: per-linear group
  sizes, bf16 keeps per projection or per layer.  Projections that share a
  fused launch (q|k|v, gate|up) run as one W4 launch when all are W4 with
  one group size; otherwise that fused set runs as a bf16 GEMV whose W4
  members carry their exact operand (the effective weight rounded to bf16,
  what the W4 kernels multiply with).
"""
from __future__ import annotations

import json
import os

import torch

from .fast import FastMossTTS, _Bf16Lin, _interleave_cols, _interleave_rows, _W4Lin, _FUSE_BLOCK
from .model import LIN_NAMES
from .quant import W4Weight

INNER_K_TILES = 8
# fused launch -> the reference projections it covers
FUSED_SETS = {"qkv": ("q", "k", "v"), "o": ("o",), "gu": ("gate", "up"), "down": ("down",)}


def int4pack_to_codes(packed: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """Codes uint8 [N, K] (0..15) of a tinygemm-packed weight (int32
    [N/8, K/128, 32, 4], inner_k_tiles 8), on packed's device."""
    if packed.dtype != torch.int32 or tuple(packed.shape) != (N // 8, K // 128, 32, INNER_K_TILES // 2):
        raise ValueError(f"packed {tuple(packed.shape)} {packed.dtype} is not the inner_k_tiles=8 layout of "
                         f"a {N} x {K} weight")
    w = packed.view(N // 8, K // 128, 8, 4, 4)                 # [nt, kt, n%8, k-pair t, word w]
    shifts = torch.arange(0, 32, 4, device=packed.device, dtype=torch.int32)
    nib = (w.unsqueeze(-1) >> shifts) & 0xF                    # [..., nibble i]
    nib = nib.view(N // 8, K // 128, 8, 4, 4, 2, 4)            # i = 4 hi + lo
    # k = 128 kt + 32 w + 8 lo + 2 t + hi ; n = 8 nt + (lane / 4)
    codes = nib.permute(0, 2, 1, 4, 6, 3, 5).reshape(N, K)
    return codes.to(torch.uint8).contiguous()


_kernel_cache: dict = {}


def kernel_linear(x: torch.Tensor, packed: torch.Tensor, g: int, qsz: torch.Tensor,
                  out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """gptq.py:577-585: x [..., K] through the W4 weight (packed, g, qsz),
    output [..., N].  The tinygemm-packed codes are converted to this
    package's tiles on first use of a (packed, qsz) pair and kept."""
    key = (packed.data_ptr(), qsz.data_ptr(), int(g))
    w = _kernel_cache.get(key)
    if w is None:
        N = int(qsz.shape[1])
        K = int(packed.shape[1]) * 128
        w = W4Weight.from_ref(int4pack_to_codes(packed.to(torch.int32), N, K), qsz, int(g))
        _kernel_cache[key] = w
    y = w.linear(x.to(torch.bfloat16).reshape(-1, x.shape[-1]).contiguous())
    return y.to(out_dtype).reshape(*x.shape[:-1], y.shape[-1])


def load_gptq_state(path: str) -> tuple[dict, dict, list]:
    """(state, group_size_map {(layer, name): g}, bf16 keeps [(layer, name) or
    layer]) of an offline GPTQ state and its ``.meta.json`` side file."""
    state = torch.load(path, map_location="cpu", weights_only=False)
    meta_path = path + ".meta.json"
    if not os.path.isfile(meta_path):
        raise FileNotFoundError(f"{meta_path} is missing: it names the per-linear group sizes and the "
                                f"projections kept in bf16, which the packed weights do not record")
    with open(meta_path) as f:
        meta = json.load(f)

    def split(key: str):
        layer, name = key.split(":")
        return int(layer), name
    gmap = {split(k): int(v) for k, v in meta.get("group_size_map", {}).items()}
    keep = [split(k) for k in meta.get("bf16_linears", [])] + [int(x) for x in meta.get("bf16_layers", [])]
    return state, gmap, keep


def load_gptq_fast(model, path: str) -> "GptqMossTTS":
    """The decoder of an offline GPTQ state (gptq.py:630-635)."""
    state, gmap, keep = load_gptq_state(path)
    return GptqMossTTS(model, state, bf16_keep=keep, group_size_map=gmap)


class GptqMossTTS(FastMossTTS):
    """``FastMossTTS`` fed GPTQ-packed weights (gptq.py:637-714)."""

    def __init__(self, model, state: dict, inner_k_tiles: int = 8, w4_group_size: int = 128, bf16_keep=(),
                 group_size_map: dict | None = None):
        if inner_k_tiles != INNER_K_TILES:
            raise ValueError(f"GPTQ states are read in the inner_k_tiles={INNER_K_TILES} layout")
        self._gptq_state = state
        keep = list(bf16_keep)
        self._keep_layers = {int(x) for x in keep if isinstance(x, int)}
        self._keep_linears = {(int(x[0]), str(x[1])) for x in keep if not isinstance(x, int)}
        self._group_size_map = {(int(k[0]), str(k[1])): int(v) for k, v in (group_size_map or {}).items()}
        super().__init__(model, quant="w4", inner_k_tiles=inner_k_tiles, w4_group_size=w4_group_size)
        self.group_size_map = {li: {name: self._group_size_map.get((li, name), self.w4_group_size)
                                    for name in LIN_NAMES} for li in range(model.n_layers)}
        del self._gptq_state

    def _kept(self, li: int, name: str) -> bool:
        return li in self._keep_layers or (li, name) in self._keep_linears

    def _quantize(self) -> None:
        m = self.m
        dev = m.device
        self.qlayers = []
        self._lins = []
        for li in range(m.n_layers):
            lyr = m.layers[li]
            recs = {}
            for name in LIN_NAMES:
                if self._kept(li, name):
                    continue
                rec = self._gptq_state[li][name]
                N, K = int(rec["qsz"].shape[1]), int(rec["packed"].shape[1]) * 128
                q = int4pack_to_codes(rec["packed"].to(device=dev, dtype=torch.int32), N, K)
                recs[name] = (q, rec["qsz"].to(device=dev, dtype=torch.bfloat16).contiguous(),
                              self._group_size_map.get((li, name), self.w4_group_size))
            lins = {}
            for fused, members in FUSED_SETS.items():
                groups = {recs[n][2] for n in members if n in recs}
                if all(n in recs for n in members) and len(groups) == 1:
                    lins[fused] = _w4_set(fused, [recs[n][:2] for n in members], groups.pop())
                else:
                    mats = []
                    for n in members:
                        if n in recs:   # the W4 kernels' own operand, as bf16
                            q, qsz, g = recs[n]
                            mats.append(W4Weight.from_ref(q, qsz, g).dequant())
                        else:
                            mats.append(lyr[n].contiguous())
                    lins[fused] = _bf16_set(fused, mats)
            self._lins.append(lins)
            self.qlayers.append(None if li in self._keep_layers else
                                {name: lins[f] for f, ms in FUSED_SETS.items() for name in ms if name in recs})
            for name in recs:
                lyr.pop(name)
            del recs
        torch.cuda.empty_cache()

    @property
    def bf16_keep_layers(self) -> tuple:
        return tuple(sorted(self._keep_layers))

    @property
    def bf16_keep_linears(self) -> tuple:
        return tuple(sorted(self._keep_linears))

    def mixed_groups(self) -> dict:
        """{(layer, name): group size} of the linears whose group size is not
        the default (gptq.py:705-714)."""
        return {(li, name): g for li, gm in self.group_size_map.items() for name, g in gm.items()
                if g != self.w4_group_size}


def _w4_set(fused: str, recs: list, g: int):
    """One fused W4 launch from [(q [N_i, K], qsz [K/g, N_i, 2])]."""
    if fused == "qkv":
        return _W4Lin(W4Weight.from_ref(torch.cat([r[0] for r in recs], 0), torch.cat([r[1] for r in recs], 1), g))
    if fused == "gu":
        (qg, sg), (qu, su) = recs
        q = _interleave_rows(qg, qu, _FUSE_BLOCK)
        s = _interleave_cols(sg, su, _FUSE_BLOCK)
        return _W4Lin(W4Weight.from_ref(q, s, g), fuse_block=_FUSE_BLOCK)
    return _W4Lin(W4Weight.from_ref(recs[0][0], recs[0][1], g))


def _bf16_set(fused: str, mats: list):
    """One fused bf16 launch (gate and up interleaved row by row for the
    SwiGLU epilogue, as fast.bf16_linears builds them)."""
    if fused == "qkv":
        return _Bf16Lin(torch.cat(mats, 0).contiguous())
    if fused == "gu":
        return _Bf16Lin(torch.stack(mats, 1).reshape(-1, mats[0].shape[1]).contiguous())
    return _Bf16Lin(mats[0].contiguous())
