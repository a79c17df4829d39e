"""A shim the reference package can carry to run its W4 linears on the B200
kernels: plain ctypes over libmtl_b200.so's C ABI (include/mtl_b200.h), no
other part of this package.

The reference builds its W4 weights in ``FastMossTTS._quantize``
(moss_tts_lite/fast.py:70-105: RTN codes q [N, K] and qsz = (scale,
zero) per group, then torch's tinygemm packer) and multiplies with
``torch._weight_int4pack_mm`` in ``FastMossTTS._linear`` (fast.py:107-121).
``pack`` replaces the packer, ``int4_mm`` the multiply, and ``install``
returns a subclass of the reference's ``FastMossTTS`` whose ``_quantize`` /
``_linear`` call them; everything else (its graphs, eager attention,
generate_fast) stays the reference's own.
"""
from __future__ import annotations

import ctypes
import os

import torch

_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmtl_b200.so")
_L = ctypes.CDLL(_LIB)
_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_L.mtl_w4a16_linear.argtypes = [_vp, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp, _f, _i, _vp, _vp, _i, _vp, _sz,
                                _vp]
_L.mtl_w4_pack_ref.argtypes = [_vp, _vp, _i, _i, _i, _vp, _vp]
_L.mtl_w4_plan.argtypes = [_i] * 5 + [ctypes.POINTER(ctypes.c_size_t)] * 2
_L.mtl_last_error.restype = ctypes.c_char_p


def _check(rc: int) -> None:
    if rc:
        raise RuntimeError(_L.mtl_last_error().decode())


def pack(q_codes: torch.Tensor, qsz: torch.Tensor, g: int):
    """Replaces _convert_weight_to_int4pack (fast.py:97-99): codes uint8
    [N, K] + qsz bf16 [K/g, N, 2] -> (tiles, scratch) on the codes' device."""
    N, K = q_codes.shape
    tb, sb = ctypes.c_size_t(), ctypes.c_size_t()
    _check(_L.mtl_w4_plan(8, K, N, g, 0, ctypes.byref(tb), ctypes.byref(sb)))
    tiles = torch.empty(tb.value, dtype=torch.uint8, device=q_codes.device)
    scratch = torch.zeros(sb.value, dtype=torch.uint8, device=q_codes.device)
    q = q_codes.to(torch.uint8).contiguous()
    z = qsz.to(torch.bfloat16).contiguous()
    _check(_L.mtl_w4_pack_ref(q.data_ptr(), z.data_ptr(), K, N, g, tiles.data_ptr(),
                              torch.cuda.current_stream().cuda_stream))
    return tiles, scratch


def int4_mm(x2: torch.Tensor, tiles: torch.Tensor, scratch: torch.Tensor, g: int, N: int) -> torch.Tensor:
    """Replaces torch._weight_int4pack_mm(x2, packed, g, qsz) (fast.py:118):
    x2 bf16 [M, K] -> bf16 [M, N]."""
    x2 = x2.to(torch.bfloat16).contiguous()
    M, K = x2.shape
    y = torch.empty(M, N, dtype=torch.bfloat16, device=x2.device)
    _check(_L.mtl_w4a16_linear(x2.data_ptr(), K, M, K, N, g, 0, tiles.data_ptr(), 0, None, None, _f(1e-6), 0, None,
                               y.data_ptr(), N, scratch.data_ptr(), scratch.numel(),
                               torch.cuda.current_stream().cuda_stream))
    return y


def install(fast_cls):
    """A subclass of the reference's ``FastMossTTS`` whose W4 weights are
    packed by ``pack`` and multiplied by ``int4_mm``.  It uses the reference's
    own RTN (gptq.rtn_quantize / pack_qsz_only, the codes and qsz its
    _quantize builds)."""
    from moss_tts_lite.gptq import pack_qsz_only, rtn_quantize

    class B200FastMossTTS(fast_cls):
        def _quantize(self) -> None:
            if self.quant != "w4":
                return super()._quantize()
            self.qlayers = []
            g = self.w4_group_size
            for lyr in self.m.layers:
                rec = {}
                for name in ("q", "k", "v", "o", "gate", "up", "down"):
                    q, s, mn = rtn_quantize(lyr[name], g)
                    qsz = pack_qsz_only(s, mn, g)
                    rec[name] = (*pack(q, qsz, g), int(qsz.shape[1]))
                    lyr.pop(name)
                self.qlayers.append(rec)
            torch.cuda.empty_cache()

        def _linear(self, x: torch.Tensor, li: int, name: str) -> torch.Tensor:
            if self.quant != "w4":
                return super()._linear(x, li, name)
            tiles, scratch, N = self.qlayers[li][name]
            y = int4_mm(x.reshape(-1, x.shape[-1]), tiles, scratch, self.w4_group_size, N)
            return y.to(self.m.dtype).reshape(*x.shape[:-1], N)

    return B200FastMossTTS
