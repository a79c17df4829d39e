"""ctypes binding of libmtl_b200.so (the C ABI declared in include/mtl_b200.h).

The shared library is built in-tree by ``moss_tts_lite_b200.build``. There
is no fallback: if the library is missing or fails to load, importing this
module raises, and every op of the package is unavailable.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmtl_b200.so")

MTL_OK = 0
MTL_E_INVALID = -1
MTL_E_ALIGN = -2
MTL_E_SCRATCH = -3
MTL_E_CUDA = -4
MTL_E_UNSUPPORTED = -5
MTL_FMT_REF = 0
MTL_FMT_GPTQ = 1
MTL_FMT_TC = 2
MTL_EPI_STORE = 0
MTL_EPI_RESIDUAL = 1
MTL_EPI_SWIGLU = 2
MTL_ATTN_KV_STABLE = 1

ABI_VERSION = 2

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_size_t = ctypes.c_size_t
_c_size_p = ctypes.POINTER(ctypes.c_size_t)
_c_u32_p = ctypes.POINTER(ctypes.c_uint32)



class ChainPhase(ctypes.Structure):
    """mtl_chain_phase (include/mtl_b200.h)."""
    _fields_ = [("tiles", _c_void_p), ("x", _c_void_p), ("norm_w", _c_void_p), ("residual", _c_void_p),
                ("y", _c_void_p), ("K", _c_int), ("N", _c_int), ("epilogue", _c_int)]


class ChainPhaseRows(ctypes.Structure):
    """mtl_chain_phase_rows (include/mtl_b200.h)."""
    _fields_ = [("tiles", _c_void_p), ("x", _c_void_p), ("norm_w", _c_void_p), ("residual", _c_void_p),
                ("y", _c_void_p), ("ldx", _c_int), ("ldr", _c_int), ("ldy", _c_int), ("K", _c_int), ("N", _c_int),
                ("epilogue", _c_int)]


# name -> (restype, argtypes); every exported symbol of include/mtl_b200.h.
SIGNATURES = {
    "mtl_last_error": (ctypes.c_char_p, []),
    "mtl_abi_version": (_c_int, []),
    "mtl_device_status": (_c_int, [_c_u32_p, _c_int]),
    "mtl_w4_plan": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_size_p, _c_size_p]),
    "mtl_w4_pack_ref": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_w4_pack_tc": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_w4_pack_gptq": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int,
                                  _c_void_p, _c_void_p]),
    "mtl_w4_dequant": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_w4_unpack_codes": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_w4a16_linear": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,
                                  _c_int, _c_void_p, _c_void_p, _c_float, _c_int, _c_void_p, _c_void_p,
                                  _c_int, _c_void_p, _c_size_t, _c_void_p]),
    "mtl_w4a16_linear_noalloc": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p,
                                          _c_int, _c_void_p, _c_void_p, _c_float, _c_int, _c_void_p, _c_void_p,
                                          _c_int, _c_void_p]),
    "mtl_w4a16_gemm": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_int, _c_void_p,
                                _c_int, _c_void_p, _c_int, _c_void_p]),
    "mtl_w4_strip_bytes": (_c_int, [_c_int, _c_int, _c_int, _c_size_p]),
    "mtl_w4_pack_strip": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_w4_chain": (_c_int, [ctypes.POINTER(ChainPhase), _c_int, _c_int, _c_float, _c_void_p, _c_void_p]),
    "mtl_w4_chain_rows": (_c_int, [ctypes.POINTER(ChainPhaseRows), _c_int, _c_int, _c_int, _c_float, _c_void_p,
                                   _c_void_p]),
    "mtl_attn_prefill": (_c_int, [_c_void_p, _c_void_p, _c_void_p, ctypes.c_longlong, _c_int, _c_int, _c_int,
                                  _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_embed_sum": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_void_p, _c_int, _c_void_p, _c_void_p]),
    "mtl_attn_scratch_bytes": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_size_p]),
    "mtl_attn_decode": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                 ctypes.c_longlong, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int,
                                 _c_int, _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "mtl_attn_append": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                 ctypes.c_longlong, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_void_p,
                                 _c_void_p]),
    "mtl_bf16_linear": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_float, _c_void_p,
                                 _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_int, _c_void_p]),
    "mtl_argmax_rows": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "mtl_argmax_masked": (_c_int, [_c_void_p, _c_int, ctypes.POINTER(ctypes.c_int32), _c_int, _c_void_p,
                                   _c_void_p, _c_void_p]),
    "mtl_feed_row": (_c_int, [_c_void_p, _c_int, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong,
                              ctypes.c_uint, _c_int, ctypes.c_longlong, _c_void_p, _c_void_p, ctypes.c_longlong,
                              _c_void_p, _c_int, _c_void_p]),
    "mtl_greedy_feed": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p]),
    "mtl_sample_rows": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, ctypes.POINTER(ctypes.c_int32), _c_float,
                                 _c_int, _c_float, _c_float, _c_void_p, _c_int, ctypes.POINTER(ctypes.c_int32),
                                 ctypes.POINTER(ctypes.c_int32), _c_int, ctypes.POINTER(ctypes.c_int32),
                                 ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, _c_void_p, _c_void_p,
                                 _c_size_t, _c_void_p]),
    "mtl_sample_scratch_bytes": (_c_size_t, [_c_int, _c_int, _c_int]),
    "mtl_rmsnorm": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_float, _c_void_p, _c_int,
                             _c_void_p]),
    "mtl_w4_rtn_quantize": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p]),
}


class MtlError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def _load() -> ctypes.CDLL:
    if not os.path.isfile(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m moss_tts_lite_b200.build` "
            "(nvcc, sm_100a). There is no CPU or PyTorch fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if lib.mtl_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH}: ABI {lib.mtl_abi_version()} != expected {ABI_VERSION}; rebuild")
    return lib


lib = _load()


def call(name: str, *args) -> None:
    """Call ``name`` and raise MtlError on a non-zero status."""
    rc = getattr(lib, name)(*args)
    if rc != MTL_OK:
        raise MtlError(name, rc, lib.mtl_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib.mtl_last_error().decode(errors="replace")


def device_status(clear: bool = True) -> int:
    """Error word that kernels set instead of trapping (0 = clean)."""
    v = ctypes.c_uint32(0)
    call("mtl_device_status", ctypes.byref(v), 1 if clear else 0)
    return int(v.value)


def w4_plan(M: int, K: int, N: int, g: int, fmt: int) -> tuple[int, int]:
    """(tiles_bytes, scratch_bytes) for a W4 linear."""
    tb = ctypes.c_size_t(0)
    sb = ctypes.c_size_t(0)
    call("mtl_w4_plan", M, K, N, g, fmt, ctypes.byref(tb), ctypes.byref(sb))
    return int(tb.value), int(sb.value)


def strip_bytes(K: int, N: int, g: int) -> int:
    """Bytes of a strip-layout W4 weight (mtl_w4_pack_strip)."""
    out = ctypes.c_size_t(0)
    call("mtl_w4_strip_bytes", K, N, g, ctypes.byref(out))
    return int(out.value)


def attn_scratch_bytes(streams: int, n_heads: int, n_kv: int, splits: int) -> int:
    out = ctypes.c_size_t(0)
    call("mtl_attn_scratch_bytes", streams, n_heads, n_kv, splits, ctypes.byref(out))
    return int(out.value)
