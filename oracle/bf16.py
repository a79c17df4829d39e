"""bfloat16 helpers for the numpy oracle (test infrastructure only).

bfloat16 values are carried as ``uint16`` bit patterns. Conversions follow
IEEE round-to-nearest-even, which is what ``torch.Tensor.to(torch.bfloat16)``
does on both CPU and CUDA.
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """Widen bfloat16 bit patterns to float32 (exact)."""
    u = np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16
    return u.view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest-even), returned as uint16 bits."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (u >> 16) & 1
    r = (u + 0x7FFF + lsb) >> 16
    r = r.astype(np.uint32) & 0xFFFF
    r = np.where(nan, 0x7FC0, r)
    return r.astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 value, returned as float32."""
    return bf16_to_f32(f32_to_bf16(x))


def f16_to_f32(u16: np.ndarray) -> np.ndarray:
    """Widen IEEE half bit patterns to float32 (exact)."""
    return np.asarray(u16, dtype=np.uint16).view(np.float16).astype(np.float32)


def torch_bf16_bits(t) -> np.ndarray:
    """uint16 bit patterns of a torch bfloat16 tensor (CPU copy)."""
    import torch
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)
