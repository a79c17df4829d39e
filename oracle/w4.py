"""W4A16 oracle: int4 unpack, dequant, RTN quantisation and the fp32 GEMV.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Two weight faces are restated here.

1. The reference's own face (moss_tts_lite/gptq.py, moss_tts_lite/fast.py):
   integer codes ``q`` uint8 [N, K] in 0..15 and a bf16 tensor
   ``qsz`` [K/g, N, 2] = (scale, zero) with ``w = (q - 8) * scale + zero``
   (gptq.py:87-97). ``zero`` is stored as ``mn + 8 * scale`` (fast.py:94-96).

2. The AutoGPTQ face named by the benchmark configuration: ``qweight`` int32
   [K/8, N], ``qzeros`` int32 [K/g, N/8], fp16 ``scales`` [K/g, N] and
   ``g_idx`` int32 [K].  The reference does not define this face, so the
   convention is declared here and used everywhere in this repository:

   * nibbles are packed LSB-first along K:
     ``q[k, n] = (qweight[k // 8, n] >> (4 * (k % 8))) & 0xF``;
   * zeros are packed LSB-first along N:
     ``z[G, n] = (qzeros[G, n // 8] >> (4 * (n % 8))) & 0xF``;
   * ``w[k, n] = (q[k, n] - (z[g_idx[k], n] + zero_offset)) * scales[g_idx[k], n]``
     with ``zero_offset = 0`` by default (``1`` reproduces the historical
     AutoGPTQ "zeros + 1" checkpoints).
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16_to_f32, f16_to_f32, f32_to_bf16

# --------------------------------------------------------------------------
# AutoGPTQ face: bit-exact pack / unpack
# --------------------------------------------------------------------------


def unpack_qweight(qweight: np.ndarray) -> np.ndarray:
    """int32 [K/8, N] -> uint8 codes [K, N] (LSB-first nibbles along K)."""
    qw = np.asarray(qweight).astype(np.uint32)
    k8, n = qw.shape
    shifts = (4 * np.arange(8, dtype=np.uint32)).reshape(1, 8, 1)
    codes = (qw.reshape(k8, 1, n) >> shifts) & 0xF
    return codes.reshape(k8 * 8, n).astype(np.uint8)


def pack_qweight(codes: np.ndarray) -> np.ndarray:
    """uint8 codes [K, N] -> int32 [K/8, N] (inverse of unpack_qweight)."""
    c = np.asarray(codes).astype(np.uint32)
    k, n = c.shape
    if k % 8:
        raise ValueError(f"K={k} is not a multiple of 8")
    c = c.reshape(k // 8, 8, n)
    shifts = (4 * np.arange(8, dtype=np.uint32)).reshape(1, 8, 1)
    return np.bitwise_or.reduce(c << shifts, axis=1).astype(np.uint32).view(np.int32)


def unpack_qzeros(qzeros: np.ndarray) -> np.ndarray:
    """int32 [G, N/8] -> uint8 zeros [G, N] (LSB-first nibbles along N)."""
    qz = np.asarray(qzeros).astype(np.uint32)
    g, n8 = qz.shape
    shifts = (4 * np.arange(8, dtype=np.uint32)).reshape(1, 1, 8)
    z = (qz.reshape(g, n8, 1) >> shifts) & 0xF
    return z.reshape(g, n8 * 8).astype(np.uint8)


def pack_qzeros(zeros: np.ndarray) -> np.ndarray:
    """uint8 zeros [G, N] -> int32 [G, N/8]."""
    z = np.asarray(zeros).astype(np.uint32)
    g, n = z.shape
    if n % 8:
        raise ValueError(f"N={n} is not a multiple of 8")
    z = z.reshape(g, n // 8, 8)
    shifts = (4 * np.arange(8, dtype=np.uint32)).reshape(1, 1, 8)
    return np.bitwise_or.reduce(z << shifts, axis=2).astype(np.uint32).view(np.int32)


def gptq_dequant(qweight, qzeros, scales_f16, g_idx, zero_offset: int = 0) -> np.ndarray:
    """Effective fp32 weight [K, N] of the AutoGPTQ face.

    ``(q - z) * s`` is exact in float32 (a 5-bit integer times an fp16).
    """
    q = unpack_qweight(qweight).astype(np.float32)
    z = unpack_qzeros(qzeros).astype(np.float32) + np.float32(zero_offset)
    s = f16_to_f32(scales_f16)
    gi = np.asarray(g_idx, dtype=np.int64)
    return (q - z[gi]) * s[gi]


# --------------------------------------------------------------------------
# Reference face: moss_tts_lite/gptq.py and moss_tts_lite/fast.py
# --------------------------------------------------------------------------


def group_scales_from_weight(w: np.ndarray, group_size: int = 128, device: str = "cuda"):
    """Restates gptq.py:35-45 (== fast.py:88-90): asymmetric group min/max,
    ``s = clamp((mx - mn) / 15, min=1e-6)``.

    ``device`` selects PyTorch's arithmetic for the division by the Python
    scalar 15: on CUDA it multiplies by the float reciprocal 1.0f/15.0f, on
    CPU it divides.  The W4 path of the reference runs on CUDA
    (fast.py:97 has no CPU kernel), so "cuda" is the default.
    ``w`` float32 [N, K]. Returns ``(s, mn)`` float32 [N, K/g]."""
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"K={k} not divisible by group_size={group_size}")
    wg = w.reshape(n, k // group_size, group_size)
    mx = wg.max(-1)
    mn = wg.min(-1)
    if device == "cuda":
        d = ((mx - mn) * (np.float32(1.0) / np.float32(15.0))).astype(np.float32)
    elif device == "cpu":
        d = ((mx - mn) / np.float32(15.0)).astype(np.float32)
    else:
        raise ValueError(f"device must be 'cuda' or 'cpu', got {device!r}")
    s = np.maximum(d, np.float32(1e-6)).astype(np.float32)
    return s, mn.astype(np.float32)


def rtn_quantize(w_bf16_bits: np.ndarray, group_size: int = 128, device: str = "cuda"):
    """Restates gptq.py:54-64 / fast.py:85-93 (round-to-nearest W4).

    ``w_bf16_bits`` uint16 [N, K] bf16 weights. Returns ``(q, s, mn)``:
    uint8 codes [N, K], float32 scale and min [N, K/g]. ``np.rint`` rounds
    half to even like ``torch.round``; ``device`` as in
    group_scales_from_weight."""
    w = bf16_to_f32(w_bf16_bits)
    n, k = w.shape
    g = group_size
    s, mn = group_scales_from_weight(w, g, device)
    wg = w.reshape(n, k // g, g)
    q = np.clip(np.rint((wg - mn[..., None]) / s[..., None]), 0, 15)
    return q.astype(np.uint8).reshape(n, k), s, mn


def pack_qsz(s: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Restates gptq.py:79-85 (``pack_qsz_only``) / fast.py:94-96.

    Returns bf16 bits [K/g, N, 2] = (scale, mn + 8 * scale)."""
    zero = (mn + np.float32(8.0) * s).astype(np.float32)
    st = np.stack([s.astype(np.float32), zero], -1)          # [N, G, 2]
    return np.ascontiguousarray(f32_to_bf16(st).transpose(1, 0, 2))


def ref_effective_weight(q: np.ndarray, qsz_bits: np.ndarray, group_size: int = 128) -> np.ndarray:
    """Restates gptq.py:87-97 (``effective_weight``): fp32 [N, K] of
    ``(q - 8) * scale + zero`` with the bf16 (scale, zero) widened exactly."""
    n, k = q.shape
    g = group_size
    qsz = bf16_to_f32(qsz_bits)                       # [G, N, 2]
    scale = qsz[:, :, 0].T                            # [N, G]
    zero = qsz[:, :, 1].T
    qf = q.astype(np.float32).reshape(n, k // g, g)
    w = (qf - np.float32(8.0)) * scale[..., None] + zero[..., None]
    return w.reshape(n, k).astype(np.float32)


def ref_operand_weight(q: np.ndarray, qsz_bits: np.ndarray, group_size: int = 128) -> np.ndarray:
    """The operand torch's int4 GEMM (``_weight_int4pack_mm``, the reference's
    W4 linear at fast.py:118 / gptq.py:582) multiplies with: the effective
    weight of gptq.py:87-97 rounded once to bf16 (bf16 FMA of the exact
    q - 8 with the bf16 scale and zero).  Returned widened to fp32 [N, K].
    Pinned against the kernel's own outputs by tests/golden/tinygemm.npz."""
    n, k = q.shape
    g = group_size
    qsz = bf16_to_f32(qsz_bits).astype(np.float64)    # [G, N, 2]
    scale = qsz[:, :, 0].T                            # [N, G]
    zero = qsz[:, :, 1].T
    qf = q.astype(np.float64).reshape(n, k // g, g)
    exact = (qf - 8.0) * scale[..., None] + zero[..., None]   # exact in fp64
    return bf16_to_f32(f32_to_bf16(exact.reshape(n, k).astype(np.float32)))


# --------------------------------------------------------------------------
# The W4A16 linear itself
# --------------------------------------------------------------------------


def linear_f64(x_bf16_bits: np.ndarray, w_kn: np.ndarray) -> np.ndarray:
    """``x @ W`` evaluated in float64 (the exact value the fp32-accumulating
    kernel approximates). ``x`` bf16 bits [M, K]; ``w_kn`` fp32 [K, N]."""
    x = bf16_to_f32(x_bf16_bits).astype(np.float64)
    return x @ np.asarray(w_kn, dtype=np.float64)


def linear_bf16(x_bf16_bits: np.ndarray, w_kn: np.ndarray) -> np.ndarray:
    """bf16 output bits of the W4A16 linear: fp32 accumulate, one final
    round-to-nearest-even (the semantics of ``torch._weight_int4pack_mm``
    named in gptq.py:577-585 and fast.py:107-121)."""
    return f32_to_bf16(linear_f64(x_bf16_bits, w_kn).astype(np.float32))


def close_enough(y_bits: np.ndarray, ref_f64: np.ndarray, atol: float = 2e-2, rtol: float = 1e-2):
    """The north-star GEMV tolerance: max-abs 2e-2 OR relative 1e-2 per
    element against the exact value (bf16 output, fp32 accumulation)."""
    y = bf16_to_f32(y_bits).astype(np.float64)
    d = np.abs(y - ref_f64)
    ok = d <= np.maximum(atol, rtol * np.abs(ref_f64))
    return bool(ok.all()), float(d.max()) if d.size else 0.0


# --------------------------------------------------------------------------
# Seeded synthetic inputs (benchmark configurations 0 and 1)
# --------------------------------------------------------------------------


def synth_gptq_linear(K: int, N: int, group_size: int = 128, seed: int = 0):
    """Seeded AutoGPTQ-layout linear with the benchmark's distributions:
    codes and zeros uniform 0..15, ``scales = |N(0,1)| * 0.01 + 1e-3`` (fp16),
    ``g_idx = k // g``, ``x ~ N(0, 1)`` bf16 [1, K]."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    zeros = rng.integers(0, 16, size=(K // group_size, N), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal((K // group_size, N))) * 0.01 + 1e-3).astype(np.float16)
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    g_idx = (np.arange(K) // group_size).astype(np.int32)
    return dict(qweight=pack_qweight(codes), qzeros=pack_qzeros(zeros),
                scales=scales.view(np.uint16), g_idx=g_idx, x=x,
                codes=codes, zeros=zeros)
