"""Torch-tensor wrappers over the C ABI of libmtl_b200.so.

torch owns the device memory and the current stream; every function here
launches one of this package's sm_100a kernels on
``torch.cuda.current_stream()`` and returns without synchronising, so all of
them can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _s() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _bf16(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")


def embed_sum(ids: torch.Tensor, emb_text: torch.Tensor, emb_audio: torch.Tensor,
              out: torch.Tensor) -> torch.Tensor:
    """ids int64 [M, 33] -> out bf16 [M, H] (model.py:156-161)."""
    M = ids.numel() // 33
    _lib.call("mtl_embed_sum", ids.data_ptr(), M, emb_text.data_ptr(), emb_text.shape[0],
              emb_audio.data_ptr(), emb_text.shape[1], out.data_ptr(), _s())
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    K = x.shape[-1]
    rows = x.numel() // K
    _lib.call("mtl_rmsnorm", x.data_ptr(), rows, K, K, weight.data_ptr(), ctypes.c_float(eps),
              out.data_ptr(), K, _s())
    return out


def attn_decode(qkv, q_norm_w, k_norm_w, rope_cos, rope_sin, k_cache_layer, v_cache_layer, pos_dev,
                n_heads: int, n_kv: int, splits: int, out, scratch, streams: int = 1,
                cache_stream_stride: int = 0, kv_stable: bool = False) -> torch.Tensor:
    """``kv_stable``: pos and cache rows [0, pos) are final before the
    preceding kernel started (graph-captured steps), so the cache may be
    streamed before the programmatic-dependent-launch wait."""
    max_seq = k_cache_layer.shape[-2]
    _lib.call("mtl_attn_decode", qkv.data_ptr(), q_norm_w.data_ptr(), k_norm_w.data_ptr(),
              rope_cos.data_ptr(), rope_sin.data_ptr(), k_cache_layer.data_ptr(), v_cache_layer.data_ptr(),
              ctypes.c_longlong(cache_stream_stride), max_seq, pos_dev.data_ptr(), streams, n_heads, n_kv,
              k_cache_layer.shape[-1], splits, _lib.MTL_ATTN_KV_STABLE if kv_stable else 0, out.data_ptr(),
              scratch.data_ptr(), scratch.numel(), _s())
    return out


def attn_append(qkv, k_norm_w, rope_cos, rope_sin, k_cache_layer, v_cache_layer, pos_dev, n_heads: int,
                n_kv: int, streams: int = 1, cache_stream_stride: int = 0, q_norm_w=None, q_out=None) -> None:
    """K/V append of `streams` rows (k norm + RoPE, v) into cache rows
    pos_dev[s]; with ``q_out`` also the rows' normed + rotated q heads."""
    max_seq = k_cache_layer.shape[-2]
    _lib.call("mtl_attn_append", qkv.data_ptr(), _p(q_norm_w), k_norm_w.data_ptr(), rope_cos.data_ptr(),
              rope_sin.data_ptr(), k_cache_layer.data_ptr(), v_cache_layer.data_ptr(),
              ctypes.c_longlong(cache_stream_stride), max_seq, pos_dev.data_ptr(), streams, n_heads, n_kv,
              k_cache_layer.shape[-1], _p(q_out), _s())


def attn_prefill(q: torch.Tensor, k_cache_layer: torch.Tensor, v_cache_layer: torch.Tensor, n_heads: int,
                 n_kv: int, out: torch.Tensor, *, rows_per_stream: int | None = None, streams: int = 1, p0: int = 0,
                 cache_stream_stride: int = 0) -> torch.Tensor:
    """Causal GQA attention over prompt rows (mtl_attn_prefill): q bf16
    [streams * rows, n_heads, 128] (normed + rotated), one layer's caches
    [n_kv, max_seq, 128] per stream, out bf16 [streams * rows, n_heads * 128]."""
    rows = rows_per_stream if rows_per_stream is not None else q.shape[0] // streams
    _lib.call("mtl_attn_prefill", q.data_ptr(), k_cache_layer.data_ptr(), v_cache_layer.data_ptr(),
              ctypes.c_longlong(cache_stream_stride), k_cache_layer.shape[-2], n_heads, n_kv, q.shape[-1], rows,
              streams, p0, out.data_ptr(), _s())
    return out


def bf16_linear(x: torch.Tensor, W: torch.Tensor, out: torch.Tensor, *, norm_weight=None, eps: float = 1e-6,
                x_normed=None, pad_period: int = 0, pad_col: int = 0, residual=None,
                swiglu: bool = False) -> torch.Tensor:
    """out = epilogue(x W^T) for bf16 W [N, K] (see include/mtl_b200.h)."""
    K = x.shape[-1]
    M = x.numel() // K
    N = W.shape[0]
    epi = _lib.MTL_EPI_SWIGLU if swiglu else (_lib.MTL_EPI_RESIDUAL if residual is not None else _lib.MTL_EPI_STORE)
    ldy = out.shape[-1]
    _lib.call("mtl_bf16_linear", x.data_ptr(), M, K, N, W.data_ptr(), _p(norm_weight), ctypes.c_float(eps),
              _p(x_normed), pad_period, pad_col, epi, _p(residual), out.data_ptr(), ldy, _s())
    return out


def argmax_rows(x: torch.Tensor, out: torch.Tensor, cols: int | None = None) -> torch.Tensor:
    """out int64 [rows] = first-index argmax of bf16 x [rows, ld]."""
    _bf16(x, "x")
    ld = x.shape[-1]
    rows = x.numel() // ld
    _lib.call("mtl_argmax_rows", x.data_ptr(), rows, ld if cols is None else cols, ld, out.data_ptr(), _s())
    return out


def argmax_scratch(device) -> torch.Tensor:
    """16 zeroed bytes for the GPU-wide argmax (one per concurrent caller)."""
    return torch.zeros(16, dtype=torch.uint8, device=device)


def argmax_masked(x: torch.Tensor, out: torch.Tensor, excluded=(), scratch: torch.Tensor | None = None) -> torch.Tensor:
    """out[0] = first-index argmax of the bf16 row ``x`` ignoring ``excluded``
    (<= 8 indices); with ``scratch`` (argmax_scratch) long rows use the whole GPU."""
    ex = list(excluded)
    arr = (ctypes.c_int32 * max(1, len(ex)))(*ex)
    _lib.call("mtl_argmax_masked", x.data_ptr(), x.numel(), arr, len(ex), out.data_ptr(), _p(scratch), _s())
    return out


def feed_row(dec: torch.Tensor, ids_row: torch.Tensor, pos_dev: torch.Tensor, pos: int, *, text_mode: int,
             text_const: int, gen_slot: int, delay_slot: int, audio_mask: int, audio_compact: bool, pad_code: int,
             seen_bits: torch.Tensor | None = None) -> None:
    """Next generate_fast input row from the step's decisions ``dec`` (int64 [33]), on the device."""
    words = seen_bits.shape[-1] if seen_bits is not None else 0
    _lib.call("mtl_feed_row", dec.data_ptr(), text_mode, text_const, gen_slot, delay_slot, audio_mask,
              int(audio_compact), pad_code, ids_row.data_ptr(), pos_dev.data_ptr(), pos, _p(seen_bits), words, _s())


def greedy_feed(la: torch.Tensor, two: torch.Tensor, ids_row: torch.Tensor, pos_dev: torch.Tensor,
                gen_slot: int, delay_slot: int, streams: int = 1) -> None:
    """Next row and position of a device-side greedy audio-phase loop, per stream."""
    _lib.call("mtl_greedy_feed", la.data_ptr(), two.data_ptr(), ids_row.data_ptr(), pos_dev.data_ptr(),
              streams, gen_slot, delay_slot, _s())


def sample_rows(logits: torch.Tensor, rows, *, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
                penalty: float = 1.0, seen_bits: torch.Tensor | None = None, seen_set=None, excluded=(),
                seed: int = 0, offset: int = 0, out: torch.Tensor, out_add: int = 0, scan_rows=None,
                sliced: bool = True) -> torch.Tensor:
    """One sampled token per listed row of bf16 ``logits`` [R, V] into out[0:len(rows)] (int64).
    ``scan_rows[i]``: rows of the reference's sample_token call that held
    row i (1 = a one-row call; default all 1), which fixes how its CUDA
    cumsum rounds the top-p partial sums.  ``sliced``: long rows with a
    top-k are selected by one CTA per slice (same draw; False = one CTA per
    row)."""
    _bf16(logits, "logits")
    V = logits.shape[-1]
    rows = list(rows)
    idx = (ctypes.c_int32 * len(rows))(*rows)
    sets = (ctypes.c_int32 * len(rows))(*(seen_set if seen_set is not None else [0] * len(rows)))
    ex = list(excluded)
    exa = (ctypes.c_int32 * max(1, len(ex)))(*ex)
    words = seen_bits.shape[-1] if seen_bits is not None else 0
    sr = (ctypes.c_int32 * len(rows))(*(scan_rows if scan_rows is not None else [1] * len(rows)))
    need = _lib.lib.mtl_sample_scratch_bytes(V, len(rows), int(top_k)) if sliced else 0
    scratch = _sample_scratch(logits.device, need) if need else None
    _lib.call("mtl_sample_rows", logits.data_ptr(), V, V, len(rows), idx, ctypes.c_float(temperature), int(top_k),
              ctypes.c_float(top_p), ctypes.c_float(penalty), _p(seen_bits), words, sets, exa, len(ex), sr,
              ctypes.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), ctypes.c_uint64(offset), ctypes.c_int64(out_add),
              out.data_ptr(), _p(scratch), need, _s())
    return out


_SAMPLE_SCRATCH: dict = {}


def _sample_scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device candidate buffer of the sliced sampling path (grows only;
    the text head's row with top-k <= 2048 needs at most 2.4 MB)."""
    buf = _SAMPLE_SCRATCH.get(device)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 148 * 2048 * 8), dtype=torch.uint8, device=device)
        _SAMPLE_SCRATCH[device] = buf
    return buf


def rtn_quantize(w: torch.Tensor, group_size: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference RTN W4 (fast.py:85-96): bf16 [N, K] -> (q uint8 [N, K], qsz bf16 [K/g, N, 2])."""
    _bf16(w, "w")
    w = w.contiguous()
    N, K = w.shape
    q = torch.empty(N, K, dtype=torch.uint8, device=w.device)
    qsz = torch.empty(K // group_size, N, 2, dtype=torch.bfloat16, device=w.device)
    _lib.call("mtl_w4_rtn_quantize", w.data_ptr(), N, K, group_size, q.data_ptr(), qsz.data_ptr(), _s())
    return q, qsz


def w4_chain(phases: list, group_size: int, barrier: torch.Tensor, eps: float = 1e-6) -> None:
    """Dependent batch-1 W4 linears in one persistent launch (mtl_w4_chain).
    ``phases``: up to 4 dicts {"w": StripWeight, "x": bf16 [K], "y": bf16
    out, "norm_w": bf16 [K] or None, "residual": bf16 [N] or None,
    "swiglu": bool}; phase i may read what phases < i wrote.  ``barrier``:
    a zeroed int32 device word (zero again after the launch)."""
    arr = (_lib.ChainPhase * len(phases))()
    for i, ph in enumerate(phases):
        w = ph["w"]
        epi = _lib.MTL_EPI_STORE
        if ph.get("swiglu"):
            epi = _lib.MTL_EPI_SWIGLU
        elif ph.get("residual") is not None:
            epi = _lib.MTL_EPI_RESIDUAL
        arr[i] = _lib.ChainPhase(w.tiles.data_ptr(), ph["x"].data_ptr(), _p(ph.get("norm_w")), _p(ph.get("residual")),
                                 ph["y"].data_ptr(), w.K, w.N, epi)
    _lib.call("mtl_w4_chain", arr, len(phases), group_size, ctypes.c_float(eps), barrier.data_ptr(), _s())


def w4_chain_rows(phases: list, group_size: int, barrier: torch.Tensor, eps: float = 1e-6) -> None:
    """w4_chain for M = 2..16 activation rows (mtl_w4_chain_rows): each
    phase's "x", "y" (and "residual") are [M, ...] row-major bf16 tensors
    with unit column stride."""
    arr = (_lib.ChainPhaseRows * len(phases))()
    M = int(phases[0]["x"].shape[0])
    for i, ph in enumerate(phases):
        w, x, y = ph["w"], ph["x"], ph["y"]
        res = ph.get("residual")
        epi = _lib.MTL_EPI_STORE
        if ph.get("swiglu"):
            epi = _lib.MTL_EPI_SWIGLU
        elif res is not None:
            epi = _lib.MTL_EPI_RESIDUAL
        if int(x.shape[0]) != M or int(y.shape[0]) != M:
            raise ValueError("every phase has the same number of rows")
        arr[i] = _lib.ChainPhaseRows(w.tiles.data_ptr(), x.data_ptr(), _p(ph.get("norm_w")), _p(res), y.data_ptr(),
                                     x.stride(0), 0 if res is None else res.stride(0), y.stride(0), w.K, w.N, epi)
    _lib.call("mtl_w4_chain_rows", arr, len(phases), M, group_size, ctypes.c_float(eps), barrier.data_ptr(), _s())
