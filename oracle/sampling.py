"""Sampling and delay-pattern FSM restated in numpy (test infrastructure only).

Restates moss_tts_lite/sampling.py (apply_top_k 9-17, apply_top_p_optimized
101-113, apply_repetition_penalty_delay_pattern 36-67, sample_token 70-98,
find_last_equal_C 116-126) and the per-step text decision / audio mask of
moss_tts_lite/fast.py:465-520 (isolated in fast_native.py:51-67).

Ties: torch.topk / torch.sort leave the order of equal values unspecified,
so where ties straddle a cut-off the kept *set* may differ between
implementations while the kept *values* agree.  The oracle keeps the lowest
indices among ties (stable order); tests compare tie-robustly.
"""
from __future__ import annotations

import numpy as np

INT64_MAX = 9223372036854775807
N_VQ = 32
PAD_TOKEN_ID = 151643
AUDIO_END_TOKEN_ID = 151653
AUDIO_DELAY_SLOT_TOKEN_ID = 151662


def apply_top_k(logits: np.ndarray, top_k: int) -> np.ndarray:
    """sampling.py:9-17: keep the k largest per row, -inf elsewhere."""
    b, v = logits.shape
    k = min(top_k, v)
    order = np.argsort(-logits, axis=-1, kind="stable")[:, :k]
    out = np.full_like(logits, -np.inf)
    rows = np.arange(b)[:, None]
    out[rows, order] = logits[rows, order]
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float64)
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(-1, keepdims=True)


def apply_top_p(logits: np.ndarray, top_p: float) -> np.ndarray:
    """sampling.py:101-113: drop the tail whose cumulative probability
    (sorted descending, shifted by one so the top token always stays)
    exceeds top_p."""
    probs = softmax(logits)
    order = np.argsort(-probs, axis=-1, kind="stable")
    sp = np.take_along_axis(probs, order, -1)
    cum = np.cumsum(sp, -1)
    remove = cum > top_p
    remove[..., 1:] = remove[..., :-1].copy()
    remove[..., 0] = False
    mask = np.zeros_like(remove)
    np.put_along_axis(mask, order, remove, -1)
    out = logits.copy()
    out[mask] = -np.inf
    return out


def apply_repetition_penalty(logits: np.ndarray, prev_tokens: np.ndarray, penalty: float) -> np.ndarray:
    """sampling.py:36-67 for [N, V] (all heads share the token set) and
    [B, H, V] (per-head token sets)."""
    if penalty == 1.0 or prev_tokens is None:
        return logits
    out = logits.copy()
    if out.ndim == 2:
        u = np.unique(prev_tokens.reshape(-1))
        t = out[:, u]
        out[:, u] = np.where(t > 0, t / np.float32(penalty), t * np.float32(penalty))
        return out
    for h in range(out.shape[1]):
        u = np.unique(prev_tokens[..., h].reshape(-1))
        if u.size == 0:
            continue
        t = out[:, h, u]
        out[:, h, u] = np.where(t > 0, t / np.float32(penalty), t * np.float32(penalty))
    return out


def argmax_first(x: np.ndarray) -> np.ndarray:
    """torch.argmax semantics: index of the first maximal value."""
    return np.argmax(x, axis=-1)


def candidate_set(logits: np.ndarray, top_k: int | None, top_p: float | None) -> np.ndarray:
    """Boolean mask of tokens with non-zero probability after top-k then
    top-p (sample_token, sampling.py:90-96)."""
    x = logits.astype(np.float32)
    if top_k is not None and top_k > 0:
        x = apply_top_k(x, top_k)
    if top_p is not None and top_p < 1.0:
        x = apply_top_p(x, top_p)
    return np.isfinite(x)


def find_last_equal(row: np.ndarray, c: int) -> int:
    """sampling.py:116-126 for one row: last index equal to c, else -1."""
    hit = np.nonzero(np.asarray(row) == c)[0]
    return int(hit[-1]) if hit.size else -1


def text_decision(dl: int, n_vq: int, wd_stop: bool, is_stopping: bool, is_audio: bool):
    """fast.py:465-478 (== fast_native.py:51-63): the forced text token of the
    delay ramp.  Returns (next_text, is_audio, sampling_text, forced)."""
    if wd_stop:
        if dl == INT64_MAX or dl < n_vq:
            return AUDIO_DELAY_SLOT_TOKEN_ID, is_audio, False, True
        return AUDIO_END_TOKEN_ID, False, False, True
    if not is_stopping and dl < n_vq:
        return AUDIO_DELAY_SLOT_TOKEN_ID, is_audio, False, True
    if not is_stopping and dl == n_vq:
        return AUDIO_END_TOKEN_ID, False, False, True
    sampling_text = (not is_stopping) and (not wd_stop) and dl > n_vq
    return PAD_TOKEN_ID, is_audio, sampling_text, False


def audio_sampling_mask(al: int, dl: int, n_vq: int) -> list:
    """fast.py:520: channel j is sampled iff al > j and (no delay ramp, or
    j > dl - 1)."""
    return [(al > j) and (dl == INT64_MAX or j > dl - 1) for j in range(n_vq)]


# --------------------------------------------------------------------------
# Fused sampling restated (the arithmetic of mtl_sample_rows)
# --------------------------------------------------------------------------

def philox4x32_10(counter, key):
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC 2011) on Python ints."""
    M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
    c = [x & 0xFFFFFFFF for x in counter]
    k0, k1 = key[0] & 0xFFFFFFFF, key[1] & 0xFFFFFFFF
    for _ in range(10):
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c = [(hi1 ^ c[1] ^ k0) & 0xFFFFFFFF, lo1, (hi0 ^ c[3] ^ k1) & 0xFFFFFFFF, lo0]
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return c


def uniform(seed: int, offset: int, row: int) -> np.float32:
    """The 24-bit uniform in [0, 1) that mtl_sample_rows draws for one row."""
    c = philox4x32_10([offset & 0xFFFFFFFF, (offset >> 32) & 0xFFFFFFFF, row, 0],
                      [seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF])
    return np.float32(c[0] >> 8) * np.float32(1.0 / 16777216.0)


def _bf(x):
    from .bf16 import round_bf16
    return round_bf16(np.asarray(x, np.float32))


# torch.cumsum of bf16 on CUDA (ATen/native/cuda/ScanUtils.cuh scan_dim, the
# PyTorch release the reference runs on): every partial sum is a bf16 value
# (the scan operator is std::plus<c10::BFloat16>: fp32 add, then round), and
# the grouping of the additions depends on the tensor's shape.
CUB_ITEMS_PER_THREAD = 30     # bf16 items per thread of the device-wide scan
CUB_TILE_THREADS = 128        # threads per tile of the device-wide scan


def _bfadd(a, b):
    return _bf(np.asarray(a, np.float32) + np.asarray(b, np.float32)).astype(np.float32)


def cumsum_device_wide(q: np.ndarray) -> np.ndarray:
    """One-row tensor ([1, n] or [n]): scan_dim hands it to CUB's
    DeviceScan::InclusiveScan.  Each thread owns CUB_ITEMS_PER_THREAD
    consecutive items and reduces them left to right; the thread totals are
    scanned per warp of 32 (Kogge-Stone: lane l adds lane l-2^i for i =
    0..4), warps chain left to right inside a tile of CUB_TILE_THREADS
    threads, tiles chain left to right; each thread then adds its items one
    by one onto its exclusive prefix."""
    q = np.asarray(q, np.float32)
    n = q.size
    ipt, tt = CUB_ITEMS_PER_THREAD, CUB_TILE_THREADS
    nthr = -(-n // ipt)
    nthr_pad = -(-nthr // tt) * tt
    x = np.zeros(nthr_pad * ipt, np.float32)
    x[:n] = q
    x = x.reshape(nthr_pad, ipt)
    agg = x[:, 0].copy()
    for i in range(1, ipt):
        agg = _bfadd(agg, x[:, i])
    # warp-level inclusive scan of the thread totals
    inc = agg.reshape(-1, 32).copy()
    for off in (1, 2, 4, 8, 16):
        nxt = inc.copy()
        nxt[:, off:] = _bfadd(inc[:, :-off], inc[:, off:])
        inc = nxt
    exc = np.zeros_like(inc)
    exc[:, 1:] = inc[:, :-1]                       # lane 0: no warp prefix
    wagg = inc[:, 31]
    wpt = tt // 32
    pre = np.zeros(nthr_pad, np.float32)
    tile_prefix = np.float32(0)
    for t0 in range(0, nthr_pad // 32, wpt):      # tiles
        ba = np.float32(0)
        for w in range(t0, t0 + wpt):
            wp = ba                                # exclusive prefix of warp w in the tile
            lane_exc = exc[w]
            if w > t0:
                lane_exc = np.where(np.arange(32) == 0, wp, _bfadd(wp, lane_exc))
            if t0 > 0:
                lane_exc = _bfadd(tile_prefix, lane_exc)
            pre[w * 32:(w + 1) * 32] = lane_exc
            ba = wagg[w] if w == t0 else _bfadd(ba, wagg[w])
        tile_prefix = ba if t0 == 0 else _bfadd(tile_prefix, ba)
    out = np.empty_like(x)
    run = pre
    for i in range(ipt):
        run = _bfadd(run, x[:, i])
        out[:, i] = run
    return out.reshape(-1)[:n]


def inner_scan_log_threads_x(num_rows: int, row_size: int) -> int:
    """get_log_num_threads_x_inner_scan (ScanUtils.cuh): threads per row of
    the shared-memory scan, as a power of two in [16, 512]."""
    lx = max(0, int(np.ceil(np.log2(row_size)))) if row_size > 1 else 0
    ly = max(0, int(np.ceil(np.log2(num_rows)))) if num_rows > 1 else 0
    return min(max(4, (9 + lx - ly) // 2), 9)


def cumsum_rows_sklansky(q: np.ndarray, log_nx: int) -> np.ndarray:
    """Rows of a [R>1, n] tensor (tensor_kernel_scan_innermost_dim): chunks
    of 2*2^log_nx items; the running total of the earlier chunks is added to
    the chunk's first item, then log_nx+1 Sklansky rounds (round m: item
    a + j, a = (x >> m << (m+1)) | 2^m, j < 2^m, adds item a - 1)."""
    q = np.atleast_2d(np.asarray(q, np.float32))
    R, n = q.shape
    nx = 1 << log_nx
    out = np.empty_like(q)
    carry = np.zeros(R, np.float32)
    x = np.arange(nx)
    for base in range(0, n, 2 * nx):
        buf = np.zeros((R, 2 * nx), np.float32)
        seg = q[:, base:base + 2 * nx]
        buf[:, :seg.shape[1]] = seg
        buf[:, 0] = _bfadd(buf[:, 0], carry)
        for m in range(log_nx + 1):
            s = 1 << m
            a = ((x >> m) << (m + 1)) | s
            ti = a + (x % s)
            si = a - 1
            buf[:, ti] = _bfadd(buf[:, ti], buf[:, si])
        out[:, base:base + seg.shape[1]] = buf[:, :seg.shape[1]]
        carry = buf[:, 2 * nx - 1].copy()
    return out


def cumsum_bf16_cuda(q: np.ndarray, num_rows: int = 1, row_size: int | None = None) -> np.ndarray:
    """torch.cumsum(dim=-1) of a bf16 tensor of ``num_rows`` rows of
    ``row_size`` on CUDA, for the leading part ``q`` of one row (positions
    depend only on the items before them, so a prefix of the row scans the
    same)."""
    q = np.asarray(q, np.float32)
    if num_rows == 1:
        return cumsum_device_wide(q)
    return cumsum_rows_sklansky(q[None, :], inner_scan_log_threads_x(num_rows, row_size or q.size))[0]


def sample_row(logits_bits: np.ndarray, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
               penalty: float = 1.0, seen=(), excluded=(), seed: int = 0, offset: int = 0, row: int = 0,
               return_probs: bool = False, device: str = "cuda", scan_rows: int = 1):
    """One row of mtl_sample_rows restated: sample_token (sampling.py:70-98)
    with the reference's bf16 rounding points (temperature as a multiply by
    the float reciprocal, bf16 penalty, top-k with lowest ids kept at a tie,
    top-p on bf16 softmax and bf16 cumsum against bf16(top_p), bf16 softmax)
    and the Philox4x32-10 categorical draw in id order.

    ``device`` selects PyTorch's cumsum of bf16: on CUDA every partial sum
    is rounded to bf16, grouped as cumsum_bf16_cuda does for a tensor of
    ``scan_rows`` rows (the rows of the reference's sample_token call that
    held this row); on CPU the sum is fp32 and only the outputs are rounded.
    The reference's decode path runs on CUDA."""
    from .bf16 import bf16_to_f32
    x = bf16_to_f32(np.asarray(logits_bits, np.uint16)).astype(np.float32)
    n = x.size
    if temperature != 1.0:
        x = _bf(x * np.float32(np.float32(1.0) / np.float32(temperature)))
    x = x.copy()
    for e in excluded:
        x[e] = -np.inf
    if penalty != 1.0 and len(seen):
        ids = np.asarray(sorted(set(int(s) for s in seen)), np.int64)
        v = x[ids]
        x[ids] = np.where(v > 0, _bf(v * np.float32(np.float32(1.0) / np.float32(penalty))),
                          _bf(v * np.float32(penalty)))
    k = top_k if 0 < top_k < n else n
    if k < n:
        order = np.lexsort((np.arange(n), -x))          # value desc, id asc
        cand = np.sort(order[:k])
    else:
        cand = np.arange(n)
    cv = x[cand].copy()

    def softmax_bf16(v):
        fin = np.isfinite(v)
        if not fin.any():
            return np.zeros_like(v)
        m = v[fin].max()
        e = np.where(fin, np.exp((v - m).astype(np.float32)), np.float32(0)).astype(np.float32)
        s = np.float32(e.sum(dtype=np.float32))
        return np.where(fin, _bf(e / s), np.float32(0)).astype(np.float32)

    if top_p < 1.0 and cv.size > 1:
        p = softmax_bf16(cv)
        order = np.lexsort((np.arange(cv.size), -p))
        thr = _bf(np.float32(top_p))
        if device == "cuda":
            cum = cumsum_bf16_cuda(p[order], scan_rows, n)
        else:
            cum = _bf(np.cumsum(p[order], dtype=np.float32))
        rem = cum > thr
        # removal shifted by one: the first sorted candidate always stays
        cv[order[1:][rem[:-1]]] = -np.inf
    p = softmax_bf16(cv)
    if return_probs:
        return cand, p
    tot = np.float32(p.sum(dtype=np.float32))
    pick = -1
    if tot > 0:
        target = np.float32(uniform(seed, offset, row) * tot)
        run = np.float32(0)
        for i in range(p.size):
            run = np.float32(run + p[i])
            if p[i] > 0 and run > target:
                pick = i
                break
        if pick < 0:
            pick = int(np.nonzero(p > 0)[0][-1])
    if pick < 0:
        pick = int(np.argmax(cv)) if np.isfinite(cv).any() else 0
    return int(cand[pick])
