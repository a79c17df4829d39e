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
