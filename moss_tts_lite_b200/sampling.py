"""Token sampling on the sm_100a kernels (mirror of moss_tts_lite.sampling).

* Greedy decisions (``do_sample=False``, sampling.py:84-85 of the reference)
  are first-index argmaxes (``mtl_argmax_rows`` / ``mtl_argmax_masked``).
* Sampled decisions (sampling.py:70-98 as used by fast.py:491-545) run in the
  fused per-row kernel ``mtl_sample_rows``: temperature, repetition penalty,
  top-k, top-p and one categorical draw per row.  Candidate sets and
  probabilities follow the reference's bf16 arithmetic; the random stream is
  Philox4x32-10 keyed by (seed, offset, row) instead of torch.multinomial's,
  so tokens agree with the reference in distribution.
"""
from __future__ import annotations

import itertools

import torch

from . import kernels
from .model import (AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_PAD_CODE, IM_END_TOKEN_ID,
                    N_VQ)

_offsets = itertools.count(1)

# Candidates one sampling CTA ranks after the top-k (kSampleMaxCand in
# csrc/sampling.cu): a top-k of at most this many over any row, or a row of
# at most this many columns with no top-k.
SAMPLE_MAX_CANDIDATES = 2048


def check_top_k(top_k, cols: int, what: str) -> None:
    """Reject, before any device work, a sampled decision the fused sampler
    does not serve: no top-k (or one beyond SAMPLE_MAX_CANDIDATES) over a row
    of more than SAMPLE_MAX_CANDIDATES columns, e.g. top-p alone over the
    151,936-way text head (the reference then sorts the whole vocabulary,
    sampling.py:101-113)."""
    k = int(top_k or 0)
    n = k if 0 < k < cols else cols
    if n > SAMPLE_MAX_CANDIDATES:
        raise NotImplementedError(
            f"{what}: sampling over {n} candidates (top_k={top_k}, {cols} columns) is not supported; "
            f"use a top_k of at most {SAMPLE_MAX_CANDIDATES} (the reference text default is 50) or greedy")


def sample_token(logits: torch.Tensor, prev_tokens: torch.Tensor | None = None, repetition_penalty: float = 1.0,
                 top_p=None, top_k=None, do_sample=True, seed: int | None = None) -> torch.Tensor:
    """sampling.py:70-98 on the device: ``logits`` bf16 [..., V] (at most 40
    rows); returns int64 [...].  ``prev_tokens`` (any shape) penalises the
    union of its ids for every row, as the reference's 2-D branch does.
    ``seed`` keys the Philox stream (default: torch.initial_seed()); each call
    advances the stream offset."""
    if logits.dtype != torch.bfloat16:
        logits = logits.to(torch.bfloat16)
    V = logits.shape[-1]
    x = logits.reshape(-1, V).contiguous()
    R = x.shape[0]
    out = torch.empty(R, dtype=torch.long, device=x.device)
    if not do_sample:
        kernels.argmax_rows(x, out)
        return out.view(logits.shape[:-1])
    check_top_k(top_k, V, "sample_token")
    seen = None
    if prev_tokens is not None and repetition_penalty != 1.0:
        # the union of the history's ids as a bit set, built on the device
        # (ids outside [0, V) land in a spare slot that is dropped)
        words = (V + 31) // 32
        ids = prev_tokens.reshape(-1).to(device=x.device, dtype=torch.long)
        ids = torch.where((ids >= 0) & (ids < V), ids, torch.full_like(ids, words * 32))
        bits = torch.zeros(words * 32 + 1, dtype=torch.bool, device=x.device)
        bits.index_fill_(0, ids, True)
        shifts = torch.arange(32, device=x.device, dtype=torch.int64)
        w = (bits[:words * 32].view(words, 32).to(torch.int64) << shifts).sum(1)
        w = torch.where(w >= 1 << 31, w - (1 << 32), w)   # two's-complement int32 words
        seen = w.to(torch.int32).view(1, words)
    kernels.sample_rows(x, list(range(R)), temperature=1.0, top_k=top_k or 0,
                        top_p=1.0 if top_p is None else float(top_p), penalty=repetition_penalty,
                        seen_bits=seen, seen_set=[0] * R, excluded=(),
                        seed=torch.initial_seed() if seed is None else seed, offset=next(_offsets), out=out,
                        scan_rows=[R] * R)
    return out.view(logits.shape[:-1])


class sample_rows:  # noqa: N801 - namespace of the two sampled decisions of generate_fast
    """Sampled text / audio decisions of one generate_fast step."""

    @staticmethod
    def text(fast, is_audio: bool, time_step: int, temperature: float, top_k, top_p, seed: int, offset: int,
             out: torch.Tensor) -> None:
        """fast.py:491-514: audio phase -> GEN/DELAY from the two-way logits
        (out[0] = 0 or 1); text phase -> a text id from the full head."""
        if is_audio:
            excluded = (1,) if time_step == 0 else ()
            kernels.sample_rows(fast.two_static.view(1, 2), [0], temperature=temperature, top_k=top_k or 0,
                                top_p=1.0 if top_p is None else top_p, excluded=excluded, seed=seed,
                                offset=offset, out=out)
        else:
            from .model import AUDIO_END_TOKEN_ID, PAD_TOKEN_ID
            ex = [PAD_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_END_TOKEN_ID]
            if time_step <= N_VQ:
                ex.append(IM_END_TOKEN_ID)
            kernels.sample_rows(fast.lt_static.view(1, -1), [0], temperature=temperature, top_k=top_k or 0,
                                top_p=1.0 if top_p is None else top_p, excluded=tuple(ex), seed=seed,
                                offset=offset, out=out)

    @staticmethod
    def audio(fast, smask, temperature: float, top_k, top_p, penalty: float, seen_bits, seed: int, offset: int,
              out: torch.Tensor) -> list:
        """fast.py:516-545: channel 0 with its own history for the penalty,
        the other sampled channels with the union of channels 1..31 (the
        reference passes generation_ids[:, :, 2:] to a 2-D sample_token).
        ``seen_bits``: device int32 [2, 33] bit sets of those two histories
        (needed when penalty != 1).  Writes one token per sampled channel to
        out[0:n]; returns the rows."""
        rows = [j for j in range(N_VQ) if smask[j]]
        sets = [0 if j == 0 else 1 for j in rows]
        # the reference scans channel 0 as [1, V] and the rest as [R, V]
        n_rest = sum(1 for j in rows if j > 0)
        scan = [1 if j == 0 else n_rest for j in rows]
        if penalty != 1.0 and seen_bits is None:
            raise ValueError("repetition penalty needs the history bit sets")
        kernels.sample_rows(fast.la_static, rows, temperature=temperature, top_k=top_k or 0,
                            top_p=1.0 if top_p is None else top_p, penalty=penalty,
                            seen_bits=seen_bits if penalty != 1.0 else None, seen_set=sets,
                            excluded=(AUDIO_PAD_CODE,), seed=seed, offset=offset, out=out, scan_rows=scan)
        return rows
