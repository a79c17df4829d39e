"""CUDA-graph W4 / bf16 decode for MOSS-TTS on the sm_100a kernels.

Drop-in for ``moss_tts_lite.fast`` (fast.py:31-610 of the reference):
``FastMossTTS(model, quant=..., w4_group_size=...)`` with ``capture()``,
``step(row, pos, audio2)``, ``prefill(input_ids)`` and the static output
buffers, plus ``generate_fast``.  What changes is the step itself:

* the reference replays 38 piecewise graphs per step with 36 eager
  attention calls between them (fast.py:308-325) and ~2,300 torch kernels;
* here ONE graph per phase holds the whole step - embedding sum, per layer
  [q|k|v W4 GEMV with the input RMSNorm fused in] -> [q/k-norm + RoPE + KV
  append + split-KV GQA attention] -> [o W4 GEMV + residual] -> [gate|up W4
  GEMV with the post-attention RMSNorm and SwiGLU fused] -> [down W4 GEMV +
  residual], then the final norm fused into the head GEMVs: 5 kernels per
  layer, 183 per step.  The decode position is read from ``pos_dev`` on the
  device, so one graph serves every cache length.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field

import torch

from . import _lib, fsm, kernels
from .generate import GenResult
from .model import (AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_END_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_PAD_CODE,
                    AUDIO_START_TOKEN_ID, AUDIO_VOCAB, IM_END_TOKEN_ID, LIN_NAMES, N_VQ, PAD_TOKEN_ID,
                    RMS_EPS, HiddenState)
from .quant import StripWeight, W4Weight, gemm_supported

_INT64_MAX = 9223372036854775807
_LIN_NAMES = LIN_NAMES
_FUSE_BLOCK = 32  # gate/up interleave granularity of the register-MMA tiles' SwiGLU epilogue
_GEMM_PREFILL_ROWS = 32  # prompts from this many rows prefill through dequantised bf16 GEMMs


# ------------------------------------------------------------------ linears
class _W4Lin:
    """A packed W4 linear (possibly fused q|k|v or gate|up)."""

    def __init__(self, w: W4Weight, fuse_block: int = _FUSE_BLOCK):
        self.w = w
        self.N = w.N
        self.fuse_block = fuse_block   # gate/up interleave of a fused SwiGLU pair

    def __call__(self, x, out, *, norm_weight=None, residual=None, swiglu=False):
        return self.w.linear(x, out=out, norm_weight=norm_weight, norm_eps=RMS_EPS,
                             residual=residual, swiglu=swiglu)


class _Bf16Lin:
    """A bf16 linear (F.linear semantics) on the bf16 GEMV kernel."""

    def __init__(self, W: torch.Tensor):
        self.W = W
        self.N = W.shape[0]

    def __call__(self, x, out, *, norm_weight=None, residual=None, swiglu=False):
        M = x.numel() // x.shape[-1]
        for r0 in range(0, M, 4):
            r1 = min(M, r0 + 4)
            kernels.bf16_linear(x.view(M, -1)[r0:r1], self.W, out.view(M, -1)[r0:r1], norm_weight=norm_weight,
                                eps=RMS_EPS, residual=None if residual is None else residual.view(M, -1)[r0:r1],
                                swiglu=swiglu)
        return out


def _interleave_rows(a: torch.Tensor, b: torch.Tensor, block: int) -> torch.Tensor:
    """[N, ...] x2 -> [2N, ...] with blocks of `block` rows alternating a, b."""
    n = a.shape[0]
    rest = a.shape[1:]
    return torch.stack([a.reshape(n // block, block, *rest), b.reshape(n // block, block, *rest)], 1) \
        .reshape(2 * n, *rest)


def _interleave_cols(a: torch.Tensor, b: torch.Tensor, block: int) -> torch.Tensor:
    """qsz [G, N, 2] x2 -> [G, 2N, 2] interleaved along N in blocks."""
    return _interleave_rows(a.transpose(0, 1), b.transpose(0, 1), block).transpose(0, 1).contiguous()


def bf16_linears(m) -> list:
    """Fused bf16 linears per layer.  The model's per-projection tensors are
    replaced by views into the fused ones (no second copy stays alive)."""
    lins = []
    for lyr in m.layers:
        qkv = torch.cat([lyr["q"], lyr["k"], lyr["v"]], 0).contiguous()
        nq, nk = lyr["q"].shape[0], lyr["k"].shape[0]
        lyr["q"], lyr["k"], lyr["v"] = qkv[:nq], qkv[nq:nq + nk], qkv[nq + nk:]
        gu = torch.stack([lyr["gate"], lyr["up"]], 1).reshape(-1, lyr["gate"].shape[1]).contiguous()
        lyr["gate"], lyr["up"] = gu[0::2], gu[1::2]
        lins.append({"qkv": _Bf16Lin(qkv), "o": _Bf16Lin(lyr["o"]), "gu": _Bf16Lin(gu),
                     "down": _Bf16Lin(lyr["down"])})
    return lins


def w4_from_codes(recs: dict, group_size: int, fmt: int | None = None) -> dict:
    """{name: (q uint8 [N, K], qsz bf16 [K/g, N, 2])} of one layer -> fused
    packed W4 linears (q|k|v concatenated, gate|up interleaved).  The
    register-MMA tiles (MTL_FMT_REF) are the decode default; ``fmt =
    MTL_FMT_TC`` selects the tensor-core tiles where they cover every shape
    of the layer (measured slower at batch 1 on B200: the A operand's TMEM
    traffic, 4 bytes per weight, bounds it below the register-MMA kernel)."""
    q = torch.cat([recs["q"][0], recs["k"][0], recs["v"][0]], 0)
    qsz = torch.cat([recs["q"][1], recs["k"][1], recs["v"][1]], 1)
    shapes = [tuple(q.shape), tuple(recs["o"][0].shape), (2 * recs["gate"][0].shape[0], recs["gate"][0].shape[1]),
              tuple(recs["down"][0].shape)]
    tc = fmt == _lib.MTL_FMT_TC and all(W4Weight.tc_supported(k, n, group_size) for n, k in shapes)
    fmt = _lib.MTL_FMT_TC if tc else _lib.MTL_FMT_REF
    blk = 1 if tc else _FUSE_BLOCK
    out = {"qkv": _W4Lin(W4Weight.from_ref(q, qsz, group_size, fmt=fmt))}
    out["o"] = _W4Lin(W4Weight.from_ref(recs["o"][0], recs["o"][1], group_size, fmt=fmt))
    gq = _interleave_rows(recs["gate"][0], recs["up"][0], blk)
    gs = _interleave_cols(recs["gate"][1], recs["up"][1], blk)
    out["gu"] = _W4Lin(W4Weight.from_ref(gq, gs, group_size, fmt=fmt), fuse_block=blk)
    out["down"] = _W4Lin(W4Weight.from_ref(recs["down"][0], recs["down"][1], group_size, fmt=fmt))
    return out


# ------------------------------------------------------------------- engine
class _StepEngine:
    """Launch sequence of one decode step (batch 1) over static buffers."""

    def __init__(self, m, lins: list, buffers=None):
        self.m = m
        self.lins = lins
        dev = m.device
        H, D = m.hidden_size, m.head_dim
        bf = torch.bfloat16
        b = buffers
        self.ids_row = b.ids_row if b is not None else torch.zeros(1, 1, N_VQ + 1, dtype=torch.long, device=dev)
        self.pos_dev = b.pos_dev if b is not None else torch.zeros(1, dtype=torch.long, device=dev)
        self.h = (b.h_static if b is not None else torch.zeros(1, 1, H, dtype=bf, device=dev)).view(1, H)
        self.h_final = b.h_final if b is not None else torch.zeros(1, H, dtype=bf, device=dev)
        self.lt = b.lt_static if b is not None else torch.zeros(m.text_vocab, dtype=bf, device=dev)
        self.la = b.la_static if b is not None else torch.zeros(N_VQ, AUDIO_VOCAB, dtype=bf, device=dev)
        self.two = b.two_static if b is not None else torch.zeros(2, dtype=bf, device=dev)
        nq = m.n_heads * D
        self.qkv = torch.zeros(1, nq + 2 * m.n_kv_heads * D, dtype=bf, device=dev)
        self.attn = torch.zeros(1, nq, dtype=bf, device=dev)
        inter = lins[0]["gu"].N // 2
        self.act = torch.zeros(1, inter, dtype=bf, device=dev)
        # KV splits per head: 8 heads x 16 splits covers the SMs once the cache
        # is long; short caches use fewer (each split holds >= 32 positions)
        self.splits = 16
        from . import _lib
        nbytes = _lib.attn_scratch_bytes(1, m.n_heads, m.n_kv_heads, self.splits)
        self.attn_scratch = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.emb_audio = getattr(m, "emb_audio", None)
        if self.emb_audio is None:   # reference MossTTSModel: stack its 32 tables once
            self.emb_audio = torch.stack(list(m.emb_ext), 0).contiguous()
        self.head_audio2d = m.head_audio.view(N_VQ * AUDIO_VOCAB, H)
        # True while a step graph is captured: every replay follows the steps
        # that wrote pos and the cache rows before it
        self.kv_stable = False
        self.strips: list | None = None

    def chain_capable(self) -> bool:
        """Whether every layer's four fused linears are reference-format W4
        weights of one group size that the persistent chain kernel serves."""
        gs = set()
        for L in self.lins:
            for n in ("qkv", "o", "gu", "down"):
                lin = L[n]
                if not isinstance(lin, _W4Lin) or lin.w.fmt != _lib.MTL_FMT_REF or lin.w.k_perm is not None:
                    return False
                if not StripWeight.supported(lin.w.K, lin.w.N, lin.w.group_size):
                    return False
                gs.add(lin.w.group_size)
        return len(gs) == 1

    def enable_chain(self) -> bool:
        """Strip-layout copies of the layers' W4 weights (the prefill keeps
        the register-MMA tiles) and one barrier word per chain launch; the
        backbone then runs each layer's o -> gate|up -> down -> next q|k|v
        as one persistent launch (mtl_w4_chain) between the attention
        launches.  Returns False (nothing changed) when not capable."""
        if self.strips is not None:
            return True
        if not self.chain_capable():
            return False
        self.strips = [{"qkv": L["qkv"].w.to_strip(), "o": L["o"].w.to_strip(),
                        "gu": L["gu"].w.to_strip(swiglu_block=L["gu"].fuse_block), "down": L["down"].w.to_strip()}
                       for L in self.lins]
        self.chain_g = self.lins[0]["qkv"].w.group_size
        # one word per launch, 128 bytes apart
        self.chain_bar = torch.zeros(self.m.n_layers + 1, 32, dtype=torch.int32, device=self.m.device)
        return True

    def _phase(self, li: int, name: str) -> dict:
        m, S = self.m, self.strips[li]
        lyr = m.layers[li]
        h = self.h.view(-1)
        if name == "qkv":
            return {"w": S["qkv"], "x": h, "y": self.qkv.view(-1), "norm_w": lyr["input_layernorm"]}
        if name == "o":
            return {"w": S["o"], "x": self.attn.view(-1), "y": h, "residual": h}
        if name == "gu":
            return {"w": S["gu"], "x": h, "y": self.act.view(-1), "norm_w": lyr["post_attention_layernorm"],
                    "swiglu": True}
        return {"w": S["down"], "x": self.act.view(-1), "y": h, "residual": h}

    def _attn(self, li: int) -> None:
        m = self.m
        lyr = m.layers[li]
        kernels.attn_decode(self.qkv, lyr["q_norm"], lyr["k_norm"], m.rope_cos, m.rope_sin,
                            m.k_cache[li], m.v_cache[li], self.pos_dev, m.n_heads, m.n_kv_heads,
                            self.splits, self.attn, self.attn_scratch, kv_stable=self.kv_stable)

    def backbone(self) -> None:
        m = self.m
        kernels.embed_sum(self.ids_row.view(1, N_VQ + 1), m.embed_tokens, self.emb_audio, self.h)
        if self.strips is not None:
            n, g, bar = m.n_layers, self.chain_g, self.chain_bar
            kernels.w4_chain([self._phase(0, "qkv")], g, bar[0], RMS_EPS)
            for li in range(n):
                self._attn(li)
                names = ("o", "gu", "down", "qkv") if li + 1 < n else ("o", "gu", "down")
                phases = [self._phase(li, nm) for nm in names[:3]]
                if li + 1 < n:
                    phases.append(self._phase(li + 1, "qkv"))
                kernels.w4_chain(phases, g, bar[li + 1], RMS_EPS)
            return
        for li in range(m.n_layers):
            lyr, L = m.layers[li], self.lins[li]
            L["qkv"](self.h, self.qkv, norm_weight=lyr["input_layernorm"])
            kernels.attn_decode(self.qkv, lyr["q_norm"], lyr["k_norm"], m.rope_cos, m.rope_sin,
                                m.k_cache[li], m.v_cache[li], self.pos_dev, m.n_heads, m.n_kv_heads,
                                self.splits, self.attn, self.attn_scratch, kv_stable=self.kv_stable)
            L["o"](self.attn, self.h, residual=self.h)
            L["gu"](self.h, self.act, norm_weight=lyr["post_attention_layernorm"], swiglu=True)
            L["down"](self.act, self.h, residual=self.h)

    def heads(self, audio2: bool) -> None:
        m = self.m
        if audio2:
            kernels.bf16_linear(self.h, m.head_2way, self.two.view(1, 2), norm_weight=m.final_norm,
                                eps=RMS_EPS, x_normed=self.h_final)
        else:
            kernels.bf16_linear(self.h, m.head_text, self.lt.view(1, -1), norm_weight=m.final_norm,
                                eps=RMS_EPS, x_normed=self.h_final)
        kernels.bf16_linear(self.h, self.head_audio2d, self.la.view(1, -1), norm_weight=m.final_norm,
                            eps=RMS_EPS, pad_period=AUDIO_VOCAB, pad_col=AUDIO_PAD_CODE)

    def final_norm(self) -> None:
        kernels.rmsnorm(self.h, self.m.final_norm, self.h_final, RMS_EPS)

    def decode_row(self, row: torch.Tensor, pos: int) -> torch.Tensor:
        """Eager decode of one row at ``pos``: returns a copy of the final-normed hidden [1, H]."""
        self.ids_row.view(-1).copy_(row.view(-1))
        self.pos_dev.fill_(pos)
        self.backbone()
        self.final_norm()
        return self.h_final.clone()

    def _prefill_chunk_rows(self) -> int:
        """Rows per prefill chunk: 8 (the register-MMA kernel's batch, the MMA
        N dimension, so 8 rows cost one pass over the weights) when every
        linear of the layer has an 8-row launch plan, else 4."""
        if getattr(self, "_chunk", None) is None:
            from . import _lib
            self._chunk = 8
            for lin in self.lins[0].values():
                w = getattr(lin, "w", None)
                if w is None:
                    continue
                try:
                    _lib.w4_plan(8, w.K, w.N, w.group_size, w.fmt)
                except Exception:
                    self._chunk = 4
        return self._chunk

    def prefill_rows(self, ids: torch.Tensor, caches=None) -> torch.Tensor:
        """Prompt rows [L, 33] -> final-normed hidden [L, H] (fast.py:218-270).
        Rows go through the layers in chunks: the projections of a chunk are
        one batched W4 launch each (the weights are read once per chunk).  The
        chunk's attention is two launches: the K/V append of all its rows,
        then one attention launch with the rows as streams over the shared
        cache, row r attending over [0, pos_r] (rows of the chunk included).
        ``caches`` = (k layers, v layers) selects another stream's KV cache
        (bf16 [n_kv, max_seq, 128] per layer; default the model's own)."""
        m = self.m
        kcs, vcs = caches if caches is not None else (m.k_cache, m.v_cache)
        L = ids.shape[0]
        if self.gemm_prefill_ok(L):
            return self._prefill_gemm(ids, kcs, vcs)
        H = m.hidden_size
        C = self._prefill_chunk_rows()
        dev = m.device
        bf = torch.bfloat16
        if getattr(self, "_p_h", None) is None or self._p_h.shape[0] < C:
            self._p_h = torch.zeros(C, H, dtype=bf, device=dev)
            self._p_qkv = torch.zeros(C, self.qkv.shape[-1], dtype=bf, device=dev)
            self._p_attn = torch.zeros(C, self.attn.shape[-1], dtype=bf, device=dev)
            self._p_act = torch.zeros(C, self.act.shape[-1], dtype=bf, device=dev)
            nbytes = _lib.attn_scratch_bytes(C, m.n_heads, m.n_kv_heads, self.splits)
            self._p_scratch = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        out = torch.empty(L, H, dtype=bf, device=dev)
        pos_all = torch.arange(L, dtype=torch.long, device=dev)
        for r0 in range(0, L, C):
            R = min(C, L - r0)
            h, qkv, attn, act = self._p_h[:R], self._p_qkv[:R], self._p_attn[:R], self._p_act[:R]
            kernels.embed_sum(ids[r0:r0 + R].contiguous(), m.embed_tokens, self.emb_audio, h)
            for li in range(m.n_layers):
                lyr, Lw = m.layers[li], self.lins[li]
                Lw["qkv"](h, qkv, norm_weight=lyr["input_layernorm"])
                pos = pos_all[r0:r0 + R]
                kernels.attn_append(qkv, lyr["k_norm"], m.rope_cos, m.rope_sin, kcs[li], vcs[li],
                                    pos, m.n_heads, m.n_kv_heads, streams=R)
                kernels.attn_decode(qkv, lyr["q_norm"], lyr["k_norm"], m.rope_cos, m.rope_sin, kcs[li],
                                    vcs[li], pos, m.n_heads, m.n_kv_heads, self.splits, attn,
                                    self._p_scratch, streams=R)
                Lw["o"](attn, h, residual=h)
                Lw["gu"](h, act, norm_weight=lyr["post_attention_layernorm"], swiglu=True)
                Lw["down"](act, h, residual=h)
            kernels.rmsnorm(h, m.final_norm, out[r0:r0 + R], RMS_EPS)
        return out

    def _prefill_gemm(self, ids: torch.Tensor, kcs, vcs, streams: int = 1) -> torch.Tensor:
        """Long prompts, layer by layer over all their rows, as the reference
        prefills (fast.py:218-270, every projection one int4 GEMM with
        M = L): each projection is one tcgen05 W4 GEMM over all rows on the
        packed weights (``mtl_w4a16_gemm``; the o and down projections add
        the residual, gate|up applies SwiGLU in its epilogue); one launch per
        stream appends its rows' normed + rotated K and V to the cache and
        writes the normed + rotated q heads, and one causal GQA attention
        launch (``mtl_attn_prefill``) reads each K/V tile once per head group
        where the reference expands K/V and runs SDPA (fast.py:237-241).

        ``streams`` > 1: ``ids`` holds that many prompts of equal length one
        after the other, and ``kcs`` / ``vcs`` [layer] are [streams, n_kv,
        max_seq, 128] caches; the GEMMs then run over all streams' rows at
        once (M = streams x L)."""
        m = self.m
        L_all = ids.shape[0]
        L = L_all // streams
        H, D = m.hidden_size, m.head_dim
        dev, bf = m.device, torch.bfloat16
        nq = m.n_heads * D
        h = torch.empty(L_all, H, dtype=bf, device=dev)
        xn = torch.empty(L_all, H, dtype=bf, device=dev)
        qn = torch.empty(L_all, m.n_heads, D, dtype=bf, device=dev)
        qkv = torch.empty(L_all, self.lins[0]["qkv"].N, dtype=bf, device=dev)
        act = torch.empty(L_all, self.lins[0]["gu"].N // 2, dtype=bf, device=dev)
        attn = torch.empty(L_all, nq, dtype=bf, device=dev)
        pos = torch.arange(L, dtype=torch.long, device=dev)
        kernels.embed_sum(ids.contiguous(), m.embed_tokens, self.emb_audio, h)
        for li in range(m.n_layers):
            lyr, Lw = m.layers[li], self.lins[li]
            kernels.rmsnorm(h, lyr["input_layernorm"], xn, RMS_EPS)
            Lw["qkv"].w.gemm(xn, out=qkv)
            if streams == 1:
                kernels.attn_append(qkv, lyr["k_norm"], m.rope_cos, m.rope_sin, kcs[li], vcs[li], pos, m.n_heads,
                                    m.n_kv_heads, streams=L, q_norm_w=lyr["q_norm"], q_out=qn)
            else:
                for s in range(streams):
                    r = slice(s * L, (s + 1) * L)
                    kernels.attn_append(qkv[r], lyr["k_norm"], m.rope_cos, m.rope_sin, kcs[li][s], vcs[li][s], pos,
                                        m.n_heads, m.n_kv_heads, streams=L, q_norm_w=lyr["q_norm"], q_out=qn[r])
            kernels.attn_prefill(qn, kcs[li], vcs[li], m.n_heads, m.n_kv_heads, attn, rows_per_stream=L,
                                 streams=streams, cache_stream_stride=kcs[li][0].numel() if streams > 1 else 0)
            Lw["o"].w.gemm(attn, residual=h, out=h)                                  # fast.py:168
            kernels.rmsnorm(h, lyr["post_attention_layernorm"], xn, RMS_EPS)
            Lw["gu"].w.gemm(xn, out=act, swiglu=True)                                 # fast.py:170-171
            Lw["down"].w.gemm(act, residual=h, out=h)                                 # fast.py:170
        out = torch.empty(L_all, H, dtype=bf, device=dev)
        kernels.rmsnorm(h, m.final_norm, out, RMS_EPS)
        return out

    def gemm_prefill_ok(self, L: int) -> bool:
        """Whether a prompt of L rows prefills through the tensor-core GEMM path."""
        return L >= _GEMM_PREFILL_ROWS and all(isinstance(self.lins[0][n], _W4Lin) and gemm_supported(self.lins[0][n].w)
                                               for n in ("qkv", "o", "gu", "down"))


# --------------------------------------------------------------- FastMossTTS
class FastMossTTS:
    """CUDA-graph decoder around a MossTTSModel (weights / cache are shared)."""

    def __init__(self, model, enable_gqa: bool = True, gqa_max_len: int = 640,
                 quant: str | None = None, inner_k_tiles: int = 8, w4_group_size: int = 128,
                 chain: bool | None = None):
        self.m = model
        dev = model.device
        if dev.type != "cuda":
            raise RuntimeError("FastMossTTS runs on CUDA (sm_100a) only")
        self.enable_gqa = enable_gqa
        self.gqa_max_len = gqa_max_len
        self.quant = quant
        if quant not in (None, "w8", "w4"):
            raise ValueError(f"unsupported quant mode {quant!r} (None, 'w8' or 'w4')")
        if quant == "w8":
            raise NotImplementedError("the W8 tier is not part of the B200 W4 decode path")
        self.inner_k_tiles = inner_k_tiles
        if w4_group_size not in (32, 64, 128, 256):
            raise ValueError("w4_group_size must be 32/64/128/256")
        self.w4_group_size = w4_group_size
        bf = model.dtype
        self.ids_row = torch.zeros(1, 1, N_VQ + 1, dtype=torch.long, device=dev)
        self.pos_dev = torch.zeros(1, dtype=torch.long, device=dev)
        self.q_static = torch.zeros(1, model.n_heads, 1, model.head_dim, dtype=bf, device=dev)
        self.o_static = torch.zeros(1, model.hidden_size, dtype=bf, device=dev)
        self.h_static = torch.zeros(1, 1, model.hidden_size, dtype=bf, device=dev)
        self.h_final = torch.zeros(1, model.hidden_size, dtype=bf, device=dev)
        self.lt_static = torch.zeros(model.text_vocab, dtype=bf, device=dev)
        self.la_static = torch.zeros(N_VQ, AUDIO_PAD_CODE + 1, dtype=bf, device=dev)
        self.two_static = torch.zeros(2, dtype=bf, device=dev)
        self.lt_buf = torch.full((model.text_vocab,), float("-inf"), dtype=bf, device=dev)
        self.qlayers: list | None = None
        if quant == "w4":
            self._quantize()
        else:
            self._lins = bf16_linears(model)
        self.engine = _StepEngine(model, self._lins, buffers=self)
        # persistent chain launches for the W4 decode step (MTL_CHAIN=0 or
        # chain=False keeps one launch per linear)
        if chain is None:
            chain = os.environ.get("MTL_CHAIN", "1") != "0"
        self.chain = bool(chain) and self.engine.enable_chain()
        self.graphs: list | None = None
        self.capture_stream = torch.cuda.Stream(device=dev)

    def _quantize(self) -> None:
        """RTN W4 of the 7 backbone linears per layer with the reference's exact
        codes and (scale, zero) (fast.py:70-105), packed into the tile layout;
        the bf16 originals are dropped like the reference does."""
        m = self.m
        self.qlayers = []
        self._lins = []
        for li in range(m.n_layers):
            lyr = m.layers[li]
            recs = {name: kernels.rtn_quantize(lyr[name], self.w4_group_size) for name in _LIN_NAMES}
            self._lins.append(w4_from_codes(recs, self.w4_group_size))
            self.qlayers.append({name: self._lins[-1] for name in ("qkv", "o", "gu", "down")})
            for name in _LIN_NAMES:
                lyr.pop(name)
            del recs
        torch.cuda.empty_cache()

    def _linear(self, x: torch.Tensor, li: int, name: str) -> torch.Tensor:
        """One named backbone projection (the reference boundary of fast.py:107-121)
        computed through the fused layer weights and sliced."""
        m = self.m
        L = self._lins[li]
        D = m.head_dim
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        if name in ("q", "k", "v"):
            out = torch.empty(x2.shape[0], L["qkv"].N, dtype=torch.bfloat16, device=x.device)
            L["qkv"](x2, out)
            nq, nk = m.n_heads * D, m.n_kv_heads * D
            sl = {"q": slice(0, nq), "k": slice(nq, nq + nk), "v": slice(nq + nk, nq + 2 * nk)}[name]
            y = out[:, sl]
        elif name in ("gate", "up"):
            lin = L["gu"]
            out = torch.empty(x2.shape[0], lin.N, dtype=torch.bfloat16, device=x.device)
            lin(x2, out)
            if isinstance(lin, _W4Lin):
                fb = lin.fuse_block
                y = out.view(x2.shape[0], -1, 2, fb)[:, :, 0 if name == "gate" else 1].reshape(x2.shape[0], -1)
            else:
                y = out[:, 0::2] if name == "gate" else out[:, 1::2]
        else:
            lin = L[name]
            y = torch.empty(x2.shape[0], lin.N, dtype=torch.bfloat16, device=x.device)
            lin(x2, y)
        return y.contiguous().reshape(*x.shape[:-1], y.shape[-1])

    def prefill(self, input_ids: torch.Tensor) -> HiddenState:
        """fast.py:251-270: prompt [1, L, 33] -> final-normed hidden [1, L, H]."""
        m = self.m
        if input_ids.dim() != 3 or input_ids.shape[0] != 1 or input_ids.shape[-1] != N_VQ + 1:
            raise ValueError(f"expected input ids [1, L, {N_VQ + 1}], got {tuple(input_ids.shape)}")
        t = int(input_ids.shape[1])
        if t > m.max_seq_len:
            raise ValueError(f"seq len {t} exceeds KV cache {m.max_seq_len}")
        m.reset()
        ids = input_ids.to(device=m.device, dtype=torch.long)
        h = self.engine.prefill_rows(ids[0])
        m._seq = t
        return HiddenState(h.view(1, t, m.hidden_size))

    def _run_eager(self, audio2: bool) -> None:
        self.engine.backbone()
        self.engine.heads(audio2)

    def capture(self) -> None:
        """Warm up, then capture one whole-step graph per phase (text / audio2)."""
        if self.graphs is not None:
            return
        m = self.m
        self.pos_dev.fill_(m.max_seq_len - 1)       # scratch slot, as fast.py:280-281
        s = torch.cuda.Stream(device=m.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                self._run_eager(False)
                self._run_eager(True)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        pool = torch.cuda.graph_pool_handle()
        self.graphs = []
        self.engine.kv_stable = True
        try:
            for audio2 in (False, True):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=pool, stream=self.capture_stream):
                    self._run_eager(audio2)
                self.graphs.append(g)
        finally:
            self.engine.kv_stable = False
        torch.cuda.synchronize()

    def capture_greedy_loop(self) -> torch.cuda.CUDAGraph:
        """Graph of one autoregressive audio-phase step with device-side
        greedy feedback (next row and position written by the feed kernel):
        replaying it repeatedly decodes with no host round trip."""
        from .model import AUDIO_DELAY_SLOT_TOKEN_ID as _DELAY, AUDIO_GEN_SLOT_TOKEN_ID as _GEN
        self.capture()

        def body():
            self._run_eager(True)
            kernels.greedy_feed(self.la_static, self.two_static, self.ids_row, self.pos_dev, _GEN, _DELAY)

        g = torch.cuda.CUDAGraph()
        self.engine.kv_stable = True
        try:
            with torch.cuda.graph(g, stream=self.capture_stream):
                body()
        finally:
            self.engine.kv_stable = False
        torch.cuda.synchronize()
        return g

    def step(self, row: torch.Tensor | None, pos: int, audio2: bool = False):
        """Replay one decode step (fast.py:308-325); outputs alias static buffers."""
        if self.graphs is None:
            raise RuntimeError("call capture() first")
        if row is not None:
            src = row if row.dim() == 2 else row[0]
            if src.data_ptr() != self.ids_row.data_ptr():
                self.ids_row.copy_(src)
        self.pos_dev.fill_(pos)
        self.graphs[1 if audio2 else 0].replay()
        return self.lt_static, self.la_static, self.h_final, self.two_static


# ------------------------------------------------------------ generate_fast
_WD_LOW_ENERGY_CH0 = fsm.WD_LOW_ENERGY_CH0
_WD_SEGMENT_FLOOR = fsm.WD_SEGMENT_FLOOR
_WD_SEGMENT_BACKSTOP_RUN = fsm.WD_SEGMENT_BACKSTOP_RUN


@dataclass
class GenResultWatchdog(GenResult):
    """GenResult + watchdog metadata (fast.py:334-340)."""

    watchdog_triggered: bool = False
    watchdog_reason: str = ""
    watchdog_stats: dict = field(default_factory=dict)


def _seen_bits(audio_cols: torch.Tensor, device) -> torch.Tensor:
    """Repetition-penalty histories of the prompt as int32 bit sets [2, 33]:
    set 0 = channel 0 ids (generation_ids[:, :, 1]), set 1 = channels 1..31
    (generation_ids[:, :, 2:]), ids outside [0, 1025) ignored."""
    words = (AUDIO_VOCAB + 31) // 32
    bits = torch.zeros(2, words * 32, dtype=torch.bool)
    for si, ids in enumerate((audio_cols[:, 0], audio_cols[:, 1:])):
        ids = torch.unique(ids.reshape(-1).cpu())
        bits[si, ids[(ids >= 0) & (ids < AUDIO_VOCAB)]] = True
    w = (bits.view(2, words, 32).to(torch.int64) << torch.arange(32)).sum(-1)
    return w.to(torch.int32).to(device)


class _DeviceOps:
    """The device side of one generate_fast call for fsm.drive: step launches
    (input-row feed, head graph, decisions into a two-slot ring) and the
    read-back of a step's decision slot (one pinned 264-byte copy)."""

    def __init__(self, fast: FastMossTTS, input_ids: torch.Tensor, sampling: dict, seen: torch.Tensor | None,
                 stats: dict | None):
        dev = fast.m.device
        self.fast = fast
        self.input_ids = input_ids
        self.sp = sampling
        self.seen = seen
        self.stats = stats
        self.dec = torch.zeros(2, N_VQ + 1, dtype=torch.long, device=dev)
        self.host = torch.zeros(2, N_VQ + 1, dtype=torch.long, pin_memory=True)
        self.ev = [torch.cuda.Event(), torch.cuda.Event()]
        self.amax = kernels.argmax_scratch(dev)
        self.times: dict = {}
        self.launches = 0

    def _event(self):
        if self.stats is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def launch(self, t: int, plan: fsm.StepPlan, prev: fsm.StepPlan | None, pos: int) -> None:
        from .sampling import sample_rows
        fast, sp = self.fast, self.sp
        self.launches += 1
        e0 = self._event()
        if t == 0:
            hs = fast.prefill(self.input_ids)
            fast.capture()
            _heads_from_hidden(fast, hs.last_hidden[0, -1:], audio2=plan.audio2)
        else:
            kernels.feed_row(self.dec[(t - 1) & 1], fast.ids_row, fast.pos_dev, pos, text_mode=prev.text_mode,
                             text_const=prev.text_const, gen_slot=AUDIO_GEN_SLOT_TOKEN_ID,
                             delay_slot=AUDIO_DELAY_SLOT_TOKEN_ID, audio_mask=prev.smask,
                             audio_compact=prev.sample_audio, pad_code=AUDIO_PAD_CODE, seen_bits=self.seen)
            fast.graphs[1 if plan.audio2 else 0].replay()
        if self.stats is not None:
            self.times[t] = (e0, self._event())
        out = self.dec[t & 1]
        if plan.greedy_audio:
            kernels.argmax_rows(fast.la_static, out[1:])
        if plan.greedy_text:
            kernels.argmax_masked(fast.two_static if plan.text_two else fast.lt_static, out[0:1], plan.excluded,
                                  scratch=self.amax)
        if plan.sample_text:
            sample_rows.text(fast, plan.is_audio, t, sp["text_temperature"], sp["text_top_k"], sp["text_top_p"],
                             sp["seed"], 2 * plan.offset, out[0:1])
        if plan.sample_audio:
            sample_rows.audio(fast, plan.smask_list, sp["audio_temperature"], sp["audio_top_k"], sp["audio_top_p"],
                              sp["audio_repetition_penalty"], self.seen, sp["seed"], 2 * plan.offset + 1, out[1:])
        self.host[t & 1].copy_(out, non_blocking=True)
        self.ev[t & 1].record()

    def fetch(self, t: int) -> list:
        self.ev[t & 1].synchronize()
        return self.host[t & 1].tolist()


@torch.inference_mode()
def generate_fast(
    fast: FastMossTTS,
    prompt: dict,
    max_new_tokens=4096,
    seed=1234,
    greedy=False,
    text_temperature=1.5,
    text_top_p=1.0,
    text_top_k=50,
    audio_temperature=1.7,
    audio_top_p=0.8,
    audio_top_k=25,
    audio_repetition_penalty=1.0,
    stats: dict | None = None,
    watchdog: bool = True,
    watchdog_silence_frames: int | None = None,
    watchdog_max_segment_frames: int | None = None,
    max_requested_pause_s: float | None = None,
    pipelined: bool = True,
) -> GenResult:
    """Delay-pattern generation on FastMossTTS with the control flow of the
    reference's generate_fast (fast.py:342-610): same text decision, per-
    channel audio mask, watchdog and stopping rules (moss_tts_lite_b200.fsm).
    Greedy decisions are first-index argmaxes computed on the device; sampled
    decisions use the fused sampling kernel (moss_tts_lite_b200.sampling).
    The next input row is built on the device from the decisions, and with
    ``pipelined`` (the default) step t+1 is enqueued before the host reads
    step t back, so the GPU does not wait for the host between steps.  With
    a stop or the step budget reached, that one speculated step may still run
    after the call returns (it only writes the static buffers and the cache
    row past the generated sequence)."""
    model = fast.m
    device = model.device
    input_ids = prompt["input_ids"].to(device=device, dtype=torch.long)
    attention_mask = prompt.get("attention_mask")
    if input_ids.dim() != 3 or input_ids.shape[0] != 1 or input_ids.shape[-1] != N_VQ + 1:
        raise ValueError(f"expected prompt input_ids [1, L, {N_VQ + 1}], got {tuple(input_ids.shape)}")
    if attention_mask is not None:
        am = attention_mask.to(device)
        if am.dim() == 1:
            am = am.unsqueeze(0)
        if tuple(am.shape) != (1, input_ids.shape[1]):
            raise ValueError(f"bad attention_mask shape {tuple(am.shape)}")
        if not bool(am.all()):
            raise NotImplementedError("batch=1 generate_fast() requires an all-True prompt mask")
    if int(input_ids.shape[1]) + max_new_tokens > model.max_seq_len:
        raise ValueError(f"prompt {int(input_ids.shape[1])} + max_new_tokens {max_new_tokens} "
                         f"exceeds KV cache {model.max_seq_len}")
    seq_len = int(input_ids.shape[1])
    if greedy:
        text_temperature = 0
        audio_temperature = 0
    text_do_sample = text_temperature > 0
    if not text_do_sample:
        text_temperature = 1
    audio_do_sample = audio_temperature > 0
    if not audio_do_sample:
        audio_temperature = 1
    if text_do_sample:
        from .sampling import check_top_k
        check_top_k(text_top_k, model.text_vocab, "generate_fast text decisions")
    if audio_do_sample:
        from .sampling import check_top_k
        check_top_k(audio_top_k, AUDIO_VOCAB, "generate_fast audio decisions")
    cfg = fsm.GenConfig.make(text_do_sample, audio_do_sample, watchdog, watchdog_silence_frames,
                             watchdog_max_segment_frames, max_requested_pause_s)
    st = fsm.FsmState.from_prompt(input_ids[0, :, 0].tolist())
    seen = None
    if audio_do_sample and audio_repetition_penalty != 1.0:
        seen = _seen_bits(input_ids[0, :, 1:], device)
    sampling = dict(seed=seed, text_temperature=text_temperature, text_top_k=text_top_k, text_top_p=text_top_p,
                    audio_temperature=audio_temperature, audio_top_k=audio_top_k, audio_top_p=audio_top_p,
                    audio_repetition_penalty=audio_repetition_penalty)
    ops = _DeviceOps(fast, input_ids, sampling, seen, stats)

    def on_step(t, plan):
        if stats is None:
            return
        if t > 0:
            stats.setdefault("audio_phase", []).append(bool(plan.audio2))
        stats.setdefault("step_wall_s", []).append(time.perf_counter())

    r = fsm.drive(ops, st, cfg, max_new_tokens, seq_len, pipelined=pipelined, on_step=on_step)
    st = r.state
    text_ids = (torch.tensor(r.text_steps, dtype=torch.long) if r.text_steps
                else torch.empty(0, dtype=torch.long))
    audio_frames = (torch.tensor(r.audio_steps, dtype=torch.long) if r.audio_steps
                    else torch.empty(0, N_VQ, dtype=torch.long))
    if stats is not None:
        torch.cuda.synchronize()
        p = ops.times.get(0)
        stats["prefill_ms"] = float(p[0].elapsed_time(p[1])) if p else None
        stats["step_ms"] = [float(a.elapsed_time(b)) for t, (a, b) in sorted(ops.times.items())
                            if 0 < t < r.n_steps]
        stats["steps"] = len(stats["step_ms"])
        stats["launches"] = ops.launches
        stats["relaunches"] = r.relaunches
    return GenResultWatchdog(text_ids=text_ids, audio_frames=audio_frames,
                             finished=bool(st.is_stopping) or bool(st.wd_stats), n_steps=r.n_steps,
                             watchdog_triggered=bool(st.wd_stats), watchdog_reason=st.wd_reason,
                             watchdog_stats=st.wd_stats)


def _heads_from_hidden(fast: FastMossTTS, hv: torch.Tensor, audio2: bool) -> None:
    """Time step 0 of generate_fast: logits of the final-normed last prompt
    row (the reference calls model.text_logits / text_logits_2way /
    audio_logits on it, fast.py:483-524)."""
    m = fast.m
    H = m.hidden_size
    if audio2:
        kernels.bf16_linear(hv, m.head_2way, fast.two_static.view(1, 2))
    else:
        kernels.bf16_linear(hv, m.head_text, fast.lt_static.view(1, -1))
    kernels.bf16_linear(hv, m.head_audio.view(N_VQ * AUDIO_VOCAB, H), fast.la_static.view(1, -1),
                        pad_period=AUDIO_VOCAB, pad_col=AUDIO_PAD_CODE)
