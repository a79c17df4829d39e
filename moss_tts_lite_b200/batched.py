"""Batched multi-stream decode: B independent utterances advanced together.

The reference decodes one utterance at a time (batch 1, moss_tts_lite/
fast.py:272-325); its throughput configuration runs streams one after the
other.  Here one decode step advances all B streams:

* every W4 projection reads its weights once for the B rows.  By default
  (up to 16 streams, the batch-1 engine running the persistent chain) each
  layer's o -> gate|up -> down -> next q|k|v is one persistent launch over
  the batch-1 engine's strip weights, the B rows as the N dimension of the
  MMAs (``mtl_w4_chain_rows``); with ``tc=True`` one launch per linear in
  tensor-core tiles (tcgen05, B rows as N, up to 16 rows per launch); with
  ``tc=False, chain=False`` one launch per linear in the register-MMA tiles
  of the batch-1 engine (launches of up to 8 rows, the mma.sync N dimension);
* attention runs the B streams in one launch, each over its own KV cache
  (``mtl_attn_decode`` with ``streams = B`` and a per-stream cache stride);
* the final norm, the two-way text head and the 32 audio heads run on the
  B rows, and the greedy audio-phase decision (first-index argmax, GEN/DELAY
  from the two-way logits) writes each stream's next row and position on the
  device, so a captured step graph replays with no host round trip.

Each stream's prompt is prefilled into its own cache slice with the
prefill of the batch-1 engine.  With ``tc=False, chain=False`` (and a batch-1
engine without the chain) stream s's results equal a
batch-1 decode of the same stream bit for bit (same kernels, same split-K
plan) while the caches hold up to 256 positions (one attention split per
head either way; past that the batched step splits each head's cache into
fewer slices than the batch-1 step, which changes the fp32 merge order);
with the tensor-core tiles they agree to within the two W4 kernels' fp32
summation orders.
"""
from __future__ import annotations

import torch

from . import _lib, kernels
from .model import AUDIO_DELAY_SLOT_TOKEN_ID, AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_PAD_CODE, AUDIO_VOCAB, N_VQ, RMS_EPS

_HEAD_ROWS = 4  # rows per bf16 head launch where they must equal one-row launches bit for bit
_HEAD_ROWS_TC = 16  # rows per launch otherwise (mtl_bf16_linear: 5..16 rows on the tensor-core kernel)


class BatchedFastMossTTS:
    """``streams`` decode streams over the weights of a FastMossTTS (shared)."""

    def __init__(self, fast, streams: int, max_seq: int | None = None, tc: bool | None = None,
                 chain: bool | None = None):
        m = fast.m
        if streams < 1:
            raise ValueError("streams must be >= 1")
        self.fast = fast
        self.m = m
        self.B = streams
        self.max_seq = int(max_seq or m.max_seq_len)
        if self.max_seq > m.max_seq_len:
            raise ValueError(f"max_seq {self.max_seq} exceeds the model's RoPE table {m.max_seq_len}")
        dev, bf = m.device, torch.bfloat16
        H, D = m.hidden_size, m.head_dim
        eng = fast.engine
        self.lins = eng.lins
        # the persistent chain over the batch-1 engine's strip weights (the
        # default when they exist, up to 16 streams, tc not asked for), else
        # per-linear launches: tensor-core tiles or register-MMA tiles
        if chain is None:
            chain = not tc and eng.strips is not None and streams <= 16
        self.chain = bool(chain) and eng.strips is not None and streams <= 16
        if chain and not self.chain:
            raise ValueError("the chain needs the batch-1 engine's strip weights (FastMossTTS(chain=True)) and "
                             "at most 16 streams")
        if tc is None:
            tc = streams >= 2 and not self.chain
        self.tc = bool(tc) and not self.chain and self._tc_capable(eng.lins)
        if self.tc:
            self.lins = self._tc_lins(eng.lins)
        if self.chain:
            self.chain_bar = torch.zeros(m.n_layers + 1, 32, dtype=torch.int32, device=m.device)
        self.emb_audio = eng.emb_audio
        self.head_audio2d = eng.head_audio2d
        B = streams
        # caches: [layer][stream] slices of one allocation per layer
        self.k_cache = torch.zeros(m.n_layers, B, m.n_kv_heads, self.max_seq, D, dtype=bf, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.ids = torch.zeros(B, N_VQ + 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(B, dtype=torch.long, device=dev)
        nq = m.n_heads * D
        self.h = torch.zeros(B, H, dtype=bf, device=dev)
        self.qkv = torch.zeros(B, nq + 2 * m.n_kv_heads * D, dtype=bf, device=dev)
        self.attn = torch.zeros(B, nq, dtype=bf, device=dev)
        self.act = torch.zeros(B, self.lins[0]["gu"].N // 2, dtype=bf, device=dev)
        self.h_final = torch.zeros(B, H, dtype=bf, device=dev)
        self.two = torch.zeros(B, 2, dtype=bf, device=dev)
        self.la = torch.zeros(B, N_VQ, AUDIO_VOCAB, dtype=bf, device=dev)
        # KV splits per (stream, head): about one CTA per SM over all streams
        # (16 streams x 8 KV heads: one split, each CTA streams its whole
        # cache slice; the batch-1 engine's 16 splits would launch 2048
        # short CTAs, one per SM at a time)
        self.splits = max(1, min(eng.splits, int(148 / (m.n_kv_heads * streams) + 0.5)))
        from . import _lib
        self.attn_scratch = torch.zeros(_lib.attn_scratch_bytes(B, m.n_heads, m.n_kv_heads, self.splits),
                                        dtype=torch.uint8, device=dev)
        self.kv_stable = False
        self.graph = None
        self.seq = [0] * B

    @staticmethod
    def _tc_capable(lins) -> bool:
        from .fast import _W4Lin
        from .quant import W4Weight
        return all(isinstance(L[n], _W4Lin) and L[n].w.fmt == _lib.MTL_FMT_REF and L[n].w.k_perm is None
                   and W4Weight.tc_supported(L[n].w.K, L[n].w.N, L[n].w.group_size)
                   for L in lins for n in ("qkv", "o", "gu", "down"))

    @staticmethod
    def _tc_lins(lins) -> list:
        """The layers' W4 weights re-packed into tensor-core tiles (same codes
        and (scale, zero); gate|up interleaved row by row)."""
        from .fast import _W4Lin
        out = []
        for L in lins:
            out.append({"qkv": _W4Lin(L["qkv"].w.to_tc()), "o": _W4Lin(L["o"].w.to_tc()),
                        "gu": _W4Lin(L["gu"].w.to_tc(swiglu_block=L["gu"].fuse_block), fuse_block=1),
                        "down": _W4Lin(L["down"].w.to_tc())})
        return out

    # ---------------------------------------------------------------- prefill
    def prefill(self, s: int, ids: torch.Tensor) -> torch.Tensor:
        """Prompt rows [L, 33] of stream ``s`` into its cache; returns the
        final-normed hidden [L, H] (the batch-1 chunked prefill)."""
        if not 0 <= s < self.B:
            raise IndexError(f"stream {s} of {self.B}")
        ids = ids.reshape(-1, N_VQ + 1).to(device=self.m.device, dtype=torch.long)
        L = int(ids.shape[0])
        if L >= self.max_seq:
            raise ValueError(f"prompt of {L} rows leaves no room in a cache of {self.max_seq}")
        k = [self.k_cache[li, s] for li in range(self.m.n_layers)]
        v = [self.v_cache[li, s] for li in range(self.m.n_layers)]
        out = self.fast.engine.prefill_rows(ids, caches=(k, v))
        self.seq[s] = L
        return out

    def prefill_all(self, prompts: list) -> torch.Tensor:
        """Every stream's prompt (rows [L, 33] each, stream s = prompts[s]) in
        one pass: with equal lengths of at least 32 rows the projections run
        as tcgen05 W4 GEMMs over all streams' rows at once (M = streams x L)
        and one attention launch covers every stream's cache; otherwise
        stream by stream.  Returns the final-normed hidden [streams * L, H]
        (or the per-stream results concatenated)."""
        if len(prompts) != self.B:
            raise ValueError(f"{len(prompts)} prompts for {self.B} streams")
        rows = [p.reshape(-1, N_VQ + 1).to(device=self.m.device, dtype=torch.long) for p in prompts]
        L = int(rows[0].shape[0])
        eng = self.fast.engine
        if all(int(r.shape[0]) == L for r in rows) and eng.gemm_prefill_ok(L) and L < self.max_seq:
            out = eng._prefill_gemm(torch.cat(rows, 0), [self.k_cache[li] for li in range(self.m.n_layers)],
                                    [self.v_cache[li] for li in range(self.m.n_layers)], streams=self.B)
            self.seq = [L] * self.B
            return out
        return torch.cat([self.prefill(s, r) for s, r in enumerate(rows)], 0)

    def start(self, s: int, row: torch.Tensor, pos: int) -> None:
        """Set stream ``s``'s next input row [33] and its cache position."""
        self.ids[s].copy_(row.reshape(-1))
        self.pos[s].fill_(pos)

    # ------------------------------------------------------------------- step
    def _phase(self, li: int, name: str) -> dict:
        lyr, S = self.m.layers[li], self.fast.engine.strips[li]
        if name == "qkv":
            return {"w": S["qkv"], "x": self.h, "y": self.qkv, "norm_w": lyr["input_layernorm"]}
        if name == "o":
            return {"w": S["o"], "x": self.attn, "y": self.h, "residual": self.h}
        if name == "gu":
            return {"w": S["gu"], "x": self.h, "y": self.act, "norm_w": lyr["post_attention_layernorm"],
                    "swiglu": True}
        return {"w": S["down"], "x": self.act, "y": self.h, "residual": self.h}

    def _attn(self, li: int) -> None:
        m, B = self.m, self.B
        lyr = m.layers[li]
        stride = m.n_kv_heads * self.max_seq * m.head_dim
        kernels.attn_decode(self.qkv, lyr["q_norm"], lyr["k_norm"], m.rope_cos, m.rope_sin,
                            self.k_cache[li], self.v_cache[li], self.pos, m.n_heads, m.n_kv_heads,
                            self.splits, self.attn, self.attn_scratch, streams=B, cache_stream_stride=stride,
                            kv_stable=self.kv_stable)

    def _step(self) -> None:
        m, B = self.m, self.B
        kernels.embed_sum(self.ids, m.embed_tokens, self.emb_audio, self.h)
        stride = m.n_kv_heads * self.max_seq * m.head_dim
        if self.chain:
            g, bar, n = self.fast.engine.chain_g, self.chain_bar, m.n_layers
            kernels.w4_chain_rows([self._phase(0, "qkv")], g, bar[0], RMS_EPS)
            for li in range(n):
                self._attn(li)
                phases = [self._phase(li, nm) for nm in ("o", "gu", "down")]
                if li + 1 < n:
                    phases.append(self._phase(li + 1, "qkv"))
                kernels.w4_chain_rows(phases, g, bar[li + 1], RMS_EPS)
            self._heads()
            return
        for li in range(m.n_layers):
            lyr, L = m.layers[li], self.lins[li]
            L["qkv"](self.h, self.qkv, norm_weight=lyr["input_layernorm"])
            kernels.attn_decode(self.qkv, lyr["q_norm"], lyr["k_norm"], m.rope_cos, m.rope_sin,
                                self.k_cache[li], self.v_cache[li], self.pos, m.n_heads, m.n_kv_heads,
                                self.splits, self.attn, self.attn_scratch, streams=B, cache_stream_stride=stride,
                                kv_stable=self.kv_stable)
            L["o"](self.attn, self.h, residual=self.h)
            L["gu"](self.h, self.act, norm_weight=lyr["post_attention_layernorm"], swiglu=True)
            L["down"](self.act, self.h, residual=self.h)
        self._heads()

    def _heads(self) -> None:
        m, B = self.m, self.B
        la2 = self.la.view(B, N_VQ * AUDIO_VOCAB)
        rows = _HEAD_ROWS_TC if (self.tc or self.chain) else _HEAD_ROWS
        for r0 in range(0, B, rows):
            r1 = min(B, r0 + rows)
            kernels.bf16_linear(self.h[r0:r1], m.head_2way, self.two[r0:r1], norm_weight=m.final_norm, eps=RMS_EPS,
                                x_normed=self.h_final[r0:r1])
            kernels.bf16_linear(self.h[r0:r1], self.head_audio2d, la2[r0:r1], norm_weight=m.final_norm, eps=RMS_EPS,
                                pad_period=AUDIO_VOCAB, pad_col=AUDIO_PAD_CODE)
        kernels.greedy_feed(self.la, self.two, self.ids, self.pos, AUDIO_GEN_SLOT_TOKEN_ID,
                            AUDIO_DELAY_SLOT_TOKEN_ID, streams=B)

    def step(self) -> None:
        """One greedy audio-phase step of every stream (graph replay once captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step()

    def capture(self) -> None:
        """Capture one batched step as a CUDA graph (warm-up launches first)."""
        if self.graph is not None:
            return
        saved = (self.ids.clone(), self.pos.clone())
        s = torch.cuda.Stream(device=self.m.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        self.kv_stable = True
        try:
            with torch.cuda.graph(g, stream=self.fast.capture_stream):
                self._step()
        finally:
            self.kv_stable = False
        torch.cuda.synchronize()
        # the warm-up and the capture advanced the streams: restore them
        self.ids.copy_(saved[0])
        self.pos.copy_(saved[1])
        self.graph = g
