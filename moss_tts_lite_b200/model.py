"""MOSS-TTS backbone container and eager decode on the B200 kernels.

Mirrors ``moss_tts_lite.model`` (constants, ``HiddenState`` and
``MossTTSModel``, model.py:10-295): same constructor, same tensors under the
same attribute names (so ``FastMossTTS`` accepts either this class or the
reference's), same ``prefill / step / text_logits / text_logits_2way /
audio_logits`` signatures and errors.  The difference is where the math runs:
``step`` and ``prefill`` drive this package's sm_100a kernels (bf16 weights)
instead of torch ops.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

N_VQ = 32
AUDIO_VOCAB = 1025
AUDIO_PAD_CODE = 1024
TEXT_VOCAB = 155648

PAD_TOKEN_ID = 151643
IM_START_TOKEN_ID = 151644
IM_END_TOKEN_ID = 151645
AUDIO_START_TOKEN_ID = 151652
AUDIO_END_TOKEN_ID = 151653
AUDIO_USER_SLOT_TOKEN_ID = 151654
AUDIO_GEN_SLOT_TOKEN_ID = 151656
AUDIO_DELAY_SLOT_TOKEN_ID = 151662

ROPE_THETA = 1_000_000.0
RMS_EPS = 1e-6

LIN_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass
class HiddenState:
    """Backbone output (final-normed hidden states)."""

    last_hidden: torch.Tensor


def rope_tables(n: int, dev, dtype, head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE cos/sin for ``n`` positions: the fp32 chain of model.py:115-124
    (theta 1e6), cast to ``dtype``.  Set-up only."""
    inv = 1.0 / (ROPE_THETA ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=dev) / head_dim))
    pos = torch.arange(n, device=dev, dtype=torch.float32)
    freqs = torch.outer(pos, inv)
    emb2 = torch.cat((freqs, freqs), dim=-1)
    return emb2.cos().to(dtype), emb2.sin().to(dtype)


class MossTTSModel:
    """MossTTSDelayModel weights + KV cache, decoded by the sm_100a kernels.

    ``weights`` uses the checkpoint key names of model.py:55-105.  Only
    ``dtype=torch.bfloat16`` on a CUDA device is served (the kernels are
    bf16 / sm_100a only)."""

    def __init__(self, weights: dict, device="cuda", dtype=torch.bfloat16, max_seq_len=8192):
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("moss_tts_lite_b200.MossTTSModel runs on CUDA (sm_100a) only")
        if dtype != torch.bfloat16:
            raise ValueError("moss_tts_lite_b200.MossTTSModel computes in bfloat16 only")
        self.device = dev
        self.dtype = dtype
        self.max_seq_len = max_seq_len
        layer_ids = sorted({int(k.split(".")[2]) for k in weights if k.startswith("language_model.layers.")})
        self.n_layers = len(layer_ids)
        if layer_ids != list(range(self.n_layers)):
            raise ValueError(f"unexpected layer ids {layer_ids}")
        emb = weights["language_model.embed_tokens.weight"]
        self.hidden_size = int(emb.shape[1])
        self.text_vocab = int(emb.shape[0])
        self.head_dim = int(weights["language_model.layers.0.self_attn.q_norm.weight"].shape[0])
        self.n_heads = int(weights["language_model.layers.0.self_attn.q_proj.weight"].shape[0]) // self.head_dim
        self.n_kv_heads = int(weights["language_model.layers.0.self_attn.k_proj.weight"].shape[0]) // self.head_dim
        if self.n_heads % self.n_kv_heads != 0:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        self.n_rep = self.n_heads // self.n_kv_heads

        def T(name: str) -> torch.Tensor:
            t = weights[name]
            if t.device != dev or t.dtype != dtype:
                t = t.to(device=dev, dtype=dtype)
            return t.contiguous()

        self.embed_tokens = T("language_model.embed_tokens.weight")
        self.final_norm = T("language_model.norm.weight")
        self.layers = []
        for i in layer_ids:
            p = f"language_model.layers.{i}"
            self.layers.append({
                "input_layernorm": T(f"{p}.input_layernorm.weight"),
                "q": T(f"{p}.self_attn.q_proj.weight"),
                "k": T(f"{p}.self_attn.k_proj.weight"),
                "v": T(f"{p}.self_attn.v_proj.weight"),
                "o": T(f"{p}.self_attn.o_proj.weight"),
                "q_norm": T(f"{p}.self_attn.q_norm.weight"),
                "k_norm": T(f"{p}.self_attn.k_norm.weight"),
                "post_attention_layernorm": T(f"{p}.post_attention_layernorm.weight"),
                "gate": T(f"{p}.mlp.gate_proj.weight"),
                "up": T(f"{p}.mlp.up_proj.weight"),
                "down": T(f"{p}.mlp.down_proj.weight"),
            })
        # The 32 audio embedding tables live in one buffer (the embedding
        # kernel indexes it as [32 * 1025, H]); emb_ext are views into it.
        self.emb_audio = torch.stack([T(f"emb_ext.{i}.weight") for i in range(N_VQ)], 0).contiguous()
        self.emb_ext = [self.emb_audio[i] for i in range(N_VQ)]
        self.head_text = T("lm_heads.0.weight")
        self.head_audio = torch.stack([weights[f"lm_heads.{i + 1}.weight"] for i in range(N_VQ)], dim=0) \
            .to(device=dev, dtype=dtype).contiguous()
        self.head_2way = self.head_text[[AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID]].contiguous()
        self.rope_cos, self.rope_sin = rope_tables(max_seq_len, dev, dtype, self.head_dim)
        self.k_cache = torch.zeros(self.n_layers, self.n_kv_heads, max_seq_len, self.head_dim,
                                   dtype=dtype, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self._seq = 0
        self._engine = None

    # ---------------------------------------------------------------- state
    def ensure_seq_len(self, n: int) -> int:
        """Grow the KV cache + rope tables so ``n`` positions fit (model.py:126-147)."""
        n = int(n)
        if n <= self.max_seq_len:
            return self.max_seq_len
        if self._seq > self.max_seq_len:
            raise RuntimeError(f"live sequence {self._seq} exceeds cache {self.max_seq_len}; cannot grow")
        old = self.max_seq_len
        ck = torch.zeros(self.n_layers, self.n_kv_heads, n, self.head_dim, dtype=self.dtype, device=self.device)
        cv = torch.zeros_like(ck)
        ck[:, :, :old].copy_(self.k_cache)
        cv[:, :, :old].copy_(self.v_cache)
        cos, sin = rope_tables(n, self.device, self.dtype, self.head_dim)
        cos[:old].copy_(self.rope_cos)
        sin[:old].copy_(self.rope_sin)
        self.k_cache, self.v_cache = ck, cv
        self.rope_cos, self.rope_sin = cos, sin
        self.max_seq_len = n
        self._engine = None
        return n

    @property
    def seq_len(self) -> int:
        return self._seq

    def reset(self) -> None:
        self._seq = 0

    # --------------------------------------------------------------- decode
    def _eng(self):
        if self._engine is None:
            from .fast import _StepEngine, bf16_linears
            self._engine = _StepEngine(self, bf16_linears(self))
        return self._engine

    def _check_ids(self, ids: torch.Tensor, t: int) -> torch.Tensor:
        if ids.shape[0] != 1 or ids.shape[-1] != N_VQ + 1 or ids.shape[1] != t:
            raise ValueError(f"expected input ids [1, {t}, {N_VQ + 1}], got {tuple(ids.shape)}")
        if self._seq + t > self.max_seq_len:
            raise ValueError(f"seq len {self._seq + t} exceeds KV cache {self.max_seq_len}")
        return ids.to(device=self.device, dtype=torch.long)

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor) -> HiddenState:
        """input_ids [1, L, 33] -> final-normed hidden [1, L, H] (model.py:206-219)."""
        if input_ids.dim() != 3 or input_ids.shape[0] != 1 or input_ids.shape[-1] != N_VQ + 1:
            raise ValueError(f"expected input ids [1, L, {N_VQ + 1}], got {tuple(input_ids.shape)}")
        t = int(input_ids.shape[1])
        self.reset()
        ids = self._check_ids(input_ids, t)
        h = self._eng().prefill_rows(ids[0])
        self._seq = t
        return HiddenState(h.view(1, t, self.hidden_size))

    @torch.inference_mode()
    def step(self, row: torch.Tensor) -> HiddenState:
        """One decode step (model.py:221-233): row [1, 1, 33] or [1, 33]."""
        if row.dim() == 2:
            row = row.unsqueeze(0)
        ids = self._check_ids(row, 1)
        h = self._eng().decode_row(ids[0, 0], self._seq)
        self._seq += 1
        return HiddenState(h.view(1, 1, self.hidden_size))

    # ---------------------------------------------------------------- heads
    def _as_vec(self, h) -> torch.Tensor:
        if isinstance(h, HiddenState):
            h = h.last_hidden
        if h.dim() == 3:
            if h.shape[0] != 1:
                raise ValueError("batch must be 1")
            return h[0]
        if h.dim() == 2 and h.shape[0] == 1:
            return h
        if h.dim() == 1:
            return h.view(1, -1)
        raise ValueError(f"unsupported hidden shape {tuple(h.shape)}")

    def _head(self, h, W: torch.Tensor, pad: bool = False) -> torch.Tensor:
        from . import kernels
        x = self._as_vec(h).contiguous()
        rows = x.shape[0]
        out = torch.empty(rows, W.shape[0], dtype=self.dtype, device=self.device)
        for r0 in range(0, rows, 4):
            r1 = min(rows, r0 + 4)
            kernels.bf16_linear(x[r0:r1], W, out[r0:r1], pad_period=AUDIO_VOCAB if pad else 0,
                                pad_col=AUDIO_PAD_CODE)
        return out

    def text_logits(self, h) -> torch.Tensor:
        """Full text head (model.py:240-253)."""
        out = self._head(h, self.head_text)
        return out[0] if out.shape[0] == 1 else out

    def text_logits_2way(self, h) -> torch.Tensor:
        """The two audio-phase text logits (model.py:255-268)."""
        out = self._head(h, self.head_2way)
        return out[0] if out.shape[0] == 1 else out

    def audio_logits(self, h) -> torch.Tensor:
        """32 audio heads, column 1024 = -inf (model.py:270-295)."""
        out = self._head(h, self.head_audio.view(N_VQ * AUDIO_VOCAB, self.hidden_size), pad=True)
        out = out.view(-1, N_VQ, AUDIO_VOCAB)
        return out[0] if out.shape[0] == 1 else out
