"""MOSS-TTS backbone container and eager decode on the B200 kernels.

Interface-compatible with ``moss_tts_lite.model`` (model.py:10-295): the
special-token constants, ``HiddenState`` and a ``MossTTSModel`` that takes a
checkpoint dict under the reference's key names and exposes its tensors under
the reference's attribute names (``embed_tokens``, ``layers[i]["q"]``,
``emb_ext``, ``head_audio``, ``k_cache`` ...), so ``FastMossTTS`` accepts
either this class or the reference's.  ``prefill`` / ``step`` /
``text_logits`` / ``text_logits_2way`` / ``audio_logits`` keep their
signatures; the arithmetic runs on this package's sm_100a kernels (bf16
weights).

The container itself is table-driven: ``_LAYER_TENSORS`` maps every per-layer
slot to its checkpoint key, ``ModelDims`` derives the architecture from the
tensor shapes once, and every tensor is placed on the device by one helper.
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

# per-layer slot -> checkpoint key suffix under "language_model.layers.<i>."
_LAYER_TENSORS = {
    "input_layernorm": "input_layernorm.weight",
    "q": "self_attn.q_proj.weight",
    "k": "self_attn.k_proj.weight",
    "v": "self_attn.v_proj.weight",
    "o": "self_attn.o_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "post_attention_layernorm": "post_attention_layernorm.weight",
    "gate": "mlp.gate_proj.weight",
    "up": "mlp.up_proj.weight",
    "down": "mlp.down_proj.weight",
}
_LAYER_PREFIX = "language_model.layers."
_EMBED_KEY = "language_model.embed_tokens.weight"
_FINAL_NORM_KEY = "language_model.norm.weight"
_TEXT_HEAD_KEY = "lm_heads.0.weight"


def _audio_emb_key(c: int) -> str:
    return f"emb_ext.{c}.weight"


def _audio_head_key(c: int) -> str:
    return f"lm_heads.{c + 1}.weight"


@dataclass
class HiddenState:
    """Backbone output (final-normed hidden states)."""

    last_hidden: torch.Tensor


@dataclass(frozen=True)
class ModelDims:
    """Architecture read off the checkpoint's tensor shapes."""

    n_layers: int
    hidden_size: int
    text_vocab: int
    head_dim: int
    n_heads: int
    n_kv_heads: int

    @staticmethod
    def infer(weights: dict) -> "ModelDims":
        ids = set()
        for key in weights:
            if key.startswith(_LAYER_PREFIX):
                ids.add(int(key[len(_LAYER_PREFIX):].split(".", 1)[0]))
        n = len(ids)
        if sorted(ids) != list(range(n)):
            raise ValueError(f"layer indices must run 0..n-1 without gaps, found {sorted(ids)}")
        vocab, hidden = (int(d) for d in weights[_EMBED_KEY].shape)
        l0 = _LAYER_PREFIX + "0."
        hd = int(weights[l0 + _LAYER_TENSORS["q_norm"]].shape[0])
        nh = int(weights[l0 + _LAYER_TENSORS["q"]].shape[0]) // hd
        nkv = int(weights[l0 + _LAYER_TENSORS["k"]].shape[0]) // hd
        if nkv <= 0 or nh % nkv:
            raise ValueError(f"{nh} query heads cannot be grouped over {nkv} key/value heads")
        return ModelDims(n, hidden, vocab, hd, nh, nkv)


def rope_tables(n: int, dev, dtype, head_dim: int) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE cos/sin for ``n`` positions.  The values must equal the
    reference's bit for bit (model.py:115-124), so the fp32 chain is the
    same: inverse frequencies theta^(-2i/d), outer product with the position,
    the half repeated, cos/sin in fp32, then the cast.  Set-up only."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32, device=dev) / head_dim
    inv_freq = 1.0 / (ROPE_THETA ** exponents)
    angles = torch.outer(torch.arange(n, device=dev, dtype=torch.float32), inv_freq)
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().to(dtype), angles.sin().to(dtype)


class MossTTSModel:
    """MossTTSDelayModel weights + KV cache, decoded by the sm_100a kernels.

    ``weights`` is a checkpoint dict under the reference key names
    (``language_model.*``, ``emb_ext.<c>``, ``lm_heads.<i>``).  Only
    ``dtype=torch.bfloat16`` on a CUDA device is served."""

    def __init__(self, weights: dict, device="cuda", dtype=torch.bfloat16, max_seq_len=8192):
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("moss_tts_lite_b200.MossTTSModel runs on CUDA (sm_100a) only")
        if dtype != torch.bfloat16:
            raise ValueError("moss_tts_lite_b200.MossTTSModel computes in bfloat16 only")
        dims = ModelDims.infer(weights)
        self.dims = dims
        self.device, self.dtype, self.max_seq_len = dev, dtype, int(max_seq_len)
        self.n_layers, self.hidden_size, self.text_vocab = dims.n_layers, dims.hidden_size, dims.text_vocab
        self.head_dim, self.n_heads, self.n_kv_heads = dims.head_dim, dims.n_heads, dims.n_kv_heads
        self.n_rep = dims.n_heads // dims.n_kv_heads

        place = self._placer(weights)
        self.embed_tokens = place(_EMBED_KEY)
        self.final_norm = place(_FINAL_NORM_KEY)
        self.layers = [{slot: place(f"{_LAYER_PREFIX}{li}.{key}") for slot, key in _LAYER_TENSORS.items()}
                       for li in range(dims.n_layers)]
        # the 32 audio embedding tables and heads each live in one stacked
        # buffer (the kernels index them as [32 * 1025, H]); emb_ext are views
        self.emb_audio = torch.stack([place(_audio_emb_key(c)) for c in range(N_VQ)]).contiguous()
        self.emb_ext = list(self.emb_audio.unbind(0))
        self.head_text = place(_TEXT_HEAD_KEY)
        self.head_audio = torch.stack([place(_audio_head_key(c)) for c in range(N_VQ)]).contiguous()
        self.head_2way = self.head_text[[AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID]].contiguous()
        self.rope_cos, self.rope_sin = rope_tables(self.max_seq_len, dev, dtype, dims.head_dim)
        self.k_cache, self.v_cache = self._new_cache(self.max_seq_len)
        self._seq = 0
        self._engine = None

    def _placer(self, weights: dict):
        dev, dtype = self.device, self.dtype

        def place(key: str) -> torch.Tensor:
            if key not in weights:
                raise KeyError(f"checkpoint has no tensor {key!r}")
            return weights[key].to(device=dev, dtype=dtype).contiguous()
        return place

    def _new_cache(self, positions: int):
        shape = (self.n_layers, self.n_kv_heads, positions, self.head_dim)
        k = torch.zeros(shape, dtype=self.dtype, device=self.device)
        return k, torch.zeros_like(k)

    # ---------------------------------------------------------------- state
    def ensure_seq_len(self, n: int) -> int:
        """Make room for ``n`` positions (reference model.py:126-147): a larger
        cache with the live rows carried over, and RoPE tables recomputed for
        the new length (the fp32 chain gives the old rows the same values)."""
        want = int(n)
        if want > self.max_seq_len:
            if self._seq > self.max_seq_len:
                raise RuntimeError(f"cannot grow: {self._seq} live positions do not fit the current "
                                   f"cache of {self.max_seq_len}")
            k, v = self._new_cache(want)
            k[:, :, :self.max_seq_len] = self.k_cache
            v[:, :, :self.max_seq_len] = self.v_cache
            self.k_cache, self.v_cache = k, v
            self.rope_cos, self.rope_sin = rope_tables(want, self.device, self.dtype, self.head_dim)
            self.max_seq_len = want
            self._engine = None
        return self.max_seq_len

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

    def _rows(self, ids: torch.Tensor, start: int) -> torch.Tensor:
        """Validated id rows [L, 33] on the device for positions start.. ."""
        shape = tuple(ids.shape)
        if len(shape) != 3 or shape[0] != 1 or shape[2] != N_VQ + 1:
            raise ValueError(f"input ids must be [1, L, {N_VQ + 1}], got {shape}")
        if start + shape[1] > self.max_seq_len:
            raise ValueError(f"{start + shape[1]} positions do not fit the KV cache of {self.max_seq_len}")
        return ids[0].to(device=self.device, dtype=torch.long)

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor) -> HiddenState:
        """Prompt [1, L, 33] from position 0 -> final-normed hidden [1, L, H]
        (reference model.py:206-219)."""
        self.reset()
        rows = self._rows(input_ids, 0)
        h = self._eng().prefill_rows(rows)
        self._seq = int(rows.shape[0])
        return HiddenState(h.view(1, self._seq, self.hidden_size))

    @torch.inference_mode()
    def step(self, row: torch.Tensor) -> HiddenState:
        """One decode step at the current position (reference model.py:221-233);
        ``row`` is [1, 1, 33] or [1, 33]."""
        rows = self._rows(row.view(1, -1, row.shape[-1]) if row.dim() == 2 else row, self._seq)
        if rows.shape[0] != 1:
            raise ValueError(f"step takes one row, got {rows.shape[0]}")
        h = self._eng().decode_row(rows[0], self._seq)
        self._seq += 1
        return HiddenState(h.view(1, 1, self.hidden_size))

    # ---------------------------------------------------------------- heads
    def _head_input(self, h) -> tuple[torch.Tensor, bool]:
        """Hidden states as rows [R, H], and whether they denote one position
        (the result then drops its row dimension).  Accepted: [1, L, H],
        [1, H] and [H] (reference model.py:240-295)."""
        t = h.last_hidden if isinstance(h, HiddenState) else h
        if t.dim() == 3 and t.shape[0] != 1:
            raise ValueError("batch must be 1")
        if t.dim() == 2 and t.shape[0] != 1 or t.dim() not in (1, 2, 3):
            raise ValueError(f"unsupported hidden shape {tuple(t.shape)}")
        rows = t.reshape(-1, t.shape[-1])
        return rows.contiguous(), rows.shape[0] == 1

    def _apply_head(self, h, weight: torch.Tensor, pad: bool) -> tuple[torch.Tensor, bool]:
        from . import kernels
        x, single = self._head_input(h)
        out = torch.empty(x.shape[0], weight.shape[0], dtype=self.dtype, device=self.device)
        for r in range(0, x.shape[0], 4):   # the head GEMV serves up to 4 rows per launch
            kernels.bf16_linear(x[r:r + 4], weight, out[r:r + 4], pad_period=AUDIO_VOCAB if pad else 0,
                                pad_col=AUDIO_PAD_CODE)
        return out, single

    def text_logits(self, h) -> torch.Tensor:
        """Full text head (reference model.py:240-253)."""
        out, single = self._apply_head(h, self.head_text, pad=False)
        return out[0] if single else out

    def text_logits_2way(self, h) -> torch.Tensor:
        """The two audio-phase text logits, GEN slot then DELAY slot (reference model.py:255-268)."""
        out, single = self._apply_head(h, self.head_2way, pad=False)
        return out[0] if single else out

    def audio_logits(self, h) -> torch.Tensor:
        """32 audio heads with column 1024 at -inf (reference model.py:270-295)."""
        out, single = self._apply_head(h, self.head_audio.view(N_VQ * AUDIO_VOCAB, self.hidden_size), pad=True)
        out = out.view(-1, N_VQ, AUDIO_VOCAB)
        return out[0] if single else out
