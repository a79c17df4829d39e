"""One MOSS-TTS decoder step restated in numpy (test infrastructure only).

Restates ``MossTTSModel`` (moss_tts_lite/model.py:46-295) and the W4 variant
that ``FastMossTTS`` runs (moss_tts_lite/fast.py:107-194) op by op, with the
same bf16 rounding points as the reference:

* embedding sum: text row, then 32 audio rows added one at a time, each add
  rounded to bf16 (model.py:156-161, fast.py:123-128);
* RMSNorm: fp32 mean of squares, ``x * rsqrt(var + eps)`` in fp32, cast to
  bf16, then ``weight * x`` rounded to bf16 (model.py:34-40);
* q/k head norm, then RoPE as ``bf16(bf16(q*cos) + bf16(rotate_half(q)*sin))``
  (model.py:175-182, fast.py:138-144);
* attention with scale 1/sqrt(head_dim) and the rounding points of
  PyTorch's flash-style SDPA for bf16 (fp32 scores and softmax statistics,
  exp(s - max) rounded to bf16 before P.V, fp32 accumulation), output
  rounded to bf16 (model.py:187-190, fast.py:149-162);
* every linear: exact fp32/fp64 accumulation, one bf16 rounding of the output;
* residual adds, ``silu(gate)`` and ``silu(gate) * up`` each rounded to bf16
  (model.py:191-196, fast.py:164-172);
* heads: text, 2-way and 32 audio heads with column 1024 set to -inf
  (model.py:240-295, fast.py:174-194).

Weights are carried as bf16 bit patterns (uint16). A linear may instead be a
W4 record ``(q uint8 [N, K], qsz bf16 bits [K/g, N, 2], g)``; its weight is
``oracle.w4.ref_operand_weight`` (the effective weight rounded to bf16, the
operand of the reference's int4 GEMM).
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16_to_f32, f32_to_bf16, round_bf16
from .w4 import ref_operand_weight

N_VQ = 32
AUDIO_PAD_CODE = 1024
AUDIO_VOCAB = 1025
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


def rms_norm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float = RMS_EPS) -> np.ndarray:
    """model.py:34-40, last axis. Returns bf16 bits."""
    x = bf16_to_f32(x_bits)
    var = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    y = f32_to_bf16((x * r).astype(np.float32))
    return f32_to_bf16(bf16_to_f32(w_bits) * bf16_to_f32(y))


def rotate_half(x: np.ndarray) -> np.ndarray:
    """model.py:42-44 on float32 values (negation is exact)."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def rope_tables(n: int, head_dim: int):
    """model.py:115-124: fp32 chain, then cast to bf16. Returns bf16 bits
    ``(cos, sin)`` [n, head_dim]."""
    inv = (np.float32(1.0) / (np.float32(ROPE_THETA) ** (
        np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)))).astype(np.float32)
    pos = np.arange(n, dtype=np.float32)
    freqs = np.outer(pos, inv).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    return f32_to_bf16(np.cos(emb).astype(np.float32)), f32_to_bf16(np.sin(emb).astype(np.float32))


def apply_rope(x_bits: np.ndarray, cos_bits: np.ndarray, sin_bits: np.ndarray) -> np.ndarray:
    """``x * cos + rotate_half(x) * sin`` with bf16 rounding after each op."""
    x = bf16_to_f32(x_bits)
    a = round_bf16(x * bf16_to_f32(cos_bits))
    b = round_bf16(rotate_half(x) * bf16_to_f32(sin_bits))
    return f32_to_bf16(a + b)


def attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool = False) -> np.ndarray:
    """Scaled dot-product attention for one head with the rounding points of
    PyTorch's flash-style SDPA kernels (CPU and CUDA) for bf16 inputs: fp32
    scores and softmax statistics, the unnormalised probabilities
    exp(s - max) rounded to bf16 before the P.V product, fp32 accumulation,
    normalisation by the fp32 row sum.  q [t, D], k/v [s, D] float64 holding
    bf16 values; returns float64 [t, D] (round to bf16 outside)."""
    sc = (q.astype(np.float32) @ k.astype(np.float32).T).astype(np.float32) * np.float32(scale)
    if causal:
        t, s = sc.shape
        sc = sc + np.triu(np.full((t, s), -np.inf, np.float32), 1 + s - t)
    m = sc.max(-1, keepdims=True)
    p = np.exp(sc - m).astype(np.float32)
    l = p.sum(-1, keepdims=True, dtype=np.float64)
    pb = round_bf16(p).astype(np.float64)
    return (pb @ v) / l


def silu_mul(gate_bits: np.ndarray, up_bits: np.ndarray) -> np.ndarray:
    """``bf16(bf16(silu(gate)) * up)`` (fast.py:170-171)."""
    g = bf16_to_f32(gate_bits)
    s = round_bf16(g / (np.float32(1.0) + np.exp(-g)))
    return f32_to_bf16(s * bf16_to_f32(up_bits))


def add_bf16(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    return f32_to_bf16(bf16_to_f32(a_bits) + bf16_to_f32(b_bits))


class OracleModel:
    """numpy MossTTSModel. ``weights`` maps reference checkpoint key names
    (tests/test_quant.py:299-327 layout) to bf16 bit arrays."""

    def __init__(self, weights: dict, max_seq_len: int = 256, fp32_linears: bool = False):
        layer_ids = sorted({int(k.split(".")[2]) for k in weights
                            if k.startswith("language_model.layers.")})
        self.n_layers = len(layer_ids)
        emb = weights["language_model.embed_tokens.weight"]
        self.hidden = int(emb.shape[1])
        self.text_vocab = int(emb.shape[0])
        self.head_dim = int(weights["language_model.layers.0.self_attn.q_norm.weight"].shape[0])
        self.n_heads = int(weights["language_model.layers.0.self_attn.q_proj.weight"].shape[0]) // self.head_dim
        self.n_kv = int(weights["language_model.layers.0.self_attn.k_proj.weight"].shape[0]) // self.head_dim
        self.n_rep = self.n_heads // self.n_kv
        self.max_seq_len = max_seq_len
        # fp32_linears: BLAS fp32 products instead of fp64 (the CPU-baseline
        # timing mode; parity tests keep the fp64 default)
        self.fp32_linears = fp32_linears
        self.embed = weights["language_model.embed_tokens.weight"]
        self.final_norm = weights["language_model.norm.weight"]
        names = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
                 "o": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj",
                 "down": "mlp.down_proj"}
        self.layers = []
        self._w_eff = []
        for i in range(self.n_layers):
            p = f"language_model.layers.{i}"
            lyr = {n: weights[f"{p}.{names[n]}.weight"] for n in LIN_NAMES}
            lyr["input_layernorm"] = weights[f"{p}.input_layernorm.weight"]
            lyr["post_attention_layernorm"] = weights[f"{p}.post_attention_layernorm.weight"]
            lyr["q_norm"] = weights[f"{p}.self_attn.q_norm.weight"]
            lyr["k_norm"] = weights[f"{p}.self_attn.k_norm.weight"]
            self.layers.append(lyr)
            self._w_eff.append({n: bf16_to_f32(lyr[n]) for n in LIN_NAMES})
        self.emb_ext = [weights[f"emb_ext.{i}.weight"] for i in range(N_VQ)]
        self.head_text = weights["lm_heads.0.weight"]
        self.head_audio = np.stack([weights[f"lm_heads.{i + 1}.weight"] for i in range(N_VQ)])
        self.head_2way = self.head_text[[AUDIO_GEN_SLOT_TOKEN_ID, AUDIO_DELAY_SLOT_TOKEN_ID]]
        self.rope_cos, self.rope_sin = rope_tables(max_seq_len, self.head_dim)
        shape = (self.n_layers, self.n_kv, max_seq_len, self.head_dim)
        self.k_cache = np.zeros(shape, np.uint16)
        self.v_cache = np.zeros(shape, np.uint16)
        self.seq = 0

    def quantize_w4(self, qrecs: dict):
        """Install W4 records ``{(li, name): (q [N,K] uint8, qsz bits, g)}``;
        those linears then multiply with the reference's int4 GEMM operand
        (gptq.py:87-97 rounded to bf16, as _weight_int4pack_mm forms it)."""
        for (li, name), (q, qsz, g) in qrecs.items():
            self._w_eff[li][name] = ref_operand_weight(q, qsz, g)

    def linear(self, x_bits: np.ndarray, li: int, name: str) -> np.ndarray:
        w = self._w_eff[li][name]                   # [N, K] fp32
        if self.fp32_linears:
            return f32_to_bf16(bf16_to_f32(x_bits) @ w.T)
        x = bf16_to_f32(x_bits).astype(np.float64)
        return f32_to_bf16((x @ w.astype(np.float64).T).astype(np.float32))

    @staticmethod
    def head(x_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
        x = bf16_to_f32(x_bits).astype(np.float64)
        return f32_to_bf16((x @ bf16_to_f32(w_bits).astype(np.float64).T).astype(np.float32))

    def embed_rows(self, ids: np.ndarray) -> np.ndarray:
        """ids int [t, 33] -> bf16 bits [t, hidden] (model.py:156-161)."""
        h = self.embed[ids[:, 0]]
        for i in range(N_VQ):
            h = add_bf16(h, self.emb_ext[i][ids[:, i + 1]])
        return h

    def layer(self, li: int, h: np.ndarray, s0: int) -> np.ndarray:
        """model.py:163-197 for t rows starting at position s0."""
        lyr = self.layers[li]
        t = h.shape[0]
        s1 = s0 + t
        D = self.head_dim
        x = rms_norm(h, lyr["input_layernorm"])
        q = self.linear(x, li, "q").reshape(t, self.n_heads, D)
        k = self.linear(x, li, "k").reshape(t, self.n_kv, D)
        v = self.linear(x, li, "v").reshape(t, self.n_kv, D)
        q = rms_norm(q, lyr["q_norm"])
        k = rms_norm(k, lyr["k_norm"])
        cos = self.rope_cos[s0:s1][:, None, :]
        sin = self.rope_sin[s0:s1][:, None, :]
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        self.k_cache[li, :, s0:s1] = k.transpose(1, 0, 2)
        self.v_cache[li, :, s0:s1] = v.transpose(1, 0, 2)
        keys = bf16_to_f32(self.k_cache[li, :, :s1]).astype(np.float64)      # [kv, s1, D]
        vals = bf16_to_f32(self.v_cache[li, :, :s1]).astype(np.float64)
        qf = bf16_to_f32(q).astype(np.float64)                                # [t, H, D]
        out = np.empty((t, self.n_heads, D), np.float64)
        scale = 1.0 / np.sqrt(D)
        for hh in range(self.n_heads):
            kv = hh // self.n_rep
            out[:, hh, :] = attend(qf[:, hh, :], keys[kv], vals[kv], scale, causal=(t > 1 and s1 == t))
        attn = f32_to_bf16(out.astype(np.float32)).reshape(t, self.n_heads * D)
        h = add_bf16(h, self.linear(attn, li, "o"))
        x = rms_norm(h, lyr["post_attention_layernorm"])
        m = silu_mul(self.linear(x, li, "gate"), self.linear(x, li, "up"))
        return add_bf16(h, self.linear(m, li, "down"))

    def prefill(self, ids: np.ndarray) -> np.ndarray:
        """model.py:206-219. ids int [L, 33] -> final-normed hidden [L, hidden]."""
        self.seq = 0
        h = self.embed_rows(ids)
        for li in range(self.n_layers):
            h = self.layer(li, h, 0)
        self.seq = ids.shape[0]
        return rms_norm(h, self.final_norm)

    def step(self, row: np.ndarray) -> np.ndarray:
        """model.py:221-233. row int [33] -> final-normed hidden [1, hidden]."""
        s0 = self.seq
        h = self.embed_rows(np.asarray(row).reshape(1, -1))
        for li in range(self.n_layers):
            h = self.layer(li, h, s0)
        self.seq = s0 + 1
        return rms_norm(h, self.final_norm)

    def text_logits(self, h_bits: np.ndarray) -> np.ndarray:
        return self.head(h_bits.reshape(-1), self.head_text)

    def text_logits_2way(self, h_bits: np.ndarray) -> np.ndarray:
        return self.head(h_bits.reshape(-1), self.head_2way)

    def audio_logits(self, h_bits: np.ndarray) -> np.ndarray:
        """model.py:270-295: [32, 1025] bf16 bits, column 1024 = -inf."""
        hv = h_bits.reshape(-1)
        out = np.stack([self.head(hv, self.head_audio[i]) for i in range(N_VQ)])
        out[:, AUDIO_PAD_CODE] = 0xFF80      # bf16 -inf
        return out


def synth_weights(hidden: int, n_layers: int, n_heads: int, n_kv: int, head_dim: int,
                  inter: int, vocab: int = 151936, seed: int = 0, std: float = 0.02,
                  norm_ones: bool = True) -> dict:
    """Seeded random-init checkpoint dict (bf16 bits) with the reference key
    names (tests/test_quant.py:299-327). numpy's PCG64 stream is stable
    across platforms, so tests regenerate these instead of storing them."""
    rng = np.random.default_rng(seed)

    def r(*shape):
        return f32_to_bf16((rng.standard_normal(shape, dtype=np.float32) * np.float32(std)))

    def ones(n):
        if norm_ones:
            return f32_to_bf16(np.ones(n, np.float32))
        return f32_to_bf16((1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32))

    w = {"language_model.embed_tokens.weight": r(vocab, hidden),
         "language_model.norm.weight": ones(hidden)}
    for li in range(n_layers):
        p = f"language_model.layers.{li}"
        w[f"{p}.input_layernorm.weight"] = ones(hidden)
        w[f"{p}.post_attention_layernorm.weight"] = ones(hidden)
        w[f"{p}.self_attn.q_proj.weight"] = r(n_heads * head_dim, hidden)
        w[f"{p}.self_attn.k_proj.weight"] = r(n_kv * head_dim, hidden)
        w[f"{p}.self_attn.v_proj.weight"] = r(n_kv * head_dim, hidden)
        w[f"{p}.self_attn.o_proj.weight"] = r(hidden, n_heads * head_dim)
        w[f"{p}.self_attn.q_norm.weight"] = ones(head_dim)
        w[f"{p}.self_attn.k_norm.weight"] = ones(head_dim)
        w[f"{p}.mlp.gate_proj.weight"] = r(inter, hidden)
        w[f"{p}.mlp.up_proj.weight"] = r(inter, hidden)
        w[f"{p}.mlp.down_proj.weight"] = r(hidden, inter)
    for i in range(N_VQ):
        w[f"emb_ext.{i}.weight"] = r(AUDIO_VOCAB, hidden)
    w["lm_heads.0.weight"] = r(vocab, hidden)
    for i in range(N_VQ):
        w[f"lm_heads.{i + 1}.weight"] = r(AUDIO_VOCAB, hidden)
    return w
