"""W4A16 linears backed by the sm_100a kernels of libmtl_b200.so.

Two faces over one packed device format (the MTL tile layout, see
include/mtl_b200.h):

* ``QuantLinear`` - the AutoGPTQ-style module named by the benchmark
  configuration: ``qweight`` int32 [K/8, N], ``qzeros`` int32 [K/g, N/8],
  fp16 ``scales`` [K/g, N], ``g_idx`` [K];  ``w = (q - (z + zero_offset)) * s``.
* ``RefW4Linear`` - the reference's own W4 weight, integer codes
  ``q`` uint8 [N, K] plus bf16 ``qsz`` [K/g, N, 2] with
  ``w = (q - 8) * scale + zero`` (moss_tts_lite/gptq.py:87-97), i.e. what
  ``FastMossTTS._quantize`` builds before the tinygemm packer
  (moss_tts_lite/fast.py:85-100).

Both call ``mtl_w4a16_linear``; torch only owns the device memory.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_GROUPS = (32, 64, 128, 256)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class W4Weight:
    """A packed W4 weight plus its split-K scratch (one per linear)."""

    def __init__(self, tiles: torch.Tensor, K: int, N: int, group_size: int, fmt: int,
                 zero_offset: int = 0, k_perm: torch.Tensor | None = None):
        self.tiles = tiles
        self.K, self.N, self.group_size, self.fmt = int(K), int(N), int(group_size), int(fmt)
        self.zero_offset = int(zero_offset)
        self.k_perm = k_perm
        _, sb = _lib.w4_plan(8, self.K, self.N, self.group_size, self.fmt)
        self.scratch = torch.zeros(sb, dtype=torch.uint8, device=tiles.device)

    @staticmethod
    def alloc_tiles(K: int, N: int, g: int, fmt: int, device) -> torch.Tensor:
        tb, _ = _lib.w4_plan(1, K, N, g, fmt)
        return torch.empty(tb, dtype=torch.uint8, device=device)

    @classmethod
    def from_ref(cls, q: torch.Tensor, qsz: torch.Tensor, group_size: int,
                 fmt: int | None = None) -> "W4Weight":
        """Codes uint8 [N, K] (0..15) + qsz bf16 [K/g, N, 2] on a CUDA device.
        ``fmt``: MTL_FMT_REF (register-MMA tiles, any batch) or MTL_FMT_TC
        (tensor-core tiles, the batch-1 decode layout; gate/up of a SwiGLU
        pair interleaved row by row)."""
        fmt = _lib.MTL_FMT_REF if fmt is None else int(fmt)
        if group_size not in _GROUPS:
            raise ValueError("w4_group_size must be 32/64/128/256")
        N, K = q.shape
        if tuple(qsz.shape) != (K // group_size, N, 2):
            raise ValueError(f"qsz shape {tuple(qsz.shape)} != {(K // group_size, N, 2)}")
        q = q.to(torch.uint8).contiguous()
        qsz = qsz.to(torch.bfloat16).contiguous()
        tiles = cls.alloc_tiles(K, N, group_size, fmt, q.device)
        fn = "mtl_w4_pack_tc" if fmt == _lib.MTL_FMT_TC else "mtl_w4_pack_ref"
        _lib.call(fn, q.data_ptr(), qsz.data_ptr(), K, N, group_size, tiles.data_ptr(), _stream())
        return cls(tiles, K, N, group_size, fmt)

    @staticmethod
    def tc_supported(K: int, N: int, group_size: int) -> bool:
        """Whether the tensor-core tile layout (MTL_FMT_TC) covers this shape."""
        return N % 128 == 0 and group_size in (32, 64, 128) and K % group_size == 0 and K <= 16384

    def unpack_codes(self) -> torch.Tensor:
        """uint8 [N, K] codes in packed row order (bit-exact inverse of packing)."""
        out = torch.empty(self.N, self.K, dtype=torch.uint8, device=self.tiles.device)
        _lib.call("mtl_w4_unpack_codes", self.tiles.data_ptr(), self.K, self.N, self.group_size,
                  self.fmt, out.data_ptr(), _stream())
        return out

    def ref_params(self) -> torch.Tensor:
        """qsz bf16 [K/g, N, 2] (scale, zero) read back from reference-format tiles."""
        if self.fmt != _lib.MTL_FMT_REF:
            raise ValueError("ref_params needs MTL_FMT_REF tiles")
        KT, nb, g = self.K // self.group_size, self.N // 64, self.group_size
        t = self.tiles.view(nb, KT, -1)[:, :, 64 * g // 2:64 * g // 2 + 256]       # [nb, KT, 64 x (scale, zero)]
        prm = t.contiguous().view(torch.bfloat16).view(nb, KT, 64, 2)
        return prm.permute(1, 0, 2, 3).reshape(KT, self.N, 2).contiguous()

    def to_tc(self, swiglu_block: int = 0) -> "W4Weight":
        """The same reference-format codes and (scale, zero) in tensor-core
        tiles (MTL_FMT_TC).  ``swiglu_block``: the weight is a gate|up pair
        interleaved in blocks of that many rows; the TC tiles interleave the
        pair row by row."""
        q, qsz = self.unpack_codes(), self.ref_params()
        if swiglu_block:
            b = swiglu_block
            q = q.view(-1, 2, b, self.K).permute(1, 0, 2, 3).reshape(2, -1, self.K)      # [gate | up][I][K]
            q = q.permute(1, 0, 2).reshape(self.N, self.K)
            z = qsz.view(qsz.shape[0], -1, 2, b, 2).permute(0, 2, 1, 3, 4).reshape(qsz.shape[0], 2, -1, 2)
            qsz = z.permute(0, 2, 1, 3).reshape(qsz.shape[0], self.N, 2)
        return W4Weight.from_ref(q.contiguous(), qsz.contiguous(), self.group_size, fmt=_lib.MTL_FMT_TC)

    def to_strip(self, swiglu_block: int = 0) -> "StripWeight":
        """The same reference-format codes and (scale, zero) in the strip
        layout of the persistent chain kernel (mtl_w4_pack_strip).
        ``swiglu_block``: the weight is a gate|up pair interleaved in blocks
        of that many rows; the strips interleave it in blocks of 8."""
        if self.fmt != _lib.MTL_FMT_REF or self.k_perm is not None:
            raise ValueError("to_strip needs reference-format tiles without a k permutation")
        q, qsz = self.unpack_codes(), self.ref_params()
        if swiglu_block:
            b, KT = swiglu_block, qsz.shape[0]
            gu = q.view(-1, 2, b, self.K).permute(1, 0, 2, 3).reshape(2, -1, self.K)          # [gate | up][I][K]
            q = torch.stack([gu[0].reshape(-1, 8, self.K), gu[1].reshape(-1, 8, self.K)], 1).reshape(self.N, self.K)
            z = qsz.view(KT, -1, 2, b, 2).permute(0, 2, 1, 3, 4).reshape(KT, 2, -1, 2)          # [KT][gate | up][I][2]
            qsz = torch.stack([z[:, 0].reshape(KT, -1, 8, 2), z[:, 1].reshape(KT, -1, 8, 2)], 2).reshape(KT, self.N, 2)
        return StripWeight.from_ref(q.contiguous(), qsz.contiguous(), self.group_size)

    def dequant(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """Effective weights bf16 [N, K] in packed column order (k_perm order
        for act-order AutoGPTQ weights), as the operand of a many-row GEMM."""
        if out is None:
            out = torch.empty(self.N, self.K, dtype=torch.bfloat16, device=self.tiles.device)
        _lib.call("mtl_w4_dequant", self.tiles.data_ptr(), self.K, self.N, self.group_size, self.fmt,
                  self.zero_offset, out.data_ptr(), _stream())
        return out

    def linear(self, x: torch.Tensor, *, out: torch.Tensor | None = None,
               residual: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
               norm_eps: float = 1e-6, swiglu: bool = False) -> torch.Tensor:
        """``x`` bf16 [..., K] -> bf16 [..., N] (or [..., N/2] with swiglu)."""
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        if x.shape[-1] != self.K:
            raise ValueError(f"x last dim {x.shape[-1]} != K={self.K}")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        M = x2.shape[0]
        nout = self.N // 2 if swiglu else self.N
        epi = _lib.MTL_EPI_STORE
        if swiglu:
            epi = _lib.MTL_EPI_SWIGLU
        elif residual is not None:
            epi = _lib.MTL_EPI_RESIDUAL
            residual = residual.reshape(M, self.N)
            if residual.dtype != torch.bfloat16 or not residual.is_contiguous():
                raise ValueError("residual must be contiguous bf16 [..., N]")
        if out is None:
            out = torch.empty(M, nout, dtype=torch.bfloat16, device=x.device)
        if M == 0:
            return out.reshape(*lead, nout)
        _lib.call("mtl_w4a16_linear", x2.data_ptr(), self.K, M, self.K, self.N, self.group_size,
                  self.fmt, self.tiles.data_ptr(), self.zero_offset, _ptr(self.k_perm),
                  _ptr(norm_weight), ctypes.c_float(norm_eps), epi, _ptr(residual), out.data_ptr(),
                  nout, self.scratch.data_ptr(), self.scratch.numel(), _stream())
        return out.reshape(*lead, nout)


class StripWeight:
    """A W4 weight in the strip layout (16 output rows x one group per tile)
    read by the persistent chain kernel (mtl_w4_chain)."""

    def __init__(self, tiles: torch.Tensor, K: int, N: int, group_size: int):
        self.tiles, self.K, self.N, self.group_size = tiles, int(K), int(N), int(group_size)

    @staticmethod
    def supported(K: int, N: int, group_size: int) -> bool:
        return group_size in (64, 128, 256) and K % group_size == 0 and N % 16 == 0 and K <= 16384

    @classmethod
    def from_ref(cls, q: torch.Tensor, qsz: torch.Tensor, group_size: int) -> "StripWeight":
        """Codes uint8 [N, K] + qsz bf16 [K/g, N, 2] on a CUDA device."""
        N, K = q.shape
        if tuple(qsz.shape) != (K // group_size, N, 2):
            raise ValueError(f"qsz shape {tuple(qsz.shape)} != {(K // group_size, N, 2)}")
        q = q.to(torch.uint8).contiguous()
        qsz = qsz.to(torch.bfloat16).contiguous()
        tiles = torch.empty(_lib.strip_bytes(K, N, group_size), dtype=torch.uint8, device=q.device)
        _lib.call("mtl_w4_pack_strip", q.data_ptr(), qsz.data_ptr(), K, N, group_size, tiles.data_ptr(), _stream())
        return cls(tiles, K, N, group_size)


def gemm_supported(w: "W4Weight") -> bool:
    """Whether the tcgen05 prefill GEMM (mtl_w4a16_gemm) serves this weight."""
    return (w.fmt == _lib.MTL_FMT_REF and w.k_perm is None and w.group_size >= 64 and w.K % 64 == 0
            and w.N % 128 == 0)


def _gemm(self: "W4Weight", x: torch.Tensor, *, out: torch.Tensor | None = None,
          residual: torch.Tensor | None = None, swiglu: bool = False) -> torch.Tensor:
    """Many-row W4 GEMM on the tensor cores (the prompt prefill): ``x`` bf16
    [M, K] -> bf16 [M, N] (or [M, N/2] with swiglu; ``residual`` [M, N] added
    and rounded as the reference's residual add, may be ``out``)."""
    if not gemm_supported(self):
        raise ValueError("mtl_w4a16_gemm needs reference-format tiles, group_size >= 64, K % 64 == 0, N % 128 == 0")
    x2 = x.reshape(-1, self.K)
    if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
        raise ValueError("x must be contiguous bf16 [M, K]")
    M = x2.shape[0]
    nout = self.N // 2 if swiglu else self.N
    epi = _lib.MTL_EPI_SWIGLU if swiglu else (_lib.MTL_EPI_RESIDUAL if residual is not None else _lib.MTL_EPI_STORE)
    if out is None:
        out = torch.empty(M, nout, dtype=torch.bfloat16, device=x.device)
    if M == 0:
        return out
    r2 = residual.reshape(M, self.N) if residual is not None else None
    _lib.call("mtl_w4a16_gemm", x2.data_ptr(), self.K, M, self.K, self.N, self.group_size, self.tiles.data_ptr(), epi,
              _ptr(r2), self.N, out.data_ptr(), nout, _stream())
    return out


W4Weight.gemm = _gemm


class RefW4Linear(torch.nn.Module):
    """The reference's W4 linear (``(packed, qsz)`` call sites of fast.py:118,
    gptq.py:582) built from the codes before tinygemm packing."""

    def __init__(self, q: torch.Tensor, qsz: torch.Tensor, group_size: int = 128):
        super().__init__()
        self.w = W4Weight.from_ref(q, qsz, group_size)
        self.in_features, self.out_features = self.w.K, self.w.N

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w.linear(x)


class QuantLinear(torch.nn.Module):
    """AutoGPTQ-style W4A16 linear (bits=4) on the B200 kernels.

    Buffers follow AutoGPTQ: ``qweight`` int32 [K/8, N], ``qzeros`` int32
    [K/g, N/8], ``scales`` fp16 [K/g, N], ``g_idx`` int32 [K]. Call
    ``post_init()`` (or use ``from_tensors``) after filling them; that packs
    the weight once into the device tile layout. Act-order checkpoints
    (non-monotone ``g_idx``) are served by sorting K by group at packing
    time and gathering x through the same permutation in the kernel.
    """

    def __init__(self, bits: int, group_size: int, infeatures: int, outfeatures: int,
                 bias: bool = False, zero_offset: int = 0, device="cuda"):
        super().__init__()
        if bits != 4:
            raise NotImplementedError("only 4-bit QuantLinear is provided")
        if group_size == -1:
            group_size = infeatures
        if group_size not in _GROUPS:
            raise ValueError(f"group_size {group_size} not in {_GROUPS}")
        if bias:
            raise NotImplementedError("MOSS-TTS linears carry no bias")
        if infeatures % group_size or outfeatures % 64:
            raise ValueError(f"infeatures {infeatures} % group_size and outfeatures {outfeatures} % 64 must be 0")
        self.bits, self.group_size = bits, group_size
        self.infeatures, self.outfeatures = infeatures, outfeatures
        self.zero_offset = int(zero_offset)
        G = infeatures // group_size
        self.register_buffer("qweight", torch.zeros(infeatures // 8, outfeatures, dtype=torch.int32, device=device))
        self.register_buffer("qzeros", torch.zeros(G, outfeatures // 8, dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.zeros(G, outfeatures, dtype=torch.float16, device=device))
        self.register_buffer("g_idx", (torch.arange(infeatures, dtype=torch.int32, device=device) // group_size))
        self.w: W4Weight | None = None

    @classmethod
    def from_tensors(cls, qweight, qzeros, scales, g_idx=None, group_size: int = 128,
                     zero_offset: int = 0, free_source: bool = True) -> "QuantLinear":
        """Pack the given AutoGPTQ tensors.  With ``free_source`` (default)
        the module's own AutoGPTQ buffers are emptied after packing: the
        caller's tensors are the source, and only the tiles stay on the
        device."""
        K = qweight.shape[0] * 8
        N = qweight.shape[1]
        m = cls(4, group_size, K, N, zero_offset=zero_offset, device=qweight.device)
        m.qweight.copy_(qweight)
        m.qzeros.copy_(qzeros)
        m.scales.copy_(scales)
        if g_idx is not None:
            m.g_idx.copy_(g_idx)
        m.post_init(free_source=free_source)
        return m

    def post_init(self, free_source: bool = False) -> None:
        """Pack the AutoGPTQ buffers into the device tiles.  ``free_source``
        empties ``qweight`` / ``qzeros`` / ``scales`` afterwards (the tiles
        hold the same codes, zeros and scales; keep them for a state_dict in
        the AutoGPTQ layout)."""
        K, N, g = self.infeatures, self.outfeatures, self.group_size
        gi = self.g_idx.to(torch.int64)
        if gi.min() < 0 or gi.max() >= K // g:
            raise ValueError("g_idx out of range")
        trivial = torch.equal(gi, torch.arange(K, device=gi.device) // g)
        perm = None
        if not trivial:
            perm = torch.argsort(gi, stable=True)
            if not torch.equal(gi[perm], torch.arange(K, device=gi.device) // g):
                raise ValueError("g_idx must assign exactly group_size rows to every group")
            perm = perm.to(torch.int32).contiguous()
        tiles = W4Weight.alloc_tiles(K, N, g, _lib.MTL_FMT_GPTQ, self.qweight.device)
        _lib.call("mtl_w4_pack_gptq", self.qweight.data_ptr(), self.qzeros.data_ptr(),
                  self.scales.data_ptr(), _ptr(perm), K, N, g, tiles.data_ptr(), _stream())
        self.w = W4Weight(tiles, K, N, g, _lib.MTL_FMT_GPTQ, self.zero_offset, perm)
        if free_source:
            self.qweight = self.qweight.new_empty(0)
            self.qzeros = self.qzeros.new_empty(0)
            self.scales = self.scales.new_empty(0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.w is None:
            self.post_init()
        return self.w.linear(x)
