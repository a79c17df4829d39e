/*
 * mtl_b200.h - C ABI of the B200 (sm_100a) kernels for the moss-tts-lite
 * W4 decode hot path.  Plain pointers, sizes and a CUDA stream; no torch
 * types.  Every function returns 0 on success or a negative MTL_E* code;
 * mtl_last_error() then describes the failure (thread-local).
 *
 * All tensor pointers are device pointers unless stated otherwise.  bf16
 * and fp16 values are passed as uint16_t bit patterns.  Nothing here
 * synchronises the stream or allocates device memory, so every entry point
 * except the mtl_w4_plan/mtl_device_status helpers can be captured in a
 * CUDA graph.
 */
#ifndef MTL_B200_H
#define MTL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mtl_stream_t; /* == cudaStream_t */

#define MTL_OK 0
#define MTL_E_INVALID (-1)     /* bad shape, group size, pointer or flag  */
#define MTL_E_ALIGN (-2)       /* pointer misaligned for the kernel       */
#define MTL_E_SCRATCH (-3)     /* scratch buffer too small                */
#define MTL_E_CUDA (-4)        /* CUDA runtime error (see mtl_last_error) */
#define MTL_E_UNSUPPORTED (-5) /* valid request this build does not serve */

/* Parameter formats of a packed W4 weight. */
#define MTL_FMT_REF 0  /* reference qsz: bf16 (scale, zero), w = (q-8)*scale+zero */
#define MTL_FMT_GPTQ 1 /* AutoGPTQ: fp16 scale + 4-bit zero, w = (q-(z+off))*s   */

/* Epilogues of mtl_w4a16_linear. */
#define MTL_EPI_STORE 0    /* y = bf16(x W^T)                                   */
#define MTL_EPI_RESIDUAL 1 /* y = bf16(residual + bf16(x W^T))                  */
#define MTL_EPI_SWIGLU 2   /* y = bf16(bf16(silu(gate)) * up), gate/up fused    */

/* ---------------------------------------------------------------- status */

/* Message for the last failing call on this thread ("" if none). */
const char* mtl_last_error(void);

/* ABI version of this library (bumped on incompatible changes). */
int mtl_abi_version(void);

/* Reads (and optionally clears) the device error word that kernels set
 * instead of trapping: bit 0 = a bounded mbarrier wait gave up, bit 1 = an
 * index failed its bound check, bit 2 = bulk copies were still in flight at
 * exit.  Synchronises the current device. */
int mtl_device_status(uint32_t* out, int clear);

/* ------------------------------------------------------------- W4 linear */

/* Sizes for a W4 linear of K inputs and N outputs:
 *   *tiles_bytes   - packed weight buffer (MTL tile layout);
 *   *scratch_bytes - split-K scratch for batch size M (M >= 1; batches
 *                    above 8 run in chunks of 8).  Zero-fill it once before
 *                    first use; every call leaves it reusable.
 * group_size in {32, 64, 128, 256}; K % group_size == 0; N % 64 == 0.
 * Host-only (no device work).  Either out pointer may be NULL. */
int mtl_w4_plan(int M, int K, int N, int group_size, int param_fmt, size_t* tiles_bytes,
                size_t* scratch_bytes);

/* Pack the reference's own W4 weight into the MTL tile layout.
 * Replaces torch.ops.aten._convert_weight_to_int4pack as called at
 * moss_tts_lite/fast.py:97-99 and gptq.py:75-76: takes the integer codes
 * before the tinygemm packer (q uint8 [N, K], values 0..15, fast.py:91-93)
 * and qsz bf16 [K/g, N, 2] = (scale, zero) (fast.py:94-96). */
int mtl_w4_pack_ref(const uint8_t* q, const uint16_t* qsz, int K, int N, int group_size, void* tiles,
                    mtl_stream_t stream);

/* Pack an AutoGPTQ weight: qweight int32 [K/8, N] (LSB-first nibbles along
 * K), qzeros int32 [K/g, N/8] (LSB-first along N), scales fp16 [K/g, N].
 * perm (nullable, int32 [K]) lists original k indices in group-sorted order
 * for act-order checkpoints: packed row k' holds original row perm[k']. */
int mtl_w4_pack_gptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                     const int32_t* perm, int K, int N, int group_size, void* tiles, mtl_stream_t stream);

/* Inverse of the packers for the codes: codes uint8 [N, K] (row n = output
 * column; packed row order, i.e. after any perm). */
int mtl_w4_unpack_codes(const void* tiles, int K, int N, int group_size, int param_fmt, uint8_t* codes,
                        mtl_stream_t stream);

/* y = epilogue(x . W_eff^T) for a packed W4 weight.
 * Replaces torch._weight_int4pack_mm(x, packed, g, qsz) at
 * moss_tts_lite/fast.py:118, gptq.py:582 and fast_native.py:169
 * (and the AutoGPTQ QuantLinear forward with param_fmt = MTL_FMT_GPTQ).
 *   x        bf16 [M, ldx] (row-major, ldx >= K)
 *   k_perm   nullable int32 [K]: x is read as x[:, k_perm[k]] (act-order)
 *   norm_w   nullable bf16 [K]: fuse RMSNorm(x) (moss_tts_lite/model.py:34-40,
 *            eps = norm_eps) into the prologue
 *   epilogue MTL_EPI_*; residual bf16 [M, N] for MTL_EPI_RESIDUAL (may
 *            alias y); MTL_EPI_SWIGLU expects gate/up interleaved in 32-column
 *            blocks (block b = gate[32b..32b+32) then up[32b..32b+32)) and
 *            writes N/2 outputs per row
 *   y        bf16 [M, ldy]
 *   scratch  device buffer of >= scratch_bytes from mtl_w4_plan, zeroed once
 *   zero_offset  MTL_FMT_GPTQ only: added to every stored zero (0 or 1). */
int mtl_w4a16_linear(const uint16_t* x, int ldx, int M, int K, int N, int group_size, int param_fmt,
                     const void* tiles, int zero_offset, const int32_t* k_perm, const uint16_t* norm_w,
                     float norm_eps, int epilogue, const uint16_t* residual, uint16_t* y, int ldy,
                     void* scratch, size_t scratch_bytes, mtl_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MTL_B200_H */
