/*
 * mtl_b200.h - C ABI of the B200 (sm_100a) kernels for the moss-tts-lite
 * W4 decode hot path.  Plain pointers, sizes and a CUDA stream; no torch
 * types.  Every function returns 0 on success or a negative MTL_E* code;
 * mtl_last_error() then describes the failure (thread-local).
 *
 * All tensor pointers are device pointers unless stated otherwise.  bf16
 * and fp16 values are passed as uint16_t bit patterns.  Nothing here
 * synchronises the stream or allocates device memory; the entry points that
 * take caller buffers (all but the mtl_w4_plan/mtl_device_status helpers and
 * mtl_w4a16_linear_noalloc) can be captured in a CUDA graph.
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
#define MTL_FMT_TC 2   /* reference qsz in the tensor-core tile layout (128-row
                          tiles, per-row (scale, zero)); mtl_w4a16_linear runs
                          the tcgen05 kernels: one row per launch for M == 1,
                          up to 16 rows per launch (the MMA N dimension)
                          otherwise.  N % 128
                          == 0, group_size 32/64/128, K <= 16384; the SwiGLU
                          epilogue expects gate and up rows interleaved one by
                          one (row 2j = gate j, row 2j + 1 = up j) */

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

/* The same reference weight (codes + qsz, as mtl_w4_pack_ref) packed into
 * the tensor-core tile layout of MTL_FMT_TC (size from mtl_w4_plan with
 * param_fmt = MTL_FMT_TC).  Same reference call sites as mtl_w4_pack_ref. */
int mtl_w4_pack_tc(const uint8_t* q, const uint16_t* qsz, int K, int N, int group_size, void* tiles,
                   mtl_stream_t stream);

/* Pack an AutoGPTQ weight: qweight int32 [K/8, N] (LSB-first nibbles along
 * K), qzeros int32 [K/g, N/8] (LSB-first along N), scales fp16 [K/g, N].
 * perm (nullable, int32 [K]) lists original k indices in group-sorted order
 * for act-order checkpoints: packed row k' holds original row perm[k']. */
int mtl_w4_pack_gptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                     const int32_t* perm, int K, int N, int group_size, void* tiles, mtl_stream_t stream);

/* Effective weights of packed tiles as bf16 w [N, K] row-major: REF
 * (q - 8) * scale + zero (gptq.py:87-97 effective_weight), GPTQ
 * (q - (z + zero_offset)) * scale, computed in fp32, rounded to bf16 — the
 * operand of the prompt-prefill GEMMs (many rows per pass over a layer),
 * where the reference runs tinygemm with M = prompt length (fast.py:218-270).
 * tiles and w 16-byte aligned (MTL_E_ALIGN otherwise). */
int mtl_w4_dequant(const void* tiles, int K, int N, int group_size, int param_fmt, int zero_offset, uint16_t* w,
                   mtl_stream_t stream);

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
 *   scratch  device buffer of >= scratch_bytes from mtl_w4_plan, zeroed once;
 *            every completed launch leaves its split-K counters at zero
 *            again.  A launch that gave up on a bounded wait (a nonzero
 *            mtl_device_status) may leave counters set: zero the scratch
 *            again before reusing it after such a status.
 *   zero_offset  MTL_FMT_GPTQ only: added to every stored zero (0 or 1). */
int mtl_w4a16_linear(const uint16_t* x, int ldx, int M, int K, int N, int group_size, int param_fmt,
                     const void* tiles, int zero_offset, const int32_t* k_perm, const uint16_t* norm_w,
                     float norm_eps, int epilogue, const uint16_t* residual, uint16_t* y, int ldy,
                     void* scratch, size_t scratch_bytes, mtl_stream_t stream);

/* mtl_w4a16_linear for callers that cannot allocate device memory (a host
 * that owns all device memory in its own pool and gives this library no
 * allocator, or a serving loop recording its step under stream capture,
 * where cudaMalloc is not permitted).  No counterpart in the reference: it
 * exists for such embedders only.  Same arguments and results as
 * mtl_w4a16_linear minus the scratch buffer: the split-K scratch is a fixed
 * 1 MiB device array inside the library (held on every GPU that loads the
 * library until exit); shapes needing more (mtl_w4_plan) fail with
 * MTL_E_SCRATCH.  Every argument is checked before anything is enqueued;
 * each call then clears the array's split-K counters on `stream` before its
 * launch.  All calls share that array: calls that can overlap on the
 * GPU (unordered streams) race, calls ordered on one stream are fine.  The
 * first call on each device resolves the array's address (with that device
 * current); make it before any stream capture.  Allocates nothing. */
int mtl_w4a16_linear_noalloc(const uint16_t* x, int ldx, int M, int K, int N, int group_size, int param_fmt,
                             const void* tiles, int zero_offset, const int32_t* k_perm, const uint16_t* norm_w,
                             float norm_eps, int epilogue, const uint16_t* residual, uint16_t* y, int ldy,
                             mtl_stream_t stream);

/* ---- persistent W4 chain (batch-1 decode) ------------------------------
 * Strip layout: the [N, K] int4 weight in tiles of 16 output rows x one
 * group (8 g + 64 bytes each, strip-major), the layout mtl_w4_chain reads.
 * Same codes and (scale, zero) as mtl_w4_pack_ref (w = bf16((q-8)*scale +
 * zero)); a gate|up pair for the SwiGLU epilogue is interleaved in blocks
 * of 8 rows (rows 0-7 of a strip gate, 8-15 up, of the same 8 outputs).
 * group_size 64/128/256, K % group_size == 0, N % 16 == 0. */
int mtl_w4_strip_bytes(int K, int N, int group_size, size_t* bytes);
int mtl_w4_pack_strip(const uint8_t* q, const uint16_t* qsz, int K, int N, int group_size, void* tiles,
                      mtl_stream_t stream);

typedef struct {
  const void* tiles;         /* strip-layout weight, K x N, 16-byte aligned */
  const uint16_t* x;         /* bf16 [K] input row, 16-byte aligned         */
  const uint16_t* norm_w;    /* nullable: RMSNorm of x first (bf16 [K])     */
  const uint16_t* residual;  /* MTL_EPI_RESIDUAL: bf16 [N], may alias y     */
  uint16_t* y;               /* bf16 [N] ([N/2] with MTL_EPI_SWIGLU)        */
  int K, N, epilogue;
} mtl_chain_phase;

/* Up to 4 dependent batch-1 W4 linears in one launch, each phase reading
 * the previous phases' outputs: the sequence o -> gate|up -> down -> next
 * q|k|v that the reference's decode step runs as separate
 * torch._weight_int4pack_mm calls (moss_tts_lite/fast.py:165-171 with
 * FastMossTTS._linear at fast.py:107-121), RMSNorm (model.py:34-40) and
 * residual / SwiGLU epilogues as mtl_w4a16_linear applies them.  One CTA
 * per SM; phases are separated by a grid barrier on `barrier`, a device
 * uint32 that must be 0 before the launch and is 0 again after it (give
 * each launch that may overlap another its own word).  A phase's y must
 * not overlap its own x (other phases' inputs and outputs may alias, as
 * the decode step's h does).  Results are
 * bitwise reproducible; they equal mtl_w4a16_linear's up to the fp32
 * summation order.  K <= 16384 per phase. */
int mtl_w4_chain(const mtl_chain_phase* phases, int nphases, int group_size, float norm_eps, uint32_t* barrier,
                 mtl_stream_t stream);

typedef struct {
  const void* tiles;         /* strip-layout weight, K x N, 16-byte aligned      */
  const uint16_t* x;         /* bf16 [M, ldx], 16-byte aligned, ldx % 8 == 0     */
  const uint16_t* norm_w;    /* nullable: RMSNorm of each row first (K <= 4096)  */
  const uint16_t* residual;  /* MTL_EPI_RESIDUAL: bf16 [M, ldr], may alias y     */
  uint16_t* y;               /* bf16 [M, ldy] ([M, N/2 columns] with SwiGLU)     */
  int ldx, ldr, ldy;
  int K, N, epilogue;
} mtl_chain_phase_rows;

/* mtl_w4_chain for M = 2..16 activation rows (the streams of a batched
 * decode step: the reference runs each stream's linears separately,
 * moss_tts_lite/fast.py:165-171).  The rows share one pass over the strip
 * weights as the N dimension of the MMAs; x is staged 4096 columns at a
 * time.  Each output is the fp32 MMA sums of the CTA's 16 warps added in
 * warp order (bitwise reproducible).  Same phase rules and barrier word as
 * mtl_w4_chain. */
int mtl_w4_chain_rows(const mtl_chain_phase_rows* phases, int nphases, int M, int group_size, float norm_eps,
                      uint32_t* barrier, mtl_stream_t stream);

/* y = epilogue(x . W^T) for a prompt of M rows on the 5th-generation tensor
 * cores (tcgen05 GEMM, the prefill path).  Replaces
 * torch._weight_int4pack_mm(x, packed, g, qsz) at M = prompt length as
 * FastMossTTS._layer_q runs it (moss_tts_lite/fast.py:218-270).
 *   tiles     reference-format tiles from mtl_w4_pack_ref (the same packed
 *             weights the decode GEMV reads); W = bf16((q-8)*scale+zero)
 *   x         bf16 [M, ldx], 16-byte aligned, ldx % 8 == 0
 *   epilogue  MTL_EPI_STORE / _RESIDUAL (residual bf16 [M, ldr], may alias
 *             y) / _SWIGLU (gate/up interleaved in 32-column blocks, N/2
 *             outputs per row)
 *   group_size 64/128/256, K % 64 == 0, N % 128 == 0 (else MTL_E_UNSUPPORTED).
 * Needs no scratch. */
int mtl_w4a16_gemm(const uint16_t* x, int ldx, int M, int K, int N, int group_size, const void* tiles, int epilogue,
                   const uint16_t* residual, int ldr, uint16_t* y, int ldy, mtl_stream_t stream);

/* ------------------------------------------------------ decoder step ops */

/* Combined embedding of one decode row per stream (model.py:156-161,
 * fast.py:123-128): out[m] = E_text[ids[m][0]] + E_audio[0][ids[m][1]] + ...
 * + E_audio[31][ids[m][32]], each add rounded to bf16, in that order.
 *   ids       int64 [M, 33] (device)
 *   emb_text  bf16 [text_vocab, hidden];  emb_audio bf16 [32 * 1025, hidden]
 *             (the 32 emb_ext tables stacked)
 *   hidden % 8 == 0.  Out-of-range ids set device-status bit 1 and read row 0. */
int mtl_embed_sum(const int64_t* ids, int M, const uint16_t* emb_text, int text_vocab,
                  const uint16_t* emb_audio, int hidden, uint16_t* out, mtl_stream_t stream);

/* Scratch for mtl_attn_decode (partials + per-KV-head counters); zero-fill
 * once before first use. */
int mtl_attn_scratch_bytes(int streams, int n_heads, int n_kv, int splits, size_t* out);

/* One layer of decode attention for `streams` independent streams, fusing the
 * q/k head RMSNorm (eps 1e-6), RoPE at the device position, the K/V append
 * and split-KV GQA attention over positions [0, pos] (fast.py:138-162,
 * model.py:175-190; replaces the eager F.scaled_dot_product_attention call
 * between graph replays at fast.py:319-324).
 *   qkv        bf16 [streams, (n_heads + 2 n_kv) * 128]: q | k | v projections
 *   q_norm_w, k_norm_w  bf16 [128];  rope_cos/sin bf16 [max_seq, 128]
 *   k_cache, v_cache    bf16 [n_kv, max_seq, 128] of this layer for stream 0;
 *              stream s starts cache_stream_stride elements later (0: the
 *              streams share one cache, see mtl_attn_append)
 *   pos        int64 [streams] (device): position being decoded
 *   splits     KV splits per head (1..64); each covers >= 64 positions
 *   flags      0 or MTL_ATTN_KV_STABLE: pos and cache rows [0, pos) were
 *              written by work that completed before the preceding kernel
 *              started (e.g. the call is one step of a CUDA graph whose
 *              replays follow the steps that wrote them); the kernel then
 *              starts streaming the cache before waiting on the preceding
 *              kernel (programmatic dependent launch)
 *   out        bf16 [streams, n_heads * 128]
 * head_dim must be 128 and n_heads / n_kv <= 8. */
#define MTL_ATTN_KV_STABLE 1
int mtl_attn_decode(const uint16_t* qkv, const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                    const uint16_t* rope_cos, const uint16_t* rope_sin, uint16_t* k_cache, uint16_t* v_cache,
                    long long cache_stream_stride, int max_seq, const int64_t* pos, int streams, int n_heads,
                    int n_kv, int head_dim, int splits, int flags, uint16_t* out, void* scratch,
                    size_t scratch_bytes, mtl_stream_t stream);

/* The K/V append of mtl_attn_decode alone, for `streams` rows at once: k
 * head RMSNorm (eps 1e-6) + RoPE at pos[s] and v, written to cache rows
 * pos[s] (fast.py:138-146).  With cache_stream_stride = 0 all rows share one
 * cache: a prefill chunk appends its rows first, then one mtl_attn_decode
 * call with the same rows as streams (cache_stream_stride 0) attends each
 * row over [0, pos[s]] (it re-writes the same K/V values).  q_out (nullable,
 * bf16 [streams, n_heads, 128]) also receives the rows' q heads after their
 * RMSNorm (q_norm_w) and RoPE, the q operand of a prefill attention over
 * many rows (fast.py:229-235).  No reference counterpart of its own: the
 * reference does this inside _p_pre and _layer_q. */
int mtl_attn_append(const uint16_t* qkv, const uint16_t* q_norm_w, const uint16_t* k_norm_w, const uint16_t* rope_cos,
                    const uint16_t* rope_sin, uint16_t* k_cache, uint16_t* v_cache, long long cache_stream_stride,
                    int max_seq, const int64_t* pos, int streams, int n_heads, int n_kv, int head_dim, uint16_t* q_out,
                    mtl_stream_t stream);

/* y = epilogue(x . W^T) for bf16 weights W [N, K] (the lm heads,
 * model.py:240-295, fast.py:174-194, and bf16 backbone linears: F.linear at
 * model.py:171-196 and the bf16 keeps of gptq.py:689-697).
 * norm_w (nullable) fuses an RMSNorm (model.py:34-40) into the prologue;
 * x_normed (nullable) then receives the normed rows.  Epilogues as for
 * mtl_w4a16_linear (MTL_EPI_*); MTL_EPI_SWIGLU expects the gate and up rows
 * interleaved (row 2j = gate j, row 2j+1 = up j) and writes N/2 outputs; the
 * residual of MTL_EPI_RESIDUAL has row stride ldy and may alias y.  When
 * pad_period > 0 (store epilogue), output column n with
 * n % pad_period == pad_col is set to -inf (AUDIO_PAD_CODE, model.py:292).
 * K <= 8192, K % 8 == 0; M <= 4 with any epilogue (CUDA-core kernel, one
 * warp per output row; each row equals a one-row call bit for bit), or
 * 5 <= M <= 16 with the store epilogue and K % 32 == 0 (tensor-core kernel:
 * m16n8k16 MMAs, W rows as A, the M rows as N; the batched decode step's
 * heads). */
int mtl_bf16_linear(const uint16_t* x, int M, int K, int N, const uint16_t* W, const uint16_t* norm_w, float eps,
                    uint16_t* x_normed, int pad_period, int pad_col, int epilogue, const uint16_t* residual,
                    uint16_t* y, int ldy, mtl_stream_t stream);

/* y[r] = RMSNorm(x[r]) * weight for bf16 rows of length K (Qwen3RMSNorm as
 * restated at model.py:34-40: fp32 statistics, bf16 rounding before and after
 * the weight multiply). */
int mtl_rmsnorm(const uint16_t* x, int rows, int K, int ldx, const uint16_t* weight, float eps, uint16_t* y,
                int ldy, mtl_stream_t stream);

/* out[r] = index of the first maximum of row r (torch.argmax semantics,
 * sampling.py:84-85) of bf16 logits [rows, ld]. */
int mtl_argmax_rows(const uint16_t* x, int rows, int cols, int ld, int64_t* out, mtl_stream_t stream);

/* out[0] = first-index argmax of one bf16 row of `cols` values, ignoring the
 * `n_excluded` (<= 8) column indices listed in HOST array `excluded` (the
 * greedy text decision of generate_fast, fast.py:481-514, with the -inf
 * writes of fast.py:487 and 507-511 folded in).  NaN never wins.  scratch:
 * optional 16 bytes, 16-byte aligned, zeroed once before first use (each
 * call leaves it zeroed); with it, rows of >= 4096 values at a 16-byte
 * aligned x are reduced by CTAs across the whole GPU, without it by one CTA.
 * One scratch must not serve two calls in flight at once. */
int mtl_argmax_masked(const uint16_t* x, int cols, const int32_t* excluded, int n_excluded, int64_t* out,
                      void* scratch, mtl_stream_t stream);

/* Device-side greedy feedback for an audio-phase decode loop with no host
 * round trip, for `streams` independent streams s (stream s's buffers at
 * s times the one-stream size): ids_row[s][1 + j] = argmax of its audio row
 * j (bf16 [32, 1025]), ids_row[s][0] = delay_slot_id if two_logits[s][1] >
 * two_logits[s][0] else gen_slot_id (the greedy 2-way decision of
 * fast.py:481-490), pos[s] += 1.  No counterpart call in the reference (its
 * loop decides on the host). */
int mtl_greedy_feed(const uint16_t* audio_logits, const uint16_t* two_logits, int64_t* ids_row, int64_t* pos,
                    int streams, int gen_slot_id, int delay_slot_id, mtl_stream_t stream);

/* Next input row of generate_fast from one step's decisions, on the device
 * (the reference builds current_input_ids from device tensors and copies it
 * into ids_row, fast.py:573-584).  dec: int64 [33], dec[0] the text decision,
 * then the audio decisions, per channel (dec[1 + j], audio_compact 0) or
 * compact over the channels set in audio_mask (audio_compact 1).
 *   ids_row[0]     = text_const               (text_mode 0)
 *                    dec[0] == 0 ? gen_slot_id : delay_slot_id   (1)
 *                    dec[0]                    (2)
 *   ids_row[1 + j] = channel j's decision if bit j of audio_mask, else pad_code
 *   pos[0]         = pos_value
 * seen_bits (optional, uint32 [2, seen_words]): the row's audio ids are ORed
 * in, channel 0 into set 0 and channels 1..31 into set 1 (the repetition-
 * penalty histories generation_ids[:, :, 1] and [:, :, 2:]).  Running it
 * again with the same arguments leaves the same state. */
int mtl_feed_row(const int64_t* dec, int text_mode, long long text_const, long long gen_slot_id,
                 long long delay_slot_id, unsigned int audio_mask, int audio_compact, long long pad_code,
                 int64_t* ids_row, int64_t* pos, long long pos_value, uint32_t* seen_bits, int seen_words,
                 mtl_stream_t stream);

/* Fused sample_token (sampling.py:70-98) for up to 40 logits rows of one
 * decode step (fast.py:491-545), one draw per row:
 *   row r = logits + row_index[r] * ld (bf16, `cols` values; row_index host
 *   array); x = bf16(x * (1/temperature)); ids in HOST array `excluded`
 *   (<= 8) -> -inf; repetition penalty (sampling.py:36-67) on the ids set in
 *   device bitmap seen_bits[seen_set_of_row[r]] (words_per_set uint32 words;
 *   penalty 1 or seen_bits NULL = off); top-k (top_k <= 0 = off, at most 2048
 *   candidates); top-p on bf16 softmax/cumsum (top_p >= 1 = off); one
 *   categorical draw from Philox4x32-10 keyed by (seed, offset, r).
 *   scan_rows (host array, NULL = all 1): how many rows the reference's
 *   sample_token call held together with row r; PyTorch's CUDA cumsum of
 *   bf16 groups its roundings differently for one-row and multi-row
 *   tensors, and the top-p cut-off follows the same grouping.
 *   out[r] (device int64) = sampled column + out_add.
 *   scratch (device, 16-byte aligned, nullable): rows of >= 16384 columns
 *   with a top-k (the text head) are cut into slices selected by one CTA
 *   each when scratch holds mtl_sample_scratch_bytes(cols, n_rows, top_k)
 *   bytes (MTL_E_SCRATCH if it is smaller); with NULL each row is one CTA.
 *   The draw is the same either way.
 * Candidate sets and probabilities follow the reference's arithmetic; the
 * random stream is this library's own (not torch.multinomial's). */
int mtl_sample_rows(const uint16_t* logits, int ld, int cols, int n_rows, const int32_t* row_index,
                    float temperature, int top_k, float top_p, float repetition_penalty, const uint32_t* seen_bits,
                    int words_per_set, const int32_t* seen_set_of_row, const int32_t* excluded, int n_excluded,
                    const int32_t* scan_rows, uint64_t seed, uint64_t offset, int64_t out_add, int64_t* out,
                    void* scratch, size_t scratch_bytes, mtl_stream_t stream);

/* Scratch bytes of mtl_sample_rows' sliced path for these arguments (0: the
 * rows are sampled one CTA each and need none). */
size_t mtl_sample_scratch_bytes(int cols, int n_rows, int top_k);

/* Round-to-nearest W4 quantisation of a bf16 weight [N, K] exactly as
 * FastMossTTS._quantize (fast.py:85-96) / gptq.rtn_quantize (gptq.py:54-64):
 * q uint8 [N, K] codes and qsz bf16 [K/g, N, 2] = (scale, min + 8 scale). */
int mtl_w4_rtn_quantize(const uint16_t* w, int N, int K, int group_size, uint8_t* q, uint16_t* qsz,
                        mtl_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MTL_B200_H */
