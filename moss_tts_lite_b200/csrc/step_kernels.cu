// Per-step decoder kernels for sm_100a: embedding sum, fused q/k-norm + RoPE
// + KV append + split-KV GQA decode attention, bf16 head GEMV with the final
// RMSNorm fused in, row argmax, and the load-time RTN W4 quantiser.
//
// Every op restates one block of the reference decoder (moss_tts_lite/
// model.py, moss_tts_lite/fast.py) with the reference's bf16 rounding points;
// the file:line of each is cited at the kernel.
#include "common.cuh"

#include <algorithm>

namespace mtl {

constexpr int kHeadDim = 128;
constexpr int kNVQ = 32;
constexpr int kAudioVocab = 1025;

// ---------------------------------------------------------------- embedding
// model.py:156-161 / fast.py:123-128: h = E_text[id0]; h = bf16(h + E_i[id_i])
// for i = 1..32 in order.  One thread owns 8 consecutive hidden elements.
__global__ void __launch_bounds__(256) embed_sum_kernel(const int64_t* __restrict__ ids, int M,
                                                        const uint16_t* __restrict__ emb_text, int text_vocab,
                                                        const uint16_t* __restrict__ emb_audio, int H,
                                                        uint16_t* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int per_row = H / 8;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= M * per_row) return;
  const int m = idx / per_row, c = idx - m * per_row;
  const int64_t* row = ids + (size_t)m * (kNVQ + 1);
  int64_t t0 = row[0];
  if (t0 < 0 || t0 >= text_vocab) {
    flag_error(kDevBadIndex);
    t0 = 0;
  }
  // all 33 row loads are independent: issue them before the ordered sum
  uint4 rows[kNVQ + 1];
  rows[0] = __ldg(reinterpret_cast<const uint4*>(emb_text + (size_t)t0 * H) + c);
#pragma unroll
  for (int i = 0; i < kNVQ; ++i) {
    int64_t a = row[i + 1];
    if (a < 0 || a >= kAudioVocab) {
      flag_error(kDevBadIndex);
      a = 0;
    }
    rows[i + 1] = __ldg(reinterpret_cast<const uint4*>(emb_audio + ((size_t)i * kAudioVocab + a) * H) + c);
  }
  float acc[8];
  {
    const uint32_t u[4] = {rows[0].x, rows[0].y, rows[0].z, rows[0].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] = __uint_as_float(u[q] << 16);
      acc[2 * q + 1] = __uint_as_float(u[q] & 0xFFFF0000u);
    }
  }
#pragma unroll
  for (int i = 1; i <= kNVQ; ++i) {
    const uint32_t w[4] = {rows[i].x, rows[i].y, rows[i].z, rows[i].w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] = round_bf16(acc[2 * q] + __uint_as_float(w[q] << 16));
      acc[2 * q + 1] = round_bf16(acc[2 * q + 1] + __uint_as_float(w[q] & 0xFFFF0000u));
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
    o[q] = (__float_as_uint(acc[2 * q]) >> 16) | (__float_as_uint(acc[2 * q + 1]) & 0xFFFF0000u);
  reinterpret_cast<uint4*>(out + (size_t)m * H)[c] = make_uint4(o[0], o[1], o[2], o[3]);
}

// --------------------------------------------------------------- bf16 GEMV
// y[m][n] = bf16(sum_k x[m][k] W[n][k]) for the lm heads (model.py:240-295,
// fast.py:174-194), optionally with the final RMSNorm fused as prologue
// (each CTA normalises x itself; CTA 0 also stores the normed rows) and with
// column `pad_col` of every `pad_period` outputs forced to -inf
// (AUDIO_PAD_CODE, model.py:292).  One warp per output row, 16-byte loads.
constexpr int kGemvThreads = 256;
constexpr int kGemvMaxK = 8192;
constexpr int kGemvMaxM = 4;
constexpr int kGemvBatch = 8;  // 16-byte weight loads in flight per lane
constexpr int kGemvCtasPerSm = 3;

struct Bf16GemvArgs {
  const uint16_t* x;
  int M, K, N;
  const uint16_t* W;  // [N, K]
  const uint16_t* norm_w;
  float eps;
  uint16_t* x_normed;  // nullable: receives the normed rows (bf16 [M, K])
  int pad_period, pad_col;
  int epi;                   // 0 store, 1 residual add, 2 SwiGLU (rows interleaved gate, up)
  const uint16_t* residual;  // bf16 [M, ldy] for epi 1 (may alias y)
  uint16_t* y;
  int ldy;
};

__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) bf16_gemv_kernel(const Bf16GemvArgs a) {
  extern __shared__ __align__(16) float xs[];  // [M][K] fp32
  __shared__ float red[kGemvThreads / 32][kGemvMaxM];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_launch_dependents();
  pdl_wait();
  for (int m = 0; m < a.M; ++m) {
    const uint16_t* xr = a.x + (size_t)m * a.K;
    float ss = 0.f;
    // elements tid, tid + 256, ... in order; eight loads issued before use
    for (int k0 = tid; k0 < a.K; k0 += 8 * kGemvThreads) {
      uint16_t xb[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) xb[e] = k0 + e * kGemvThreads < a.K ? xr[k0 + e * kGemvThreads] : (uint16_t)0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = k0 + e * kGemvThreads;
        if (k < a.K) {
          const float v = bf16_bits_to_f32(xb[e]);
          xs[(size_t)m * a.K + k] = v;
          ss = fmaf(v, v, ss);
        }
      }
    }
    if (a.norm_w) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp][m] = ss;
    }
  }
  __syncthreads();
  if (a.norm_w) {
    for (int m = 0; m < a.M; ++m) {
      float ss = 0.f;
      for (int w = 0; w < kGemvThreads / 32; ++w) ss += red[w][m];
      const float rinv = rsqrtf(ss / (float)a.K + a.eps);
      for (int k0 = tid; k0 < a.K; k0 += 8 * kGemvThreads) {
        uint16_t nb[8];  // norm weights of this thread's next eight elements, loaded together
#pragma unroll
        for (int e = 0; e < 8; ++e) nb[e] = k0 + e * kGemvThreads < a.K ? __ldg(a.norm_w + k0 + e * kGemvThreads) : (uint16_t)0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int k = k0 + e * kGemvThreads;
          if (k < a.K) {
            // model.py:34-40
            const float v = round_bf16(bf16_bits_to_f32(nb[e]) * round_bf16(xs[(size_t)m * a.K + k] * rinv));
            xs[(size_t)m * a.K + k] = v;
            if (a.x_normed && blockIdx.x == 0) a.x_normed[(size_t)m * a.K + k] = f32_to_bf16_bits(v);
          }
        }
      }
    }
    __syncthreads();
  }
  const int nwarps_total = gridDim.x * (kGemvThreads / 32);
  const int chunks = a.K / 8;  // 16-byte chunks per row
  const int rows_per_out = (a.epi == 2) ? 2 : 1;  // SwiGLU: a warp owns the (gate, up) row pair
  const int nout = a.N / rows_per_out;
  for (int n = blockIdx.x * (kGemvThreads / 32) + warp; n < nout; n += nwarps_total) {
    float res[2][kGemvMaxM];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      if (rr >= rows_per_out) {
#pragma unroll
        for (int m = 0; m < kGemvMaxM; ++m) res[rr][m] = 0.f;
        continue;
      }
      const uint4* wr = reinterpret_cast<const uint4*>(a.W + (size_t)(n * rows_per_out + rr) * a.K);
      float acc[kGemvMaxM];
#pragma unroll
      for (int m = 0; m < kGemvMaxM; ++m) acc[m] = 0.f;
      // all loads of a batch of kGemvBatch chunks are issued before any is
      // used: 4 KB per warp in flight
      for (int c0 = lane; c0 < chunks; c0 += 32 * kGemvBatch) {
        uint4 vb[kGemvBatch];
#pragma unroll
        for (int i = 0; i < kGemvBatch; ++i)
          vb[i] = (c0 + 32 * i < chunks) ? __ldg(wr + c0 + 32 * i) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int i = 0; i < kGemvBatch; ++i) {
          const int c = c0 + 32 * i;
          if (c >= chunks) break;
          const uint32_t u[4] = {vb[i].x, vb[i].y, vb[i].z, vb[i].w};
#pragma unroll
          for (int m = 0; m < kGemvMaxM; ++m) {
            if (m < a.M) {
              const float4 x0 = reinterpret_cast<const float4*>(xs + (size_t)m * a.K)[2 * c];
              const float4 x1 = reinterpret_cast<const float4*>(xs + (size_t)m * a.K)[2 * c + 1];
              float s = acc[m];
              s = fmaf(__uint_as_float(u[0] << 16), x0.x, s);
              s = fmaf(__uint_as_float(u[0] & 0xFFFF0000u), x0.y, s);
              s = fmaf(__uint_as_float(u[1] << 16), x0.z, s);
              s = fmaf(__uint_as_float(u[1] & 0xFFFF0000u), x0.w, s);
              s = fmaf(__uint_as_float(u[2] << 16), x1.x, s);
              s = fmaf(__uint_as_float(u[2] & 0xFFFF0000u), x1.y, s);
              s = fmaf(__uint_as_float(u[3] << 16), x1.z, s);
              s = fmaf(__uint_as_float(u[3] & 0xFFFF0000u), x1.w, s);
              acc[m] = s;
            }
          }
        }
      }
#pragma unroll
      for (int m = 0; m < kGemvMaxM; ++m) res[rr][m] = (m < a.M) ? warp_sum(acc[m]) : 0.f;
    }
    if (lane == 0) {
      for (int m = 0; m < a.M; ++m) {
        uint16_t b;
        if (a.epi == 2) {
          // fast.py:170-171: bf16(silu(gate)) * up, each op rounded to bf16
          const float gt = round_bf16(res[0][m]), up = round_bf16(res[1][m]);
          b = f32_to_bf16_bits(round_bf16(gt / (1.0f + expf(-gt))) * up);
        } else if (a.epi == 1) {
          b = f32_to_bf16_bits(bf16_bits_to_f32(a.residual[(size_t)m * a.ldy + n]) + round_bf16(res[0][m]));
        } else {
          b = f32_to_bf16_bits(res[0][m]);
          if (a.pad_period > 0 && (n % a.pad_period) == a.pad_col) b = 0xFF80u;  // -inf
        }
        a.y[(size_t)m * a.ldy + n] = b;
      }
    }
  }
}

// ----------------------------------------------------------------- RMSNorm
// model.py:34-40 on rows of length K: fp32 mean of squares, bf16(x * rsqrt),
// then bf16(weight * that).  One CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const uint16_t* __restrict__ x, int K, int ldx,
                                                           const uint16_t* __restrict__ w, float eps,
                                                           uint16_t* __restrict__ y, int ldy) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  const uint16_t* xr = x + (size_t)blockIdx.x * ldx;
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float v = bf16_bits_to_f32(xr[k]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float rinv = rsqrtf(tot / (float)K + eps);
  for (int k = threadIdx.x; k < K; k += 256)
    y[(size_t)blockIdx.x * ldy + k] =
        f32_to_bf16_bits(bf16_bits_to_f32(w[k]) * round_bf16(bf16_bits_to_f32(xr[k]) * rinv));
}

// ------------------------------------------------------------------ argmax
// torch.argmax over the last dim of bf16 rows: first index of the maximum
// (NaN-free logits; -inf entries are never selected unless the row is all
// -inf, then index 0).  One CTA per row.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const uint16_t* __restrict__ x, int cols, int ld,
                                                          int64_t* __restrict__ out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  pdl_launch_dependents();
  pdl_wait();
  const uint16_t* r = x + (size_t)blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < cols; c += 256) {
    const float v = bf16_bits_to_f32(r[c]);
    if (v > best) {
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[blockIdx.x] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

// -------------------------------------------------------- masked argmax
// Greedy text decision of generate_fast (fast.py:481-514): first-index argmax
// of one bf16 row with up to 8 indices excluded (the -inf index_fill /
// element writes of fast.py:487,507-511).  One CTA.
struct ExcludeList {
  int n;
  int idx[8];
};

__global__ void __launch_bounds__(256) argmax_masked_kernel(const uint16_t* __restrict__ x, int cols, ExcludeList ex,
                                                            int64_t* __restrict__ out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  pdl_launch_dependents();
  pdl_wait();
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < cols; c += 256) {
    bool skip = false;
#pragma unroll
    for (int e = 0; e < 8; ++e) skip |= (e < ex.n) && (ex.idx[e] == c);
    if (skip) continue;
    const float v = bf16_bits_to_f32(x[c]);
    if (v > best) {
      best = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[0] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

// The same decision spread over the whole GPU for long rows (the 155,648-way
// text head): each CTA reduces its chunks to one 64-bit key (order-preserving
// value bits << 32 | ~index, so the largest key is the largest value at the
// smallest index), merges it with atomicMax into key_slot[0], and the last
// CTA to arrive (counter key_slot[1]) writes the index and re-arms both
// words for the next call.  NaN never wins and -0 ranks as +0, as in the
// one-CTA kernel.  x must be 16-byte aligned.
__device__ __forceinline__ unsigned long long argmax_key(uint32_t bits, int idx) {
  if ((bits & 0x7FFFFFFFu) > 0x7F800000u) return 0ull;  // NaN
  if ((bits & 0x7FFFFFFFu) == 0u) bits = 0u;            // -0 == +0
  const uint32_t ord = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(256) argmax_masked_grid_kernel(const uint16_t* __restrict__ x, int cols,
                                                                 ExcludeList ex, int64_t* __restrict__ out,
                                                                 unsigned long long* key_slot) {
  __shared__ unsigned long long sk[8];
  __shared__ int last;
  pdl_launch_dependents();
  pdl_wait();
  unsigned long long best = 0ull;
  const int nchunks = cols >> 3;
  const int stride = gridDim.x * blockDim.x;
  auto take = [&](uint32_t bits, int idx) {
    bool skip = false;
#pragma unroll
    for (int e = 0; e < 8; ++e) skip |= (e < ex.n) && (ex.idx[e] == idx);
    const unsigned long long k = skip ? 0ull : argmax_key(bits, idx);
    best = k > best ? k : best;
  };
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < nchunks; c += stride) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x) + c);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      take(u[q] << 16, 8 * c + 2 * q);
      take(u[q] & 0xFFFF0000u, 8 * c + 2 * q + 1);
    }
  }
  for (int i = 8 * nchunks + blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += stride)
    take((uint32_t)x[i] << 16, i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = sk[w] > best ? sk[w] : best;
    atomicMax(&key_slot[0], best);
    __threadfence();
    last = atomicAdd(&key_slot[1], 1ull) == (unsigned long long)(gridDim.x - 1);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    const unsigned long long k = atomicExch(&key_slot[0], 0ull);
    atomicExch(&key_slot[1], 0ull);
    out[0] = k ? (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
  }
}

// ---------------------------------------------------------- greedy feed
// Device-side greedy feedback for an autoregressive audio-phase decode loop
// without host round trips: next row = [GEN_SLOT or DELAY_SLOT by the 2-way
// argmax (fast.py:481-490), argmax of each of the 32 audio rows] and
// pos += 1.  One warp per audio row; warp 0 also takes the text decision.
__global__ void __launch_bounds__(1024) greedy_feed_kernel(const uint16_t* __restrict__ la,
                                                           const uint16_t* __restrict__ two, int64_t* ids,
                                                           int64_t* pos, int gen_slot, int delay_slot) {
  // one CTA per stream: stream blockIdx.x's logits, row and position
  la += (size_t)blockIdx.x * kNVQ * kAudioVocab;
  two += 2 * (size_t)blockIdx.x;
  ids += (size_t)blockIdx.x * (kNVQ + 1);
  pos += blockIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < kNVQ) {
    const uint16_t* r = la + (size_t)warp * kAudioVocab;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < kAudioVocab; c += 32) {
      const float v = bf16_bits_to_f32(r[c]);
      if (v > best) {
        best = v;
        bi = c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) ids[1 + warp] = (bi == 0x7fffffff) ? 0 : bi;
  }
  if (threadIdx.x == 0) {
    const float a = bf16_bits_to_f32(two[0]), b = bf16_bits_to_f32(two[1]);
    ids[0] = (b > a) ? delay_slot : gen_slot;
    pos[0] += 1;
  }
}

// Next input row of generate_fast built on the device from the step's
// decisions (the reference builds current_input_ids with device tensors,
// fast.py:573-584): dec = [text decision, audio decisions], the audio ones
// either per channel (dec[1 + j]) or compact over the sampled channels
// (dec[1 + rank of j in audio_mask]).  Also sets pos and ORs the new audio
// ids into the repetition-penalty sets (channel 0 -> set 0, 1..31 -> set 1).
// Re-running it with the same inputs writes the same row (the OR is
// idempotent), which the pipelined host loop relies on.
struct FeedArgs {
  const int64_t* dec;
  int64_t* ids;
  int64_t* pos_dev;
  uint32_t* seen;
  long long pos, text_const, gen_slot, delay_slot, pad_code;
  unsigned int audio_mask;
  int text_mode, audio_compact, seen_words;
};

__global__ void __launch_bounds__(32) feed_row_kernel(const FeedArgs f) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = threadIdx.x;
  const unsigned bit = 1u << j;
  int64_t tok = f.pad_code;
  if (f.audio_mask & bit) tok = f.dec[1 + (f.audio_compact ? __popc(f.audio_mask & (bit - 1u)) : j)];
  f.ids[1 + j] = tok;
  if (f.seen && tok >= 0 && tok < (int64_t)f.seen_words * 32)
    atomicOr(f.seen + (j ? f.seen_words : 0) + (int)(tok >> 5), 1u << (tok & 31));
  if (j == 0) {
    int64_t t = f.text_const;
    if (f.text_mode == 1) t = f.dec[0] == 0 ? f.gen_slot : f.delay_slot;
    if (f.text_mode == 2) t = f.dec[0];
    f.ids[0] = t;
    f.pos_dev[0] = f.pos;
  }
}

// -------------------------------------------------------- RTN quantisation
// fast.py:85-96 / gptq.py:35-64: per (row n, group G) of a bf16 weight
// [N, K]: mx/mn over the group, s = clamp((mx - mn) * (1/15), min=1e-6),
// q = clamp(round_half_even((w - mn) / s), 0, 15), and
// qsz[G][n] = (bf16(s), bf16(mn + 8 s)).  One warp per (n, G).
__global__ void __launch_bounds__(256) rtn_quantize_kernel(const uint16_t* __restrict__ w, int N, int K, int g,
                                                           uint8_t* __restrict__ q, uint16_t* __restrict__ qsz) {
  const int KT = K / g;
  const int job = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (job >= N * KT) return;
  const int n = job / KT, G = job - n * KT;
  const uint16_t* src = w + (size_t)n * K + (size_t)G * g;
  float mx = -INFINITY, mn = INFINITY;
  for (int i = lane; i < g; i += 32) {
    const float v = bf16_bits_to_f32(src[i]);
    mx = fmaxf(mx, v);
    mn = fminf(mn, v);
  }
  mx = warp_max(mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  // PyTorch on CUDA divides by a Python scalar as a multiply by its float
  // reciprocal; the reference's W4 path runs on CUDA.
  const float s = fmaxf(__fmul_rn(__fsub_rn(mx, mn), 1.0f / 15.0f), 1e-6f);
  for (int i = lane; i < g; i += 32) {
    const float v = bf16_bits_to_f32(src[i]);
    const float r = rintf(__fdiv_rn(__fsub_rn(v, mn), s));
    q[(size_t)n * K + (size_t)G * g + i] = (uint8_t)fminf(fmaxf(r, 0.f), 15.f);
  }
  if (lane == 0) {
    qsz[((size_t)G * N + n) * 2 + 0] = f32_to_bf16_bits(s);
    qsz[((size_t)G * N + n) * 2 + 1] = f32_to_bf16_bits(__fadd_rn(mn, __fmul_rn(8.0f, s)));
  }
}

// ------------------------------------------------------------------ host side

namespace {
cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute* attr,
                           int use_pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl ? 1 : 0;
  return cfg;
}
}  // namespace

cudaError_t launch_embed_sum(const int64_t* ids, int M, const uint16_t* emb_text, int text_vocab,
                             const uint16_t* emb_audio, int H, uint16_t* out, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  const int total = M * (H / 8);
  cudaLaunchConfig_t cfg = pdl_cfg(dim3((total + 255) / 256), dim3(256), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, embed_sum_kernel, ids, M, emb_text, text_vocab, emb_audio, H, out);
}

cudaError_t launch_bf16_gemv(const Bf16GemvArgs& a, int num_sms, cudaStream_t s, int use_pdl) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(bf16_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kGemvMaxM * kGemvMaxK * 4);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int rows_per_cta = kGemvThreads / 32;
  const int nout = (a.epi == 2) ? a.N / 2 : a.N;
  const int grid = std::max(1, std::min((nout + rows_per_cta - 1) / rows_per_cta, num_sms * kGemvCtasPerSm));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(grid), dim3(kGemvThreads), (size_t)a.M * a.K * 4, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, bf16_gemv_kernel, a);
}

cudaError_t launch_argmax_rows(const uint16_t* x, int rows, int cols, int ld, int64_t* out, cudaStream_t s,
                               int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(256), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, argmax_rows_kernel, x, cols, ld, out);
}

cudaError_t launch_rmsnorm_rows(const uint16_t* x, int rows, int K, int ldx, const uint16_t* w, float eps,
                                uint16_t* y, int ldy, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(256), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, rmsnorm_rows_kernel, x, K, ldx, w, eps, y, ldy);
}

cudaError_t launch_argmax_masked(const uint16_t* x, int cols, const int* excl, int n_excl, int64_t* out,
                                 void* scratch, int num_sms, cudaStream_t s, int use_pdl) {
  ExcludeList ex{};
  ex.n = n_excl;
  for (int i = 0; i < n_excl && i < 8; ++i) ex.idx[i] = excl[i];
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(256), 0, s, attr, use_pdl);
  if (scratch && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && cols >= 4096) {
    const int grid = std::max(1, std::min(num_sms, (cols / 8 + 255) / 256));
    cudaLaunchConfig_t gcfg = pdl_cfg(dim3(grid), dim3(256), 0, s, attr, use_pdl);
    return cudaLaunchKernelEx(&gcfg, argmax_masked_grid_kernel, x, cols, ex, out,
                              reinterpret_cast<unsigned long long*>(scratch));
  }
  return cudaLaunchKernelEx(&cfg, argmax_masked_kernel, x, cols, ex, out);
}

cudaError_t launch_greedy_feed(const uint16_t* la, const uint16_t* two, int64_t* ids, int64_t* pos, int streams,
                               int gen_slot, int delay_slot, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(streams), dim3(kNVQ * 32), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, greedy_feed_kernel, la, two, ids, pos, gen_slot, delay_slot);
}

cudaError_t launch_feed_row(const FeedArgs& f, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(kNVQ), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, feed_row_kernel, f);
}

cudaError_t launch_rtn_quantize(const uint16_t* w, int N, int K, int g, uint8_t* q, uint16_t* qsz, cudaStream_t s) {
  const int jobs = N * (K / g);
  rtn_quantize_kernel<<<(jobs + 7) / 8, 256, 0, s>>>(w, N, K, g, q, qsz);
  return cudaGetLastError();
}

}  // namespace mtl
