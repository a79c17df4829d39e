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

// ----------------------------------------------------- decode attention
// Fused _p_pre tail + _p_attn (fast.py:138-162, model.py:175-190) for one
// layer and one decode position per stream:
//   q/k head RMSNorm (model.py:34-40 over head_dim), RoPE
//   bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)) at position pos, K/V append
//   at pos, then softmax(q k^T / sqrt(128)) v over positions [0, pos] for
//   the n_rep query heads sharing each KV head (GQA).
// Grid: (n_kv, splits, streams).  Split p covers a contiguous slice of
// [0, pos]; each writes (max, sum, o[128]) per query head to scratch and the
// last split to finish (atomic counter per KV head) merges them in split
// order.  Probabilities exp(s - split_max) are rounded to bf16 before P.V
// with fp32 accumulation (the rounding point of PyTorch's flash-style SDPA).
struct AttnArgs {
  const uint16_t* qkv;  // bf16 [streams, (nh + 2 nkv) * 128]
  const uint16_t* q_norm_w;
  const uint16_t* k_norm_w;
  const uint16_t* rope_cos;  // bf16 [max_seq, 128]
  const uint16_t* rope_sin;
  uint16_t* k_cache;  // bf16 [streams][nkv][max_seq][128] for this layer (stream stride given)
  uint16_t* v_cache;
  long long cache_stream_stride;  // elements between streams (0 for one stream)
  int max_seq;
  const int64_t* pos;  // [streams] decode position of each stream
  int nh, nkv, splits;
  uint16_t* out;  // bf16 [streams, nh * 128]
  float* partials;  // [streams][nkv][splits][n_rep][2 + 128]
  int* counters;    // [streams][nkv]
  float scale;
};

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxRep = 8;
constexpr int kAttnTile = 32;       // positions per tile (4 warps x 8)
constexpr int kAttnMinChunk = 32;   // positions per split at least

__device__ __forceinline__ float rope_rot(const float* x, int d) {
  // rotate_half (model.py:42-44): [-x2, x1]
  return d < kHeadDim / 2 ? -x[d + kHeadDim / 2] : x[d - kHeadDim / 2];
}

// Registers of one tile: each lane holds 32 K dims of one position (scores)
// and 4 V dims of 8 positions (P.V).
struct KVTile {
  uint4 k[4];
  uint2 v[8];
};

__device__ __forceinline__ void load_tile(KVTile& t, const uint16_t* kc, const uint16_t* vc, int base, int hi,
                                          int pos, int warp, int lane) {
  const int ps = lane >> 2, dg = lane & 3;
  const int sk = base + warp * 8 + ps;
  if (sk < hi && sk != pos) {
    const uint4* kp = reinterpret_cast<const uint4*>(kc + (size_t)sk * kHeadDim + dg * 32);
#pragma unroll
    for (int j = 0; j < 4; ++j) t.k[j] = __ldg(kp + j);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int sv = base + warp * 8 + i;
    if (sv < hi && sv != pos) t.v[i] = __ldg(reinterpret_cast<const uint2*>(vc + (size_t)sv * kHeadDim) + lane);
  }
}

__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  __shared__ float sq[kAttnMaxRep][kHeadDim];  // normed + roped q (bf16 values)
  __shared__ float sk[kHeadDim], sv[kHeadDim];
  __shared__ float sc[kAttnMaxRep][kAttnTile];
  __shared__ float so[4][kAttnMaxRep][kHeadDim];  // per-warp P.V partials
  __shared__ float mrun_s[kAttnMaxRep], alpha_s[kAttnMaxRep];
  __shared__ int last_flag;
  const int h = blockIdx.x, sp = blockIdx.y, st = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rep = a.nh / a.nkv;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t pos64 = a.pos[st];
  if (pos64 < 0 || pos64 >= a.max_seq) {
    if (tid == 0) flag_error(kDevBadIndex);
    return;
  }
  const int pos = (int)pos64, s1 = pos + 1;
  const int chunk = max(kAttnMinChunk, (s1 + a.splits - 1) / a.splits);
  const int lo = min(sp * chunk, s1), hi = min(lo + chunk, s1);
  const int n = hi - lo;
  uint16_t* kc = a.k_cache + st * a.cache_stream_stride + (size_t)h * a.max_seq * kHeadDim;
  uint16_t* vc = a.v_cache + st * a.cache_stream_stride + (size_t)h * a.max_seq * kHeadDim;
  float* part = a.partials + ((((size_t)st * a.nkv + h) * a.splits + sp) * rep) * (2 + kHeadDim);

  if (n > 0) {
    // first tile's loads go out before the q/k prologue (they do not depend on it)
    KVTile cur;
    load_tile(cur, kc, vc, lo, hi, pos, warp, lane);
    const uint16_t* qkv = a.qkv + (size_t)st * (a.nh + 2 * a.nkv) * kHeadDim;
    const uint16_t* cs = a.rope_cos + (size_t)pos * kHeadDim;
    const uint16_t* sn = a.rope_sin + (size_t)pos * kHeadDim;
    // --- q/k RMSNorm over head_dim + RoPE; one warp per head (rep q heads + k)
    for (int r = warp; r <= rep; r += 4) {
      const uint16_t* src = (r < rep) ? qkv + (size_t)(h * rep + r) * kHeadDim : qkv + (size_t)(a.nh + h) * kHeadDim;
      const uint16_t* nw = (r < rep) ? a.q_norm_w : a.k_norm_w;
      float x[4];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[j] = bf16_bits_to_f32(src[lane + 32 * j]);
        ss = fmaf(x[j], x[j], ss);
      }
      ss = warp_sum(ss);
      const float rinv = rsqrtf(ss / (float)kHeadDim + 1e-6f);
      float* dst = (r < rep) ? sq[r] : sk;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        dst[d] = round_bf16(bf16_bits_to_f32(nw[d]) * round_bf16(x[j] * rinv));
      }
      __syncwarp();
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        const float t1 = round_bf16(dst[d] * bf16_bits_to_f32(cs[d]));
        const float t2 = round_bf16(rope_rot(dst, d) * bf16_bits_to_f32(sn[d]));
        y[j] = round_bf16(t1 + t2);
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = y[j];
    }
    // v is used as is (fast.py:137,140)
    sv[tid] = bf16_bits_to_f32(qkv[(size_t)(a.nh + a.nkv + h) * kHeadDim + tid]);
    if (tid < kAttnMaxRep) mrun_s[tid] = -INFINITY;
    __syncthreads();
    // K/V append at pos (fast.py:145-146) by the split holding pos; every split
    // uses sk / sv for position pos instead of re-reading the cache.
    if (hi == s1) {
      kc[(size_t)pos * kHeadDim + tid] = f32_to_bf16_bits(sk[tid]);
      vc[(size_t)pos * kHeadDim + tid] = f32_to_bf16_bits(sv[tid]);
    }

    const int ps = lane >> 2, dg = lane & 3;
    float o[kAttnMaxRep][4];
#pragma unroll
    for (int r = 0; r < kAttnMaxRep; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[r][c] = 0.f;
    float lsum[kAttnMaxRep];
#pragma unroll
    for (int r = 0; r < kAttnMaxRep; ++r) lsum[r] = 0.f;

    for (int base = lo; base < hi; base += kAttnTile) {
      KVTile nxt;
      if (base + kAttnTile < hi) load_tile(nxt, kc, vc, base + kAttnTile, hi, pos, warp, lane);
      // --- scores of this tile: lane = (position ps, dim group dg)
      const int s = base + warp * 8 + ps;
      float kv[32];
      if (s == pos) {
#pragma unroll
        for (int j = 0; j < 32; ++j) kv[j] = sk[dg * 32 + j];
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t u[4] = {cur.k[j].x, cur.k[j].y, cur.k[j].z, cur.k[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            kv[8 * j + 2 * q] = __uint_as_float(u[q] << 16);
            kv[8 * j + 2 * q + 1] = __uint_as_float(u[q] & 0xFFFF0000u);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kAttnMaxRep; ++r) {
        if (r < rep) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) acc = fmaf(sq[r][dg * 32 + j], kv[j], acc);
          acc += __shfl_xor_sync(0xffffffffu, acc, 1);
          acc += __shfl_xor_sync(0xffffffffu, acc, 2);
          if (dg == 0) sc[r][warp * 8 + ps] = (s < hi) ? acc * a.scale : -INFINITY;
        }
      }
      __syncthreads();
      // --- running max per head (warp r owns head r..), rescale factor
      for (int r = warp; r < rep; r += 4) {
        const float tmx = warp_max(sc[r][lane]);
        if (lane == 0) {
          const float mnew = fmaxf(mrun_s[r], tmx);
          alpha_s[r] = (mrun_s[r] == -INFINITY) ? 0.f : expf(mrun_s[r] - mnew);
          mrun_s[r] = mnew;
        }
      }
      __syncthreads();
      // --- probabilities exp(s - m) rounded to bf16 (flash-style), P.V over
      //     this warp's 8 positions for 4 dims per lane
      const int dbase = lane * 4;
#pragma unroll
      for (int r = 0; r < kAttnMaxRep; ++r) {
        if (r < rep) {
          const float al = alpha_s[r], m = mrun_s[r];
#pragma unroll
          for (int c = 0; c < 4; ++c) o[r][c] *= al;
          lsum[r] *= al;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int sp2 = base + warp * 8 + i;
            if (sp2 < hi) {
              const float pf = expf(sc[r][warp * 8 + i] - m);
              lsum[r] += pf;
              const float pb = round_bf16(pf);
              float vv[4];
              if (sp2 == pos) {
#pragma unroll
                for (int c = 0; c < 4; ++c) vv[c] = sv[dbase + c];
              } else {
                vv[0] = __uint_as_float(cur.v[i].x << 16);
                vv[1] = __uint_as_float(cur.v[i].x & 0xFFFF0000u);
                vv[2] = __uint_as_float(cur.v[i].y << 16);
                vv[3] = __uint_as_float(cur.v[i].y & 0xFFFF0000u);
              }
#pragma unroll
              for (int c = 0; c < 4; ++c) o[r][c] = fmaf(pb, vv[c], o[r][c]);
            }
          }
        }
      }
      __syncthreads();  // sc / alpha reuse
      if (base + kAttnTile < hi) cur = nxt;
    }
    // --- combine the 4 warps' partials (same running max) and publish
    for (int r = 0; r < rep; ++r) {
#pragma unroll
      for (int c = 0; c < 4; ++c) so[warp][r][lane * 4 + c] = o[r][c];
    }
    float* lred = &sc[0][0];  // reuse: [4 warps][rep] row sums
    for (int r = 0; r < rep; ++r) {
      // lsum is identical across lanes of a warp (every lane saw the same p's)
      if (lane == 0) lred[warp * kAttnMaxRep + r] = lsum[r];
    }
    __syncthreads();
    for (int r = 0; r < rep; ++r) {
      part[(size_t)r * (2 + kHeadDim) + 2 + tid] = so[0][r][tid] + so[1][r][tid] + so[2][r][tid] + so[3][r][tid];
      if (tid == 0) {
        part[(size_t)r * (2 + kHeadDim) + 0] = mrun_s[r];
        part[(size_t)r * (2 + kHeadDim) + 1] = lred[0 * kAttnMaxRep + r] + lred[1 * kAttnMaxRep + r] +
                                                lred[2 * kAttnMaxRep + r] + lred[3 * kAttnMaxRep + r];
      }
    }
  } else if (tid < rep) {
    part[(size_t)tid * (2 + kHeadDim) + 0] = -INFINITY;
    part[(size_t)tid * (2 + kHeadDim) + 1] = 0.f;
  }
  // --- last split to finish merges all splits in order
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    int* ctr = a.counters + (size_t)st * a.nkv + h;
    const int old = atomicAdd(ctr, 1);
    last_flag = (old == a.splits - 1);
    if (last_flag) {
      __threadfence();
      *ctr = 0;
    }
  }
  __syncthreads();
  if (!last_flag) return;
  // --- merge: all (max, sum) pairs in one round of independent loads, the
  //     rescale factors per split, then each thread's 128-dim slice with its
  //     partial loads issued back to back.  Only splits that held positions.
  __shared__ float mg_m[kAttnMaxRep * 64], mg_l[kAttnMaxRep * 64], mg_lsum[kAttnMaxRep];
  const int nact = min(a.splits, (s1 + chunk - 1) / chunk);
  const float* basep = a.partials + (((size_t)st * a.nkv + h) * a.splits * rep) * (2 + kHeadDim);
  for (int i = tid; i < rep * nact; i += kAttnThreads) {
    const int r = i / nact, j = i - r * nact;
    const float* pj = basep + ((size_t)j * rep + r) * (2 + kHeadDim);
    mg_m[r * 64 + j] = __ldcg(pj);
    mg_l[r * 64 + j] = __ldcg(pj + 1);
  }
  __syncthreads();
  for (int r = warp; r < rep; r += 4) {
    float m = -INFINITY;
    for (int j = lane; j < nact; j += 32) m = fmaxf(m, mg_m[r * 64 + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < nact; j += 32) {
      const float mj = mg_m[r * 64 + j];
      const float f = (mj == -INFINITY) ? 0.f : expf(mj - m);
      mg_m[r * 64 + j] = f;  // becomes the rescale factor of split j
      l = fmaf(mg_l[r * 64 + j], f, l);
    }
    l = warp_sum(l);
    if (lane == 0) mg_lsum[r] = l;
  }
  __syncthreads();
  for (int r = 0; r < rep; ++r) {
    float acc = 0.f;
#pragma unroll 8
    for (int j = 0; j < nact; ++j)
      acc = fmaf(__ldcg(basep + ((size_t)j * rep + r) * (2 + kHeadDim) + 2 + tid), mg_m[r * 64 + j], acc);
    a.out[(size_t)st * a.nh * kHeadDim + (size_t)(h * rep + r) * kHeadDim + tid] = f32_to_bf16_bits(acc / mg_lsum[r]);
  }
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

__global__ void __launch_bounds__(kGemvThreads) bf16_gemv_kernel(const Bf16GemvArgs a) {
  extern __shared__ __align__(16) float xs[];  // [M][K] fp32
  __shared__ float red[kGemvThreads / 32][kGemvMaxM];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_launch_dependents();
  pdl_wait();
  for (int m = 0; m < a.M; ++m) {
    const uint16_t* xr = a.x + (size_t)m * a.K;
    float ss = 0.f;
    for (int k = tid; k < a.K; k += kGemvThreads) {
      const float v = bf16_bits_to_f32(xr[k]);
      xs[(size_t)m * a.K + k] = v;
      ss = fmaf(v, v, ss);
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
      for (int k = tid; k < a.K; k += kGemvThreads) {
        // model.py:34-40
        const float v = round_bf16(bf16_bits_to_f32(a.norm_w[k]) * round_bf16(xs[(size_t)m * a.K + k] * rinv));
        xs[(size_t)m * a.K + k] = v;
        if (a.x_normed && blockIdx.x == 0) a.x_normed[(size_t)m * a.K + k] = f32_to_bf16_bits(v);
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
    for (int rr = 0; rr < rows_per_out; ++rr) {
      const uint4* wr = reinterpret_cast<const uint4*>(a.W + (size_t)(n * rows_per_out + rr) * a.K);
      float acc[kGemvMaxM];
#pragma unroll
      for (int m = 0; m < kGemvMaxM; ++m) acc[m] = 0.f;
#pragma unroll 4
      for (int c = lane; c < chunks; c += 32) {
        const uint4 v = __ldg(wr + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
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

// ---------------------------------------------------------- greedy feed
// Device-side greedy feedback for an autoregressive audio-phase decode loop
// without host round trips: next row = [GEN_SLOT or DELAY_SLOT by the 2-way
// argmax (fast.py:481-490), argmax of each of the 32 audio rows] and
// pos += 1.  One warp per audio row; warp 0 also takes the text decision.
__global__ void __launch_bounds__(1024) greedy_feed_kernel(const uint16_t* __restrict__ la,
                                                           const uint16_t* __restrict__ two, int64_t* ids,
                                                           int64_t* pos, int gen_slot, int delay_slot) {
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

cudaError_t launch_attn_decode(const AttnArgs& a, int streams, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.nkv, a.splits, streams), dim3(kAttnThreads), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel, a);
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
  const int grid = std::max(1, std::min((nout + rows_per_cta - 1) / rows_per_cta, num_sms * 4));
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
                                 cudaStream_t s, int use_pdl) {
  ExcludeList ex{};
  ex.n = n_excl;
  for (int i = 0; i < n_excl && i < 8; ++i) ex.idx[i] = excl[i];
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(256), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, argmax_masked_kernel, x, cols, ex, out);
}

cudaError_t launch_greedy_feed(const uint16_t* la, const uint16_t* two, int64_t* ids, int64_t* pos, int gen_slot,
                               int delay_slot, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(1), dim3(kNVQ * 32), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, greedy_feed_kernel, la, two, ids, pos, gen_slot, delay_slot);
}

cudaError_t launch_rtn_quantize(const uint16_t* w, int N, int K, int g, uint8_t* q, uint16_t* qsz, cudaStream_t s) {
  const int jobs = N * (K / g);
  rtn_quantize_kernel<<<(jobs + 7) / 8, 256, 0, s>>>(w, N, K, g, q, qsz);
  return cudaGetLastError();
}

}  // namespace mtl
