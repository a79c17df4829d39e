// Decode attention for sm_100a: the _p_pre tail and _p_attn of the
// reference (fast.py:138-162, model.py:175-190) for one layer and one decode
// position per stream, as one kernel:
//
//   q/k head RMSNorm over head_dim (model.py:34-40), RoPE
//   bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)) at position pos, K/V append
//   at pos, then softmax(q k^T / sqrt(128)) v over positions [0, pos] for the
//   n_rep query heads sharing each KV head (GQA).
//
// Grid (n_kv, splits, streams), 8 warps per CTA in two pipelines of 4 that
// take alternate tiles.  Split p owns a contiguous, 64-aligned slice of
// [0, pos]; its K/V rows stream into a 4-stage shared memory ring as
// 64-position x 64-dim tensor tiles (TMA, 128-byte swizzle, so the fragment
// loads below are free of bank conflicts).  Each warp of a pipeline owns 16
// positions of a tile and computes on the tensor cores (mma.sync m16n8k16,
// bf16 in, fp32 accumulate):
//   S^T[16 pos x 8 heads] = K[16 pos x 128] . Q^T[128 x 8 heads]
//   O^T[128 x 8 heads]   += V^T[128 x 16 pos] . P^T[16 pos x 8 heads]
// with an online softmax per warp; probabilities exp(s - m) are rounded to
// bf16 before P.V and the normaliser sums the unrounded values (the rounding
// point of PyTorch's flash-style SDPA).  The eight warps, then the splits
// are merged with the usual max/sum rescaling: the last-arriving CTA of a
// head fetches every split's record with one bulk copy into its idle tile
// ring (one round trip whatever the split count) and merges them in split
// order from shared memory.
#include "common.cuh"

#include <cuda.h>

namespace mtl {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = 8;   // two pipelines of 4 warps, alternate tiles
constexpr int kAttnGroupThreads = 128;
constexpr int kAttnMaxRep = 8;
constexpr int kAttnTile = 64;                              // positions per tile, 16 per warp of a pipeline
constexpr int kAttnStages = 4;   // ring stages up to 16 splits; 3 (two CTAs per SM) above
// Positions per split: at least kAttnMinChunk, and a cache of up to
// kAttnSoloMax positions goes to one CTA per KV head with no split merge
// (measured on B200 over cache lengths 140..4200: lowest step time).
constexpr int kAttnMinChunk = 128;
constexpr int kAttnSoloMax = 256;
constexpr int kAttnBoxBytes = kAttnTile * 128;             // 64 rows x 64 dims x bf16
constexpr int kAttnStageBytes = 4 * kAttnBoxBytes;         // K dims 0-63, K 64-127, V 0-63, V 64-127
__host__ __device__ constexpr int attn_dyn_smem(int stages) { return stages * kAttnStageBytes + 1024; }  // + swizzle alignment
constexpr unsigned kAttnKvStable = 1u;  // rows [0, pos) are final before this grid starts
constexpr int kAttnRec = 132;           // floats per (split, head) partial: o[128], max, sum, pad

struct AttnArgs {
  const uint16_t* qkv;  // bf16 [streams, (nh + 2 nkv) * 128]
  const uint16_t* q_norm_w;
  const uint16_t* k_norm_w;
  const uint16_t* rope_cos;  // bf16 [max_seq, 128]
  const uint16_t* rope_sin;
  uint16_t* k_cache;  // bf16 [streams][nkv][max_seq][128] for this layer (stream stride given)
  uint16_t* v_cache;
  long long cache_stream_stride;  // elements between streams
  int max_seq;
  const int64_t* pos;  // [streams] decode position of each stream
  int nh, nkv, splits;
  unsigned flags;
  uint16_t* out;    // bf16 [streams, nh * 128]
  float* partials;  // [streams][nkv][splits][n_rep][kAttnRec]
  int* counters;    // [streams][nkv]
  float scale;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 3-D tensor tile global -> shared, completing on an mbarrier (no multicast).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of (row, 16-byte chunk) inside one 128-byte-swizzled box.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int kAttnStages>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const AttnArgs a) {
  extern __shared__ uint8_t attn_dyn[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kAttnStages];
  __shared__ __align__(8) uint64_t mrg;  // the split records of the merge landed
  __shared__ __align__(16) uint16_t sq[kAttnMaxRep][kHeadDim];      // normed + roped q (bf16), zero padded
  __shared__ __align__(16) uint16_t snew[2][kHeadDim];              // k, v of position pos (bf16)
  __shared__ __align__(16) uint16_t pbuf[kAttnWarps][kAttnMaxRep][16];
  __shared__ float wm[kAttnWarps][kAttnMaxRep], wl[kAttnWarps][kAttnMaxRep];
  // the warps' partial outputs of the merge, in the ring once the tiles are
  // consumed (keeps the static shared memory small: two CTAs fit an SM)
  float(*wo)[kAttnMaxRep][kHeadDim] = reinterpret_cast<float(*)[kAttnMaxRep][kHeadDim]>(ring);
  __shared__ int sh_flag[2];  // [0] bail (a wait timed out), [1] last split
  __shared__ int last_tile[kAttnStages];  // tile last issued into each stage (drain after a bail)

  const int h = blockIdx.x, sp = blockIdx.y, st = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = warp >> 2, tg = tid & (kAttnGroupThreads - 1);  // pipeline, thread in it
  const int g = lane >> 2, t = lane & 3;
  const int rep = a.nh / a.nkv;
  const bool early = (a.flags & kAttnKvStable) != 0;
  pdl_launch_dependents();

  if (tid == 0) {
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&full[s], 1);
    mbar_init(&mrg, 1);
    fence_mbar_init();
    sh_flag[0] = 0;
    sh_flag[1] = 0;
  }
  for (int i = tid; i < kAttnMaxRep * kHeadDim; i += kAttnThreads) (&sq[0][0])[i] = 0;
  __syncthreads();

  // ---- the split's positions (pos is final before this grid in both modes:
  //      with kAttnKvStable the caller guarantees it, otherwise after the wait)
  int pos = -1, lo = 0, hi = 0, ntiles = 0, s1 = 0, chunk = kAttnTile;
  auto plan = [&]() {
    const int64_t p64 = a.pos[st];
    if (p64 < 0 || p64 >= a.max_seq) {
      pos = -1;
      return;
    }
    pos = (int)p64;
    s1 = pos + 1;
    const int per = (s1 + a.splits - 1) / a.splits;
    chunk = s1 <= kAttnSoloMax ? kAttnSoloMax : max(kAttnMinChunk, (per + kAttnTile - 1) / kAttnTile * kAttnTile);
    lo = min(sp * chunk, s1);
    hi = min(lo + chunk, s1);
    ntiles = (hi - lo + kAttnTile - 1) / kAttnTile;
  };
  const int row0 = h * a.max_seq;  // first cache row of this KV head in the 2-D view
  auto issue = [&](int i) {         // one thread: tile i into stage i % S
    uint8_t* sb = ring + (size_t)(i % kAttnStages) * kAttnStageBytes;
    uint64_t* bar = &full[i % kAttnStages];
    last_tile[i % kAttnStages] = i;
    const int y = row0 + lo + i * kAttnTile;
    const int z = a.cache_stream_stride ? st : 0;  // streams may share one cache (prefill rows)
    mbar_arrive_expect_tx(bar, kAttnStageBytes);
    tma_load_3d(sb + 0 * kAttnBoxBytes, &tm_k, 0, y, z, bar);
    tma_load_3d(sb + 1 * kAttnBoxBytes, &tm_k, 64, y, z, bar);
    tma_load_3d(sb + 2 * kAttnBoxBytes, &tm_v, 0, y, z, bar);
    tma_load_3d(sb + 3 * kAttnBoxBytes, &tm_v, 64, y, z, bar);
  };
  // layer constants: norm weights and the RoPE row of pos (lane's dims lane + 32 j)
  float qw[4], kw[4], cv[4], sv[4];
  auto load_consts = [&]() {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = lane + 32 * j;
      qw[j] = bf16_bits_to_f32(a.q_norm_w[d]);
      kw[j] = bf16_bits_to_f32(a.k_norm_w[d]);
      cv[j] = bf16_bits_to_f32(a.rope_cos[(size_t)pos * kHeadDim + d]);
      sv[j] = bf16_bits_to_f32(a.rope_sin[(size_t)pos * kHeadDim + d]);
    }
  };
  int issued = 0;
  if (early) {
    plan();
    if (tid == 0 && pos >= 0)
      for (; issued < min(kAttnStages, ntiles); ++issued) issue(issued);
    if (pos >= 0 && lo < hi) load_consts();
  }
  pdl_wait();
  if (!early) {
    plan();
    if (tid == 0 && pos >= 0) {
      fence_proxy_async_smem();
      for (; issued < min(kAttnStages, ntiles); ++issued) issue(issued);
    }
    if (pos >= 0 && lo < hi) load_consts();
  }
  if (pos < 0) {
    if (tid == 0) flag_error(kDevBadIndex);
    return;  // nothing was issued
  }
  const int n = hi - lo;
  // one non-empty split: it writes the output itself, the others just exit
  const bool solo = (s1 + chunk - 1) / chunk == 1;
  if (solo && n == 0) return;
  uint16_t* kc = a.k_cache + st * a.cache_stream_stride + (size_t)row0 * kHeadDim;
  uint16_t* vc = a.v_cache + st * a.cache_stream_stride + (size_t)row0 * kHeadDim;
  float* part = a.partials + ((((size_t)st * a.nkv + h) * a.splits + sp) * rep) * kAttnRec;
  const bool has_pos = (n > 0) && (hi == s1);

  if (n > 0) {
    // ---- q (and, for the split holding pos, k and v): all loads first.
    //      warp w: q heads w and w + 4; warp 0 also k, warp 1 also v.
    const uint16_t* qkv = a.qkv + (size_t)st * (a.nh + 2 * a.nkv) * kHeadDim;
    float x[3][4];
    int rows[3];
    int nr = 0;
    for (int r = warp; r < rep; r += kAttnWarps) rows[nr++] = r;
    if (has_pos && warp == 0) rows[nr++] = rep;      // k
    if (has_pos && warp == 1) rows[nr++] = rep + 1;  // v
#pragma unroll
    for (int i = 0; i < 3; ++i)
      if (i < nr) {
        const int r = rows[i];
        const uint16_t* src = r < rep ? qkv + (size_t)(h * rep + r) * kHeadDim
                                      : qkv + (size_t)((r == rep ? a.nh : a.nh + a.nkv) + h) * kHeadDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) x[i][j] = bf16_bits_to_f32(src[lane + 32 * j]);
      }
#pragma unroll
    for (int i = 0; i < 3; ++i)
      if (i < nr) {
        const int r = rows[i];
        uint16_t* dst = r < rep ? sq[r] : snew[r - rep];
        if (r == rep + 1) {  // v is used as is (fast.py:137,140)
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = f32_to_bf16_bits(x[i][j]);
          continue;
        }
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss = fmaf(x[i][j], x[i][j], ss);
        ss = warp_sum(ss);
        const float rinv = rsqrtf(ss / (float)kHeadDim + 1e-6f);
        float xn[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xn[j] = round_bf16((r < rep ? qw[j] : kw[j]) * round_bf16(x[i][j] * rinv));
        // rotate_half (model.py:42-44): dims d and d + 64 sit in this lane at j and j + 2
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float rot = j < 2 ? -xn[j + 2] : xn[j - 2];
          const float t1 = round_bf16(xn[j] * cv[j]);
          const float t2 = round_bf16(rot * sv[j]);
          dst[lane + 32 * j] = f32_to_bf16_bits(t1 + t2);
        }
      }
    __syncthreads();
    // K/V append at pos (fast.py:145-146) by the split holding pos
    if (has_pos && tid < kHeadDim) {
      kc[(size_t)pos * kHeadDim + tid] = snew[0][tid];
      vc[(size_t)pos * kHeadDim + tid] = snew[1][tid];
    }
    // q as the B operand (k = dim, n = head): b0 = q[g][16j+2t, +1], b1 = q[g][16j+2t+8, +9]
    uint32_t bq[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      bq[j][0] = *reinterpret_cast<const uint32_t*>(&sq[g][16 * j + 2 * t]);
      bq[j][1] = *reinterpret_cast<const uint32_t*>(&sq[g][16 * j + 2 * t + 8]);
    }
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[i][c] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2t, 2t+1
    const uint64_t deadline = globaltimer_ns() + kWaitNs;
    const int rb = (warp & 3) * 16;
    const int bar_id = 1 + grp;  // the pipeline's named barrier

    for (int i = grp; i < ntiles; i += 2) {
      const int s = i % kAttnStages;
      uint8_t* sb = ring + (size_t)s * kAttnStageBytes;
      if (!mbar_wait_until(&full[s], (i / kAttnStages) & 1, deadline)) sh_flag[0] = 1;
      const int p0 = lo + i * kAttnTile;
      // the stale row pos is replaced by the new k/v; rows >= hi of V are
      // zeroed (P is 0 there, and 0 * a stale NaN would not be)
      if (has_pos && pos >= p0 && pos < p0 + kAttnTile && tg < 32) {
        const int rr = pos - p0, box = tg >> 3, c = tg & 7;  // box: K lo, K hi, V lo, V hi
        const uint16_t* srcv = snew[box >> 1] + (box & 1) * 64 + c * 8;
        *reinterpret_cast<uint4*>(sb + box * kAttnBoxBytes + swz(rr, c)) = *reinterpret_cast<const uint4*>(srcv);
      }
      if (hi < p0 + kAttnTile) {
        const int z0 = hi - p0;
        for (int e = tg; e < (kAttnTile - z0) * 16; e += kAttnGroupThreads) {
          const int row = z0 + (e >> 4), box = 2 + ((e >> 3) & 1), c = e & 7;
          *reinterpret_cast<uint4*>(sb + box * kAttnBoxBytes + row * 128 + c * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(kAttnGroupThreads) : "memory");
      if (sh_flag[0]) break;
      const uint32_t kb = smem_addr(sb), vb = kb + 2 * kAttnBoxBytes;
      // ---- S^T = K . Q^T over 8 k-steps of 16 dims
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int row = rb + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t af[4];
          ldsm_x4(af, kb + (j >> 2) * kAttnBoxBytes + swz(row, 2 * (j & 3) + (lane >> 4)));
          mma_bf16(sc, af, bq[j][0], bq[j][1]);
        }
      }
      // ---- online softmax per head over this warp's 16 positions
      const bool v0 = p0 + rb + g < hi, v1 = p0 + rb + g + 8 < hi;
      float s00 = v0 ? sc[0] * a.scale : -INFINITY, s01 = v0 ? sc[1] * a.scale : -INFINITY;
      float s10 = v1 ? sc[2] * a.scale : -INFINITY, s11 = v1 ? sc[3] * a.scale : -INFINITY;
      float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float mr0 = mn0 == -INFINITY ? 0.f : mn0, mr1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = expf(m0 - mr0), al1 = expf(m1 - mr1);
      m0 = mn0;
      m1 = mn1;
      const float p00 = expf(s00 - mr0), p01 = expf(s01 - mr1), p10 = expf(s10 - mr0), p11 = expf(s11 - mr1);
      l0 = fmaf(l0, al0, p00 + p10);
      l1 = fmaf(l1, al1, p01 + p11);
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        o[d][0] *= al0;
        o[d][1] *= al1;
        o[d][2] *= al0;
        o[d][3] *= al1;
      }
      // P^T as the B operand (k = position, n = head), through a per-warp transpose
      pbuf[warp][2 * t][g] = f32_to_bf16_bits(p00);
      pbuf[warp][2 * t + 1][g] = f32_to_bf16_bits(p01);
      pbuf[warp][2 * t][g + 8] = f32_to_bf16_bits(p10);
      pbuf[warp][2 * t + 1][g + 8] = f32_to_bf16_bits(p11);
      __syncwarp();
      const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(&pbuf[warp][g][2 * t]);
      const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(&pbuf[warp][g][2 * t + 8]);
      // ---- O^T += V^T . P^T, 16 dims per MMA
      {
        const int row = rb + (lane & 7) + 8 * (lane >> 4);
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          uint32_t af[4];
          ldsm_x4_trans(af, vb + (d >> 2) * kAttnBoxBytes + swz(row, 2 * (d & 3) + ((lane >> 3) & 1)));
          mma_bf16(o[d], af, pb0, pb1);
        }
      }
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(kAttnGroupThreads) : "memory");  // stage s free
      if (tg == 0 && i + kAttnStages < ntiles) {  // the refill: this pipeline's leader
        fence_proxy_async_smem();
        issue(i + kAttnStages);
      }
    }
    __syncthreads();  // both pipelines done (and last_tile visible)
    // ---- every issued copy has landed before the CTA goes on (and exits)
    if (tid == 0 && sh_flag[0]) {
      const uint64_t dl = globaltimer_ns() + kWaitNs;
      for (int s = 0; s < kAttnStages && s < min(issued, ntiles); ++s) {
        const int last = last_tile[s];
        if (!mbar_wait_until(&full[s], (last / kAttnStages) & 1, dl)) {
          flag_error(kDevCopyDrainTimeout);
          break;
        }
      }
      flag_error(kDevWaitTimeout);
    }
    // ---- merge the 8 warps: row sums over the 8 lanes of each head pair
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0) {
      wm[warp][2 * t] = m0;
      wm[warp][2 * t + 1] = m1;
      wl[warp][2 * t] = l0;
      wl[warp][2 * t + 1] = l1;
    }
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      wo[warp][2 * t][16 * d + g] = o[d][0];
      wo[warp][2 * t + 1][16 * d + g] = o[d][1];
      wo[warp][2 * t][16 * d + g + 8] = o[d][2];
      wo[warp][2 * t + 1][16 * d + g + 8] = o[d][3];
    }
    __syncthreads();
    for (int r = 0; r < rep && tid < kHeadDim; ++r) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][r]);
      float acc = 0.f, L = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = wm[w][r] == -INFINITY ? 0.f : expf(wm[w][r] - M);
        acc = fmaf(wo[w][r][tid], f, acc);
        L = fmaf(wl[w][r], f, L);
      }
      if (solo) {  // the split merge below with a single record, without the round trip
        a.out[(size_t)st * a.nh * kHeadDim + (size_t)(h * rep + r) * kHeadDim + tid] =
            f32_to_bf16_bits(acc * (1.0f / L));
        continue;
      }
      part[(size_t)r * kAttnRec + tid] = acc;
      if (tid == 0) {
        part[(size_t)r * kAttnRec + kHeadDim] = M;
        part[(size_t)r * kAttnRec + kHeadDim + 1] = L;
      }
    }
    if (solo) return;
  } else if (tid < rep) {
    part[(size_t)tid * kAttnRec + kHeadDim] = -INFINITY;
    part[(size_t)tid * kAttnRec + kHeadDim + 1] = 0.f;
  }
  // ---- the last split to finish merges all splits in split order
  __syncthreads();
  if (tid == 0) {
    // release this split's records (ordered before by the barrier) and, for
    // the last split, acquire the others'
    int* ctr = a.counters + (size_t)st * a.nkv + h;
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ctr) : "memory");
    sh_flag[1] = (old == a.splits - 1);
    if (sh_flag[1]) *ctr = 0;  // re-armed for the next launch
  }
  __syncthreads();
  if (!sh_flag[1]) return;
  const int nact_all = min(a.splits, (s1 + chunk - 1) / chunk);
  const uint32_t rec_bytes = (uint32_t)(nact_all * rep * kAttnRec * 4);
  if (rec_bytes <= (uint32_t)(kAttnStages * kAttnStageBytes)) {
    // every split's records into the idle ring by one bulk copy (one round
    // trip whatever the split count), merged from shared memory: per head
    // the largest running max first, then the rescaled sums in split order
    const float* src = a.partials + (((size_t)st * a.nkv + h) * a.splits * rep) * kAttnRec;
    const float* rec_s = reinterpret_cast<const float*>(ring);
    if (tid == 0) {
      fence_proxy_async_smem();                                // the warp merge's accesses of the ring
      asm volatile("fence.proxy.async.global;" ::: "memory");  // the records acquired above
      mbar_arrive_expect_tx(&mrg, rec_bytes);
      bulk_g2s(ring, src, rec_bytes, &mrg);
    }
    if (!mbar_wait(&mrg, 0)) return;  // flagged; the copy is bounded by the wait
    for (int task = tid; task < rep * 32; task += kAttnThreads) {
      const int r = task >> 5, d4 = task & 31;
      float M = -INFINITY;
      for (int j = 0; j < nact_all; ++j) M = fmaxf(M, rec_s[((size_t)j * rep + r) * kAttnRec + kHeadDim]);
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < nact_all; ++j) {
        const float* rec = rec_s + ((size_t)j * rep + r) * kAttnRec;
        const float mj = rec[kHeadDim];
        const float f = (mj == -INFINITY) ? 0.f : expf(mj - M);
        const float4 ov = reinterpret_cast<const float4*>(rec)[d4];
        acc.x = fmaf(ov.x, f, acc.x);
        acc.y = fmaf(ov.y, f, acc.y);
        acc.z = fmaf(ov.z, f, acc.z);
        acc.w = fmaf(ov.w, f, acc.w);
        L = fmaf(rec[kHeadDim + 1], f, L);
      }
      const float inv = 1.0f / L;
      uint16_t* dst = a.out + (size_t)st * a.nh * kHeadDim + (size_t)(h * rep + r) * kHeadDim + 4 * d4;
      const uint32_t lo2 = (uint32_t)f32_to_bf16_bits(acc.x * inv) | ((uint32_t)f32_to_bf16_bits(acc.y * inv) << 16);
      const uint32_t hi2 = (uint32_t)f32_to_bf16_bits(acc.z * inv) | ((uint32_t)f32_to_bf16_bits(acc.w * inv) << 16);
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo2, hi2);
    }
    return;
  }
  // records beyond the ring: from global memory, 8 splits per round trip.
  // thread task (head r, dims 4 d4 .. 4 d4 + 3): the splits' records are
  // read 8 at a time with every load issued before any is used; running
  // max / rescale across the groups, sums in split order
  const int nact = min(a.splits, (s1 + chunk - 1) / chunk);
  const float* basep = a.partials + (((size_t)st * a.nkv + h) * a.splits * rep) * kAttnRec;
  for (int task = tid; task < rep * 32; task += kAttnThreads) {
    const int r = task >> 5, d4 = task & 31;
    float M = -INFINITY, L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < nact; j0 += 8) {
      float4 ov[8];
      float mv[8], lv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < nact) {
          const float* rec = basep + ((size_t)(j0 + j) * rep + r) * kAttnRec;
          ov[j] = __ldcg(reinterpret_cast<const float4*>(rec) + d4);
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(rec + kHeadDim));
          mv[j] = ml.x;
          lv[j] = ml.y;
        }
      float Mn = M;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < nact) Mn = fmaxf(Mn, mv[j]);
      const float rs = (M == -INFINITY) ? 0.f : expf(M - Mn);
      acc.x *= rs;
      acc.y *= rs;
      acc.z *= rs;
      acc.w *= rs;
      L *= rs;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j0 + j < nact) {
          const float f = (mv[j] == -INFINITY) ? 0.f : expf(mv[j] - Mn);
          acc.x = fmaf(ov[j].x, f, acc.x);
          acc.y = fmaf(ov[j].y, f, acc.y);
          acc.z = fmaf(ov[j].z, f, acc.z);
          acc.w = fmaf(ov[j].w, f, acc.w);
          L = fmaf(lv[j], f, L);
        }
      M = Mn;
    }
    const float inv = 1.0f / L;
    uint16_t* dst = a.out + (size_t)st * a.nh * kHeadDim + (size_t)(h * rep + r) * kHeadDim + 4 * d4;
    const uint32_t lo2 = (uint32_t)f32_to_bf16_bits(acc.x * inv) | ((uint32_t)f32_to_bf16_bits(acc.y * inv) << 16);
    const uint32_t hi2 = (uint32_t)f32_to_bf16_bits(acc.z * inv) | ((uint32_t)f32_to_bf16_bits(acc.w * inv) << 16);
    *reinterpret_cast<uint2*>(dst) = make_uint2(lo2, hi2);
  }
}

// K/V append alone (the `_p_pre` tail, fast.py:138-146): k head RMSNorm +
// RoPE at pos[s] and v, written to cache rows pos[s] of every KV head, for
// `streams` rows at once; with a.out set, also the rows' q heads normed and
// rotated into a.out ([streams, nh, 128], the operand of a prefill attention
// over many rows, fast.py:229-235).  Prefill runs it for prompt rows before
// their attention (the decode attention re-writes the same K/V values).
// Grid (n_kv, streams), 128 threads: warp 0 k, warp 1 v, warps 2-3 the
// group's q heads.
__device__ __forceinline__ void norm_rope_row(const uint16_t* src, const uint16_t* w, const uint16_t* cosr,
                                              const uint16_t* sinr, uint16_t* dst, int lane) {
  float x[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = bf16_bits_to_f32(src[lane + 32 * j]);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = fmaf(x[j], x[j], ss);
  ss = warp_sum(ss);
  const float rinv = rsqrtf(ss / (float)kHeadDim + 1e-6f);
  float xn[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) xn[j] = round_bf16(bf16_bits_to_f32(w[lane + 32 * j]) * round_bf16(x[j] * rinv));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = lane + 32 * j;
    const float rot = j < 2 ? -xn[j + 2] : xn[j - 2];
    const float t1 = round_bf16(xn[j] * bf16_bits_to_f32(cosr[d]));
    const float t2 = round_bf16(rot * bf16_bits_to_f32(sinr[d]));
    dst[d] = f32_to_bf16_bits(t1 + t2);
  }
}

constexpr int kAppendThreads = 128;  // warps 0 / 1: k / v; warps 2, 3: the q heads

__global__ void __launch_bounds__(kAppendThreads) attn_append_kernel(const AttnArgs a) {
  const int h = blockIdx.x, st = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t p64 = a.pos[st];
  if (p64 < 0 || p64 >= a.max_seq) {
    if (threadIdx.x == 0) flag_error(kDevBadIndex);
    return;
  }
  const int pos = (int)p64;
  const uint16_t* qkv = a.qkv + (size_t)st * (a.nh + 2 * a.nkv) * kHeadDim;
  const uint16_t* cosr = a.rope_cos + (size_t)pos * kHeadDim;
  const uint16_t* sinr = a.rope_sin + (size_t)pos * kHeadDim;
  if (warp >= 2) {
    if (!a.out) return;
    const int rep = a.nh / a.nkv;
    for (int r = warp - 2; r < rep; r += 2) {
      const int qh = h * rep + r;
      norm_rope_row(qkv + (size_t)qh * kHeadDim, a.q_norm_w, cosr, sinr,
                    a.out + ((size_t)st * a.nh + qh) * kHeadDim, lane);
    }
    return;
  }
  uint16_t* dst = (warp == 0 ? a.k_cache : a.v_cache) + st * a.cache_stream_stride +
                  ((size_t)h * a.max_seq + pos) * kHeadDim;
  const uint16_t* src = qkv + (size_t)((warp == 0 ? a.nh : a.nh + a.nkv) + h) * kHeadDim;
  if (warp == 1) {  // v is used as is (fast.py:137,140)
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = src[lane + 32 * j];
    return;
  }
  norm_rope_row(src, a.k_norm_w, cosr, sinr, dst, lane);
}

// ------------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D view of one layer's cache: (dim, row = head * max_seq + position,
// stream), boxes of 64 dims x 64 rows with the 128-byte swizzle.
static cudaError_t make_kv_map(CUtensorMap* m, void* base, int nkv, int max_seq, int streams,
                               long long stream_stride) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t rows = (cuuint64_t)nkv * max_seq;
  cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, rows, (cuuint64_t)streams};
  cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2,
                           streams > 1 ? (cuuint64_t)stream_stride * 2 : rows * kHeadDim * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)kAttnTile, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_attn_decode(const AttnArgs& a, int streams, cudaStream_t s, int use_pdl) {
  // 4 ring stages up to 16 splits; 3 above, so that two CTAs fit an SM
  const bool three = a.splits > 16;
  auto kern = three ? attn_decode_kernel<3> : attn_decode_kernel<4>;
  const int dyn = attn_dyn_smem(three ? 3 : 4);
  static bool attr_done[2] = {false, false};
  if (!attr_done[three]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return e;
    attr_done[three] = true;
  }
  CUtensorMap tk, tv;
  const int map_streams = a.cache_stream_stride ? streams : 1;
  cudaError_t e = make_kv_map(&tk, a.k_cache, a.nkv, a.max_seq, map_streams, a.cache_stream_stride);
  if (e == cudaSuccess) e = make_kv_map(&tv, a.v_cache, a.nkv, a.max_seq, map_streams, a.cache_stream_stride);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.nkv, a.splits, streams), dim3(kAttnThreads), dyn, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, kern, tk, tv, a);
}

}  // namespace mtl

namespace mtl {
cudaError_t launch_attn_append(const AttnArgs& a, int streams, cudaStream_t s, int use_pdl) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(a.nkv, streams), dim3(kAppendThreads), 0, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, attn_append_kernel, a);
}
}  // namespace mtl
