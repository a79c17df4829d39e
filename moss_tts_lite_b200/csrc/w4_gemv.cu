// W4A16 GEMV / small-batch GEMM for sm_100a.
//
// Replaces torch._weight_int4pack_mm as called by the reference at
// moss_tts_lite/fast.py:118 (FastMossTTS._linear), gptq.py:582
// (kernel_linear) and fast_native.py:169 (_lin_fused): y = x . W^T, fp32
// accumulation, bf16 output.  Reference format: W = bf16((q - 8) * scale +
// zero) per group (gptq.py:87-97), rounded to bf16 once as torch's int4 GEMM
// forms its operand, so the products are those of the reference's kernel and
// only the fp32 summation order differs.  AutoGPTQ format: W = (q - z) * s,
// exact (the group affine is applied in fp32).
//
// Design (HBM-bound at batch 1):
//  * weights stream through a shared-memory ring filled by 1-D bulk copies
//    (cp.async.bulk, ~16 KB = several 64-column x group tiles each) issued
//    by a producer
//    warp as soon as the CTA starts - before the upstream kernel has
//    finished when launched with programmatic dependent launch;
//  * stream-K partition: CTA c owns tiles [T c / G, T (c+1) / G), so every
//    CTA streams the same number of bytes whatever N and K are;
//  * codes go register -> bf16 pairs (128 + q) with three shifts and four
//    LOP3 per 8 codes and into m16n8k16 bf16 MMAs whose B operand is the
//    bf16 activation itself (batch in the MMA N dimension).  Reference
//    format: each pair becomes bf16((q - 8) s + z) by two bf16x2 FMAs
//    (exact q - 8, then one rounding) and the MMAs accumulate a column
//    block over all its groups.  AutoGPTQ format: the per-group affine is
//    applied after the group's MMAs, y += s (D - (z + 128) Sx) with Sx the
//    group's activation sum (products of bf16 values are exact in fp32);
//  * split-K partials from different CTAs are combined by the last CTA to
//    arrive at a column block, in fixed contributor order (deterministic),
//    followed by the fused epilogue (store / residual add / SwiGLU).
#include "common.cuh"
#include "w4_gemv.cuh"

#include <algorithm>
#include <cmath>
#include <cstdlib>

namespace mtl {

namespace {

// The CTA whose range [T c / G, T (c + 1) / G) holds tile t.  32-bit
// arithmetic ((t + 1) G <= T G < 2^32, checked by w4_plan): the fixup calls
// this on its critical path, where an emulated 64-bit divide costs hundreds
// of cycles.
__host__ __device__ __forceinline__ int cta_of_tile(long long t, int G, int T) {
  return (int)(((uint32_t)(t + 1) * (uint32_t)G - 1u) / (uint32_t)T);
}

__host__ __device__ __forceinline__ size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr int kMiscWords = 320;  // [0,128) reductions, [128,136) 1/rms, [144] bail, [160,160+nblk) last flags
constexpr int kW4CThreads = kW4Warps * 32;  // consumer threads

struct SmemLayout {
  size_t bar, ring, xs, bsum, gsum, part, fin, misc, total;
};

__host__ __device__ inline SmemLayout smem_layout(const W4Plan& p, int g, int M) {
  SmemLayout L;
  size_t o = 0;
  L.bar = o;
  o += align_up((size_t)2 * p.stages * 8, 128);
  L.ring = o;
  o += (size_t)p.stages * p.tps * p.tile_bytes;
  o = align_up(o, 16);
  L.xs = o;
  o += (size_t)p.ng_max * M * g * 2;
  o = align_up(o, 16);
  L.bsum = o;
  o += (size_t)p.ng_max * M * (g / 16) * 4;
  L.gsum = o;
  o += (size_t)p.ng_max * M * 4;
  o = align_up(o, 16);
  L.part = o;
  o += (size_t)p.nblk_max * kW4Warps * kNT * M * 4;
  L.fin = o;
  o += (size_t)p.nblk_max * kNT * M * 4;
  L.misc = o;
  o += kMiscWords * 4;
  L.total = align_up(o, 128);
  return L;
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kW4CThreads) : "memory"); }

// m16n8k16 bf16 MMA with fp32 accumulate (register-sourced operands).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int FMT>
__global__ void __launch_bounds__((kW4Warps + 1) * 32, 2) w4_gemv_kernel(const W4Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const W4Plan& p = a.p;
  const int M = a.M, g = a.g, KT = p.KT;
  const int cta = blockIdx.x;
  // stream-K range of this CTA (32-bit: T G < 2^32, checked by the plan)
  const int t0 = (int)(((uint32_t)p.T * (uint32_t)cta) / (uint32_t)p.G);
  const int t1 = (int)(((uint32_t)p.T * (uint32_t)(cta + 1)) / (uint32_t)p.G);
  const int nt = t1 - t0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages, tps = p.tps;
  const size_t stage_bytes = (size_t)tps * p.tile_bytes;
  const SmemLayout L = smem_layout(p, g, M);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* empty = full + S;
  uint8_t* ring = smem + L.ring;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + L.xs);
  float* bsum = reinterpret_cast<float*>(smem + L.bsum);
  float* gsum = reinterpret_cast<float*>(smem + L.gsum);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* fin = reinterpret_cast<float*>(smem + L.fin);
  float* misc = reinterpret_cast<float*>(smem + L.misc);
  int* imisc = reinterpret_cast<int*>(misc);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], tps);  // every warp that consumes a tile of the stage arrives
    }
    fence_mbar_init();
  }
  if (threadIdx.x < kMiscWords - 144) imisc[144 + threadIdx.x] = 0;
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kW4Warps) {
    // ------------------------------------------------------------ producer
    // Weights do not depend on the upstream kernel: start streaming at once.
    if (lane == 0) {
      const int nst = (nt + tps - 1) / tps;
      int issued = 0;
      for (int st = 0; st < nst; ++st) {
        const int s = st % S;
        // the first stage lands before the rest are requested: every CTA's
        // first tile is served ahead of the other CTAs' later stages
        if (st == 1 && !mbar_wait(&full[0], 0)) break;
        if (st >= S && !mbar_wait(&empty[s], ((st / S) - 1) & 1)) break;
        const int ntile = min(tps, nt - st * tps);
        const uint32_t bytes = (uint32_t)(ntile * p.tile_bytes);
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(ring + (size_t)s * stage_bytes, a.tiles + (size_t)(t0 + st * tps) * p.tile_bytes, bytes, &full[s]);
        issued = st + 1;
      }
      // The last copy issued on each stage must land before the CTA exits
      // (consumers normally waited on every one of them already).
      const uint64_t deadline = globaltimer_ns() + kWaitNs;
      for (int s = 0; s < S && s < issued; ++s) {
        const int last = s + ((issued - 1 - s) / S) * S;
        if (!mbar_wait_until(&full[s], (last / S) & 1, deadline)) {
          flag_error(kDevCopyDrainTimeout);
          break;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int tid = threadIdx.x;  // consumer thread 0..kW4CThreads-1
  const int ng = min(KT, nt);   // groups touched: cyclic interval [gbeg, gbeg + ng)
  const int gbeg = t0 % KT;
  const int nb16 = g / 16;
  float* red = misc;
  const int njobs = ng * M * nb16;  // staging jobs: 16 values of one row of one group
  auto job_k0 = [&](int job, int& slot, int& m, int& b) {
    slot = job / (M * nb16);
    const int rem = job - slot * (M * nb16);
    m = rem / nb16;
    b = rem - m * nb16;
    return ((gbeg + slot) % KT) * g + b * 16;
  };
  // The first two staging jobs of this thread keep their inputs in
  // registers: the norm weight (a layer constant) is loaded before the
  // wait, x right after it together with the statistics loads.
  uint4 nwc[2][2], xc[2][2];
  if (a.xvec) {
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int job = tid + kW4CThreads * jj;
      if (job < njobs && a.norm_w) {
        int sl, m, b;
        const int k0 = job_k0(job, sl, m, b);
        nwc[jj][0] = __ldg(reinterpret_cast<const uint4*>(a.norm_w + k0));
        nwc[jj][1] = __ldg(reinterpret_cast<const uint4*>(a.norm_w + k0 + 8));
      }
    }
  }
  pdl_wait();
  if (a.xvec) {
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int job = tid + kW4CThreads * jj;
      if (job < njobs) {
        int sl, m, b;
        const int k0 = job_k0(job, sl, m, b);
        const uint16_t* xr = a.x + (size_t)m * a.ldx;
        xc[jj][0] = __ldg(reinterpret_cast<const uint4*>(xr + k0));
        xc[jj][1] = __ldg(reinterpret_cast<const uint4*>(xr + k0 + 8));
      }
    }
  }

  // (a) RMSNorm statistics over the full row (permutation-invariant).
  if (a.norm_w) {
    for (int m = 0; m < M; ++m) {
      float ss = 0.f;
      const uint16_t* xr = a.x + (size_t)m * a.ldx;
      if (a.xvec) {
        // chunks tid, tid + 256, ... in order; four loads issued before use
        const int nc = a.K / 8;
        for (int c0 = tid; c0 < nc; c0 += 4 * kW4CThreads) {
          uint4 v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            v[e] = c0 + e * kW4CThreads < nc ? __ldg(reinterpret_cast<const uint4*>(xr) + c0 + e * kW4CThreads)
                                             : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (c0 + e * kW4CThreads < nc) {
              const uint32_t u[4] = {v[e].x, v[e].y, v[e].z, v[e].w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float lo = __uint_as_float(u[q] << 16), hi = __uint_as_float(u[q] & 0xFFFF0000u);
                ss = fmaf(lo, lo, ss);
                ss = fmaf(hi, hi, ss);
              }
            }
          }
        }
      } else {
        for (int k = tid; k < a.K; k += kW4CThreads) {
          const float h = bf16_bits_to_f32(xr[k]);
          ss = fmaf(h, h, ss);
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp * kW4MaxM + m] = ss;
    }
    consumer_sync();
    if (tid < M) {
      float ss = 0.f;
      for (int w = 0; w < kW4Warps; ++w) ss += red[w * kW4MaxM + tid];
      misc[128 + tid] = rsqrtf(ss / (float)a.K + a.norm_eps);
    }
    consumer_sync();
  }

  // (b) stage the groups this CTA needs as bf16 in MMA-B order: within each
  //     16-block lane t reads [2t, 2t+1, 2t+8, 2t+9] at positions 4t..4t+3,
  //     i.e. 32-bit words [w0, w4, w1, w5, w2, w6, w3, w7] of the input.
  //     The per-16-block sums feed the bias / offset terms.
  auto stage_job = [&](int job, bool cached, const uint4 (&xcj)[2], const uint4 (&nwj)[2]) {
    int slot, m, b;
    const int k0 = job_k0(job, slot, m, b);
    const uint16_t* xr = a.x + (size_t)m * a.ldx;
    uint32_t u[8], nw[8];
    if (a.xvec) {
      uint4 v0, v1, n0, n1;
      if (cached) {
        v0 = xcj[0];
        v1 = xcj[1];
        n0 = nwj[0];
        n1 = nwj[1];
      } else {
        v0 = __ldg(reinterpret_cast<const uint4*>(xr + k0));
        v1 = __ldg(reinterpret_cast<const uint4*>(xr + k0 + 8));
        if (a.norm_w) {
          n0 = __ldg(reinterpret_cast<const uint4*>(a.norm_w + k0));
          n1 = __ldg(reinterpret_cast<const uint4*>(a.norm_w + k0 + 8));
        }
      }
      u[0] = v0.x; u[1] = v0.y; u[2] = v0.z; u[3] = v0.w; u[4] = v1.x; u[5] = v1.y; u[6] = v1.z; u[7] = v1.w;
      if (a.norm_w) {
        nw[0] = n0.x; nw[1] = n0.y; nw[2] = n0.z; nw[3] = n0.w; nw[4] = n1.x; nw[5] = n1.y; nw[6] = n1.z; nw[7] = n1.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int ka = a.k_perm ? a.k_perm[k0 + 2 * q] : k0 + 2 * q;
        const int kb = a.k_perm ? a.k_perm[k0 + 2 * q + 1] : k0 + 2 * q + 1;
        u[q] = (uint32_t)xr[ka] | ((uint32_t)xr[kb] << 16);
        if (a.norm_w) nw[q] = (uint32_t)a.norm_w[ka] | ((uint32_t)a.norm_w[kb] << 16);
      }
    }
    float bs = 0.f;
    if (a.norm_w) {
      const float rinv = misc[128 + m];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        // model.py:34-40: bf16(h * rsqrt(var + eps)), then bf16(weight * that)
        const float v0 = round_bf16(__uint_as_float(nw[q] << 16) * round_bf16(__uint_as_float(u[q] << 16) * rinv));
        const float v1 = round_bf16(__uint_as_float(nw[q] & 0xFFFF0000u) *
                                    round_bf16(__uint_as_float(u[q] & 0xFFFF0000u) * rinv));
        u[q] = (__float_as_uint(v0) >> 16) | (__float_as_uint(v1) & 0xFFFF0000u);
      }
    }
    uint16_t* dst = xs + ((size_t)slot * M + m) * g + b * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(u[0], u[4], u[1], u[5]);
    *reinterpret_cast<uint4*>(dst + 8) = make_uint4(u[2], u[6], u[3], u[7]);
    if (FMT != kFmtRef) {
#pragma unroll
      for (int q = 0; q < 8; ++q) bs += __uint_as_float(u[q] << 16) + __uint_as_float(u[q] & 0xFFFF0000u);
      bsum[(slot * M + m) * nb16 + b] = bs;
    }
  };
  if (tid < njobs) stage_job(tid, a.xvec != 0, xc[0], nwc[0]);
  if (tid + kW4CThreads < njobs) stage_job(tid + kW4CThreads, a.xvec != 0, xc[1], nwc[1]);
  for (int job = tid + 2 * kW4CThreads; job < njobs; job += kW4CThreads) stage_job(job, false, xc[0], nwc[0]);
  for (int i = tid; i < p.nblk_max * kW4Warps * kNT * M; i += kW4CThreads) part[i] = 0.f;
  consumer_sync();
  if (FMT != kFmtRef) {
    // group sums of the activations for the GPTQ affine: the 16-value block
    // sums in order, all loads issued before the adds
    for (int job = tid; job < ng * M; job += kW4CThreads) {
      float bv[16];
#pragma unroll
      for (int b = 0; b < 16; ++b) bv[b] = b < nb16 ? bsum[job * nb16 + b] : 0.f;
      float s = 0.f;
#pragma unroll
      for (int b = 0; b < 16; ++b)
        if (b < nb16) s += bv[b];
      gsum[job] = s;
    }
    consumer_sync();
  }

  // ------------------------------------------------------------ main loop
  const int gr = lane >> 2, tq = lane & 3;
  const int mrow = min(gr, M - 1);
  const int KS = g >> 4;
  const int blk_first = t0 / KT;
  // Column-block accumulators.  Reference format: the MMAs take the bf16
  // effective weights themselves, so a block accumulates over all its groups
  // in two chains (even / odd k16-steps).  GPTQ format: per-group MMA sums
  // of (128 + q) x, folded into yacc by the group affine.
  float yacc[4][4], yacc2[4][4];
  int cur = -1;
  bool bail = false;

  auto flush = [&](int blk) {
    float* dst = part + ((size_t)(blk - blk_first) * kW4Warps + warp) * kNT * M;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = 16 * j + gr + ((e & 2) ? 8 : 0);
        const int m = 2 * tq + (e & 1);
        if (m < M) dst[col * M + m] = (FMT == kFmtRef) ? yacc[j][e] + yacc2[j][e] : yacc[j][e];
      }
  };

  int nb = (t0 + warp) / KT;
  int G = (t0 + warp) - nb * KT;
  int slot = (G - gbeg + KT) % KT;
  // ring position of this warp's tile, advanced incrementally (tps is a power of two)
  int ltps = 0;
  while ((1 << ltps) < tps) ++ltps;
  const int dst = kW4Warps >> ltps;  // stages between two tiles of this warp
  int s = (warp >> ltps) % S, q = (warp >> ltps) / S;
  for (int i = warp; i < nt; i += kW4Warps) {
    if (nb != cur) {
      if (cur >= 0) flush(cur);
      cur = nb;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) yacc[j][e] = yacc2[j][e] = 0.f;
    }
    if (!mbar_wait(&full[s], q & 1)) {
      bail = true;
      break;
    }
    const uint8_t* tile = ring + (size_t)s * stage_bytes + (size_t)(i & (tps - 1)) * p.tile_bytes;
    const uint4* wt = reinterpret_cast<const uint4*>(tile);
    const uint16_t* xg = xs + ((size_t)slot * M + mrow) * g + 4 * tq;
    const uint8_t* prm = tile + kNT * g / 2;
    if (FMT == kFmtRef) {
      // (scale, scale) and (zero, zero) bf16 pairs of this lane's 8 columns
      // 16 j + gr (+ 8): rows r0 / r1 of the A fragments
      uint32_t sc2[4][2], zr2[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const uint32_t pw = reinterpret_cast<const uint32_t*>(prm)[16 * j + gr + 8 * hr];
          sc2[j][hr] = __byte_perm(pw, 0u, 0x1010);
          zr2[j][hr] = __byte_perm(pw, 0u, 0x3232);
        }
#pragma unroll 2
      for (int ks = 0; ks < KS; ks += 2) {
        const uint4 wv = wt[ks * 32 + lane];
        const uint4 wv2 = wt[(ks + 1) * 32 + lane];
        const uint2 bx = *reinterpret_cast<const uint2*>(xg + ks * 16);
        const uint2 bx2 = *reinterpret_cast<const uint2*>(xg + (ks + 1) * 16);
        const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint32_t wr2[4] = {wv2.x, wv2.y, wv2.z, wv2.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t w = wr[j], v = wr2[j];
          mma_bf16_16816(yacc[j], w4_ref_pair(lop3_and_or(w, 0x000F000Fu, 0x43004300u), sc2[j][0], zr2[j][0]),
                         w4_ref_pair(lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u), sc2[j][1], zr2[j][1]),
                         w4_ref_pair(lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u), sc2[j][0], zr2[j][0]),
                         w4_ref_pair(lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u), sc2[j][1], zr2[j][1]),
                         bx.x, bx.y);
          mma_bf16_16816(yacc2[j], w4_ref_pair(lop3_and_or(v, 0x000F000Fu, 0x43004300u), sc2[j][0], zr2[j][0]),
                         w4_ref_pair(lop3_and_or(v >> 4, 0x000F000Fu, 0x43004300u), sc2[j][1], zr2[j][1]),
                         w4_ref_pair(lop3_and_or(v >> 8, 0x000F000Fu, 0x43004300u), sc2[j][0], zr2[j][0]),
                         w4_ref_pair(lop3_and_or(v >> 12, 0x000F000Fu, 0x43004300u), sc2[j][1], zr2[j][1]),
                         bx2.x, bx2.y);
        }
      }
    } else {
      // even and odd k16-steps accumulate separately: eight independent MMA
      // chains per warp instead of four
      float d[4][4], d2[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[j][e] = d2[j][e] = 0.f;
#pragma unroll 2
      for (int ks = 0; ks < KS; ks += 2) {
        const uint4 wv = wt[ks * 32 + lane];
        const uint4 wv2 = wt[(ks + 1) * 32 + lane];
        const uint2 bx = *reinterpret_cast<const uint2*>(xg + ks * 16);
        const uint2 bx2 = *reinterpret_cast<const uint2*>(xg + (ks + 1) * 16);
        const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint32_t wr2[4] = {wv2.x, wv2.y, wv2.z, wv2.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t w = wr[j], v = wr2[j];
          mma_bf16_16816(d[j], lop3_and_or(w, 0x000F000Fu, 0x43004300u), lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u),
                         lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u), lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u),
                         bx.x, bx.y);
          mma_bf16_16816(d2[j], lop3_and_or(v, 0x000F000Fu, 0x43004300u), lop3_and_or(v >> 4, 0x000F000Fu, 0x43004300u),
                         lop3_and_or(v >> 8, 0x000F000Fu, 0x43004300u), lop3_and_or(v >> 12, 0x000F000Fu, 0x43004300u),
                         bx2.x, bx2.y);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[j][e] += d2[j][e];
      // group affine: D = sum x (128 + q)  =>  w = (q - (z + zero_offset)) s gives
      // y += s D + C Sx with C = -(z + zero_offset + 128) s
      const float sx0 = gsum[slot * M + min(2 * tq, M - 1)];
      const float sx1 = gsum[slot * M + min(2 * tq + 1, M - 1)];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int col = 16 * j + gr + 8 * hr;
          const float A = __half2float(reinterpret_cast<const __half*>(prm)[col]);
          const uint32_t zw = reinterpret_cast<const uint32_t*>(prm + 128)[col >> 3];
          const int z = (int)((zw >> (4 * (col & 7))) & 0xFu) + a.zero_offset;
          const float C = -(float)(z + 128) * A;
          yacc[j][2 * hr + 0] = fmaf(A, d[j][2 * hr + 0], fmaf(C, sx0, yacc[j][2 * hr + 0]));
          yacc[j][2 * hr + 1] = fmaf(A, d[j][2 * hr + 1], fmaf(C, sx1, yacc[j][2 * hr + 1]));
        }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // next tile of this warp: kW4Warps further along
    s += dst;
    while (s >= S) {
      s -= S;
      ++q;
    }
    G += kW4Warps;
    slot += kW4Warps;
    while (G >= KT) {
      G -= KT;
      ++nb;
    }
    while (slot >= KT) slot -= KT;
  }
  if (cur >= 0 && !bail) flush(cur);
  if (bail) imisc[144] = 1;
  consumer_sync();
  if (imisc[144] == 1) return;

  // ------------------------------------- CTA reduce + split-K fixup (all blocks at once)
  const int blk_last = (t1 - 1) / KT;
  const int nblk = blk_last - blk_first + 1;
  const int per = kNT * M;
  // the residual does not depend on the split-K partials: load it now
  float rpf[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.epi == kEpiResidual && tid < per) {
    const int col = tid / M, m = tid - (tid / M) * M;
#pragma unroll
    for (int bl = 0; bl < 4; ++bl)
      if (bl < nblk) rpf[bl] = bf16_bits_to_f32(a.residual[(size_t)m * a.ldr + (blk_first + bl) * kNT + col]);
  }
  for (int i = tid; i < nblk * per; i += kW4CThreads) {
    const int bl = i / per, r = i - bl * per;
    float v = 0.f;
    for (int w = 0; w < kW4Warps; ++w) v += part[((size_t)bl * kW4Warps + w) * per + r];
    fin[i] = v;
  }
  consumer_sync();
  bool any_partial = false;
  for (int bl = 0; bl < nblk; ++bl) {
    const int blk = blk_first + bl;
    any_partial |= !((blk * KT >= t0) && ((blk + 1) * KT <= t1));
  }
  if (any_partial) {
    for (int i = tid; i < nblk * per; i += kW4CThreads) {
      const int bl = i / per, r = i - bl * per;
      const int blk = blk_first + bl;
      if ((blk * KT >= t0) && ((blk + 1) * KT <= t1)) continue;
      const int c_lo = cta_of_tile((long long)blk * KT, p.G, p.T);
      a.partials[((size_t)blk * p.maxc + (cta - c_lo)) * per + r] = fin[i];
    }
    consumer_sync();
    if (tid < nblk) {
      const int blk = blk_first + tid;
      if (!((blk * KT >= t0) && ((blk + 1) * KT <= t1))) {
        const int c_lo = cta_of_tile((long long)blk * KT, p.G, p.T);
        const int c_hi = cta_of_tile((long long)(blk + 1) * KT - 1, p.G, p.T);
        // release this CTA's partials (ordered before by the barrier) and,
        // for the last contributor, acquire the others'
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.counters + blk) : "memory");
        if (old == c_hi - c_lo) {
          imisc[160 + tid] = 1;
          a.counters[blk] = 0;  // re-arm for the next launch
        }
      }
    }
    consumer_sync();
    for (int i = tid; i < nblk * per; i += kW4CThreads) {
      const int bl = i / per, r = i - bl * per;
      if (!imisc[160 + bl]) continue;
      const int blk = blk_first + bl;
      const int c_lo = cta_of_tile((long long)blk * KT, p.G, p.T);
      const int c_hi = cta_of_tile((long long)(blk + 1) * KT - 1, p.G, p.T);
      // contributors in order; up to 8 partial loads issued before the adds
      const int ncon = c_hi - c_lo + 1;
      const float* pp = a.partials + (size_t)blk * p.maxc * per + r;
      float pv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) pv[j] = j < ncon ? __ldcg(pp + (size_t)j * per) : 0.f;
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < ncon) v += pv[j];
      for (int j = 8; j < ncon; ++j) v += __ldcg(pp + (size_t)j * per);
      fin[i] = v;
    }
    consumer_sync();
  }

  // ---------------------------------------------------------------- epilogue
  for (int bl = 0; bl < nblk; ++bl) {
    const int blk = blk_first + bl;
    const bool complete = (blk * KT >= t0) && ((blk + 1) * KT <= t1);
    if (!complete && !imisc[160 + bl]) continue;
    const float* f = fin + (size_t)bl * per;
    if (a.epi == kEpiSwiGLU) {
      for (int i = tid; i < (kNT / 2) * M; i += kW4CThreads) {
        const int col = i / M, m = i - (i / M) * M;
        // fast.py:170-171: bf16(silu(gate)) * up, each op rounded to bf16
        const float gt = round_bf16(f[col * M + m]);
        const float up = round_bf16(f[(col + kNT / 2) * M + m]);
        const float sg = round_bf16(gt / (1.0f + expf(-gt)));
        a.y[(size_t)m * a.ldy + blk * (kNT / 2) + col] = f32_to_bf16_bits(sg * up);
      }
    } else {
      for (int i = tid; i < per; i += kW4CThreads) {
        const int col = i / M, m = i - (i / M) * M;
        const int n = blk * kNT + col;
        float v = f[i];
        if (a.epi == kEpiResidual) {
          // fast.py:168 / :170: residual + bf16(linear(...)), rounded to bf16
          float r = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k == bl) r = rpf[k];
          if (bl >= 4 || i >= kW4CThreads) r = bf16_bits_to_f32(a.residual[(size_t)m * a.ldr + n]);
          v = r + round_bf16(v);
        }
        a.y[(size_t)m * a.ldy + n] = f32_to_bf16_bits(v);
      }
    }
  }
}

}  // namespace

int w4_plan(int M, int K, int N, int g, int fmt, int num_sms, W4Plan* out) {
  if (M < 1 || M > kW4MaxM || K <= 0 || N <= 0 || (N % kNT) || (K % g) || (g % 16) || g > 256) return -1;
  W4Plan p{};
  p.KT = K / g;
  p.nblocks = N / kNT;
  if ((long long)p.nblocks * p.KT * 2 * num_sms >= (1ll << 32)) return -1;  // cta_of_tile's 32-bit range
  p.T = p.nblocks * p.KT;
  p.tile_bytes = tile_bytes(g, fmt);
  // ~16 KB per bulk copy (large copies stream markedly better than 4 KB ones)
  p.tps = 1;
  while (p.tps < kW4Warps && (p.tps * 2) * p.tile_bytes <= 18 * 1024) p.tps *= 2;
  const int ngroups = kW4Warps / p.tps;  // stage s is consumed by warp group s % ngroups
  // CTAs per SM: 2 by default.  With 1, a CTA uses at most ~113 KB when it
  // can, so that the next kernel of a chain (programmatic dependent launch)
  // co-resides and starts streaming its weights while this one finishes.
  static int ctas_per_sm = -1;
  if (ctas_per_sm < 0) {
    const char* e = std::getenv("MTL_W4_CTAS_PER_SM");
    ctas_per_sm = (e && e[0] == '1') ? 1 : 2;
  }
  struct Try { int per_sm; size_t budget; };
  const Try tries[3] = {{2, 113 * 1024}, {1, 113 * 1024}, {1, 225 * 1024}};
  bool ok = false;
  for (const Try& tr : tries) {
    if (tr.per_sm > ctas_per_sm) continue;
    int G = std::min(p.T, num_sms * tr.per_sm);
    G = std::max(1, std::min(G, std::max(1, p.T / 2)));
    p.G = G;
    const int ntmax = (p.T + G - 1) / G;
    p.ng_max = std::min(p.KT, ntmax);
    p.nblk_max = std::min(p.nblocks, ntmax / p.KT + 2);
    const int nst = (ntmax + p.tps - 1) / p.tps;
    p.stages = std::max(ngroups, std::min(8, (nst + ngroups - 1) / ngroups * ngroups));
    for (;;) {
      SmemLayout L = smem_layout(p, g, M);
      p.smem = L.total;
      if (L.total <= tr.budget || p.stages <= ngroups) break;
      p.stages -= ngroups;
    }
    if (p.smem <= tr.budget) { ok = true; break; }
  }
  if (!ok) return -2;
  int maxc = 1;
  for (int b = 0; b < p.nblocks; ++b) {
    const int lo = cta_of_tile((long long)b * p.KT, p.G, p.T);
    const int hi = cta_of_tile((long long)(b + 1) * p.KT - 1, p.G, p.T);
    maxc = std::max(maxc, hi - lo + 1);
  }
  p.maxc = maxc;
  p.partial_bytes = align_up((size_t)p.nblocks * p.maxc * kNT * M * 4, 256);
  *out = p;
  return 0;
}

cudaError_t w4_launch(const W4Args& args, int fmt, cudaStream_t stream, int use_pdl) {
  const W4Args& a = args;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.p.G);
  cfg.blockDim = dim3((kW4Warps + 1) * 32);
  cfg.dynamicSmemBytes = a.p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl ? 1 : 0;
  // The shared-memory opt-in is set once per kernel (to the largest size any
  // plan uses) so that launches inside a stream capture make no attribute calls.
  static bool attr_done[2] = {false, false};
  auto kern = (fmt == kFmtRef) ? w4_gemv_kernel<kFmtRef> : w4_gemv_kernel<kFmtGptq>;
  const int fi = (fmt == kFmtRef) ? 0 : 1;
  if (!attr_done[fi]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[fi] = true;
  }
  return cudaLaunchKernelEx(&cfg, kern, a);
}

// ------------------------------------------------------------------ packing

namespace {

// Source accessors for one code W[n][k] (n = output column).
struct GptqSrc {
  const int32_t* qweight;  // [K/8, N]
  const int32_t* perm;     // nullable, sorted-k -> original k
  int N;
  __device__ __forceinline__ uint32_t code(int n, int k) const {
    int kk = perm ? perm[k] : k;
    return ((uint32_t)qweight[(size_t)(kk >> 3) * N + n] >> (4 * (kk & 7))) & 0xFu;
  }
};
struct RefSrc {
  const uint8_t* q;  // [N, K]
  int K;
  __device__ __forceinline__ uint32_t code(int n, int k) const { return q[(size_t)n * K + k] & 0xFu; }
};

template <class Src>
__global__ void pack_words_kernel(Src src, int K, int N, int g, int tile_bytes, uint8_t* tiles) {
  const int KT = K / g, KS = g / 16;
  const long long words_per_tile = (long long)KS * 32 * 4;
  const long long total = (long long)(N / kNT) * KT * words_per_tile;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long t = idx / words_per_tile;
    const int wi = (int)(idx % words_per_tile);
    const int j = wi & 3, lane = (wi >> 2) & 31, ks = wi >> 7;
    const int nb = (int)(t / KT), G = (int)(t % KT);
    const int gr = lane >> 2, tq = lane & 3;
    const int r0 = nb * kNT + 16 * j + gr, r1 = r0 + 8;
    const int kb = G * g + 16 * ks;
    uint32_t w = 0;
    w |= src.code(r0, kb + 2 * tq) << 0;
    w |= src.code(r1, kb + 2 * tq) << 4;
    w |= src.code(r0, kb + 2 * tq + 8) << 8;
    w |= src.code(r1, kb + 2 * tq + 8) << 12;
    w |= src.code(r0, kb + 2 * tq + 1) << 16;
    w |= src.code(r1, kb + 2 * tq + 1) << 20;
    w |= src.code(r0, kb + 2 * tq + 9) << 24;
    w |= src.code(r1, kb + 2 * tq + 9) << 28;
    reinterpret_cast<uint32_t*>(tiles + t * tile_bytes)[wi] = w;
  }
}

__global__ void pack_params_ref_kernel(const uint16_t* qsz, int K, int N, int g, int tile_bytes, uint8_t* tiles) {
  const int KT = K / g;
  const long long total = (long long)N * KT;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(idx % N), G = (int)(idx / N);
    const long long t = (long long)(n / kNT) * KT + G;
    const uint32_t sc = qsz[((size_t)G * N + n) * 2 + 0];
    const uint32_t zr = qsz[((size_t)G * N + n) * 2 + 1];
    reinterpret_cast<uint32_t*>(tiles + t * tile_bytes + kNT * g / 2)[n % kNT] = sc | (zr << 16);
  }
}

__global__ void pack_params_gptq_kernel(const uint16_t* scales, const int32_t* qzeros, int K, int N, int g,
                                        int tile_bytes, uint8_t* tiles) {
  const int KT = K / g;
  const long long total = (long long)N * KT;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(idx % N), G = (int)(idx / N);
    const long long t = (long long)(n / kNT) * KT + G;
    uint8_t* prm = tiles + t * tile_bytes + kNT * g / 2;
    reinterpret_cast<uint16_t*>(prm)[n % kNT] = scales[(size_t)G * N + n];
    if ((n & 7) == 0)
      reinterpret_cast<uint32_t*>(prm + 128)[(n % kNT) >> 3] = (uint32_t)qzeros[(size_t)G * (N / 8) + n / 8];
  }
}

// Inverse of the word packing, for bit-exact round-trip checks: codes[n][k].
__global__ void unpack_codes_kernel(const uint8_t* tiles, int K, int N, int g, int tile_bytes, uint8_t* codes) {
  const int KT = K / g;
  const long long total = (long long)N * K;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(idx / K), k = (int)(idx % K);
    const int nb = n / kNT, c = n % kNT, G = k / g, kin = k % g;
    const int j = c / 16, rr = c % 16, gr = rr & 7, hi_row = rr >> 3;
    const int ks = kin / 16, k16 = kin % 16;
    const int hi_k = k16 >= 8 ? 1 : 0;
    const int kk = k16 & 7, tq = kk >> 1, odd = kk & 1;
    const int lane = gr * 4 + tq;
    const int slot = (hi_row ? 1 : 0) + (hi_k ? 2 : 0) + (odd ? 4 : 0);
    const long long t = (long long)nb * KT + G;
    const uint32_t w = reinterpret_cast<const uint32_t*>(tiles + t * tile_bytes)[(ks * 32 + lane) * 4 + j];
    codes[idx] = (uint8_t)((w >> (4 * slot)) & 0xFu);
  }
}

// Effective bf16 weights W[n][k] from the tiles (the prefill GEMM operand):
// REF  w = (q - 8) * scale + zero            (gptq.py:87-97)
// GPTQ w = (q - (z + zero_offset)) * scale    (AutoGPTQ)
// computed in fp32 and rounded to bf16; two consecutive k per thread.
// One 64-column x group tile per CTA iteration: warp w unpacks k16-steps
// w, w + 8, ... in the MMA lane layout the tiles are packed in (one uint4 of
// codes per lane: rows 16 j + gr (+8), columns 16 ks + 2 tq (+1, +8, +9)),
// writes bf16 pairs into a padded shared-memory tile (row stride g + 8
// elements: the 32 lanes of a store hit 32 distinct banks), and the CTA then
// writes the tile's 64 rows as 16-byte chunks.  (q - 8) comes from the float
// 2^23 + q minus (2^23 + 8), exact, so v = fmaf(q - 8, scale, zero) is the
// same single-rounding FMA as the GEMV's group affine.
template <int FMT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* tiles, int K, int N, int g, int tile_bytes,
                                                      int zero_offset, uint16_t* w) {
  extern __shared__ __align__(16) uint16_t sout[];  // [kNT][g + 8]
  const int KT = K / g, KS = g / 16, ld = g + 8, cpr = g / 8;
  const int ntiles = (N / kNT) * KT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gr = lane >> 2, tq = lane & 3;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int nb = t / KT, G = t - nb * KT;
    const uint8_t* tile = tiles + (size_t)t * tile_bytes;
    const uint8_t* prm = tile + kNT * g / 2;
    float sc[4][2], zo[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int c = 16 * j + gr + 8 * hr;
        if (FMT == kFmtRef) {
          const uint32_t pw = reinterpret_cast<const uint32_t*>(prm)[c];
          sc[j][hr] = __uint_as_float(pw << 16);
          zo[j][hr] = __uint_as_float(pw & 0xFFFF0000u);
        } else {
          sc[j][hr] = __half2float(reinterpret_cast<const __half*>(prm)[c]);
          const uint32_t zw = reinterpret_cast<const uint32_t*>(prm + 128)[c >> 3];
          zo[j][hr] = (float)((int)((zw >> (4 * (c & 7))) & 0xFu) + zero_offset);
        }
      }
    for (int ks = warp; ks < KS; ks += 8) {
      const uint4 wv = reinterpret_cast<const uint4*>(tile)[ks * 32 + lane];
      const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr)
#pragma unroll
          for (int hk = 0; hk < 2; ++hk) {
            const int slot = hr + 2 * hk;
            const uint32_t n0 = (wr[j] >> (4 * slot)) & 0xFu, n1 = (wr[j] >> (4 * (slot + 4))) & 0xFu;
            float v0, v1;
            if (FMT == kFmtRef) {
              v0 = fmaf(__uint_as_float(0x4B000000u | n0) - 8388616.f, sc[j][hr], zo[j][hr]);
              v1 = fmaf(__uint_as_float(0x4B000000u | n1) - 8388616.f, sc[j][hr], zo[j][hr]);
            } else {
              v0 = ((__uint_as_float(0x4B000000u | n0) - 8388608.f) - zo[j][hr]) * sc[j][hr];
              v1 = ((__uint_as_float(0x4B000000u | n1) - 8388608.f) - zo[j][hr]) * sc[j][hr];
            }
            const int c = 16 * j + gr + 8 * hr, k = 16 * ks + 8 * hk + 2 * tq;
            *reinterpret_cast<uint32_t*>(sout + c * ld + k) =
                (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
          }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kNT * cpr; i += blockDim.x) {
      const int r = i / cpr, ch = i - r * cpr;
      *reinterpret_cast<uint4*>(w + (size_t)(nb * kNT + r) * K + (size_t)G * g + ch * 8) =
          *reinterpret_cast<const uint4*>(sout + r * ld + ch * 8);
    }
    __syncthreads();
  }
}

inline int grid_for(long long work) {
  long long b = (work + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(b, 148LL * 32));
}

}  // namespace

cudaError_t w4_pack_gptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                         const int32_t* perm, int K, int N, int g, uint8_t* tiles, cudaStream_t s) {
  const int tb = tile_bytes(g, kFmtGptq);
  GptqSrc src{qweight, perm, N};
  long long words = (long long)(N / kNT) * (K / g) * (g / 16) * 128;
  pack_words_kernel<<<grid_for(words), 256, 0, s>>>(src, K, N, g, tb, tiles);
  pack_params_gptq_kernel<<<grid_for((long long)N * (K / g)), 256, 0, s>>>(scales, qzeros, K, N, g, tb, tiles);
  return cudaGetLastError();
}

cudaError_t w4_pack_ref(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles,
                        cudaStream_t s) {
  const int tb = tile_bytes(g, kFmtRef);
  RefSrc src{q, K};
  long long words = (long long)(N / kNT) * (K / g) * (g / 16) * 128;
  pack_words_kernel<<<grid_for(words), 256, 0, s>>>(src, K, N, g, tb, tiles);
  pack_params_ref_kernel<<<grid_for((long long)N * (K / g)), 256, 0, s>>>(qsz, K, N, g, tb, tiles);
  return cudaGetLastError();
}

cudaError_t w4_dequant(const uint8_t* tiles, int K, int N, int g, int fmt, int zero_offset, uint16_t* w,
                       cudaStream_t s) {
  const int ntiles = (N / kNT) * (K / g);
  const int grid = std::max(1, std::min(ntiles, 148 * 8));
  const size_t smem = (size_t)kNT * (g + 8) * 2;
  if (smem > 48 * 1024) return cudaErrorInvalidValue;  // g <= 376
  if (fmt == kFmtRef)
    dequant_kernel<kFmtRef><<<grid, 256, smem, s>>>(tiles, K, N, g, tile_bytes(g, fmt), zero_offset, w);
  else
    dequant_kernel<kFmtGptq><<<grid, 256, smem, s>>>(tiles, K, N, g, tile_bytes(g, fmt), zero_offset, w);
  return cudaGetLastError();
}

cudaError_t w4_unpack_codes(const uint8_t* tiles, int K, int N, int g, int fmt, uint8_t* codes, cudaStream_t s) {
  unpack_codes_kernel<<<grid_for((long long)N * K), 256, 0, s>>>(tiles, K, N, g, tile_bytes(g, fmt), codes);
  return cudaGetLastError();
}

}  // namespace mtl
