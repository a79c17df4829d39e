// Persistent W4A16 GEMV chain for the batched multi-stream decode step
// (2..16 activation rows: the streams of BatchedFastMossTTS), sm_100a.
//
// The batch-1 chain (w4_chain.cu) with the rows of the batch as the N
// dimension of the m16n8k16 MMAs (one or two 8-row n-tiles): the same strip
// weights, the same one-CTA-per-SM grid with a grid barrier between phases
// (o -> gate|up -> down -> next q|k|v, as the reference's decode step calls
// torch._weight_int4pack_mm once per stream, moss_tts_lite/fast.py:165-171),
// the same bf16 operand bf16((q - 8) s + z).  What changes:
//
//  * x is staged per K-slice of up to 4096 columns (16 rows x 4096 bf16 do
//    not leave room for more): the rows land by bulk copies in their natural
//    order (RMSNorm phases normalise them in place); the CTA walks its pieces
//    slice by slice, strip by strip within a slice, and re-stages x between
//    slices (RMSNorm phases have K <= 4096, one slice);
//  * after each strip every consumer warp writes its fp32 MMA sums (16 rows
//    x the batch rows) to one of two shared-memory partial buffers and
//    arrives on the buffer's mbarrier; a reducer warp sums the 16 partials
//    in warp order - the results are bitwise reproducible - frees the
//    buffer and applies the epilogue (store / residual / SwiGLU, per batch
//    row) while the consumers go on with the next strip.  Phases with
//    several x slices add each slice's sums into fp32 strip accumulators, in
//    slice order.
#include "w4_chain.cuh"

namespace mtl {

namespace {

constexpr int kCbSlice = 4096;                    // max x columns staged at once
constexpr int kCbPieces = kChainWarps;            // pieces per ring stage: one per consumer warp
constexpr int kCbMiscWords = 64;                  // [0] bail, [1] reducer phases, [8, 8 + kCW) warp sums of squares

struct CbLayout {
  size_t bar, ring, xs, pbuf, acc, res, misc, total;
};

// x row stride in bytes: a slice of bf16 plus 64 bytes, so that the 8 rows
// one MMA fragment load touches fall in different banks
__host__ __device__ inline int cb_xstride(int kslice) { return kslice * 2 + 64; }

__host__ __device__ inline CbLayout cb_layout(int stages, int tile_bytes, int kslice, int rows, int uaux) {
  CbLayout L;
  size_t o = 0;
  L.bar = o;
  o += round_up((size_t)(2 * stages + 5) * 8, 128);
  L.ring = o;
  o += (size_t)stages * kCbPieces * tile_bytes;
  o = round_up(o, 128);
  L.xs = o;
  o += (size_t)rows * cb_xstride(kslice);
  o = round_up(o, 16);
  L.pbuf = o;  // [2][warps][32 lanes][rows / 2] fp32 strip partials
  o += (size_t)2 * kChainWarps * 32 * (rows / 2) * 4;
  L.acc = o;   // [uaux][16][rows] fp32 slice sums
  o += (size_t)uaux * 16 * rows * 4;
  L.res = o;   // [uaux][16][rows] bf16 residual of the CTA's strips
  o += round_up((size_t)uaux * 16 * rows * 2, 16);
  L.misc = o;
  o += kCbMiscWords * 4;
  L.total = round_up(o, 128);
  return L;
}

// Pieces of a phase in the CTA's order: slice sl, strip u in [u0, u1),
// groups of the slice; a "run" is one (slice, strip) pair, contiguous in
// memory (strip-major tiles).
struct CbRun {
  int KT, gps, nsl, nu;  // groups, groups per slice, slices, strips
};

template <int GS, int NT>
__global__ void __launch_bounds__((kChainWarps + 2) * 32, 1) w4_chainb_kernel(const ChainBArgs a) {
  extern __shared__ __align__(128) uint8_t cb_sm[];
  constexpr int kCW = kChainWarps;
  constexpr int kCThr = kCW * 32;
  constexpr int TB = 8 * GS + 64;
  constexpr uint32_t kStageBytes = (uint32_t)kCbPieces * TB;
  constexpr int MR = 8 * NT;  // staged rows (batch rows padded to the n-tiles)
  const int S = a.stages, M = a.M, KSL = a.kslice;
  const int XS = cb_xstride(KSL);
  const CbLayout L = cb_layout(S, TB, KSL, MR, a.uaux);
  uint64_t* full = reinterpret_cast<uint64_t*>(cb_sm + L.bar);
  uint64_t* empty = full + S;
  uint64_t* xbar = empty + S;  // x rows of a slice landed
  uint64_t* sfull = xbar + 1;  // [2] every consumer warp's partial of a strip written
  uint64_t* sfree = sfull + 2; // [2] the reducer is done with a partial buffer
  uint8_t* ring = cb_sm + L.ring;
  uint8_t* xs = cb_sm + L.xs;
  float* pbuf = reinterpret_cast<float*>(cb_sm + L.pbuf);
  float* acc_s = reinterpret_cast<float*>(cb_sm + L.acc);
  uint16_t* res_s = reinterpret_cast<uint16_t*>(cb_sm + L.res);
  float* misc = reinterpret_cast<float*>(cb_sm + L.misc);
  int* imisc = reinterpret_cast<int*>(misc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    mbar_init(xbar, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], kCW);
      mbar_init(&sfree[b], 1);
    }
    fence_mbar_init();
    imisc[0] = 0;
    imisc[1] = 0;  // phases the reducer has finished (a counter: a CTA with no strips in a phase
                   // finishes it at once, so a parity wait could not tell two phases apart)
  }
  __syncthreads();
  pdl_launch_dependents();

  auto runs = [&](const ChainBPhase& P, int& u0, int& u1) {
    CbRun r;
    r.KT = P.K / GS;
    r.gps = KSL / GS;
    r.nsl = (r.KT + r.gps - 1) / r.gps;
    strip_range(P.N / 16, c, G, u0, u1);
    r.nu = u1 - u0;
    return r;
  };

  if (warp == kCW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int st = 0;
      bool ok = true;
      for (int ph = 0; ph < a.nphases && ok; ++ph) {
        const ChainBPhase& P = a.ph[ph];
        int u0, u1;
        const CbRun r = runs(P, u0, u1);
        for (int sl = 0; sl < r.nsl && ok; ++sl) {
          const int g0 = sl * r.gps, g1 = min(r.KT, g0 + r.gps);
          for (int u = u0; u < u1 && ok; ++u) {
            const uint8_t* src = P.tiles + ((size_t)u * r.KT + g0) * TB;
            for (int s0 = 0; s0 < g1 - g0; s0 += kCbPieces) {
              const int slot = st % S;
              if (st >= S && !mbar_wait(&empty[slot], ((st / S) - 1) & 1)) {
                ok = false;
                break;
              }
              const uint32_t bytes = (uint32_t)min(kCbPieces, g1 - g0 - s0) * TB;
              mbar_arrive_expect_tx(&full[slot], bytes);
              bulk_g2s(ring + (size_t)slot * kStageBytes, src + (size_t)s0 * TB, bytes, &full[slot]);
              ++st;
            }
          }
        }
      }
      const uint64_t deadline = globaltimer_ns() + kWaitNs;
      for (int s = 0; s < S && s < st; ++s) {
        const int last = s + ((st - 1 - s) / S) * S;
        if (!mbar_wait_until(&full[s], (last / S) & 1, deadline)) {
          flag_error(kDevCopyDrainTimeout);
          break;
        }
      }
    }
    return;
  }

  if (warp == kCW + 1) {
    // -------------------------------------------------------------- reducer
    // For each strip, in the consumers' order: wait until all 16 warps have
    // written their partials, sum them in warp order (each lane: rows gr /
    // gr + 8 of the strip, batch rows 8 nt + 2 tq (+1)), add slices in slice
    // order, apply the epilogue after the last slice, free the buffer.
    const int gr = lane >> 2, tq = lane & 3;
    int sq = 0;
    bool ok = true;
    for (int ph = 0; ph < a.nphases && ok; ++ph) {
      const ChainBPhase& P = a.ph[ph];
      int u0, u1;
      const CbRun r = runs(P, u0, u1);
      for (int sl = 0; sl < r.nsl && ok; ++sl) {
        for (int ul = 0; ul < r.nu; ++ul, ++sq) {
          const int bsel = sq & 1;
          const bool landed = mbar_wait(&sfull[bsel], (sq >> 1) & 1);
          if (__any_sync(0xffffffffu, !landed)) {
            ok = false;
            break;
          }
          float v[4 * NT];
#pragma unroll
          for (int i = 0; i < 4 * NT; ++i) v[i] = 0.f;
          for (int w = 0; w < kCW; ++w) {
            const float* src = pbuf + (((size_t)bsel * kCW + w) * NT * 32 + lane) * 4;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const float4 p4 = *reinterpret_cast<const float4*>(src + nt * 128);
              v[4 * nt] += p4.x;
              v[4 * nt + 1] += p4.y;
              v[4 * nt + 2] += p4.z;
              v[4 * nt + 3] += p4.w;
            }
          }
          __syncwarp();  // every lane's reads of the buffer before it is freed
          if (lane == 0) mbar_arrive(&sfree[bsel]);
          if (r.nsl > 1) {  // slices add up in slice order
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int row = gr + ((e & 2) ? 8 : 0), m = 8 * nt + 2 * tq + (e & 1);
                float& cell = acc_s[((size_t)ul * 16 + row) * MR + m];
                cell += v[4 * nt + e];
                v[4 * nt + e] = cell;
              }
          }
          if (sl != r.nsl - 1) continue;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int row = gr + ((e & 2) ? 8 : 0), m = 8 * nt + 2 * tq + (e & 1);
              if (m >= M) continue;
              if (P.epi == kEpiSwiGLU) {
                if (e & 2) continue;  // the up row (gr + 8) is paired with gate row gr in this lane
                // fast.py:170-171: bf16(silu(gate)) * up, each op rounded to bf16
                const float gt = round_bf16(v[4 * nt + e]), up = round_bf16(v[4 * nt + e + 2]);
                const float sg = round_bf16(gt / (1.0f + expf(-gt)));
                P.y[(size_t)m * P.ldy + 8 * (u0 + ul) + gr] = f32_to_bf16_bits(sg * up);
              } else {
                float o = v[4 * nt + e];
                if (P.epi == kEpiResidual)  // fast.py:168 / :170: residual + bf16(linear(...)), rounded to bf16
                  o = bf16_bits_to_f32(res_s[((size_t)ul * 16 + row) * MR + m]) + round_bf16(o);
                P.y[(size_t)m * P.ldy + 16 * (u0 + ul) + row] = f32_to_bf16_bits(o);
              }
            }
        }
      }
      __syncwarp();
      if (ok && lane == 0) {
        __threadfence_block();  // this phase's outputs before the count
        *reinterpret_cast<volatile int*>(imisc + 1) = ph + 1;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int tid = threadIdx.x;
  const int gr = lane >> 2, tq = lane & 3;
  int slot = 0;
  uint32_t par = 0;
  uint32_t xpar = 0;  // phase parity of xbar
  int arrived = 0;
  int sq = 0;  // strips flushed in this launch (partial buffer sq & 1)
  static_assert(kChainWarps == 16, "partial buffers hold 16 warps");
  bool bail = false;
  // staging roles: thread t stages rows t / tpr (tpr threads per row), its
  // 32-column blocks t % tpr, t % tpr + tpr, ... of the slice
  constexpr int kTpr = kCThr / MR;
  const int srow = tid / kTpr, scol = tid % kTpr;
  const int swarps = kTpr / 32;  // warps per staged row (1 or 2)

  for (int ph = 0; ph < a.nphases && !bail; ++ph) {
    const ChainBPhase& P = a.ph[ph];
    int u0, u1;
    const CbRun r = runs(P, u0, u1);
    if (r.nsl > 1)  // slice sums (such phases own at most uaux strips)
      for (int i = tid; i < r.nu * 16 * MR; i += kCThr) acc_s[i] = 0.f;

    if (ph == 0) {
      pdl_wait();
    } else {
      if (tid == 0 && !grid_wait(a.barrier, (unsigned)G * ph)) {
        flag_error(kDevWaitTimeout);
        imisc[0] = 1;
      }
      chain_sync();
      if (imisc[0]) {
        bail = true;
        break;
      }
    }
    // the residual of this CTA's strips (written before this phase), read
    // by the reducing warps; ordered by the staging barrier below
    if (P.epi == kEpiResidual) {
      for (int i = tid; i < r.nu * 16 * M; i += kCThr) {
        const int ul = i / (16 * M), rem = i - ul * 16 * M, row = rem / M, m = rem - row * M;
        res_s[((size_t)ul * 16 + row) * MR + m] = __ldcg(P.residual + (size_t)m * P.ldr + 16 * (u0 + ul) + row);
      }
    }

    float acc[NT][4], acc2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = acc2[nt][e] = 0.f;
    // this warp's sums of a strip into partial buffer sq & 1 (once the
    // reducer warp is done with the strip two back that used it)
    auto flush = [&](int sq) {
      const int bsel = sq & 1;
      if (sq >= 2) {
        const bool freed = mbar_wait(&sfree[bsel], ((sq >> 1) - 1) & 1);
        if (__any_sync(0xffffffffu, !freed)) imisc[0] = 1;
      }
      // [buffer][warp][n-tile][lane] float4: a store covers 512 contiguous bytes
      float* dst = pbuf + (((size_t)bsel * kCW + warp) * NT * 32 + lane) * 4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float4*>(dst + nt * 128) = make_float4(acc[nt][0] + acc2[nt][0], acc[nt][1] + acc2[nt][1],
                                                                 acc[nt][2] + acc2[nt][2], acc[nt][3] + acc2[nt][3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nt][e] = acc2[nt][e] = 0.f;
      __syncwarp();  // the warp's partial stores before lane 0's release
      if (lane == 0) mbar_arrive(&sfull[bsel]);
    };

    for (int sl = 0; sl < r.nsl && !bail; ++sl) {
      const int g0 = sl * r.gps, g1 = min(r.KT, g0 + r.gps);
      const int kc = (g1 - g0) * GS;  // columns of this slice
      // ---- stage x[:, slice] (RMSNorm phases have a single slice): the M
      //      rows land in shared memory by bulk copies (one round trip) and
      //      are normalised there
      if (sl > 0) chain_sync();  // every warp is done with the previous slice
      const int nblk = kc / 32;
      if (tid == 0) {
        // generic-proxy accesses of xs (the previous slice) and the phase
        // inputs written through the grid barrier before the async copies
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arrive_expect_tx(xbar, (uint32_t)(M * kc * 2));
        for (int mm = 0; mm < M; ++mm)
          bulk_g2s(xs + (size_t)mm * XS, P.x + (size_t)mm * P.ldx + g0 * GS, (uint32_t)(kc * 2), xbar);
      }
      if (!mbar_wait(xbar, xpar)) imisc[0] = 1;
      xpar ^= 1u;
      uint8_t* xrow = xs + (size_t)srow * XS;
      float rinv = 1.f;
      if (P.norm_w) {
        float ss = 0.f;
        if (srow < M) {
          for (int cc = scol; cc < 4 * nblk; cc += kTpr) {  // 16-byte chunks, consecutive per lane
            {
              const uint4 v = reinterpret_cast<const uint4*>(xrow)[cc];
              const uint32_t u4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float lo = __uint_as_float(u4[q] << 16), hi = __uint_as_float(u4[q] & 0xFFFF0000u);
                ss = fmaf(lo, lo, ss);
                ss = fmaf(hi, hi, ss);
              }
            }
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) misc[8 + warp] = ss;
        chain_sync();
        float t = 0.f;
        for (int w = 0; w < swarps; ++w) t += misc[8 + srow * swarps + w];
        rinv = rsqrtf(t / (float)P.K + a.eps);
      }
      // x stays in its natural order (the strip packing permutes the MMAs'
      // k positions to match); RMSNorm phases normalise it in place.  Rows
      // past M are never written: they only feed output columns past M,
      // which are not stored.
      if (P.norm_w && srow < M) {
        // 16-byte chunks, consecutive per lane (no bank conflicts); the norm
        // weights of four chunks are loaded before they are used
        const int nch = 4 * nblk;
        const uint4* nwp = reinterpret_cast<const uint4*>(P.norm_w + g0 * GS);
        uint4* xr4 = reinterpret_cast<uint4*>(xrow);
        for (int c0 = scol; c0 < nch; c0 += 4 * kTpr) {
          uint4 nv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (c0 + e * kTpr < nch) nv[e] = __ldg(nwp + c0 + e * kTpr);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int cc = c0 + e * kTpr;
            if (cc >= nch) break;
            const uint4 v = xr4[cc];
            uint32_t u4[4] = {v.x, v.y, v.z, v.w};
            const uint32_t w4[4] = {nv[e].x, nv[e].y, nv[e].z, nv[e].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              // model.py:34-40: bf16(h * rsqrt(var + eps)), then bf16(weight * that)
              const float v0 = round_bf16(__uint_as_float(w4[q] << 16) * round_bf16(__uint_as_float(u4[q] << 16) * rinv));
              const float v1 = round_bf16(__uint_as_float(w4[q] & 0xFFFF0000u) *
                                          round_bf16(__uint_as_float(u4[q] & 0xFFFF0000u) * rinv));
              u4[q] = (__float_as_uint(v0) >> 16) | (__float_as_uint(v1) & 0xFFFF0000u);
            }
            xr4[cc] = make_uint4(u4[0], u4[1], u4[2], u4[3]);
          }
        }
      }
      chain_sync();
      if (imisc[0]) {
        bail = true;
        break;
      }

      // ---- this slice's pieces: strip by strip, one piece per warp per stage
      for (int ul = 0; ul < r.nu; ++ul) {
        for (int s0 = 0; s0 < g1 - g0; s0 += kCbPieces) {
          const bool landed = mbar_wait(&full[slot], par);
          if (__any_sync(0xffffffffu, !landed)) {
            bail = true;
            break;
          }
          const int k = g0 + s0 + warp;  // this warp's group
          if (k < g1) {
            const uint8_t* tile = ring + (size_t)slot * kStageBytes + (size_t)warp * TB;
            const uint2 pw = *reinterpret_cast<const uint2*>(tile + 8 * GS + 8 * gr);
            const uint32_t sc0 = __byte_perm(pw.x, 0u, 0x1010), zr0 = __byte_perm(pw.x, 0u, 0x3232);
            const uint32_t sc1 = __byte_perm(pw.y, 0u, 0x1010), zr1 = __byte_perm(pw.y, 0u, 0x3232);
            const uint4* wt = reinterpret_cast<const uint4*>(tile);
            const size_t xo = (size_t)(k - g0) * GS * 2 + 16 * tq;
#pragma unroll
            for (int h = 0; h < GS / 64; ++h) {
              const uint4 wv = wt[h * 32 + lane];
              const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
              uint32_t bx[NT][8];
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                const uint8_t* xb = xs + (size_t)(gr + 8 * nt) * XS + xo + 128 * h;
                const uint4 xa = *reinterpret_cast<const uint4*>(xb);
                const uint4 xc = *reinterpret_cast<const uint4*>(xb + 64);
                bx[nt][0] = xa.x;
                bx[nt][1] = xa.y;
                bx[nt][2] = xa.z;
                bx[nt][3] = xa.w;
                bx[nt][4] = xc.x;
                bx[nt][5] = xc.y;
                bx[nt][6] = xc.z;
                bx[nt][7] = xc.w;
              }
#pragma unroll
              for (int l = 0; l < 4; ++l) {
                const uint32_t w = wr[l];
                const uint32_t a0 = w4_ref_pair(lop3_and_or(w, 0x000F000Fu, 0x43004300u), sc0, zr0);
                const uint32_t a1 = w4_ref_pair(lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u), sc1, zr1);
                const uint32_t a2 = w4_ref_pair(lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u), sc0, zr0);
                const uint32_t a3 = w4_ref_pair(lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u), sc1, zr1);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  if (l & 1)
                    mma_bf16(acc2[nt], a0, a1, a2, a3, bx[nt][2 * l], bx[nt][2 * l + 1]);
                  else
                    mma_bf16(acc[nt], a0, a1, a2, a3, bx[nt][2 * l], bx[nt][2 * l + 1]);
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
          if (++slot == S) {
            slot = 0;
            par ^= 1u;
          }
        }
        if (bail) break;
        flush(sq++);  // every warp, pieces or not
      }
      if (bail) imisc[0] = 1;
    }
    // the reducer warp has written every strip of the phase (and is done
    // with acc_s / res_s before the next phase refills them)
    if (tid == 0) {
      const volatile int* done = imisc + 1;
      if (*done < ph + 1) {
        const uint64_t deadline = globaltimer_ns() + kWaitNs;
        for (uint32_t i = 1; *done < ph + 1; ++i)
          if ((i & 63) == 0 && globaltimer_ns() > deadline) {
            flag_error(kDevWaitTimeout);
            imisc[0] = 1;
            break;
          }
      }
      __threadfence_block();
    }
    chain_sync();
    if (imisc[0]) {
      bail = true;
      break;
    }
    if (ph + 1 < a.nphases && tid == 0) {
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.barrier), "r"(1u) : "memory");
      ++arrived;
    }
  }

  if (tid == 0) {
    if (bail) flag_error(kDevWaitTimeout);
    const unsigned rem = (unsigned)(a.nphases - arrived);
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a.barrier), "r"(rem) : "memory");
    if (old + rem == (unsigned)G * (unsigned)a.nphases) atomicExch(a.barrier, 0u);
  }
}

}  // namespace

int w4_chainb_plan(const int* K, const int* N, const int* norm, const int* epi, int nphases, int M, int g,
                   int num_sms, ChainPlan* out) {
  if (nphases < 1 || nphases > kChainMaxPhases || M < 1 || M > 16 || (g != 64 && g != 128 && g != 256) ||
      num_sms < 1)
    return -1;
  ChainPlan p{};
  p.G = num_sms;
  p.kmax = 0;
  p.umax = 1;
  p.uaux = 1;
  for (int i = 0; i < nphases; ++i) {
    if (K[i] <= 0 || N[i] <= 0 || K[i] % g || N[i] % 16) return -1;
    if (norm[i] && K[i] > kCbSlice) return -1;  // RMSNorm statistics need the row in one slice
    p.kmax = std::max(p.kmax, std::min(K[i], kCbSlice));
  }
  for (int i = 0; i < nphases; ++i) {
    const int u = (N[i] / 16 + p.G - 1) / p.G;
    p.umax = std::max(p.umax, u);
    if (epi[i] == kEpiResidual || K[i] > p.kmax) p.uaux = std::max(p.uaux, u);
  }
  const int rows = M > 8 ? 16 : 8;
  const int tb = strip_tile_bytes(g);
  p.stages = 0;
  for (int s = 12; s >= 2; --s) {
    if (cb_layout(s, tb, p.kmax, rows, p.uaux).total <= 227 * 1024) {
      p.stages = s;
      break;
    }
  }
  if (p.stages == 0) return -2;
  p.smem = cb_layout(p.stages, tb, p.kmax, rows, p.uaux).total;
  *out = p;
  return 0;
}

cudaError_t w4_chainb_launch(const ChainBArgs& args, int g, const ChainPlan& p, cudaStream_t stream, int use_pdl) {
  ChainBArgs a = args;
  a.stages = p.stages;
  a.kslice = p.kmax;
  a.uaux = p.uaux;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.G);
  cfg.blockDim = dim3((kChainWarps + 2) * 32);  // + producer + reducer
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl ? 1 : 0;
  const int two = a.M > 8 ? 1 : 0;
  const int gi = (g == 64 ? 0 : (g == 128 ? 1 : 2)) * 2 + two;
  using K_t = void (*)(const ChainBArgs);
  static const K_t kerns[6] = {w4_chainb_kernel<64, 1>,  w4_chainb_kernel<64, 2>,  w4_chainb_kernel<128, 1>,
                               w4_chainb_kernel<128, 2>, w4_chainb_kernel<256, 1>, w4_chainb_kernel<256, 2>};
  static bool done[6] = {false, false, false, false, false, false};
  if (!done[gi]) {
    cudaError_t e = cudaFuncSetAttribute(kerns[gi], cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kerns[gi], (kChainWarps + 2) * 32, 227 * 1024);
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorInvalidConfiguration;
    done[gi] = true;
  }
  return cudaLaunchKernelEx(&cfg, kerns[gi], a);
}

}  // namespace mtl
