// Persistent W4A16 GEMV chain for the batch-1 decode step (sm_100a).
//
// One launch runs a sequence of dependent W4 linears of the decoder - o ->
// gate|up -> down -> the next layer's q|k|v, the order in which the
// reference's decode step calls torch._weight_int4pack_mm
// (moss_tts_lite/fast.py:165-171, FastMossTTS._linear at fast.py:107-121),
// with the RMSNorm before gate|up and q|k|v, the residual adds after o and
// down and the SwiGLU between gate|up and down fused in - on one CTA per SM:
//
//  * each phase's N/16 strips (w4_chain.cuh) are split over the CTAs in
//    contiguous ranges; a CTA owns whole strips over the full K, so no
//    output needs another CTA's partial sums (no split-K fixup);
//  * a producer warp streams every phase's strips of its CTA, in order,
//    through one shared-memory ring of bulk copies: the next phase's
//    weights land while the current phase drains and the grid waits at
//    the phase barrier;
//  * 16 consumer warps take two pieces (16 rows x one group) each per ring
//    stage and multiply with the reference's operand bf16((q - 8) s + z)
//    (one rounding, as the register-MMA GEMV forms it) in m16n8k16 MMAs
//    with fp32 accumulation, even / odd k16-steps in two chains;
//  * the CTA sums its warps' per-strip partials in fixed order (results
//    are bitwise reproducible) and applies the phase's epilogue; one thread
//    then releases an add on a grid counter, and the next phase starts when
//    the counter reaches G x (phases done) - a bounded acquire spin;
//  * every CTA adds exactly `nphases` to the counter; the add that brings it
//    to G x nphases resets it to 0 for the next launch.
//
// All CTAs must be resident at once: the grid is one CTA per SM and the
// plan checks that the shared memory admits it.  Every wait (ring
// mbarriers, the grid counter) is bounded (kWaitNs); a CTA that gives up
// flags the device status, adds its remaining arrivals so that no other CTA
// waits on it, and returns after its copies in flight have landed.
#include "common.cuh"
#include "w4_gemv.cuh"
#include "w4_chain.cuh"

#include <algorithm>

namespace mtl {

namespace {

constexpr int kCW = kChainWarps;
constexpr int kCThr = kCW * 32;
constexpr int kPer = 2;                    // pieces per consumer warp per ring stage
constexpr int kStagePieces = kCW * kPer;   // pieces per ring stage (one bulk copy)
constexpr int kChainMiscWords = 64;  // [0] bail flag, [4] 1/rms, [8, 8 + kCW) warp sums of squares

struct ChainLayout {
  size_t bar, ring, xs, part, misc, total;
};

__host__ __device__ __forceinline__ size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline ChainLayout chain_layout(int stages, int tile_bytes, int kmax, int umax) {
  ChainLayout L;
  size_t o = 0;
  L.bar = o;
  o += round_up((size_t)2 * stages * 8, 128);
  L.ring = o;
  o += (size_t)stages * kStagePieces * tile_bytes;
  o = round_up(o, 128);
  L.xs = o;
  o += (size_t)kmax * 2;
  o = round_up(o, 16);
  L.part = o;
  o += (size_t)umax * kCW * 16 * 4;
  L.misc = o;
  o += kChainMiscWords * 4;
  L.total = round_up(o, 128);
  return L;
}

__device__ __forceinline__ void chain_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCThr) : "memory"); }

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Spin (bounded) until *bar >= target.  (Relaxed polls with one acquire
// fence at the end measured slower on B200.)
__device__ bool grid_wait(const unsigned* bar, unsigned target) {
  if (ld_acquire_gpu(bar) >= target) return true;
  const uint64_t deadline = globaltimer_ns() + kWaitNs;
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_gpu(bar) >= target) return true;
    if ((i & 15) == 0 && globaltimer_ns() > deadline) return false;
  }
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A CTA's strip range [u0, u1) of a phase with U strips.
__device__ __forceinline__ void strip_range(int U, int c, int G, int& u0, int& u1) {
  u0 = (int)(((long long)U * c) / G);
  u1 = (int)(((long long)U * (c + 1)) / G);
}

template <int GS>
__global__ void __launch_bounds__((kCW + 1) * 32, 1) w4_chain_kernel(const ChainArgs a) {
  extern __shared__ __align__(128) uint8_t chain_sm[];
  constexpr int TB = 8 * GS + 64;  // strip tile bytes
  constexpr uint32_t kStageBytes = (uint32_t)kStagePieces * TB;
  const int S = a.stages;
  const ChainLayout L = chain_layout(S, TB, a.kmax, a.umax);
  uint64_t* full = reinterpret_cast<uint64_t*>(chain_sm + L.bar);
  uint64_t* empty = full + S;
  uint8_t* ring = chain_sm + L.ring;
  uint16_t* xs = reinterpret_cast<uint16_t*>(chain_sm + L.xs);
  float* part = reinterpret_cast<float*>(chain_sm + L.part);
  float* misc = reinterpret_cast<float*>(chain_sm + L.misc);
  int* imisc = reinterpret_cast<int*>(misc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);  // every consumer warp arrives once per stage
    }
    fence_mbar_init();
    imisc[0] = 0;
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kCW) {
    // ------------------------------------------------------------ producer
    // Weights do not depend on any phase's input: stream them all, as far
    // ahead as the ring allows.
    if (lane == 0) {
      int st = 0;
      bool ok = true;
      for (int ph = 0; ph < a.nphases && ok; ++ph) {
        const ChainPhase& P = a.ph[ph];
        const int KT = P.K / GS;
        int u0, u1;
        strip_range(P.N / 16, c, G, u0, u1);
        const int n = (u1 - u0) * KT;
        const uint8_t* src = P.tiles + (size_t)u0 * KT * TB;
        for (int s0 = 0; s0 < n; s0 += kStagePieces) {
          const int slot = st % S;
          if (st >= S && !mbar_wait(&empty[slot], ((st / S) - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t bytes = (uint32_t)min(kStagePieces, n - s0) * TB;
          mbar_arrive_expect_tx(&full[slot], bytes);
          bulk_g2s(ring + (size_t)slot * kStageBytes, src + (size_t)s0 * TB, bytes, &full[slot]);
          ++st;
        }
      }
      // the last copy issued on each slot lands before the CTA exits
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

  // -------------------------------------------------------------- consumers
  const int tid = threadIdx.x;
  const int gr = lane >> 2, tq = lane & 3;
  int slot = 0;        // ring slot and phase parity of the next stage (all phases)
  uint32_t par = 0;
  int arrived = 0;     // grid-counter adds of this CTA (thread 0)
  bool bail = false;

  for (int ph = 0; ph < a.nphases && !bail; ++ph) {
    const ChainPhase& P = a.ph[ph];
    const int K = P.K, KT = K / GS;
    int u0, u1;
    strip_range(P.N / 16, c, G, u0, u1);
    const int nu = u1 - u0, n = nu * KT;

    // x staging: thread t owns the 16-byte chunks t, t + 512, ... (consecutive
    // threads on consecutive chunks: coalesced loads, conflict-free stores)
    const int nch = K / 8;  // <= 4 kCThr (K <= kChainMaxK)
    // layer constants first: the norm weights of this thread's chunks
    uint4 nw[4];
    if (P.norm_w) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (tid + e * kCThr < nch) nw[e] = __ldg(reinterpret_cast<const uint4*>(P.norm_w) + tid + e * kCThr);
    }
    for (int i = tid; i < nu * kCW * 16; i += kCThr) part[i] = 0.f;

    // wait for this phase's input: the upstream kernel, or the grid
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

    // x (L2 loads: it may have been written by this launch), its RMSNorm
    // statistics and the residual this thread's epilogue adds
    uint4 xv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (tid + e * kCThr < nch) xv[e] = __ldcg(reinterpret_cast<const uint4*>(P.x) + tid + e * kCThr);
    float rres = 0.f;
    if (P.epi == kEpiResidual && tid < nu * 16) rres = bf16_bits_to_f32(__ldcg(P.residual + 16 * u0 + tid));
    float rinv = 1.f;
    if (P.norm_w) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (tid + e * kCThr < nch) {
          const uint32_t u4[4] = {xv[e].x, xv[e].y, xv[e].z, xv[e].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float lo = __uint_as_float(u4[q] << 16), hi = __uint_as_float(u4[q] & 0xFFFF0000u);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
          }
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) misc[8 + warp] = ss;
      chain_sync();
      // every thread sums the warps' partials in the same order
      float tss = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) tss += misc[8 + w];
      rinv = rsqrtf(tss / (float)K + a.eps);
    }
    // stage x as bf16 in its natural order (the strip packing permutes the
    // MMAs' k positions to match)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (tid + e * kCThr >= nch) break;
      uint32_t u4[4] = {xv[e].x, xv[e].y, xv[e].z, xv[e].w};
      if (P.norm_w) {
        const uint32_t w4[4] = {nw[e].x, nw[e].y, nw[e].z, nw[e].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          // model.py:34-40: bf16(h * rsqrt(var + eps)), then bf16(weight * that)
          const float v0 = round_bf16(__uint_as_float(w4[q] << 16) * round_bf16(__uint_as_float(u4[q] << 16) * rinv));
          const float v1 = round_bf16(__uint_as_float(w4[q] & 0xFFFF0000u) *
                                      round_bf16(__uint_as_float(u4[q] & 0xFFFF0000u) * rinv));
          u4[q] = (__float_as_uint(v0) >> 16) | (__float_as_uint(v1) & 0xFFFF0000u);
        }
      }
      reinterpret_cast<uint4*>(xs)[tid + e * kCThr] = make_uint4(u4[0], u4[1], u4[2], u4[3]);
    }
    chain_sync();

    // ------------------------------------------------------------ main loop
    // stage = kCW x kPer consecutive pieces; warp w takes pieces
    // kPer w .. kPer w + kPer - 1 of each stage.  (su, sk) = strip and group
    // of the warp's first piece of the current stage.
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    int cur = -1;
    int su = (kPer * warp) / KT, sk = (kPer * warp) % KT;
    for (int s0 = 0; s0 < n; s0 += kStagePieces) {
      const bool landed = mbar_wait(&full[slot], par);
      if (__any_sync(0xffffffffu, !landed)) {  // warp-uniform: the MMAs below are .aligned
        bail = true;
        break;
      }
      int pu = su, pk = sk;
#pragma unroll
      for (int pp = 0; pp < kPer; ++pp) {
        if (s0 + kPer * warp + pp < n) {
          if (pu != cur) {
            if (cur >= 0 && tq == 0) {
              float* d = part + ((size_t)cur * kCW + warp) * 16;
              d[gr] = acc[0] + acc2[0];
              d[gr + 8] = acc[2] + acc2[2];
            }
            cur = pu;
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = acc2[e] = 0.f;
          }
          const uint8_t* tile = ring + (size_t)slot * kStageBytes + (size_t)(kPer * warp + pp) * TB;
          // params of rows gr and gr + 8, adjacent: one 8-byte load
          const uint2 pw = *reinterpret_cast<const uint2*>(tile + 8 * GS + 8 * gr);
          const uint32_t sc0 = __byte_perm(pw.x, 0u, 0x1010), zr0 = __byte_perm(pw.x, 0u, 0x3232);
          const uint32_t sc1 = __byte_perm(pw.y, 0u, 0x1010), zr1 = __byte_perm(pw.y, 0u, 0x3232);
          const uint4* wt = reinterpret_cast<const uint4*>(tile);
          const uint4* xg = reinterpret_cast<const uint4*>(xs + (size_t)pk * GS) + tq;
#pragma unroll
          for (int h = 0; h < GS / 64; ++h) {
            const uint4 wv = wt[h * 32 + lane];
            const uint4 xa = xg[(2 * h) * 4], xb = xg[(2 * h + 1) * 4];  // x[32q + 8t ..], q = 2h | 2h + 1
            const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
            const uint32_t bx[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int l = 0; l < 4; ++l) {
              const uint32_t w = wr[l];
              const uint32_t a0 = w4_ref_pair(lop3_and_or(w, 0x000F000Fu, 0x43004300u), sc0, zr0);
              const uint32_t a1 = w4_ref_pair(lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u), sc1, zr1);
              const uint32_t a2 = w4_ref_pair(lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u), sc0, zr0);
              const uint32_t a3 = w4_ref_pair(lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u), sc1, zr1);
              if (l & 1)
                mma_bf16(acc2, a0, a1, a2, a3, bx[2 * l], bx[2 * l + 1]);
              else
                mma_bf16(acc, a0, a1, a2, a3, bx[2 * l], bx[2 * l + 1]);
            }
          }
        }
        if (++pk == KT) {
          pk = 0;
          ++pu;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == S) {
        slot = 0;
        par ^= 1u;
      }
      sk += kStagePieces;
      while (sk >= KT) {
        sk -= KT;
        ++su;
      }
    }
    if (bail) imisc[0] = 1;
    if (!bail && cur >= 0 && tq == 0) {
      float* d = part + ((size_t)cur * kCW + warp) * 16;
      d[gr] = acc[0] + acc2[0];
      d[gr + 8] = acc[2] + acc2[2];
    }
    chain_sync();
    if (imisc[0]) {
      bail = true;
      break;
    }

    // ------------------------------------------ CTA reduce (fixed order) + epilogue
    if (P.epi == kEpiSwiGLU) {
      for (int t = tid; t < nu * 8; t += kCThr) {
        const int ul = t >> 3, r = t & 7;
        const float* pp = part + (size_t)ul * kCW * 16;
        float vg = 0.f, vu = 0.f;
        for (int w = 0; w < kCW; ++w) {
          vg += pp[w * 16 + r];
          vu += pp[w * 16 + r + 8];
        }
        // fast.py:170-171: bf16(silu(gate)) * up, each op rounded to bf16
        const float gt = round_bf16(vg), up = round_bf16(vu);
        const float sg = round_bf16(gt / (1.0f + expf(-gt)));
        P.y[(size_t)8 * (u0 + ul) + r] = f32_to_bf16_bits(sg * up);
      }
    } else {
      for (int t = tid; t < nu * 16; t += kCThr) {
        const int ul = t >> 4, r = t & 15;
        const float* pp = part + (size_t)ul * kCW * 16 + r;
        float v = 0.f;
        for (int w = 0; w < kCW; ++w) v += pp[w * 16];
        const int nn = 16 * u0 + t;
        if (P.epi == kEpiResidual) {
          // fast.py:168 / :170: residual + bf16(linear(...)), rounded to bf16
          const float rv = t < kCThr ? rres : bf16_bits_to_f32(__ldcg(P.residual + nn));
          v = rv + round_bf16(v);
        }
        P.y[nn] = f32_to_bf16_bits(v);
      }
    }
    chain_sync();
    if (ph + 1 < a.nphases && tid == 0) {
      // release: this CTA's outputs (ordered before by the barrier) are
      // visible before the add
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.barrier), "r"(1u) : "memory");
      ++arrived;
    }
  }

  // Every CTA adds nphases in total (fewer phases done -> the rest now, so
  // that no CTA waits on this one); the add reaching G x nphases re-arms.
  if (tid == 0) {
    const unsigned rem = (unsigned)(a.nphases - arrived);
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a.barrier), "r"(rem) : "memory");
    if (old + rem == (unsigned)G * (unsigned)a.nphases) atomicExch(a.barrier, 0u);
  }
}

// Strip packing: one thread per uint32 word of a tile.
__global__ void pack_strip_kernel(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles) {
  const int KT = K / g, wpt = 2 * g + 16;
  const long long total = (long long)(N / 16) * KT * wpt;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int wi = (int)(idx % wpt);
  const long long tile = idx / wpt;
  const int k = (int)(tile % KT), u = (int)(tile / KT);
  uint32_t* out = reinterpret_cast<uint32_t*>(tiles + (size_t)tile * strip_tile_bytes(g));
  if (wi < 2 * g) {
    const int h = wi >> 7, lane = (wi >> 2) & 31, l = wi & 3;
    const int gr = lane >> 2, t = lane & 3;
    const int r0 = 16 * u + gr, c0 = k * g + 32 * (2 * h + (l >> 1)) + 8 * t + 4 * (l & 1);
    uint32_t w = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int row = r0 + ((s & 1) ? 8 : 0);
      const int col = c0 + ((s & 2) ? 2 : 0) + (s >> 2);
      w |= (uint32_t)(q[(size_t)row * K + col] & 0xFu) << (4 * s);
    }
    out[wi] = w;
  } else {
    const int p = wi - 2 * g;  // param word p: row (p / 2) + 8 (p % 2)
    const size_t n = (size_t)16 * u + (p >> 1) + 8 * (p & 1);
    const size_t o = ((size_t)k * N + n) * 2;
    out[wi] = (uint32_t)qsz[o] | ((uint32_t)qsz[o + 1] << 16);
  }
}

}  // namespace

int w4_chain_plan(const int* K, const int* N, int nphases, int g, int num_sms, ChainPlan* out) {
  if (nphases < 1 || nphases > kChainMaxPhases || (g != 64 && g != 128 && g != 256) || num_sms < 1) return -1;
  ChainPlan p{};
  p.G = num_sms;
  p.kmax = 0;
  p.umax = 1;
  for (int i = 0; i < nphases; ++i) {
    if (K[i] <= 0 || N[i] <= 0 || K[i] % g || N[i] % 16 || K[i] > kChainMaxK) return -1;
    p.kmax = std::max(p.kmax, K[i]);
    p.umax = std::max(p.umax, (N[i] / 16 + p.G - 1) / p.G);
  }
  const int tb = strip_tile_bytes(g);
  const size_t budget = 227 * 1024;
  p.stages = 0;
  for (int s = 16; s >= 2; --s) {
    if (chain_layout(s, tb, p.kmax, p.umax).total <= budget) {
      p.stages = s;
      break;
    }
  }
  if (p.stages == 0) return -2;
  p.smem = chain_layout(p.stages, tb, p.kmax, p.umax).total;
  *out = p;
  return 0;
}

cudaError_t w4_chain_launch(const ChainArgs& args, int g, const ChainPlan& p, cudaStream_t stream, int use_pdl) {
  ChainArgs a = args;
  a.stages = p.stages;
  a.kmax = p.kmax;
  a.umax = p.umax;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.G);
  cfg.blockDim = dim3((kCW + 1) * 32);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl ? 1 : 0;
  auto kern = g == 64 ? w4_chain_kernel<64> : (g == 128 ? w4_chain_kernel<128> : w4_chain_kernel<256>);
  const int gi = g == 64 ? 0 : (g == 128 ? 1 : 2);
  // Once per kernel (the first call, outside any capture): the shared-memory
  // opt-in, and the check that a CTA fits on an SM at the largest size a
  // plan uses - the grid is one CTA per SM, all resident together.
  static bool done[3] = {false, false, false};
  if (!done[gi]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (kCW + 1) * 32, 227 * 1024);
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorInvalidConfiguration;
    done[gi] = true;
  }
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t w4_pack_strip(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles,
                          cudaStream_t s) {
  const long long total = (long long)(N / 16) * (K / g) * (2 * g + 16);
  const int threads = 256;
  const long long blocks = (total + threads - 1) / threads;
  pack_strip_kernel<<<(unsigned)blocks, threads, 0, s>>>(q, qsz, K, N, g, tiles);
  return cudaGetLastError();
}

}  // namespace mtl
