// W4A16 GEMV for batch 1 on the 5th-generation tensor cores (tcgen05).
//
// Replaces torch._weight_int4pack_mm for one activation row as the reference
// calls it in its decode step (moss_tts_lite/fast.py:118, gptq.py:582,
// fast_native.py:169): y = x . W^T, W = bf16((q - 8) * scale + zero) per
// group (gptq.py:87-97; rounded once to bf16, as torch's int4 GEMM forms its
// operand), fp32 accumulation, bf16 output, with the same fused
// RMSNorm prologue and store / residual / SwiGLU epilogues as the
// register-MMA kernel in w4_gemv.cu.
//
// Why tcgen05: at batch 1 every weight passes through one multiply-add, and
// the legacy warp MMA (mma.sync m16n8k16, 256 weights per instruction)
// cannot keep up with HBM on sm_100.  Here one thread issues one
// tcgen05.mma per 128 rows x 16 k = 2048 weights:
//
//   A (weights)      TMEM, 128 lanes (rows) x 8 columns per k16 step, written
//                    by the dequantising warps with tcgen05.st: each thread
//                    owns one output row and turns 16 int4 codes into eight
//                    bf16 pairs of effective weights (one shift + LOP3 per
//                    pair for 128 + q, then two bf16x2 FMAs: q - 8, exact,
//                    and (q - 8) scale + zero, one rounding);
//   B (activations)  shared memory, K-major, no swizzle.  Only column 0 of
//                    the N = 16 MMA is used: with the k-chunk stride (LBO) set
//                    to 16 bytes the canonical core matrices overlap and row 0
//                    of every core matrix is the next 8 activations, so B is
//                    the activation vector itself, contiguous (columns 1..15
//                    of D hold sums against shifted activations and are never
//                    read);
//   D (fp32)         TMEM, 128 lanes x 16 columns, one group of k per MMA
//                    chain; the dequantising warps read column 0 back
//                    (tcgen05.ld) and add it to the row's fp32 sum.
//
// Pipeline per CTA (2 per SM): warp 0 streams tiles with 1-D bulk copies into
// a shared-memory ring (before the programmatic-dependent-launch wait: the
// weights do not depend on the upstream kernel); warp 1 owns TMEM and issues
// the MMAs; warps 2-5 dequantise tile i into A buffer i % 3 and then read
// back the accumulator of tile i - 2, so two tiles' MMAs are in flight while
// the next one is dequantised.  Stream-K over tiles with the same
// deterministic last-arriver split-K fixup as the register-MMA kernel.
//
// Tile layout ("TC tile"): 128 output rows x one group, n-block-major
// (tile t = nb * (K/g) + G):
//   words  : [g/16 k16-steps][128 rows][2] uint32 — word 0 holds codes
//            k0..k7 of the step with nibble i = k_{2i} and nibble i + 4 =
//            k_{2i+1}; word 1 holds k8..k15 the same way
//   params : [128 rows] uint32 = bf16 scale | bf16 zero << 16
#include "common.cuh"

#include <algorithm>

namespace mtl {

constexpr int kTcRows = 128;  // UMMA M: output rows per tile
constexpr int kTcWarps = 6;   // 0 producer, 1 MMA + TMEM owner, 2..5 dequantise / epilogue
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcMaxK = 16384;
constexpr int kTcTmemCols = 256;
constexpr int kTcBufs = 3;    // A / D buffers in flight (TMEM: 3 x (8 g/16) + 3 x 16 columns)
// kind::f16, D fp32, A and B bf16, both K-major, N = 16, M = 128
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

struct TcPlan {
  int T, KT, nblocks, G, tps, stages, maxc, tile_bytes;
  size_t smem, partial_bytes;
};

struct TcArgs {
  const uint16_t* x;  // bf16 [K]
  int K, N, g;
  const uint8_t* tiles;
  const uint16_t* norm_w;  // nullable: fused RMSNorm prologue (bf16 [K])
  float norm_eps;
  int epi;
  const uint16_t* residual;  // bf16 [N] (kEpiResidual; may alias y)
  uint16_t* y;
  float* partials;  // [nblocks][maxc][128]
  int* counters;    // [nblocks]
  TcPlan p;
};

inline int tc_tile_bytes(int g) { return kTcRows * g / 2 + kTcRows * 4; }

namespace {

// The CTA whose stream-K range holds tile t (32-bit: (t + 1) G <= T G < 2^32,
// checked by w4_tc_plan).
__host__ __device__ __forceinline__ int tc_cta_of_tile(long long t, int G, int T) {
  return (int)(((uint32_t)(t + 1) * (uint32_t)G - 1u) / (uint32_t)T);
}
__host__ __device__ __forceinline__ size_t tc_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct TcSmem {
  size_t bar, misc, ring, xs, total;
};
__host__ __device__ inline TcSmem tc_smem(const TcPlan& p, int K, int g) {
  TcSmem L;
  size_t o = 0;
  L.bar = o;
  o += tc_align((size_t)(2 * p.stages + 3 * kTcBufs) * 8, 128);
  L.misc = o;
  o += 128;
  L.ring = o;
  o += (size_t)p.stages * p.tps * p.tile_bytes;
  o = tc_align(o, 128);
  L.xs = o;
  o += (size_t)(K + 128) * 2;  // + overreach of the last overlapping core matrix
  L.total = tc_align(o, 128);
  return L;
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t v;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v) : "r"(taddr) : "memory");
  return v;
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld with the loaded register as an operand (no use of it can
// be scheduled before the wait).
__device__ __forceinline__ void tmem_wait_ld1(uint32_t& r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r) : : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[tmem] . B[smem desc], issued by one thread
__device__ __forceinline__ void tc_mma(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` once every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem_tc() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, no swizzle, start address `addr`,
// leading (k-chunk) byte offset 16, stride (8-row group) byte offset 128.
__device__ __forceinline__ uint64_t b_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
         (1ull << 46);
}

__global__ void __launch_bounds__(kTcThreads, 2) w4_tc_kernel(const __grid_constant__ TcArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const TcPlan& p = a.p;
  const int K = a.K, g = a.g, KT = p.KT, KS = g >> 4;
  const int cta = blockIdx.x;
  // stream-K range of this CTA (32-bit: T G < 2^32, checked by the plan)
  const int t0 = (int)(((uint32_t)p.T * (uint32_t)cta) / (uint32_t)p.G);
  const int t1 = (int)(((uint32_t)p.T * (uint32_t)(cta + 1)) / (uint32_t)p.G);
  const int nt = t1 - t0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages, tps = p.tps;
  const size_t stage_bytes = (size_t)tps * p.tile_bytes;
  const TcSmem L = tc_smem(p, K, g);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;         // [kTcBufs] A buffer written
  uint64_t* dfull = afull + kTcBufs;   // [kTcBufs] MMAs of the buffer done (A free, D ready)
  uint64_t* dfree = dfull + kTcBufs;   // [kTcBufs] accumulator read back
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L.misc);
  int* imisc = reinterpret_cast<int*>(smem + L.misc);  // [1] bail, [2] last-arriver flag
  float* red = reinterpret_cast<float*>(smem + L.misc) + 8;  // [4] norm partials
  uint8_t* ring = smem + L.ring;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + L.xs);
  const int acols = KS * 8;                       // TMEM columns of one A buffer
  const int dcol0 = kTcBufs * acols;              // first accumulator column

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTcRows * tps);  // every dequantising thread, per tile of the stage
    }
    for (int b = 0; b < kTcBufs; ++b) {
      mbar_init(&afull[b], kTcRows);
      mbar_init(&dfull[b], 1);
      mbar_init(&dfree[b], kTcRows);
    }
    fence_mbar_init();
    imisc[1] = 0;
    imisc[2] = 0;
  }
  if (warp == 1) {
    tmem_alloc(tslot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int nst = (nt + tps - 1) / tps;
      int issued = 0;
      for (int st = 0; st < nst; ++st) {
        const int s = st % S;
        if (st >= S && !mbar_wait(&empty[s], ((st / S) - 1) & 1)) break;
        const int ntile = min(tps, nt - st * tps);
        const uint32_t bytes = (uint32_t)(ntile * p.tile_bytes);
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(ring + (size_t)s * stage_bytes, a.tiles + (size_t)(t0 + st * tps) * p.tile_bytes, bytes, &full[s]);
        issued = st + 1;
      }
      const uint64_t deadline = globaltimer_ns() + kWaitNs;
      for (int s = 0; s < S && s < issued; ++s) {
        const int last = s + ((issued - 1 - s) / S) * S;
        if (!mbar_wait_until(&full[s], (last / S) & 1, deadline)) {
          flag_error(kDevCopyDrainTimeout);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    named_sync(2, 160);  // activations staged
    if (lane == 0) {
      const uint32_t xaddr = smem_addr(xs);
      int G = t0 % KT;
      int done = 0;
      for (int i = 0; i < nt; ++i) {
        const int buf = i % kTcBufs;
        if (!mbar_wait(&afull[buf], (i / kTcBufs) & 1)) break;
        if (i >= kTcBufs && !mbar_wait(&dfree[buf], ((i - kTcBufs) / kTcBufs) & 1)) break;
        tc_fence_after();
        const uint32_t d = tbase + (uint32_t)(dcol0 + 16 * buf);
        const uint32_t at = tbase + (uint32_t)(buf * acols);
        const uint32_t xg = xaddr + (uint32_t)(G * g * 2);
        for (int ks = 0; ks < KS; ++ks) tc_mma(d, at + 8 * ks, b_desc(xg + 32 * ks), kTcIdesc, ks > 0 ? 1u : 0u);
        tc_commit(&dfull[buf]);
        done = i + 1;
        if (++G == KT) G = 0;
      }
      // every MMA issued has completed before TMEM is released
      if (done > 0) {
        const uint64_t dl = globaltimer_ns() + kWaitNs;
        const int i = done - 1;
        if (!mbar_wait_until(&dfull[i % kTcBufs], (i / kTcBufs) & 1, dl)) flag_error(kDevWaitTimeout);
      }
    }
  } else {
    // ------------------------------------------ dequantise + epilogue (rows)
    const int lt = threadIdx.x - 64;         // 0..127 (staging)
    const int row = 32 * (warp & 3) + lane;  // TMEM lane = output row of the tile
    const uint32_t trow = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
    constexpr int kCh = kTcMaxK / 8 / 128;   // 16-byte chunks of x per thread
    const int nch = K / 8;
    // (a) the norm weight is a layer constant: load it before the wait
    uint4 nv[kCh];
    if (a.norm_w) {
#pragma unroll
      for (int j = 0; j < kCh; ++j)
        if (lt + 128 * j < nch) nv[j] = __ldg(reinterpret_cast<const uint4*>(a.norm_w) + lt + 128 * j);
    }
    pdl_wait();
    // (b) activations (normed if norm_w) as bf16 into xs, 8-value sums into bs
    uint4 xv[kCh];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int c = lt + 128 * j;
      if (c < nch) {
        xv[j] = __ldg(reinterpret_cast<const uint4*>(a.x) + c);
        if (a.norm_w) {
          const uint32_t u[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float lo = __uint_as_float(u[q] << 16), hi = __uint_as_float(u[q] & 0xFFFF0000u);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
          }
        }
      }
    }
    float rinv = 0.f;
    if (a.norm_w) {
      ss = warp_sum(ss);
      if (lane == 0) red[warp - 2] = ss;
      named_sync(1, 128);
      rinv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)K + a.norm_eps);
    }
#pragma unroll
    for (int j = 0; j < kCh; ++j) {
      const int c = lt + 128 * j;
      if (c < nch) {
        uint32_t u[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
        if (a.norm_w) {
          const uint32_t nw[4] = {nv[j].x, nv[j].y, nv[j].z, nv[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // model.py:34-40: bf16(h * rsqrt(var + eps)), then bf16(weight * that)
            const float v0 = round_bf16(__uint_as_float(nw[q] << 16) * round_bf16(__uint_as_float(u[q] << 16) * rinv));
            const float v1 = round_bf16(__uint_as_float(nw[q] & 0xFFFF0000u) *
                                        round_bf16(__uint_as_float(u[q] & 0xFFFF0000u) * rinv));
            u[q] = (__float_as_uint(v0) >> 16) | (__float_as_uint(v1) & 0xFFFF0000u);
          }
        }
        reinterpret_cast<uint4*>(xs)[c] = make_uint4(u[0], u[1], u[2], u[3]);
      }
    }
    if (lt < 16) reinterpret_cast<uint4*>(xs + K)[lt] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem_tc();  // xs is read by the tensor cores (async proxy)
    named_sync(1, 128);
    named_sync(2, 160);           // the MMA issuer may start

    // (c) main loop: dequantise tile i, then read back tile i - lag
    constexpr int lag = kTcBufs - 1;
    int G = t0 % KT, nb = t0 / KT;
    int cur = -1;
    float yacc = 0.f;
    // column block of the tiles whose MMAs are in flight, oldest first
    int qB[lag];
#pragma unroll
    for (int k = 0; k < lag; ++k) qB[k] = -1;
    bool bail = false;
    // A wait that times out sets `bail` (and the CTA flag, so that the other
    // threads stop waiting too) but the warp-collective tcgen05 ld/st and
    // the named barriers still execute in the same order in every thread.
    volatile int* vbail = imisc + 1;
    auto wait_or_bail = [&](uint64_t* bar, uint32_t parity) {
      if (!bail && *vbail) bail = true;
      if (!bail && !mbar_wait(bar, parity)) {
        bail = true;
        *vbail = 1;
      }
    };
    auto flush = [&](int blk, float v) {
      const bool complete = (blk * KT >= t0) && ((blk + 1) * KT <= t1);
      const int n = blk * kTcRows + row;
      // the residual does not depend on the split-K partials: load it first
      const float res = (a.epi == kEpiResidual) ? bf16_bits_to_f32(a.residual[n]) : 0.f;
      if (!complete) {
        const int c_lo = tc_cta_of_tile((long long)blk * KT, p.G, p.T);
        const int c_hi = tc_cta_of_tile((long long)(blk + 1) * KT - 1, p.G, p.T);
        a.partials[((size_t)blk * p.maxc + (cta - c_lo)) * kTcRows + row] = v;
        named_sync(1, 128);
        if (lt == 0) {
          // release this CTA's partials (ordered by the barrier), acquire the
          // other contributors' partials when last
          int old;
          asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.counters + blk) : "memory");
          const int last = (old == c_hi - c_lo);
          if (last) a.counters[blk] = 0;  // re-armed for the next launch
          imisc[2] = last;
        }
        named_sync(1, 128);
        const int last = imisc[2];
        named_sync(1, 128);  // imisc[2] is reused by the next flush
        if (!last) return;
        // contributors in order; up to 8 partial loads issued before the adds
        const int ncon = c_hi - c_lo + 1;
        const float* pp = a.partials + (size_t)blk * p.maxc * kTcRows + row;
        float pv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) pv[j] = j < ncon ? __ldcg(pp + (size_t)j * kTcRows) : 0.f;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < ncon) s += pv[j];
        for (int j = 8; j < ncon; ++j) s += __ldcg(pp + (size_t)j * kTcRows);
        v = s;
      }
      if (a.epi == kEpiSwiGLU) {
        // rows interleaved: 2j = gate j, 2j + 1 = up j (fast.py:170-171:
        // bf16(silu(gate)) * up, each op rounded to bf16)
        const float other = __shfl_xor_sync(0xffffffffu, v, 1);
        if ((row & 1) == 0) {
          const float gt = round_bf16(v), up = round_bf16(other);
          const float sg = round_bf16(gt / (1.0f + expf(-gt)));
          a.y[n >> 1] = f32_to_bf16_bits(sg * up);
        }
      } else if (a.epi == kEpiResidual) {
        // fast.py:168 / :170: residual + bf16(linear(...)), rounded to bf16
        a.y[n] = f32_to_bf16_bits(res + round_bf16(v));
      } else {
        a.y[n] = f32_to_bf16_bits(v);
      }
    };
    // accumulator of tile j (the oldest in flight) -> y: the TMEM load is
    // issued before the next tile's dequantisation (readback_issue) and
    // completed after it (readback)
    uint32_t draw = 0;
    auto readback_issue = [&](int j) {
      const int buf = j % kTcBufs;
      wait_or_bail(&dfull[buf], (j / kTcBufs) & 1);
      tc_fence_after();
      draw = tmem_ld1(trow + (uint32_t)(dcol0 + 16 * buf));
    };
    auto readback = [&](int j) {
      const int buf = j % kTcBufs;
      tmem_wait_ld1(draw);
      const float d = __uint_as_float(draw);
      tc_fence_before();
      mbar_arrive(&dfree[buf]);
      if (qB[0] != cur) {
        if (cur >= 0) flush(cur, yacc);
        cur = qB[0];
        yacc = 0.f;
      }
      yacc += d;   // the group's products of bf16 effective weights, summed in fp32
#pragma unroll
      for (int k = 0; k + 1 < lag; ++k) qB[k] = qB[k + 1];
    };

    for (int i = 0; i < nt; ++i) {
      const int st = i / tps, s = st % S, buf = i % kTcBufs;
      if (i >= lag) readback_issue(i - lag);
      wait_or_bail(&full[s], (st / S) & 1);
      const uint8_t* tile = ring + (size_t)s * stage_bytes + (size_t)(i % tps) * p.tile_bytes;
      const uint2* wp = reinterpret_cast<const uint2*>(tile) + row;
      const uint32_t at = trow + (uint32_t)(buf * acols);
      // this row's (scale, scale) and (zero, zero) bf16 pairs of the group
      const uint32_t pw = reinterpret_cast<const uint32_t*>(tile + kTcRows * g / 2)[row];
      const uint32_t sc2 = __byte_perm(pw, 0u, 0x1010), zr2 = __byte_perm(pw, 0u, 0x3232);
      // A buffer `buf` is free: the MMAs of tile i - kTcBufs completed
      // (observed by its read-back in iteration i - 1).  A = the bf16
      // effective weights bf16((q - 8) scale + zero) (gptq.py:87-97, rounded
      // once as torch's int4 GEMM rounds its operand)
#pragma unroll 4
      for (int ks = 0; ks < KS; ++ks) {
        const uint2 w = wp[ks * kTcRows];
        uint32_t r[8];
        r[0] = w4_ref_pair(lop3_and_or(w.x, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[1] = w4_ref_pair(lop3_and_or(w.x >> 4, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[2] = w4_ref_pair(lop3_and_or(w.x >> 8, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[3] = w4_ref_pair(lop3_and_or(w.x >> 12, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[4] = w4_ref_pair(lop3_and_or(w.y, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[5] = w4_ref_pair(lop3_and_or(w.y >> 4, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[6] = w4_ref_pair(lop3_and_or(w.y >> 8, 0x000F000Fu, 0x43004300u), sc2, zr2);
        r[7] = w4_ref_pair(lop3_and_or(w.y >> 12, 0x000F000Fu, 0x43004300u), sc2, zr2);
        tmem_st8(at + 8 * ks, r);
      }
      mbar_arrive(&empty[s]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull[buf]);
      const int slot = i < lag ? i : lag - 1;  // queue position of tile i after this iteration
      if (i >= lag) readback(i - lag);
#pragma unroll
      for (int k = 0; k < lag; ++k)
        if (k == slot) qB[k] = nb;
      if (++G == KT) {
        G = 0;
        ++nb;
      }
    }
    for (int j = max(0, nt - lag); j < nt; ++j) {
      readback_issue(j);
      readback(j);
    }
    if (cur >= 0) flush(cur, yacc);  // a bail is reported by the device status word
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTcTmemCols);
  }
}

// ------------------------------------------------------------------ packing
// Codes q [N][K] (0..15) + qsz bf16 [K/g][N][2] (scale, zero) -> TC tiles.
__global__ void tc_pack_words_kernel(const uint8_t* q, int K, int N, int g, int tile_bytes, uint8_t* tiles) {
  const int KT = K / g, KS = g / 16;
  const long long per_tile = (long long)KS * kTcRows * 2;
  const long long total = (long long)(N / kTcRows) * KT * per_tile;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long t = idx / per_tile;
    const int wi = (int)(idx % per_tile);
    const int half = wi & 1, row = (wi >> 1) & (kTcRows - 1), ks = wi >> 8;
    const int nb = (int)(t / KT), G = (int)(t % KT);
    const int n = nb * kTcRows + row;
    const uint8_t* src = q + (size_t)n * K + (size_t)G * g + 16 * ks + 8 * half;
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      w |= (uint32_t)(src[2 * i] & 0xF) << (4 * i);
      w |= (uint32_t)(src[2 * i + 1] & 0xF) << (4 * i + 16);
    }
    reinterpret_cast<uint32_t*>(tiles + t * tile_bytes)[wi] = w;
  }
}

__global__ void tc_pack_params_kernel(const uint16_t* qsz, int K, int N, int g, int tile_bytes, uint8_t* tiles) {
  const int KT = K / g;
  const long long total = (long long)N * KT;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(idx % N), G = (int)(idx / N);
    const long long t = (long long)(n / kTcRows) * KT + G;
    const uint32_t sc = qsz[((size_t)G * N + n) * 2 + 0];
    const uint32_t zr = qsz[((size_t)G * N + n) * 2 + 1];
    reinterpret_cast<uint32_t*>(tiles + t * tile_bytes + kTcRows * g / 2)[n % kTcRows] = sc | (zr << 16);
  }
}

__global__ void tc_unpack_codes_kernel(const uint8_t* tiles, int K, int N, int g, int tile_bytes, uint8_t* codes) {
  const int KT = K / g;
  const long long total = (long long)N * K;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(idx / K), k = (int)(idx % K);
    const int nb = n / kTcRows, row = n % kTcRows, G = k / g, kin = k % g;
    const int ks = kin / 16, k16 = kin % 16, half = k16 >> 3, kk = k16 & 7;
    const long long t = (long long)nb * KT + G;
    const uint32_t w = reinterpret_cast<const uint32_t*>(tiles + t * tile_bytes)[(ks * kTcRows + row) * 2 + half];
    const int nib = (kk >> 1) + 4 * (kk & 1);
    codes[idx] = (uint8_t)((w >> (4 * nib)) & 0xFu);
  }
}

inline int tc_grid_for(long long work) {
  long long b = (work + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(b, 148LL * 32));
}

}  // namespace

// Host planning for one shape on `num_sms` SMs (2 CTAs per SM).
int w4_tc_plan(int K, int N, int g, int num_sms, TcPlan* out) {
  if (K <= 0 || N <= 0 || (N % kTcRows) || (g != 32 && g != 64 && g != 128) || (K % g) || K > kTcMaxK) return -1;
  TcPlan p{};
  p.KT = K / g;
  p.nblocks = N / kTcRows;
  if ((long long)p.nblocks * p.KT * 2 * num_sms >= (1ll << 32)) return -1;  // tc_cta_of_tile's 32-bit range
  p.T = p.nblocks * p.KT;
  p.tile_bytes = tc_tile_bytes(g);
  p.tps = 1;
  while (p.tps < 4 && (p.tps * 2) * p.tile_bytes <= 18 * 1024) p.tps *= 2;
  int G = std::min(p.T, num_sms * 2);
  G = std::max(1, std::min(G, std::max(1, p.T / 2)));
  p.G = G;
  const int ntmax = (p.T + G - 1) / G;
  const int nst = (ntmax + p.tps - 1) / p.tps;
  p.stages = std::max(1, std::min(8, nst));
  for (;;) {
    const TcSmem L = tc_smem(p, K, g);
    p.smem = L.total;
    if (L.total <= 112 * 1024 || p.stages <= 2) break;
    --p.stages;
  }
  if (p.smem > 112 * 1024) return -2;
  int maxc = 1;
  for (int b = 0; b < p.nblocks; ++b) {
    const int lo = tc_cta_of_tile((long long)b * p.KT, p.G, p.T);
    const int hi = tc_cta_of_tile((long long)(b + 1) * p.KT - 1, p.G, p.T);
    maxc = std::max(maxc, hi - lo + 1);
  }
  p.maxc = maxc;
  p.partial_bytes = tc_align((size_t)p.nblocks * p.maxc * kTcRows * 4, 256);
  *out = p;
  return 0;
}

cudaError_t w4_tc_launch(const TcArgs& a, cudaStream_t stream, int use_pdl) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(w4_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.p.G);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = a.p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, w4_tc_kernel, a);
}

cudaError_t w4_tc_pack(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles, cudaStream_t s) {
  const int tb = tc_tile_bytes(g);
  const long long words = (long long)(N / kTcRows) * (K / g) * (g / 16) * kTcRows * 2;
  tc_pack_words_kernel<<<tc_grid_for(words), 256, 0, s>>>(q, K, N, g, tb, tiles);
  tc_pack_params_kernel<<<tc_grid_for((long long)N * (K / g)), 256, 0, s>>>(qsz, K, N, g, tb, tiles);
  return cudaGetLastError();
}

cudaError_t w4_tc_unpack_codes(const uint8_t* tiles, int K, int N, int g, uint8_t* codes, cudaStream_t s) {
  tc_unpack_codes_kernel<<<tc_grid_for((long long)N * K), 256, 0, s>>>(tiles, K, N, g, tc_tile_bytes(g), codes);
  return cudaGetLastError();
}

}  // namespace mtl
