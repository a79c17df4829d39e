// W4A16 linear for 2..16 activation rows on the 5th-generation tensor cores:
// the TC tile format (w4_tc.cu) with the rows of a batch as the N = 16
// dimension of tcgen05.mma, so one pass over the weights serves every row
// (the batched multi-stream decode step and short prompts).
//
// Per tile (128 output rows x one group of k), as in w4_tc.cu: the four
// dequantising warps write A = the bf16 effective weights bf16((q - 8) scale
// + zero) into TMEM, one thread issues g/16 MMAs M = 128, N = 16, K = 16, and
// the accumulator comes back two tiles later (tcgen05.ld, 16 columns = 16
// batch rows) and is added to the rows' fp32 sums.  What changes is B:
// instead of one activation vector staged once, each tile's [16 rows x g]
// slice of the activations is staged by the dequantising warps into a B
// buffer in the canonical K-major layout (core matrices of 8 rows x 16
// bytes; k-chunk stride 256 bytes, 8-row stride 128 bytes), RMSNorm applied
// when fused, one tile ahead of its MMAs (its global loads are issued a tile
// earlier).  Thread (warp w, lane l) stages chunks c = 2 (l % 8) and c + 1 of
// row m = 4 w + l / 8.
//
// Batch rows beyond M are zero in B and never read.  The split-K partials
// are [block][contributor][row m][128] floats; the last CTA to arrive at a
// column block sums them in contributor order (deterministic).

namespace mtl {

constexpr int kTcbMaxM = 16;

struct TcbArgs {
  const uint16_t* x;  // bf16 [M, ldx]
  int ldx, M, K, N, g;
  const uint8_t* tiles;
  const uint16_t* norm_w;  // nullable: fused RMSNorm prologue (bf16 [K])
  float norm_eps;
  int epi;
  const uint16_t* residual;  // bf16 [M, N] (kEpiResidual; may alias y)
  uint16_t* y;
  int ldy;
  float* partials;  // [nblocks][maxc][kTcbMaxM][128]
  int* counters;    // [nblocks]
  TcPlan p;         // w4_tc_plan of the shape; smem replaced by tcb_smem
};

namespace {

struct TcbSmem {
  size_t bar, misc, ring, bbuf, total;
};
__host__ __device__ inline TcbSmem tcb_smem(const TcPlan& p, int g) {
  TcbSmem L;
  size_t o = 0;
  L.bar = o;
  o += tc_align((size_t)(2 * p.stages + 3 * kTcBufs) * 8, 128);
  L.misc = o;
  o += 2048;  // [0,16) ints; floats: rinv [16] at 128, group sums [3][16] at 160, chunk sums [16][16] at 256
  L.ring = o;
  o += (size_t)p.stages * p.tps * p.tile_bytes;
  o = tc_align(o, 128);
  L.bbuf = o;
  o += (size_t)kTcBufs * kTcbMaxM * g * 2;
  L.total = tc_align(o, 128);
  return L;
}

// B descriptor: K-major, no swizzle, k-chunk (leading) stride 256 B, 8-row
// (stride) offset 128 B.
__device__ __forceinline__ uint64_t bb_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(256 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
         (1ull << 46);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// tcgen05.wait::ld with the loaded registers as operands, so that no use of
// them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 2) w4_tcb_kernel(const __grid_constant__ TcbArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const TcPlan& p = a.p;
  const int K = a.K, g = a.g, KT = p.KT, KS = g >> 4, M = a.M;
  const int cta = blockIdx.x;
  // stream-K range of this CTA (32-bit: T G < 2^32, checked by the plan)
  const int t0 = (int)(((uint32_t)p.T * (uint32_t)cta) / (uint32_t)p.G);
  const int t1 = (int)(((uint32_t)p.T * (uint32_t)(cta + 1)) / (uint32_t)p.G);
  const int nt = t1 - t0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages, tps = p.tps;
  const size_t stage_bytes = (size_t)tps * p.tile_bytes;
  const TcbSmem L = tcb_smem(p, g);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;        // [kTcBufs] A and B of the buffer written
  uint64_t* dfull = afull + kTcBufs;  // [kTcBufs] MMAs of the buffer done
  uint64_t* dfree = dfull + kTcBufs;  // [kTcBufs] accumulator read back
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L.misc);
  int* imisc = reinterpret_cast<int*>(smem + L.misc);        // [1] bail, [2] last-arriver flag
  float* rinv_s = reinterpret_cast<float*>(smem + L.misc) + 128;  // [16]
  uint8_t* ring = smem + L.ring;
  uint8_t* bbuf = smem + L.bbuf;
  const size_t bbytes = (size_t)kTcbMaxM * g * 2;  // one B buffer
  const int acols = KS * 8;
  const int dcol0 = kTcBufs * acols;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTcRows * tps);
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
    if (lane == 0) {
      const uint32_t b0 = smem_addr(bbuf);
      int done = 0;
      for (int i = 0; i < nt; ++i) {
        const int buf = i % kTcBufs;
        if (!mbar_wait(&afull[buf], (i / kTcBufs) & 1)) break;
        if (i >= kTcBufs && !mbar_wait(&dfree[buf], ((i - kTcBufs) / kTcBufs) & 1)) break;
        tc_fence_after();
        const uint32_t d = tbase + (uint32_t)(dcol0 + 16 * buf);
        const uint32_t at = tbase + (uint32_t)(buf * acols);
        const uint32_t bb = b0 + (uint32_t)(buf * bbytes);
        for (int ks = 0; ks < KS; ++ks) tc_mma(d, at + 8 * ks, bb_desc(bb + 512 * ks), kTcIdesc, ks > 0 ? 1u : 0u);
        tc_commit(&dfull[buf]);
        done = i + 1;
      }
      if (done > 0) {
        const uint64_t dl = globaltimer_ns() + kWaitNs;
        const int i = done - 1;
        if (!mbar_wait_until(&dfull[i % kTcBufs], (i / kTcBufs) & 1, dl)) flag_error(kDevWaitTimeout);
      }
    }
  } else {
    // --------------------------- dequantise A, stage B, epilogue (output rows)
    const int lt = threadIdx.x - 64;         // 0..127
    const int row = 32 * (warp & 3) + lane;  // TMEM lane = output row of the tile
    const uint32_t trow = tbase + ((uint32_t)(32 * (warp & 3)) << 16);
    // B staging role: batch row bm, k-chunks bc and bc + 1 of the group
    const int bm = 4 * (warp - 2) + (lane >> 3);
    const int bc = 2 * (lane & 7);
    const int nch = g / 8;                   // 8-value chunks of a group (4..16)
    const bool bact = bm < M && bc < nch;    // this thread stages real values
    const uint16_t* xrow = a.x + (size_t)min(bm, M - 1) * a.ldx;
    pdl_wait();
    // (a) RMSNorm statistics per batch row: the 8 lanes that stage row bm
    //     sum its squares, four independent loads in flight per lane
    if (a.norm_w) {
      float ss[4] = {0.f, 0.f, 0.f, 0.f};
      if (bm < M) {
        const uint4* xr = reinterpret_cast<const uint4*>(a.x + (size_t)bm * a.ldx);
        const int nc = K / 8, j = lane & 7;
        for (int c = j; c < nc; c += 32) {
          uint4 v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = c + 8 * e < nc ? __ldg(xr + c + 8 * e) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t u[4] = {v[e].x, v[e].y, v[e].z, v[e].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float lo = __uint_as_float(u[q] << 16), hi = __uint_as_float(u[q] & 0xFFFF0000u);
              ss[e] = fmaf(lo, lo, ss[e]);
              ss[e] = fmaf(hi, hi, ss[e]);
            }
          }
        }
      }
      float t = (ss[0] + ss[1]) + (ss[2] + ss[3]);
      t += __shfl_xor_sync(0xFFFFFFFFu, t, 1);
      t += __shfl_xor_sync(0xFFFFFFFFu, t, 2);
      t += __shfl_xor_sync(0xFFFFFFFFu, t, 4);
      if ((lane & 7) == 0 && bm < M) rinv_s[bm] = rsqrtf(t / (float)K + a.norm_eps);
      named_sync(1, 128);
    }
    const float rinv = a.norm_w && bm < M ? rinv_s[bm] : 0.f;
    // the two 16-byte chunks of x (and of the norm weight) for group G
    auto load_b = [&](int G, uint4 (&xv)[2], uint4 (&nv)[2]) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        xv[h] = make_uint4(0u, 0u, 0u, 0u);
        nv[h] = make_uint4(0u, 0u, 0u, 0u);
        if (bact) {
          const int k0 = G * g + 8 * (bc + h);
          xv[h] = __ldg(reinterpret_cast<const uint4*>(xrow + k0));
          if (a.norm_w) nv[h] = __ldg(reinterpret_cast<const uint4*>(a.norm_w + k0));
        }
      }
    };
    // normed bf16 chunks into B buffer `buf`
    auto stage_b = [&](int buf, const uint4 (&xv)[2], const uint4 (&nv)[2]) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t u[4] = {xv[h].x, xv[h].y, xv[h].z, xv[h].w};
        if (a.norm_w) {
          const uint32_t nw[4] = {nv[h].x, nv[h].y, nv[h].z, nv[h].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // model.py:34-40: bf16(h * rsqrt(var + eps)), then bf16(weight * that);
            // each pair rounded by one packed conversion (low half = even k)
            const uint32_t r = bf16x2_rn(__uint_as_float(u[q] << 16) * rinv, __uint_as_float(u[q] & 0xFFFF0000u) * rinv);
            u[q] = bf16x2_rn(__uint_as_float(nw[q] << 16) * __uint_as_float(r << 16),
                             __uint_as_float(nw[q] & 0xFFFF0000u) * __uint_as_float(r & 0xFFFF0000u));
          }
        }
        if (!bact) u[0] = u[1] = u[2] = u[3] = 0u;
        if (bc + h < nch)
          *reinterpret_cast<uint4*>(bbuf + buf * bbytes + ((size_t)(bc + h) * kTcbMaxM + bm) * 16) =
              make_uint4(u[0], u[1], u[2], u[3]);
      }
    };

    constexpr int lag = kTcBufs - 1;
    int G = t0 % KT, nb = t0 / KT;
    int cur = -1;
    float yacc[kTcbMaxM];
#pragma unroll
    for (int m = 0; m < kTcbMaxM; ++m) yacc[m] = 0.f;
    int qB[lag];
#pragma unroll
    for (int k = 0; k < lag; ++k) qB[k] = -1;
    bool bail = false;
    volatile int* vbail = imisc + 1;
    auto wait_or_bail = [&](uint64_t* bar, uint32_t parity) {
      if (!bail && *vbail) bail = true;
      if (!bail && !mbar_wait(bar, parity)) {
        bail = true;
        *vbail = 1;
      }
    };
    auto flush = [&](int blk) {
      const bool complete = (blk * KT >= t0) && ((blk + 1) * KT <= t1);
      const int n = blk * kTcRows + row;
      if (!complete) {
        const int c_lo = tc_cta_of_tile((long long)blk * KT, p.G, p.T);
        const int c_hi = tc_cta_of_tile((long long)(blk + 1) * KT - 1, p.G, p.T);
        float* dst = a.partials + (((size_t)blk * p.maxc + (cta - c_lo)) * kTcbMaxM) * kTcRows + row;
#pragma unroll
        for (int m = 0; m < kTcbMaxM; ++m)
          if (m < M) dst[(size_t)m * kTcRows] = yacc[m];
        named_sync(1, 128);
        if (lt == 0) {
          int old;
          asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.counters + blk) : "memory");
          const int last = (old == c_hi - c_lo);
          if (last) a.counters[blk] = 0;  // re-armed for the next launch
          imisc[2] = last;
        }
        named_sync(1, 128);
        const int last = imisc[2];
        named_sync(1, 128);
        if (!last) return;
#pragma unroll
        for (int m = 0; m < kTcbMaxM; ++m) yacc[m] = 0.f;
        // contributor order per row; the rows' loads of one contributor are
        // independent and issued together
        for (int j = 0; j <= c_hi - c_lo; ++j) {
          float v[kTcbMaxM];
#pragma unroll
          for (int m = 0; m < kTcbMaxM; ++m)
            v[m] = m < M ? __ldcg(a.partials + (((size_t)blk * p.maxc + j) * kTcbMaxM + m) * kTcRows + row) : 0.f;
#pragma unroll
          for (int m = 0; m < kTcbMaxM; ++m) yacc[m] += v[m];
        }
      }
#pragma unroll
      for (int m = 0; m < kTcbMaxM; ++m) {
        if (m >= M) continue;
        const float v = yacc[m];
        if (a.epi == kEpiSwiGLU) {
          // rows interleaved: 2j = gate j, 2j + 1 = up j (fast.py:170-171)
          const float other = __shfl_xor_sync(0xffffffffu, v, 1);
          if ((row & 1) == 0) {
            const float gt = round_bf16(v), up = round_bf16(other);
            const float sg = round_bf16(gt / (1.0f + expf(-gt)));
            a.y[(size_t)m * a.ldy + (n >> 1)] = f32_to_bf16_bits(sg * up);
          }
        } else if (a.epi == kEpiResidual) {
          // fast.py:168 / :170: residual + bf16(linear(...)), rounded to bf16
          const float r = bf16_bits_to_f32(a.residual[(size_t)m * a.N + n]);
          a.y[(size_t)m * a.ldy + n] = f32_to_bf16_bits(r + round_bf16(v));
        } else {
          a.y[(size_t)m * a.ldy + n] = f32_to_bf16_bits(v);
        }
      }
    };
    // accumulator of tile j (the oldest in flight) -> yacc: the TMEM load is
    // issued first (readback_issue, before the next tile's dequantisation)
    // and completed by readback
    uint32_t d[16];
    auto readback_issue = [&](int j) {
      const int buf = j % kTcBufs;
      wait_or_bail(&dfull[buf], (j / kTcBufs) & 1);
      tc_fence_after();
      tmem_ld16(trow + (uint32_t)(dcol0 + 16 * buf), d);
    };
    auto readback = [&](int j) {
      const int buf = j % kTcBufs;
      tmem_wait_ld16(d);
      tc_fence_before();
      mbar_arrive(&dfree[buf]);
      if (qB[0] != cur) {
        if (cur >= 0) flush(cur);
        cur = qB[0];
#pragma unroll
        for (int m = 0; m < kTcbMaxM; ++m) yacc[m] = 0.f;
      }
      // the group's products of bf16 effective weights, summed in fp32
#pragma unroll
      for (int m = 0; m < kTcbMaxM; ++m) yacc[m] += __uint_as_float(d[m]);
#pragma unroll
      for (int k = 0; k + 1 < lag; ++k) qB[k] = qB[k + 1];
    };

    uint4 xv[2], nv[2];
    if (nt > 0) load_b(G, xv, nv);
    for (int i = 0; i < nt; ++i) {
      const int st = i / tps, s = st % S, buf = i % kTcBufs;
      // every thread is done with iteration i - 1, whose read-back waited
      // for the MMAs of buffer `buf`: refill its B
      named_sync(1, 128);
      // B of tile i (its x was loaded an iteration ago), then the next x
      stage_b(buf, xv, nv);
      if (i + 1 < nt) load_b(G + 1 == KT ? 0 : G + 1, xv, nv);
      if (i >= lag) readback_issue(i - lag);
      wait_or_bail(&full[s], (st / S) & 1);
      const uint8_t* tile = ring + (size_t)s * stage_bytes + (size_t)(i % tps) * p.tile_bytes;
      const uint2* wp = reinterpret_cast<const uint2*>(tile) + row;
      const uint32_t at = trow + (uint32_t)(buf * acols);
      // A = the bf16 effective weights bf16((q - 8) scale + zero) of this row
      // (gptq.py:87-97, one rounding as torch's int4 GEMM forms its operand)
      const uint32_t pw = reinterpret_cast<const uint32_t*>(tile + kTcRows * g / 2)[row];
      const uint32_t sc2 = __byte_perm(pw, 0u, 0x1010), zr2 = __byte_perm(pw, 0u, 0x3232);
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
      fence_proxy_async_smem_tc();  // B is read by the tensor cores (async proxy)
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&afull[buf]);
      const int slot = i < lag ? i : lag - 1;
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
    if (cur >= 0) flush(cur);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTcTmemCols);
  }
}

}  // namespace

// Plan for M rows: the batch-1 plan of the shape with the ring shrunk until
// the B buffers fit; partial_bytes for 16 rows.
int w4_tcb_plan(int K, int N, int g, int num_sms, TcPlan* out) {
  TcPlan p;
  if (int r = w4_tc_plan(K, N, g, num_sms, &p)) return r;
  for (;;) {
    const TcbSmem L = tcb_smem(p, g);
    p.smem = L.total;
    if (L.total <= 112 * 1024 || p.stages <= 2) break;
    --p.stages;
  }
  if (p.smem > 112 * 1024) return -2;
  p.partial_bytes = tc_align((size_t)p.nblocks * p.maxc * kTcbMaxM * kTcRows * 4, 256);
  *out = p;
  return 0;
}

cudaError_t w4_tcb_launch(const TcbArgs& a, cudaStream_t stream, int use_pdl) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(w4_tcb_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
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
  return cudaLaunchKernelEx(&cfg, w4_tcb_kernel, a);
}

}  // namespace mtl
