// W4A16 GEMM for prompt prefill on the 5th-generation tensor cores.
//
// Replaces torch._weight_int4pack_mm at M = prompt rows, as the reference
// prefills a prompt (moss_tts_lite/fast.py:218-270, _layer_q: every
// projection of a layer is one int4 GEMM over all L rows): y[L, N] =
// x[L, K] . W^T with W = bf16((q - 8) * scale + zero) per group
// (gptq.py:87-97; rounded once to bf16 as that kernel forms its operand),
// fp32 accumulation, bf16 output, optional residual-add or SwiGLU epilogue
// (fast.py:168-171).  It reads the same packed weights as the decode GEMV
// (the register-MMA "MTL tile layout" of w4_gemv.cuh, reference format), so
// a model keeps one copy of its W4 weights.
//
// One output tile = 128 weight rows (two 64-column tile blocks) x NT prompt
// rows (64, 128 or 256); the CTAs (one per SM) walk the tiles round-robin.
// Per 64-wide k-stage:
//   * warp 8 (producer) loads the stage's activations with 8 TMA tensor
//     copies (8 k x NT rows each, no swizzle, no multicast) into the
//     canonical K-major layout (core matrix = 8 rows x 16 bytes; k-chunk
//     stride NT * 16 bytes, 8-row stride 128 bytes), and the stage's packed
//     codes + (scale, zero) of the two tile blocks with 1-D bulk copies;
//   * warps 0-3 dequantise the codes into A, 128 rows x 64 k of bf16
//     effective weights in the same canonical layout (k-chunk stride 2048
//     bytes): each lane turns one 32-bit word (8 codes of its MMA-lane
//     layout) into four bf16 pairs, 128 + q by one shift + LOP3, then q - 8
//     (exact) and (q - 8) scale + zero (one rounding) by two bf16x2 FMAs,
//     stored as 4-byte pairs (32 lanes cover 128 contiguous bytes);
//   * warp 9 (one thread) issues 4 tcgen05.mma kind::f16 (M = 128, N = NT,
//     K = 16, A and B from shared memory) into a TMEM accumulator and
//     commits the stage back to the producer and the dequantisers;
//   * warps 4-7 (epilogue) read the finished accumulator (tcgen05.ld, one
//     TMEM lane = one weight row per thread, 32 prompt rows at a time) and
//     write bf16 outputs.  Two accumulators (2 x NT TMEM columns) let the
//     epilogue of tile t overlap the main loop of tile t + 1.
// No split-K, so no scratch.  Every wait is bounded (device status word).
#include "common.cuh"

namespace mtl {

constexpr int kGemmRows = 128;     // weight rows per tile (UMMA M)
constexpr int kGemmK = 64;         // k per stage
constexpr int kGemmStages = 4;     // A / B stages
constexpr int kGemmWSlots = 4;     // packed-weight slots
constexpr int kGemmThreads = 320;  // warps 0-3 dequantise, 4-7 epilogue, 8 producer, 9 MMA
constexpr int kGemmWSlotBytes = 2 * (4 * 512 + 256);  // two tile blocks: 4 k16-steps of words + params

struct GemmArgs {
  int L, K, N, g, NT;
  const uint8_t* tiles;      // MTL tile layout, reference format
  int tile_bytes;
  int epi;                   // kEpiStore / kEpiResidual / kEpiSwiGLU
  const uint16_t* residual;  // bf16 [L, ldr] (may alias y)
  int ldr;
  uint16_t* y;  // bf16 [L, ldy]
  int ldy;
  int ntiles, nblk128;  // tiles = nblk128 (weight blocks of 128) x token blocks
};

namespace {

struct GemmSmem {
  size_t bar, misc, a, b, w, total;
};
__host__ __device__ inline GemmSmem gemm_smem(int NT) {
  GemmSmem L;
  size_t o = 0;
  L.bar = o;
  o += 256;  // mbarriers
  L.misc = o;
  o = 1024;  // operand buffers 1024-byte aligned (TMA destinations)
  L.a = o;
  o += (size_t)kGemmStages * kGemmRows * kGemmK * 2;
  L.b = o;
  o += (size_t)kGemmStages * NT * kGemmK * 2;
  L.w = o;
  o += (size_t)kGemmWSlots * kGemmWSlotBytes;
  L.total = (o + 127) / 128 * 128;
  return L;
}

__device__ __forceinline__ void gtma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// K-major, no swizzle: leading (k-chunk) byte offset `lbo`, stride (8-row) offset 128.
__device__ __forceinline__ uint64_t gemm_desc(uint32_t addr, uint32_t lbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void gemm_mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void gemm_tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void gemm_tmem_wait_ld32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    w4_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t gemm_sm[];
  uint8_t* smem = gemm_sm;
  const int NT = a.NT, K = a.K, g = a.g;
  const GemmSmem L = gemm_smem(NT);
  uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + L.bar);  // [S] activations landed
  uint64_t* afull = bfull + kGemmStages;                         // [S] A written (128 arrivals)
  uint64_t* sempty = afull + kGemmStages;                        // [S] stage read by the MMAs
  uint64_t* wfull = sempty + kGemmStages;                        // [WS] packed weights landed
  uint64_t* wempty = wfull + kGemmWSlots;                        // [WS] packed weights read (4 warps)
  uint64_t* accfull = wempty + kGemmWSlots;                      // [2] accumulator complete
  uint64_t* accempty = accfull + 2;                              // [2] accumulator read (128 arrivals)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L.misc);
  volatile int* vbail = reinterpret_cast<volatile int*>(smem + L.misc + 16);
  uint8_t* abuf = smem + L.a;
  uint8_t* bbuf = smem + L.b;
  uint8_t* wbuf = smem + L.w;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nks = K / kGemmK;  // k-stages per tile
  const uint32_t abytes = kGemmRows * kGemmK * 2, bbytes = (uint32_t)NT * kGemmK * 2;
  const uint32_t tmem_cols = NT <= 64 ? 128 : (NT <= 128 ? 256 : 512);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&afull[s], 128);
      mbar_init(&sempty[s], 1);
    }
    for (int s = 0; s < kGemmWSlots; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 128);
    }
    fence_mbar_init();
    *vbail = 0;
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tbase = *tslot;
  pdl_launch_dependents();
  pdl_wait();  // activations (and the residual) come from the upstream kernel

  bool bail = false;
  auto wait_or_bail = [&](uint64_t* bar, uint32_t parity) {
    if (!bail && *vbail) bail = true;
    if (!bail && !mbar_wait(bar, parity)) {
      bail = true;
      *vbail = 1;
    }
  };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0, last_b = -1, last_w = -1;
      for (int tile = blockIdx.x; tile < a.ntiles && !bail; tile += gridDim.x) {
        const int wb = tile % a.nblk128, tb = tile / a.nblk128;
        for (int kst = 0; kst < nks; ++kst, ++it) {
          const int s = it % kGemmStages, ws = it % kGemmWSlots;
          if (it >= kGemmStages) wait_or_bail(&sempty[s], ((it / kGemmStages) - 1) & 1);
          if (it >= kGemmWSlots) wait_or_bail(&wempty[ws], ((it / kGemmWSlots) - 1) & 1);
          if (bail) break;
          // activations: 8 boxes of 8 k x NT rows (rows past L read as zeros)
          mbar_arrive_expect_tx(&bfull[s], bbytes);
          uint8_t* bs = bbuf + (size_t)s * bbytes;
#pragma unroll
          for (int c = 0; c < 8; ++c) gtma_load_2d(bs + (size_t)c * NT * 16, &tm_x, kst * kGemmK + 8 * c, tb * NT, &bfull[s]);
          last_b = it;
          // packed codes (4 k16-steps) + (scale, zero) of the two tile blocks
          const int k0 = kst * kGemmK, G = k0 / g, ks0 = (k0 % g) / 16;
          uint8_t* wd = wbuf + (size_t)ws * kGemmWSlotBytes;
          mbar_arrive_expect_tx(&wfull[ws], kGemmWSlotBytes);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint8_t* tsrc = a.tiles + ((size_t)(2 * wb + h) * (K / g) + G) * a.tile_bytes;
            bulk_g2s(wd + h * (4 * 512 + 256), tsrc + (size_t)ks0 * 512, 4 * 512, &wfull[ws]);
            bulk_g2s(wd + h * (4 * 512 + 256) + 4 * 512, tsrc + 64 * g / 2, 256, &wfull[ws]);
          }
          last_w = it;
        }
      }
      // copies in flight land before the CTA exits
      const uint64_t dl = globaltimer_ns() + kWaitNs;
      if (last_b >= 0 && !mbar_wait_until(&bfull[last_b % kGemmStages], (last_b / kGemmStages) & 1, dl))
        flag_error(kDevCopyDrainTimeout);
      if (last_w >= 0 && !mbar_wait_until(&wfull[last_w % kGemmWSlots], (last_w / kGemmWSlots) & 1, dl))
        flag_error(kDevCopyDrainTimeout);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | ((128u >> 4) << 24);
      int it = 0, tl = 0, last_commit = -1;
      for (int tile = blockIdx.x; tile < a.ntiles && !bail; tile += gridDim.x, ++tl) {
        const int ab = tl & 1;
        if (tl >= 2) wait_or_bail(&accempty[ab], ((tl >> 1) - 1) & 1);
        const uint32_t d = tbase + (uint32_t)(ab * NT);
        for (int kst = 0; kst < nks && !bail; ++kst, ++it) {
          const int s = it % kGemmStages;
          wait_or_bail(&bfull[s], (it / kGemmStages) & 1);
          wait_or_bail(&afull[s], (it / kGemmStages) & 1);
          if (bail) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a0 = smem_addr(abuf + (size_t)s * abytes), b0 = smem_addr(bbuf + (size_t)s * bbytes);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            gemm_mma(d, gemm_desc(a0 + i * 2 * 2048, 2048), gemm_desc(b0 + i * 2 * NT * 16, NT * 16), idesc,
                     (kst > 0 || i > 0) ? 1u : 0u);
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_addr(&sempty[s]))
                       : "memory");
          last_commit = it;
        }
        if (!bail)
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_addr(&accfull[ab]))
                       : "memory");
      }
      // every MMA issued has completed before TMEM is released
      if (last_commit >= 0) {
        const uint64_t dl = globaltimer_ns() + kWaitNs;
        if (!mbar_wait_until(&sempty[last_commit % kGemmStages], (last_commit / kGemmStages) & 1, dl))
          flag_error(kDevWaitTimeout);
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ dequantise
    const int h = warp >> 1;              // tile block (64 weight rows) of this warp
    const int gr = lane >> 2, tq = lane & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < a.ntiles && !bail; tile += gridDim.x) {
      for (int kst = 0; kst < nks; ++kst, ++it) {
        const int s = it % kGemmStages, ws = it % kGemmWSlots;
        wait_or_bail(&wfull[ws], (it / kGemmWSlots) & 1);
        if (it >= kGemmStages) wait_or_bail(&sempty[s], ((it / kGemmStages) - 1) & 1);
        if (bail) break;
        const uint8_t* wd = wbuf + (size_t)ws * kGemmWSlotBytes + h * (4 * 512 + 256);
        const uint32_t* prm = reinterpret_cast<const uint32_t*>(wd + 4 * 512);
        uint32_t sc2[4][2], zr2[4][2];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const uint32_t pw = prm[16 * j + gr + 8 * hr];
            sc2[j][hr] = __byte_perm(pw, 0u, 0x1010);
            zr2[j][hr] = __byte_perm(pw, 0u, 0x3232);
          }
        uint8_t* as = abuf + (size_t)s * abytes;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
          const int ksl = 2 * (warp & 1) + kk;  // k16-step of the stage (0..3)
          const uint4 wv = reinterpret_cast<const uint4*>(wd)[ksl * 32 + lane];
          const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t w = wr[j];
            // weight rows 64 h + 16 j + gr and + 8, k = 16 ksl + 2 tq (+8).
            // SwiGLU tiles place subtile j at A rows 64 h + 32 (j & 1) +
            // 16 (j >> 1): each 32-row TMEM lane quarter then holds 16 gate
            // rows and the 16 up rows of the same outputs
            const int rg = 8 * h + (a.epi == kEpiSwiGLU ? 4 * (j & 1) + 2 * (j >> 1) : 2 * j);
            uint8_t* base = as + (size_t)(2 * ksl) * 2048 + rg * 128 + gr * 16 + tq * 4;
            *reinterpret_cast<uint32_t*>(base) =
                w4_ref_pair(lop3_and_or(w, 0x000F000Fu, 0x43004300u), sc2[j][0], zr2[j][0]);
            *reinterpret_cast<uint32_t*>(base + 128) =
                w4_ref_pair(lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u), sc2[j][1], zr2[j][1]);
            *reinterpret_cast<uint32_t*>(base + 2048) =
                w4_ref_pair(lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u), sc2[j][0], zr2[j][0]);
            *reinterpret_cast<uint32_t*>(base + 2048 + 128) =
                w4_ref_pair(lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u), sc2[j][1], zr2[j][1]);
          }
        }
        // A is read by the tensor cores (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(&afull[s]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[ws]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q4 = warp & 3;           // TMEM lane quarter
    const int row = 32 * q4 + lane;    // A row of the tile
    const uint32_t tlane = tbase + ((uint32_t)(32 * q4) << 16);
    int tl = 0;
    for (int tile = blockIdx.x; tile < a.ntiles && !bail; tile += gridDim.x, ++tl) {
      const int wb = tile % a.nblk128, tb = tile / a.nblk128;
      const int ab = tl & 1;
      wait_or_bail(&accfull[ab], (tl >> 1) & 1);
      if (bail) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int n = wb * kGemmRows + row;
      // SwiGLU: lanes 0-15 hold gate rows, 16-31 the up rows of the same
      // outputs: 32 (2 wb + q4 / 2) + 16 (q4 & 1) + lane % 16
      const int o = 32 * (2 * wb + (q4 >> 1)) + 16 * (q4 & 1) + (lane & 15);
      for (int c0 = 0; c0 < NT; c0 += 32) {
        uint32_t r[32];
        gemm_tmem_ld32(tlane + (uint32_t)(ab * NT + c0), r);
        gemm_tmem_wait_ld32(r);
        const int t0 = tb * NT + c0;
        if (a.epi == kEpiSwiGLU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float up = __shfl_xor_sync(0xffffffffu, __uint_as_float(r[i]), 16);
            if (lane < 16 && t0 + i < a.L) {
              // fast.py:170-171: bf16(silu(gate)) * up, each op rounded to bf16
              const float gt = round_bf16(__uint_as_float(r[i]));
              const float sg = round_bf16(gt / (1.0f + expf(-gt)));
              a.y[(size_t)(t0 + i) * a.ldy + o] = f32_to_bf16_bits(sg * round_bf16(up));
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (t0 + i < a.L) {
              float v = __uint_as_float(r[i]);
              if (a.epi == kEpiResidual) {
                // fast.py:168 / :170: residual + bf16(linear(...)), rounded to bf16
                v = bf16_bits_to_f32(a.residual[(size_t)(t0 + i) * a.ldr + n]) + round_bf16(v);
              }
              a.y[(size_t)(t0 + i) * a.ldy + n] = f32_to_bf16_bits(v);
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&accempty[ab]);
    }
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 9) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(tmem_cols) : "memory");
  }
}

}  // namespace

// Prompt-row tile for L rows: 64, 128 or 256.
inline int gemm_nt(int L) { return L <= 64 ? 64 : (L <= 128 ? 128 : 256); }

size_t w4_gemm_smem(int L) { return gemm_smem(gemm_nt(L)).total; }

cudaError_t w4_gemm_launch(const uint16_t* x, int ldx, int L, int K, int N, int g, const uint8_t* tiles, int epi,
                           const uint16_t* residual, int ldr, uint16_t* y, int ldy, int num_sms, cudaStream_t s,
                           int use_pdl) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(w4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  GemmArgs a{};
  a.L = L;
  a.K = K;
  a.N = N;
  a.g = g;
  a.NT = gemm_nt(L);
  a.tiles = tiles;
  a.tile_bytes = tile_bytes(g, kFmtRef);
  a.epi = epi;
  a.residual = residual;
  a.ldr = ldr;
  a.y = y;
  a.ldy = ldy;
  a.nblk128 = N / kGemmRows;
  a.ntiles = a.nblk128 * ((L + a.NT - 1) / a.NT);
  // activations as a 2-D tensor (k, row); boxes of 8 k x NT rows
  EncodeTiledFn enc = encode_tiled_fn();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)L};
  cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  cuuint32_t box[2] = {8, (cuuint32_t)a.NT};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const int grid = a.ntiles < num_sms ? a.ntiles : num_sms;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(grid), dim3(kGemmThreads), gemm_smem(a.NT).total, s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, w4_gemm_kernel, tm, a);
}

}  // namespace mtl
