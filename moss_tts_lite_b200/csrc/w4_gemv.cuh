// W4A16 linear for batch <= 8: tile layout, planning and launch interface.
//
// Device weight layout ("MTL tile layout"): the [N, K] int4 matrix is cut
// into tiles of 64 output columns x one quantisation group of K (g rows).
// Tiles are stored n-block-major (tile t = nb * (K/g) + G); each tile is one
// contiguous record:
//
//   words  : [g/16 k16-steps][32 lanes][4 subtiles] uint32  (64*g/2 bytes)
//   params : REF  -> [64] uint32 = bf16 scale | bf16 zero << 16   (256 B)
//            GPTQ -> [64] fp16 scale, then [8] uint32 packed zeros (160 B)
//
// Word (ks, lane, j) holds exactly the eight codes that lane (gr = lane/4,
// t = lane%4) feeds as the A fragment of one m16n8k16 bf16 MMA for subtile
// j: rows r0 = 16j + gr and r1 = r0 + 8 (output columns), k = 16ks + {2t,
// 2t+1, 2t+8, 2t+9}.  Slot s occupies bits 4s..4s+3:
//   s0 = W[r0][2t]    s4 = W[r0][2t+1]     -> A register a0
//   s1 = W[r1][2t]    s5 = W[r1][2t+1]     -> a1
//   s2 = W[r0][2t+8]  s6 = W[r0][2t+9]     -> a2
//   s3 = W[r1][2t+8]  s7 = W[r1][2t+9]     -> a3
// so a_i = ((w >> 4i) & 0x000F000F) | 0x43004300 is the bf16 pair
// (128 + q_lo, 128 + q_hi): three shifts and four LOP3s per eight codes.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace mtl {

constexpr int kNT = 64;       // output columns per tile
constexpr int kW4Warps = 8;   // consumer warps per CTA (+1 producer warp)
constexpr int kW4MaxM = 8;    // batch rows per launch (MMA N dimension)

enum ParamFmt : int { kFmtRef = 0, kFmtGptq = 1 };
enum Epilogue : int { kEpiStore = 0, kEpiResidual = 1, kEpiSwiGLU = 2 };

inline int param_bytes(int fmt) { return fmt == kFmtRef ? 256 : 160; }
inline int tile_bytes(int g, int fmt) { return kNT * g / 2 + param_bytes(fmt); }

struct W4Plan {
  int T;          // tiles
  int KT;         // groups along K (= tiles per column block)
  int nblocks;    // column blocks (N / 64)
  int G;          // CTAs
  int tps;        // tiles per ring stage (one bulk copy), divides kW4Warps
  int stages;     // ring depth, a multiple of kW4Warps / tps
  int ng_max;     // max groups a CTA stages
  int nblk_max;   // max column blocks a CTA touches
  int maxc;       // max CTAs contributing to one column block
  int tile_bytes;
  size_t smem;
  size_t partial_bytes;  // split-K partials (scratch, after the counters)
};

struct W4Args {
  const uint16_t* x;  // bf16 [M, ldx]
  int ldx;
  int M, K, N, g;
  const uint8_t* tiles;
  const int32_t* k_perm;    // nullable: x is gathered as x[k_perm[k]]
  const uint16_t* norm_w;   // nullable: fused RMSNorm prologue (bf16 [K])
  float norm_eps;
  int epi;
  const uint16_t* residual;  // bf16 [M, ldr] (kEpiResidual)
  int ldr;
  uint16_t* y;  // bf16 [M, ldy]
  int ldy;
  float* partials;
  int* counters;
  int zero_offset;
  int xvec;  // x rows and norm_w 16-byte aligned, K % 16 == 0, no k_perm
  W4Plan p;
};

// Host planning (grid, ring depth, shared memory, scratch) for one shape.
int w4_plan(int M, int K, int N, int g, int fmt, int num_sms, W4Plan* out);

// Effective bf16 weights [N, K] row-major from the tiles (REF or GPTQ).
cudaError_t w4_dequant(const uint8_t* tiles, int K, int N, int g, int fmt, int zero_offset, uint16_t* w,
                       cudaStream_t s);

// Launch on `stream` (programmatic dependent launch when use_pdl != 0).
cudaError_t w4_launch(const W4Args& a, int fmt, cudaStream_t stream, int use_pdl);

}  // namespace mtl
