// Persistent W4A16 GEMV chain (batch-1 decode): strip layout, phase
// descriptors, planning and launch interface.
//
// Strip layout (MTL_FMT_STRIP): the [N, K] int4 matrix is cut into tiles of
// 16 output rows (a "strip") x one quantisation group of K (g columns).
// Tile (u, k) - rows [16u, 16u + 16), group k - sits at (u * K/g + k) *
// (8 g + 64) bytes, so a strip's groups are contiguous:
//
//   words  : [g/64][32 lanes][4] uint32  (8 g bytes)
//   params : [8][2] uint32 = bf16 scale | bf16 zero << 16; word (r, h) is
//            row r + 8h, so a lane's two rows (gr, gr + 8) are adjacent
//
// Word (h, lane, l) holds the eight codes lane (gr = lane/4, t = lane%4)
// feeds as the A fragment of one m16n8k16 MMA, the l-th of word group h:
// rows r0 = gr, r1 = gr + 8 of the strip, and columns of the 32-column block
// q = 2h + l/2 at c = 32 q + 8 t + 4 (l % 2); slot s (bits 4s..4s+3) holds
//   s0 = W[r0][c]     s4 = W[r0][c+1]      -> A register a0
//   s1 = W[r1][c]     s5 = W[r1][c+1]      -> a1
//   s2 = W[r0][c+2]   s6 = W[r0][c+3]      -> a2
//   s3 = W[r1][c+2]   s7 = W[r1][c+3]      -> a3
// The MMA's k positions are permuted within each 32-column block - the
// same way for A and for B - so that lane t's B fragments of MMAs l = 0, 1
// are the 16 contiguous bytes x[32q + 8t .. 32q + 8t + 7]: x is used in its
// natural order (no staging permutation).  A gate|up pair for the SwiGLU epilogue is interleaved in
// blocks of 8 rows: rows 0-7 of strip u are gate rows 8u..8u+7, rows 8-15
// the up rows of the same outputs, so the MMA lane that holds a gate sum
// also holds its up sum.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace mtl {

constexpr int kChainMaxPhases = 4;
constexpr int kChainWarps = 16;  // consumer warps per CTA (+1 producer warp)
constexpr int kChainMaxK = kChainWarps * 32 * 32;  // x staged from registers: one 32-block per thread

__host__ __device__ inline int strip_tile_bytes(int g) { return 8 * g + 64; }

struct ChainPhase {
  const uint8_t* tiles;      // strip layout, K x N
  const uint16_t* x;         // bf16 [K] input row
  const uint16_t* norm_w;    // nullable: RMSNorm of x before the linear (bf16 [K])
  const uint16_t* residual;  // kEpiResidual: bf16 [N] (may alias y)
  uint16_t* y;               // bf16 [N] (or [N/2] with SwiGLU)
  int K, N, epi;
};

struct ChainArgs {
  ChainPhase ph[kChainMaxPhases];
  int nphases;
  float eps;
  unsigned* barrier;  // grid counter: 0 before the launch, reset to 0 by it
  int stages, kmax, umax;
};

struct ChainPlan {
  int G;       // CTAs (one per SM)
  int stages;  // ring stages of kChainWarps tiles
  int kmax;    // largest K of the phases (x staging)
  int umax;    // most strips one CTA owns in any phase
  int uaux;    // batched chain: most strips of a phase with a residual or several x slices
  size_t smem;
};

// Plan for phases with the given (K, N) and group size g (64/128/256).
// Returns 0, or -1 (shape not served) / -2 (does not fit).
int w4_chain_plan(const int* K, const int* N, int nphases, int g, int num_sms, ChainPlan* out);

cudaError_t w4_chain_launch(const ChainArgs& a, int g, const ChainPlan& p, cudaStream_t stream, int use_pdl);

// Batched chain (w4_chainb.cu): M = 2..16 activation rows per phase.
struct ChainBPhase {
  const uint8_t* tiles;      // strip layout, K x N
  const uint16_t* x;         // bf16 [M, ldx]
  const uint16_t* norm_w;    // nullable: RMSNorm of each row first (K <= 4096)
  const uint16_t* residual;  // kEpiResidual: bf16 [M, ldr] (may alias y)
  uint16_t* y;               // bf16 [M, ldy]
  int ldx, ldr, ldy;
  int K, N, epi;
};

struct ChainBArgs {
  ChainBPhase ph[kChainMaxPhases];
  int nphases, M;
  float eps;
  unsigned* barrier;  // grid counter: 0 before the launch, reset to 0 by it
  int stages, kslice, uaux;
};

int w4_chainb_plan(const int* K, const int* N, const int* norm, const int* epi, int nphases, int M, int g,
                   int num_sms, ChainPlan* out);
cudaError_t w4_chainb_launch(const ChainBArgs& a, int g, const ChainPlan& p, cudaStream_t stream, int use_pdl);

cudaError_t w4_pack_strip(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles,
                          cudaStream_t s);

}  // namespace mtl
