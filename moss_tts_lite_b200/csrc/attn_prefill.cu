// Causal GQA attention over a prompt for sm_100a: the attention step of the
// reference's prefill (moss_tts_lite/fast.py:218-270 _layer_q, model.py:
// 184-190): out = softmax(q k^T / sqrt(128) + causal mask) v per query head,
// where the reference expands K/V over the head groups (repeat_interleave)
// and runs PyTorch's SDPA.  Here each K/V tile is loaded once per head group.
//
// Inputs: q [rows][nh][128] bf16 (RMSNorm'd and rotated by mtl_attn_append
// with q_out), the layer's K/V cache [nkv][max_seq][128] per stream (rows
// [0, p0 + rows_per_stream) written), rows_per_stream prompt rows per stream
// at positions p0.. (row i of a stream attends to cache positions
// [0, p0 + i]).
//
// Grid (query blocks, nkv, streams), 8 warps.  A CTA serves QB query rows of
// all rep = nh / nkv heads of one KV head (warp w: head w % rep, rows
// 16 (w / rep) .. +16; QB = 128 / rep).  K/V tiles of 64 positions x 128
// dims stream through a two-stage shared-memory ring (cp.async, 16-byte
// chunks XOR-swizzled by row so that ldmatrix is conflict-free), and every
// warp computes on the tensor cores (mma.sync m16n8k16, bf16 in, fp32
// accumulate): S = Q K^T (Q fragments kept in registers), an online softmax
// per row with exp(s - m) rounded to bf16 before P V and the normaliser
// summing the unrounded values (the rounding point of flash-style SDPA, as
// the decode kernel), O += P V.  Query blocks are launched heaviest (latest
// positions) first.
#include "common.cuh"

namespace mtl {

constexpr int kPfWarps = 8;
constexpr int kPfThreads = kPfWarps * 32;
constexpr int kPfTile = 64;                      // positions per K/V tile
constexpr int kPfTileBytes = kPfTile * 128 * 2;  // one of K or V
constexpr int kPfSmem = 2 * 2 * kPfTileBytes;    // two stages of K and V

struct PrefillAttnArgs {
  const uint16_t* q;  // bf16 [streams * rows_per_stream][nh][128]
  const uint16_t* k_cache;
  const uint16_t* v_cache;
  long long cache_stream_stride;  // elements
  int max_seq, nh, nkv, rows_per_stream, p0;
  float scale;
  uint16_t* out;  // bf16 [streams * rows_per_stream][nh * 128]
};

namespace {

__device__ __forceinline__ void pf_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void pf_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pf_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void pf_ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void pf_ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void pf_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of (row, 16-byte chunk) in a 64 x 256-byte tile, chunk XOR row.
__device__ __forceinline__ uint32_t pf_off(int row, int chunk) {
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kPfThreads, 1) attn_prefill_kernel(const PrefillAttnArgs a) {
  extern __shared__ __align__(128) uint8_t pf_sm[];
  const int rep = a.nh / a.nkv;
  const int QB = 128 / rep;                       // query rows per CTA
  const int nqb = (a.rows_per_stream + QB - 1) / QB;
  const int qb = nqb - 1 - blockIdx.x;            // heaviest blocks first
  const int kvh = blockIdx.y, s = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = kvh * rep + warp % rep;
  const int r0 = qb * QB + 16 * (warp / rep);     // this warp's first query row (in the stream)
  const int g = lane >> 2, t = lane & 3;
  const uint16_t* kc = a.k_cache + (size_t)s * a.cache_stream_stride + (size_t)kvh * a.max_seq * 128;
  const uint16_t* vc = a.v_cache + (size_t)s * a.cache_stream_stride + (size_t)kvh * a.max_seq * 128;
  const size_t row_base = (size_t)s * a.rows_per_stream;
  const int last_row = min(qb * QB + QB, a.rows_per_stream) - 1;
  const int kv_end = a.p0 + last_row + 1;         // positions [0, kv_end) for this CTA
  const int ntiles = (kv_end + kPfTile - 1) / kPfTile;
  const uint32_t sbase = smem_addr(pf_sm);

  // stage st: K at st * 2 * kPfTileBytes, V after it
  auto load_tile = [&](int tile, int st) {
    const uint32_t kd = sbase + (uint32_t)(st * 2 * kPfTileBytes), vd = kd + kPfTileBytes;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = threadIdx.x + kPfThreads * i;  // 0..1023: row (64) x chunk (16)
      const int row = idx >> 4, ch = idx & 15;
      const int p = min(tile * kPfTile + row, kv_end - 1);  // rows past the end repeat the last (masked)
      pf_cp16(kd + pf_off(row, ch), kc + (size_t)p * 128 + ch * 8);
      pf_cp16(vd + pf_off(row, ch), vc + (size_t)p * 128 + ch * 8);
    }
    pf_commit();
  };
  load_tile(0, 0);

  // Q fragments (16 rows x 128 dims: 8 k16-steps x 4 registers), rows past
  // the stream's prompt read as zeros
  uint32_t qf[8][4];
  {
    const int ra = r0 + g, rb = r0 + g + 8;
    const uint16_t* qa = a.q + ((row_base + ra) * a.nh + head) * 128;
    const uint16_t* qbp = a.q + ((row_base + rb) * a.nh + head) * 128;
    const bool va = ra < a.rows_per_stream, vb = rb < a.rows_per_stream;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d = 16 * ks + 2 * t;
      qf[ks][0] = va ? *reinterpret_cast<const uint32_t*>(qa + d) : 0u;
      qf[ks][1] = vb ? *reinterpret_cast<const uint32_t*>(qbp + d) : 0u;
      qf[ks][2] = va ? *reinterpret_cast<const uint32_t*>(qa + d + 8) : 0u;
      qf[ks][3] = vb ? *reinterpret_cast<const uint32_t*>(qbp + d + 8) : 0u;
    }
  }
  const int pa = a.p0 + r0 + g, pb = pa + 8;  // positions of this lane's two rows
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
  // the last tile this warp needs (its own rows' causal limit)
  const int warp_end = min(a.p0 + r0 + 16, kv_end);
  const int wtiles = r0 < a.rows_per_stream ? (warp_end + kPfTile - 1) / kPfTile : 0;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int st = tile & 1;
    if (tile + 1 < ntiles) {
      load_tile(tile + 1, st ^ 1);
      pf_wait<1>();
    } else {
      pf_wait<0>();
    }
    __syncthreads();
    if (tile < wtiles) {
      const uint32_t kd = sbase + (uint32_t)(st * 2 * kPfTileBytes), vd = kd + kPfTileBytes;
      // S = Q K^T: 8 n8 tiles (positions) x 8 k16 steps (dims)
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int kp = 0; kp < 4; ++kp) {
          // 8 positions (rows 8 j + lane % 8) x 32 dims (chunks 4 kp + lane / 8)
          uint32_t b[4];
          pf_ldsm_x4(b, kd + pf_off(8 * j + (lane & 7), 4 * kp + (lane >> 3)));
          pf_mma(sc[j], qf[2 * kp][0], qf[2 * kp][1], qf[2 * kp][2], qf[2 * kp][3], b[0], b[1]);
          pf_mma(sc[j], qf[2 * kp + 1][0], qf[2 * kp + 1][1], qf[2 * kp + 1][2], qf[2 * kp + 1][3], b[2], b[3]);
        }
      }
      // scale, causal mask, online softmax
      float mxa = ma, mxb = mb;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = tile * kPfTile + 8 * j + 2 * t;
        sc[j][0] = c <= pa ? sc[j][0] * a.scale : -INFINITY;
        sc[j][1] = c + 1 <= pa ? sc[j][1] * a.scale : -INFINITY;
        sc[j][2] = c <= pb ? sc[j][2] * a.scale : -INFINITY;
        sc[j][3] = c + 1 <= pb ? sc[j][3] * a.scale : -INFINITY;
        mxa = fmaxf(mxa, fmaxf(sc[j][0], sc[j][1]));
        mxb = fmaxf(mxb, fmaxf(sc[j][2], sc[j][3]));
      }
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
      mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
      mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
      const float ala = mxa == -INFINITY ? 1.f : expf(ma - mxa);
      const float alb = mxb == -INFINITY ? 1.f : expf(mb - mxb);
      ma = mxa;
      mb = mxb;
      uint32_t pf[4][4];   // P as A fragments: k16 step kk = positions 16 kk .. +16
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p0 = mxa == -INFINITY ? 0.f : expf(sc[j][0] - mxa);
        const float p1 = mxa == -INFINITY ? 0.f : expf(sc[j][1] - mxa);
        const float p2 = mxb == -INFINITY ? 0.f : expf(sc[j][2] - mxb);
        const float p3 = mxb == -INFINITY ? 0.f : expf(sc[j][3] - mxb);
        sa += p0 + p1;
        sb += p2 + p3;
        const uint32_t lo = bf16x2_rn(p0, p1), hi = bf16x2_rn(p2, p3);
        pf[j >> 1][(j & 1) ? 2 : 0] = lo;
        pf[j >> 1][(j & 1) ? 3 : 1] = hi;
      }
      sa += __shfl_xor_sync(0xffffffffu, sa, 1);
      sa += __shfl_xor_sync(0xffffffffu, sa, 2);
      sb += __shfl_xor_sync(0xffffffffu, sb, 1);
      sb += __shfl_xor_sync(0xffffffffu, sb, 2);
      la = la * ala + sa;
      lb = lb * alb + sb;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= ala;
        o[j][1] *= ala;
        o[j][2] *= alb;
        o[j][3] *= alb;
      }
      // O += P V: 16 n8 tiles (dims) x 4 k16 steps (positions)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 8; ++jp) {
          // positions 16 kk + (lane % 16), dims 16 jp + 8 (lane / 16): two n8 tiles
          uint32_t b[4];
          pf_ldsm_x4_t(b, vd + pf_off(16 * kk + (lane & 15), 2 * jp + (lane >> 4)));
          pf_mma(o[2 * jp], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b[0], b[1]);
          pf_mma(o[2 * jp + 1], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b[2], b[3]);
        }
      }
    }
    __syncthreads();  // the stage is refilled next iteration
  }
  // normalise and store (bf16), rows of this stream's prompt only
  const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
  const int ra = r0 + g, rb = r0 + g + 8;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 8 * j + 2 * t;
    if (ra < a.rows_per_stream)
      *reinterpret_cast<uint32_t*>(a.out + (row_base + ra) * (size_t)a.nh * 128 + head * 128 + d) =
          bf16x2_rn(o[j][0] * ia, o[j][1] * ia);
    if (rb < a.rows_per_stream)
      *reinterpret_cast<uint32_t*>(a.out + (row_base + rb) * (size_t)a.nh * 128 + head * 128 + d) =
          bf16x2_rn(o[j][2] * ib, o[j][3] * ib);
  }
}

}  // namespace

cudaError_t launch_attn_prefill(const PrefillAttnArgs& a, int streams, cudaStream_t s) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const int rep = a.nh / a.nkv;
  const int QB = 128 / rep;
  dim3 grid((a.rows_per_stream + QB - 1) / QB, a.nkv, streams);
  attn_prefill_kernel<<<grid, kPfThreads, kPfSmem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace mtl
