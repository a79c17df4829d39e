// bf16 linear for 2..16 activation rows on the tensor cores (sm_100a): the
// heads of the batched decode step (the reference runs them per stream,
// moss_tts_lite/fast.py:174-194 / model.py:240-295), with the final RMSNorm
// fused as prologue and the audio heads' pad column forced to -inf.
//
// Each warp owns a 16-row strip of W over the whole K: the strip rows are the
// A operand of m16n8k16 MMAs (16-byte global loads straight into the A
// fragments), the batch rows the N dimension (one or two 8-row n-tiles, B
// from shared memory), so no partial sums cross warps.  Within each 32-column
// block the k positions are permuted the same way in A and B (lane t holds
// columns 8t..8t+7 of its two rows: MMA j takes 8t+4j..8t+4j+3), so both
// operands load 16 contiguous bytes per lane and x is staged in natural
// order.  Each output is one MMA accumulator summed over K in fp32.
namespace mtl {

namespace {

constexpr int kRowsWarps = 16;
constexpr int kRowsThreads = kRowsWarps * 32;
constexpr int kRowsUnroll = 4;  // 32-column blocks whose W loads are issued together

__host__ __device__ inline int rows_xstride(int K) { return K * 2 + 64; }  // bytes; rows fall in different banks

template <int NT>
__global__ void __launch_bounds__(kRowsThreads, 1) bf16_rows_kernel(const Bf16GemvArgs a) {
  extern __shared__ __align__(16) uint8_t rows_sm[];
  constexpr int MR = 8 * NT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, tq = lane & 3;
  const int M = a.M, K = a.K, N = a.N, XS = rows_xstride(K);
  pdl_launch_dependents();
  pdl_wait();

  // ---- stage x (RMSNorm fused): warp w stages row w (rows >= M are zero)
  if (warp < MR) {
    uint8_t* xrow = rows_sm + (size_t)warp * XS;
    const int nc = K / 8;  // 16-byte chunks
    if (warp < M) {
      const uint4* xr = reinterpret_cast<const uint4*>(a.x + (size_t)warp * K);
      float rinv = 1.f;
      if (a.norm_w) {
        float ss = 0.f;
        for (int c0 = lane; c0 < nc; c0 += 32 * 4) {
          uint4 v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = c0 + 32 * e < nc ? __ldg(xr + c0 + 32 * e) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t u[4] = {v[e].x, v[e].y, v[e].z, v[e].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float lo = __uint_as_float(u[q] << 16), hi = __uint_as_float(u[q] & 0xFFFF0000u);
              ss = fmaf(lo, lo, ss);
              ss = fmaf(hi, hi, ss);
            }
          }
        }
        ss = warp_sum(ss);
        rinv = rsqrtf(ss / (float)K + a.eps);
      }
      for (int c0 = lane; c0 < nc; c0 += 32 * 4) {
        uint4 v[4], nv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[e] = c0 + 32 * e < nc ? __ldg(xr + c0 + 32 * e) : make_uint4(0u, 0u, 0u, 0u);
          nv[e] = (a.norm_w && c0 + 32 * e < nc) ? __ldg(reinterpret_cast<const uint4*>(a.norm_w) + c0 + 32 * e)
                                                 : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = c0 + 32 * e;
          if (c >= nc) break;
          uint32_t u[4] = {v[e].x, v[e].y, v[e].z, v[e].w};
          if (a.norm_w) {
            const uint32_t w4[4] = {nv[e].x, nv[e].y, nv[e].z, nv[e].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              // model.py:34-40: bf16(h * rsqrt(var + eps)), then bf16(weight * that)
              const float v0 = round_bf16(__uint_as_float(w4[q] << 16) * round_bf16(__uint_as_float(u[q] << 16) * rinv));
              const float v1 = round_bf16(__uint_as_float(w4[q] & 0xFFFF0000u) *
                                          round_bf16(__uint_as_float(u[q] & 0xFFFF0000u) * rinv));
              u[q] = (__float_as_uint(v0) >> 16) | (__float_as_uint(v1) & 0xFFFF0000u);
            }
          }
          const uint4 o = make_uint4(u[0], u[1], u[2], u[3]);
          reinterpret_cast<uint4*>(xrow)[c] = o;
          if (a.x_normed && blockIdx.x == 0) reinterpret_cast<uint4*>(a.x_normed + (size_t)warp * K)[c] = o;
        }
      }
    } else {
      for (int c = lane; c < nc; c += 32) reinterpret_cast<uint4*>(xrow)[c] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __syncthreads();

  // ---- strips: warp-owned, the whole K each
  const int U = (N + 15) / 16;
  const int nblk = K / 32;
  for (int u = blockIdx.x * kRowsWarps + warp; u < U; u += gridDim.x * kRowsWarps) {
    const int r0 = 16 * u + gr, r1 = r0 + 8;
    const uint4* w0 = reinterpret_cast<const uint4*>(a.W + (size_t)min(r0, N - 1) * K) + tq;
    const uint4* w1 = reinterpret_cast<const uint4*>(a.W + (size_t)min(r1, N - 1) * K) + tq;
    const bool v0 = r0 < N, v1 = r1 < N;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    for (int c0 = 0; c0 < nblk; c0 += kRowsUnroll) {
      uint4 wa[kRowsUnroll], wb[kRowsUnroll];
#pragma unroll
      for (int i = 0; i < kRowsUnroll; ++i) {
        const bool in = c0 + i < nblk;
        wa[i] = (in && v0) ? __ldg(w0 + 4 * (c0 + i)) : make_uint4(0u, 0u, 0u, 0u);
        wb[i] = (in && v1) ? __ldg(w1 + 4 * (c0 + i)) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < kRowsUnroll; ++i) {
        if (c0 + i >= nblk) break;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 xb = *reinterpret_cast<const uint4*>(rows_sm + (size_t)(gr + 8 * nt) * XS + 64 * (c0 + i) + 16 * tq);
          mma_bf16_16816(acc[nt], wa[i].x, wb[i].x, wa[i].y, wb[i].y, xb.x, xb.y);
          mma_bf16_16816(acc[nt], wa[i].z, wb[i].z, wa[i].w, wb[i].w, xb.z, xb.w);
        }
      }
    }
    // lane holds rows gr / gr + 8 for batch rows 8 nt + 2 tq (+1)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = (e & 2) ? r1 : r0, m = 8 * nt + 2 * tq + (e & 1);
        if (row < N && m < M) {
          uint16_t b = f32_to_bf16_bits(acc[nt][e]);
          if (a.pad_period > 0 && (row % a.pad_period) == a.pad_col) b = 0xFF80u;  // -inf
          a.y[(size_t)m * a.ldy + row] = b;
        }
      }
  }
}

}  // namespace

size_t bf16_rows_smem(int M, int K) { return (size_t)(M > 8 ? 16 : 8) * rows_xstride(K); }

cudaError_t launch_bf16_rows(const Bf16GemvArgs& a, int num_sms, cudaStream_t s, int use_pdl) {
  const bool two = a.M > 8;
  auto kern = two ? bf16_rows_kernel<2> : bf16_rows_kernel<1>;
  static bool done[2] = {false, false};
  if (!done[two]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    done[two] = true;
  }
  const int U = (a.N + 15) / 16;
  const int grid = std::max(1, std::min((U + kRowsWarps - 1) / kRowsWarps, num_sms));
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_cfg(dim3(grid), dim3(kRowsThreads), bf16_rows_smem(a.M, a.K), s, attr, use_pdl);
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace mtl
