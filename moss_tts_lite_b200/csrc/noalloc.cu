// W4A16 linear for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc: an FFI/plugin host that
// owns all device memory in its own pool and hands the library no
// allocator, or a serving loop that records its decode step under CUDA
// stream capture (where cudaMalloc is not permitted) and must not stall on
// the device synchronisation an allocation can cause.  For them,
// mtl_w4a16_linear_noalloc runs the same kernel as mtl_w4a16_linear with its
// split-K scratch taken from a fixed file-scope device array instead of a
// caller buffer.
//
// Limits and sharing:
//  * the array holds kNoAllocScratchBytes (1 MiB) on every GPU that loads
//    the library, for as long as the library stays loaded;
//  * every argument is checked before any device work; shapes whose scratch
//    (mtl_w4_plan) exceeds the array are rejected with MTL_E_SCRATCH;
//  * every call shares the one array: calls that may run at the same time on
//    the GPU (different streams without ordering) race and must not be used;
//    calls ordered on one stream are fine;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make
//    that first call before any stream capture.
#include "../../include/mtl_b200.h"

#include <cstdint>
#include <mutex>

namespace mtl {

constexpr size_t kNoAllocScratchBytes = 1u << 20;

// The scratch itself: split-K counters (must be zero when a launch starts)
// followed by the split-K partials.  Host code never dereferences this name:
// on the host it is only a handle for cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;

// Device address of g_noalloc_scratch per device ordinal (nullptr = not set up).
void* noalloc_scratch_ptr(int* err) {
  static std::mutex mu;
  static void* ptrs[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = (e != cudaSuccess) ? (int)e : -1;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // with device `dev` current
    if (e != cudaSuccess || p == nullptr) {
      *err = (e != cudaSuccess) ? (int)e : -1;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *err = 0;
  return ptrs[dev];
}

}  // namespace
}  // namespace mtl

extern "C" int mtl_w4a16_linear_noalloc(const uint16_t* x, int ldx, int M, int K, int N, int group_size,
                                        int param_fmt, const void* tiles, int zero_offset, const int32_t* k_perm,
                                        const uint16_t* norm_w, float norm_eps, int epilogue,
                                        const uint16_t* residual, uint16_t* y, int ldy, mtl_stream_t stream) {
  // every argument is checked before anything is put on the caller's stream
  size_t need = 0;
  if (int r = check_w4_linear_args(x, ldx, M, K, N, group_size, param_fmt, tiles, zero_offset, k_perm, norm_w,
                                   epilogue, residual, y, ldy, &need))
    return r;
  if (need > mtl::kNoAllocScratchBytes)
    return fail(MTL_E_SCRATCH, "mtl_w4a16_linear_noalloc: shape needs %zu scratch bytes, the fixed device array holds %zu",
                need, mtl::kNoAllocScratchBytes);
  int err = 0;
  void* scratch = mtl::noalloc_scratch_ptr(&err);
  if (!scratch)
    return fail(MTL_E_CUDA, "mtl_w4a16_linear_noalloc: cannot resolve the device scratch array (error %d)", err);
  // The split-K counters at the head of the array must start at zero.  A
  // completed launch leaves them zero, but clear them anyway so that an
  // interrupted earlier call cannot leak into this one (a memset on the
  // caller's stream allocates nothing).  The two tile formats keep one
  // counter per 64- or 128-column block.
  const size_t cbytes = param_fmt == MTL_FMT_TC ? tc_counters_bytes(N) : counters_bytes(N);
  cudaError_t e = cudaMemsetAsync(scratch, 0, cbytes, stream);
  if (e != cudaSuccess) return cuda_fail(e, "mtl_w4a16_linear_noalloc: clear counters");
  return mtl_w4a16_linear(x, ldx, M, K, N, group_size, param_fmt, tiles, zero_offset, k_perm, norm_w, norm_eps,
                          epilogue, residual, y, ldy, scratch, mtl::kNoAllocScratchBytes, stream);
}
