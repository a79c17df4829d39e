// extern "C" entry points of libmtl_b200.so: argument validation, plan
// caching and launches.  Declarations and reference citations live in
// include/mtl_b200.h.
#include "../../include/mtl_b200.h"
#include "common.cuh"
#include "w4_gemv.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

namespace mtl {
cudaError_t w4_pack_gptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                         const int32_t* perm, int K, int N, int g, uint8_t* tiles, cudaStream_t s);
cudaError_t w4_pack_ref(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles,
                        cudaStream_t s);
cudaError_t w4_unpack_codes(const uint8_t* tiles, int K, int N, int g, int fmt, uint8_t* codes, cudaStream_t s);
}  // namespace mtl

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MTL_E_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool valid_group(int g) { return g == 32 || g == 64 || g == 128 || g == 256; }

int num_sms() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  cache[dev] = n;
  return n;
}

bool use_pdl() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MTL_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

int get_plan(int M, int K, int N, int g, int fmt, mtl::W4Plan* out) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int>, mtl::W4Plan> cache;
  const int sms = num_sms();
  auto key = std::make_tuple(M, K, N, g, fmt, sms);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return 0;
    }
  }
  mtl::W4Plan p;
  int r = mtl::w4_plan(M, K, N, g, fmt, sms, &p);
  if (r != 0) return r;
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = p;
  *out = p;
  return 0;
}

int check_w4_shape(int K, int N, int g, int fmt) {
  if (!valid_group(g)) return fail(MTL_E_INVALID, "group_size %d not in {32,64,128,256}", g);
  if (K <= 0 || N <= 0) return fail(MTL_E_INVALID, "K=%d N=%d must be positive", K, N);
  if (K % g) return fail(MTL_E_INVALID, "K=%d is not a multiple of group_size %d", K, g);
  if (N % mtl::kNT) return fail(MTL_E_INVALID, "N=%d is not a multiple of %d", N, mtl::kNT);
  if (fmt != MTL_FMT_REF && fmt != MTL_FMT_GPTQ) return fail(MTL_E_INVALID, "unknown param_fmt %d", fmt);
  return 0;
}

size_t counters_bytes(int N) { return ((size_t)(N / mtl::kNT) * 4 + 255) / 256 * 256; }

}  // namespace

extern "C" {

const char* mtl_last_error(void) { return g_err; }

int mtl_abi_version(void) { return 1; }

int mtl_device_status(uint32_t* out, int clear) {
  if (!out) return fail(MTL_E_INVALID, "mtl_device_status: out is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "mtl_device_status: synchronize");
  uint32_t v = 0;
  e = cudaMemcpyFromSymbol(&v, mtl::g_device_status, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "mtl_device_status: read");
  *out = v;
  if (clear) {
    uint32_t z = 0;
    e = cudaMemcpyToSymbol(mtl::g_device_status, &z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e, "mtl_device_status: clear");
  }
  return MTL_OK;
}

int mtl_w4_plan(int M, int K, int N, int group_size, int param_fmt, size_t* tiles_bytes, size_t* scratch_bytes) {
  if (int r = check_w4_shape(K, N, group_size, param_fmt)) return r;
  if (M < 1) return fail(MTL_E_INVALID, "M=%d must be >= 1", M);
  const int mc = M < mtl::kW4MaxM ? M : mtl::kW4MaxM;
  mtl::W4Plan p;
  int r = get_plan(mc, K, N, group_size, param_fmt, &p);
  if (r != 0) return fail(MTL_E_UNSUPPORTED, "no launch plan for M=%d K=%d N=%d g=%d", mc, K, N, group_size);
  if (tiles_bytes) *tiles_bytes = (size_t)p.T * p.tile_bytes;
  if (scratch_bytes) *scratch_bytes = counters_bytes(N) + p.partial_bytes;
  return MTL_OK;
}

int mtl_w4_pack_ref(const uint8_t* q, const uint16_t* qsz, int K, int N, int group_size, void* tiles,
                    mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, MTL_FMT_REF)) return r;
  if (!q || !qsz || !tiles) return fail(MTL_E_INVALID, "mtl_w4_pack_ref: NULL pointer");
  if (!aligned(tiles, 16)) return fail(MTL_E_ALIGN, "tiles must be 16-byte aligned");
  cudaError_t e = mtl::w4_pack_ref(q, qsz, K, N, group_size, static_cast<uint8_t*>(tiles), stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_pack_ref");
}

int mtl_w4_pack_gptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales, const int32_t* perm,
                     int K, int N, int group_size, void* tiles, mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, MTL_FMT_GPTQ)) return r;
  if (!qweight || !qzeros || !scales || !tiles) return fail(MTL_E_INVALID, "mtl_w4_pack_gptq: NULL pointer");
  if (!aligned(tiles, 16)) return fail(MTL_E_ALIGN, "tiles must be 16-byte aligned");
  cudaError_t e = mtl::w4_pack_gptq(qweight, qzeros, scales, perm, K, N, group_size,
                                    static_cast<uint8_t*>(tiles), stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_pack_gptq");
}

int mtl_w4_unpack_codes(const void* tiles, int K, int N, int group_size, int param_fmt, uint8_t* codes,
                        mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, param_fmt)) return r;
  if (!tiles || !codes) return fail(MTL_E_INVALID, "mtl_w4_unpack_codes: NULL pointer");
  cudaError_t e = mtl::w4_unpack_codes(static_cast<const uint8_t*>(tiles), K, N, group_size, param_fmt, codes,
                                       stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_unpack_codes");
}

int mtl_w4a16_linear(const uint16_t* x, int ldx, int M, int K, int N, int group_size, int param_fmt,
                     const void* tiles, int zero_offset, const int32_t* k_perm, const uint16_t* norm_w,
                     float norm_eps, int epilogue, const uint16_t* residual, uint16_t* y, int ldy, void* scratch,
                     size_t scratch_bytes, mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, param_fmt)) return r;
  if (!x || !tiles || !y || !scratch) return fail(MTL_E_INVALID, "mtl_w4a16_linear: NULL pointer");
  if (M < 1) return fail(MTL_E_INVALID, "M=%d must be >= 1", M);
  if (ldx < K) return fail(MTL_E_INVALID, "ldx=%d < K=%d", ldx, K);
  if (epilogue != MTL_EPI_STORE && epilogue != MTL_EPI_RESIDUAL && epilogue != MTL_EPI_SWIGLU)
    return fail(MTL_E_INVALID, "unknown epilogue %d", epilogue);
  const int nout = epilogue == MTL_EPI_SWIGLU ? N / 2 : N;
  if (ldy < nout) return fail(MTL_E_INVALID, "ldy=%d < %d outputs", ldy, nout);
  if (epilogue == MTL_EPI_RESIDUAL && !residual) return fail(MTL_E_INVALID, "residual epilogue needs residual");
  if (zero_offset < 0 || zero_offset > 1) return fail(MTL_E_INVALID, "zero_offset must be 0 or 1");
  if (!aligned(tiles, 16)) return fail(MTL_E_ALIGN, "tiles must be 16-byte aligned");
  if (!aligned(scratch, 256)) return fail(MTL_E_ALIGN, "scratch must be 256-byte aligned");
  if (!aligned(x, 2) || !aligned(y, 2)) return fail(MTL_E_ALIGN, "x/y must be 2-byte aligned");
  size_t need = 0;
  if (int r = mtl_w4_plan(M, K, N, group_size, param_fmt, nullptr, &need)) return r;
  if (scratch_bytes < need) return fail(MTL_E_SCRATCH, "scratch %zu < required %zu bytes", scratch_bytes, need);

  for (int m0 = 0; m0 < M; m0 += mtl::kW4MaxM) {
    const int mc = (M - m0) < mtl::kW4MaxM ? (M - m0) : mtl::kW4MaxM;
    mtl::W4Args a{};
    if (get_plan(mc, K, N, group_size, param_fmt, &a.p))
      return fail(MTL_E_UNSUPPORTED, "no launch plan for M=%d K=%d N=%d", mc, K, N);
    a.x = x + (size_t)m0 * ldx;
    a.ldx = ldx;
    a.M = mc;
    a.K = K;
    a.N = N;
    a.g = group_size;
    a.tiles = static_cast<const uint8_t*>(tiles);
    a.k_perm = k_perm;
    a.norm_w = norm_w;
    a.norm_eps = norm_eps;
    a.epi = epilogue;
    a.residual = residual ? residual + (size_t)m0 * N : nullptr;
    a.ldr = N;
    a.y = y + (size_t)m0 * ldy;
    a.ldy = ldy;
    a.counters = static_cast<int*>(scratch);
    a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + counters_bytes(N));
    a.zero_offset = zero_offset;
    a.xvec = (aligned(a.x, 16) && (ldx % 8) == 0 && (K % 16) == 0 && !k_perm && (!norm_w || aligned(norm_w, 16)))
                 ? 1 : 0;
    cudaError_t e = mtl::w4_launch(a, param_fmt, stream, use_pdl() ? 1 : 0);
    if (e != cudaSuccess) return cuda_fail(e, "mtl_w4a16_linear launch");
  }
  return MTL_OK;
}

}  // extern "C"
