// extern "C" entry points of libmtl_b200.so: argument validation, plan
// caching and launches.  Declarations and reference citations live in
// include/mtl_b200.h.
#include "../../include/mtl_b200.h"
#include "common.cuh"
#include "w4_gemv.cuh"
#include "w4_chain.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

namespace mtl {
cudaError_t launch_embed_sum(const int64_t* ids, int M, const uint16_t* emb_text, int text_vocab,
                             const uint16_t* emb_audio, int H, uint16_t* out, cudaStream_t s, int use_pdl);
cudaError_t launch_attn_decode(const AttnArgs& a, int streams, cudaStream_t s, int use_pdl);
cudaError_t launch_attn_append(const AttnArgs& a, int streams, cudaStream_t s, int use_pdl);
cudaError_t launch_bf16_gemv(const Bf16GemvArgs& a, int num_sms, cudaStream_t s, int use_pdl);
cudaError_t launch_bf16_rows(const Bf16GemvArgs& a, int num_sms, cudaStream_t s, int use_pdl);
size_t bf16_rows_smem(int M, int K);
cudaError_t launch_argmax_rows(const uint16_t* x, int rows, int cols, int ld, int64_t* out, cudaStream_t s,
                               int use_pdl);
cudaError_t launch_rtn_quantize(const uint16_t* w, int N, int K, int g, uint8_t* q, uint16_t* qsz, cudaStream_t s);
cudaError_t launch_argmax_masked(const uint16_t* x, int cols, const int* excl, int n_excl, int64_t* out,
                                 void* scratch, int num_sms, cudaStream_t s, int use_pdl);
struct FeedArgs;
cudaError_t launch_feed_row(const FeedArgs& f, cudaStream_t s, int use_pdl);
cudaError_t launch_greedy_feed(const uint16_t* la, const uint16_t* two, int64_t* ids, int64_t* pos, int streams,
                               int gen_slot, int delay_slot, cudaStream_t s, int use_pdl);
cudaError_t launch_rmsnorm_rows(const uint16_t* x, int rows, int K, int ldx, const uint16_t* w, float eps,
                                uint16_t* y, int ldy, cudaStream_t s, int use_pdl);
cudaError_t launch_sample_rows(const SampleArgs& a, cudaStream_t s);
cudaError_t w4_pack_gptq(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                         const int32_t* perm, int K, int N, int g, uint8_t* tiles, cudaStream_t s);
cudaError_t w4_pack_ref(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles,
                        cudaStream_t s);
cudaError_t w4_unpack_codes(const uint8_t* tiles, int K, int N, int g, int fmt, uint8_t* codes, cudaStream_t s);
int w4_tc_plan(int K, int N, int g, int num_sms, TcPlan* out);
cudaError_t w4_tc_launch(const TcArgs& a, cudaStream_t stream, int use_pdl);
int w4_tcb_plan(int K, int N, int g, int num_sms, TcPlan* out);
cudaError_t w4_tcb_launch(const TcbArgs& a, cudaStream_t stream, int use_pdl);
cudaError_t w4_tc_pack(const uint8_t* q, const uint16_t* qsz, int K, int N, int g, uint8_t* tiles, cudaStream_t s);
cudaError_t w4_tc_unpack_codes(const uint8_t* tiles, int K, int N, int g, uint8_t* codes, cudaStream_t s);
struct PrefillAttnArgs;
cudaError_t launch_attn_prefill(const PrefillAttnArgs& a, int streams, cudaStream_t s);
cudaError_t w4_gemm_launch(const uint16_t* x, int ldx, int L, int K, int N, int g, const uint8_t* tiles, int epi,
                           const uint16_t* residual, int ldr, uint16_t* y, int ldy, int num_sms, cudaStream_t s,
                           int use_pdl);
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

int get_tc_plan(int K, int N, int g, mtl::TcPlan* out) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, mtl::TcPlan> cache;
  const int sms = num_sms();
  auto key = std::make_tuple(K, N, g, sms);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return 0;
    }
  }
  mtl::TcPlan p;
  int r = mtl::w4_tc_plan(K, N, g, sms, &p);
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
  if (fmt != MTL_FMT_REF && fmt != MTL_FMT_GPTQ && fmt != MTL_FMT_TC)
    return fail(MTL_E_INVALID, "unknown param_fmt %d", fmt);
  if (fmt == MTL_FMT_TC) {
    if (N % mtl::kTcRows) return fail(MTL_E_INVALID, "N=%d is not a multiple of %d", N, mtl::kTcRows);
    if (g == 256) return fail(MTL_E_UNSUPPORTED, "MTL_FMT_TC supports group_size 32/64/128");
    if (K > mtl::kTcMaxK) return fail(MTL_E_UNSUPPORTED, "MTL_FMT_TC supports K <= %d", mtl::kTcMaxK);
    return 0;
  }
  if (N % mtl::kNT) return fail(MTL_E_INVALID, "N=%d is not a multiple of %d", N, mtl::kNT);
  return 0;
}

size_t counters_bytes(int N) { return ((size_t)(N / mtl::kNT) * 4 + 255) / 256 * 256; }
size_t tc_counters_bytes(int N) { return ((size_t)(N / mtl::kTcRows) * 4 + 255) / 256 * 256; }

}  // namespace

extern "C" {

const char* mtl_last_error(void) { return g_err; }

int mtl_abi_version(void) { return 2; }

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
  if (param_fmt == MTL_FMT_TC) {
    mtl::TcPlan p;
    if (get_tc_plan(K, N, group_size, &p))
      return fail(MTL_E_UNSUPPORTED, "no tensor-core plan for K=%d N=%d g=%d", K, N, group_size);
    size_t part = p.partial_bytes;
    mtl::TcPlan pb;
    if (M > 1 && mtl::w4_tcb_plan(K, N, group_size, num_sms(), &pb) == 0 && pb.partial_bytes > part)
      part = pb.partial_bytes;
    if (tiles_bytes) *tiles_bytes = (size_t)p.T * p.tile_bytes;
    if (scratch_bytes) *scratch_bytes = tc_counters_bytes(N) + part;
    return MTL_OK;
  }
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

int mtl_w4_pack_tc(const uint8_t* q, const uint16_t* qsz, int K, int N, int group_size, void* tiles,
                   mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, MTL_FMT_TC)) return r;
  if (!q || !qsz || !tiles) return fail(MTL_E_INVALID, "mtl_w4_pack_tc: NULL pointer");
  if (!aligned(tiles, 16)) return fail(MTL_E_ALIGN, "tiles must be 16-byte aligned");
  cudaError_t e = mtl::w4_tc_pack(q, qsz, K, N, group_size, static_cast<uint8_t*>(tiles), stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_pack_tc");
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
  if (param_fmt == MTL_FMT_TC) {
    cudaError_t e = mtl::w4_tc_unpack_codes(static_cast<const uint8_t*>(tiles), K, N, group_size, codes, stream);
    return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_unpack_codes");
  }
  cudaError_t e = mtl::w4_unpack_codes(static_cast<const uint8_t*>(tiles), K, N, group_size, param_fmt, codes,
                                       stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_unpack_codes");
}

int mtl_w4_dequant(const void* tiles, int K, int N, int group_size, int param_fmt, int zero_offset, uint16_t* w,
                   mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, param_fmt)) return r;
  if (param_fmt == MTL_FMT_TC) return fail(MTL_E_UNSUPPORTED, "mtl_w4_dequant: MTL_FMT_TC tiles");
  if (!tiles || !w) return fail(MTL_E_INVALID, "mtl_w4_dequant: NULL pointer");
  if (!aligned(tiles, 16) || !aligned(w, 16)) return fail(MTL_E_ALIGN, "mtl_w4_dequant: tiles / w must be 16-byte aligned");
  if (zero_offset < 0 || zero_offset > 1) return fail(MTL_E_INVALID, "zero_offset must be 0 or 1");
  cudaError_t e = mtl::w4_dequant(static_cast<const uint8_t*>(tiles), K, N, group_size, param_fmt, zero_offset, w,
                                  stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_dequant");
}

}  // extern "C"

namespace {

// Every argument check of mtl_w4a16_linear except those on the scratch
// buffer: no device work happens before these pass.  On success *need is
// the scratch the call requires (mtl_w4_plan).
int check_w4_linear_args(const uint16_t* x, int ldx, int M, int K, int N, int group_size, int param_fmt,
                         const void* tiles, int zero_offset, const int32_t* k_perm, const uint16_t* norm_w,
                         int epilogue, const uint16_t* residual, const uint16_t* y, int ldy, size_t* need) {
  if (int r = check_w4_shape(K, N, group_size, param_fmt)) return r;
  if (!x || !tiles || !y) return fail(MTL_E_INVALID, "mtl_w4a16_linear: NULL pointer");
  if (M < 1) return fail(MTL_E_INVALID, "M=%d must be >= 1", M);
  if (ldx < K) return fail(MTL_E_INVALID, "ldx=%d < K=%d", ldx, K);
  if (epilogue != MTL_EPI_STORE && epilogue != MTL_EPI_RESIDUAL && epilogue != MTL_EPI_SWIGLU)
    return fail(MTL_E_INVALID, "unknown epilogue %d", epilogue);
  const int nout = epilogue == MTL_EPI_SWIGLU ? N / 2 : N;
  if (ldy < nout) return fail(MTL_E_INVALID, "ldy=%d < %d outputs", ldy, nout);
  if (epilogue == MTL_EPI_RESIDUAL && !residual) return fail(MTL_E_INVALID, "residual epilogue needs residual");
  if (zero_offset < 0 || zero_offset > 1) return fail(MTL_E_INVALID, "zero_offset must be 0 or 1");
  if (!aligned(tiles, 16)) return fail(MTL_E_ALIGN, "tiles must be 16-byte aligned");
  if (!aligned(x, 2) || !aligned(y, 2)) return fail(MTL_E_ALIGN, "x/y must be 2-byte aligned");
  if (param_fmt == MTL_FMT_TC) {
    if (zero_offset != 0 || k_perm) return fail(MTL_E_UNSUPPORTED, "MTL_FMT_TC has no zero offset or k_perm");
    if (!aligned(x, 16) || (ldx % 8) || (norm_w && !aligned(norm_w, 16)))
      return fail(MTL_E_ALIGN, "MTL_FMT_TC needs 16-byte aligned x rows and norm_w");
  }
  return mtl_w4_plan(M, K, N, group_size, param_fmt, nullptr, need);
}

}  // namespace

extern "C" {

int mtl_w4a16_linear(const uint16_t* x, int ldx, int M, int K, int N, int group_size, int param_fmt,
                     const void* tiles, int zero_offset, const int32_t* k_perm, const uint16_t* norm_w,
                     float norm_eps, int epilogue, const uint16_t* residual, uint16_t* y, int ldy, void* scratch,
                     size_t scratch_bytes, mtl_stream_t stream) {
  size_t need = 0;
  if (int r = check_w4_linear_args(x, ldx, M, K, N, group_size, param_fmt, tiles, zero_offset, k_perm, norm_w,
                                   epilogue, residual, y, ldy, &need))
    return r;
  if (!scratch) return fail(MTL_E_INVALID, "mtl_w4a16_linear: NULL pointer");
  if (!aligned(scratch, 256)) return fail(MTL_E_ALIGN, "scratch must be 256-byte aligned");
  if (scratch_bytes < need) return fail(MTL_E_SCRATCH, "scratch %zu < required %zu bytes", scratch_bytes, need);

  if (param_fmt == MTL_FMT_TC) {
    // tensor-core kernel: one launch per activation row (batch-1 decode path)
    mtl::TcArgs a{};
    if (get_tc_plan(K, N, group_size, &a.p)) return fail(MTL_E_UNSUPPORTED, "no tensor-core plan");
    a.K = K;
    a.N = N;
    a.g = group_size;
    a.tiles = static_cast<const uint8_t*>(tiles);
    a.norm_w = norm_w;
    a.norm_eps = norm_eps;
    a.epi = epilogue;
    a.counters = static_cast<int*>(scratch);
    a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + tc_counters_bytes(N));
    if (M > 1) {
      // several rows: the batch is the N = 16 dimension of the MMAs
      mtl::TcbArgs b{};
      if (mtl::w4_tcb_plan(K, N, group_size, num_sms(), &b.p))
        return fail(MTL_E_UNSUPPORTED, "no batched tensor-core plan");
      b.ldx = ldx;
      b.K = K;
      b.N = N;
      b.g = group_size;
      b.tiles = a.tiles;
      b.norm_w = norm_w;
      b.norm_eps = norm_eps;
      b.epi = epilogue;
      b.ldy = ldy;
      b.counters = a.counters;
      b.partials = a.partials;
      for (int m0 = 0; m0 < M; m0 += mtl::kTcbMaxM) {
        b.M = (M - m0) < mtl::kTcbMaxM ? (M - m0) : mtl::kTcbMaxM;
        b.x = x + (size_t)m0 * ldx;
        b.residual = residual ? residual + (size_t)m0 * N : nullptr;
        b.y = y + (size_t)m0 * ldy;
        cudaError_t e = mtl::w4_tcb_launch(b, stream, use_pdl() ? 1 : 0);
        if (e != cudaSuccess) return cuda_fail(e, "mtl_w4a16_linear (tensor cores, batched) launch");
      }
      return MTL_OK;
    }
    for (int m = 0; m < M; ++m) {
      a.x = x + (size_t)m * ldx;
      a.residual = residual ? residual + (size_t)m * N : nullptr;
      a.y = y + (size_t)m * ldy;
      cudaError_t e = mtl::w4_tc_launch(a, stream, use_pdl() ? 1 : 0);
      if (e != cudaSuccess) return cuda_fail(e, "mtl_w4a16_linear (tensor cores) launch");
    }
    return MTL_OK;
  }

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

int mtl_w4a16_gemm(const uint16_t* x, int ldx, int M, int K, int N, int group_size, const void* tiles, int epilogue,
                   const uint16_t* residual, int ldr, uint16_t* y, int ldy, mtl_stream_t stream) {
  if (int r = check_w4_shape(K, N, group_size, MTL_FMT_REF)) return r;
  if (!x || !tiles || !y) return fail(MTL_E_INVALID, "mtl_w4a16_gemm: NULL pointer");
  if (M < 1) return fail(MTL_E_INVALID, "M=%d must be >= 1", M);
  if (group_size < 64) return fail(MTL_E_UNSUPPORTED, "mtl_w4a16_gemm: group_size %d (64/128/256 served)", group_size);
  if (K % 64 || N % 128) return fail(MTL_E_UNSUPPORTED, "mtl_w4a16_gemm: K=%d N=%d (K %% 64, N %% 128 must be 0)", K, N);
  if (ldx < K || (ldx % 8)) return fail(MTL_E_INVALID, "ldx=%d (>= K, multiple of 8)", ldx);
  if (epilogue != MTL_EPI_STORE && epilogue != MTL_EPI_RESIDUAL && epilogue != MTL_EPI_SWIGLU)
    return fail(MTL_E_INVALID, "unknown epilogue %d", epilogue);
  const int nout = epilogue == MTL_EPI_SWIGLU ? N / 2 : N;
  if (ldy < nout) return fail(MTL_E_INVALID, "ldy=%d < %d outputs", ldy, nout);
  if (epilogue == MTL_EPI_RESIDUAL && (!residual || ldr < N))
    return fail(MTL_E_INVALID, "residual epilogue needs residual with ldr >= N");
  if (!aligned(x, 16) || !aligned(tiles, 16)) return fail(MTL_E_ALIGN, "x and tiles must be 16-byte aligned");
  if (!aligned(y, 2)) return fail(MTL_E_ALIGN, "y must be 2-byte aligned");
  cudaError_t e = mtl::w4_gemm_launch(x, ldx, M, K, N, group_size, static_cast<const uint8_t*>(tiles), epilogue,
                                      residual, ldr, y, ldy, num_sms(), stream, use_pdl() ? 1 : 0);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4a16_gemm");
}

int mtl_w4_strip_bytes(int K, int N, int group_size, size_t* bytes) {
  if (!bytes) return fail(MTL_E_INVALID, "mtl_w4_strip_bytes: NULL output");
  if (group_size != 64 && group_size != 128 && group_size != 256)
    return fail(MTL_E_UNSUPPORTED, "strip layout: group_size %d (64/128/256 served)", group_size);
  if (K <= 0 || N <= 0 || K % group_size || N % 16)
    return fail(MTL_E_INVALID, "strip layout: K=%d (multiple of %d), N=%d (multiple of 16)", K, group_size, N);
  *bytes = (size_t)(N / 16) * (K / group_size) * mtl::strip_tile_bytes(group_size);
  return MTL_OK;
}

int mtl_w4_pack_strip(const uint8_t* q, const uint16_t* qsz, int K, int N, int group_size, void* tiles,
                      mtl_stream_t stream) {
  size_t nb = 0;
  if (int r = mtl_w4_strip_bytes(K, N, group_size, &nb)) return r;
  if (!q || !qsz || !tiles) return fail(MTL_E_INVALID, "mtl_w4_pack_strip: NULL pointer");
  if (!aligned(tiles, 16) || !aligned(qsz, 2)) return fail(MTL_E_ALIGN, "tiles 16-byte, qsz 2-byte aligned");
  cudaError_t e = mtl::w4_pack_strip(q, qsz, K, N, group_size, static_cast<uint8_t*>(tiles), stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_pack_strip");
}

int mtl_w4_chain(const mtl_chain_phase* phases, int nphases, int group_size, float norm_eps, uint32_t* barrier,
                 mtl_stream_t stream) {
  if (!phases || nphases < 1 || nphases > mtl::kChainMaxPhases)
    return fail(MTL_E_INVALID, "mtl_w4_chain: %d phases (1..%d)", nphases, mtl::kChainMaxPhases);
  if (group_size != 64 && group_size != 128 && group_size != 256)
    return fail(MTL_E_UNSUPPORTED, "mtl_w4_chain: group_size %d (64/128/256 served)", group_size);
  if (!barrier || !aligned(barrier, 4)) return fail(MTL_E_INVALID, "mtl_w4_chain: barrier word NULL or misaligned");
  if (!(norm_eps > 0.f)) return fail(MTL_E_INVALID, "mtl_w4_chain: norm_eps must be > 0");
  mtl::ChainArgs a{};
  int Ks[mtl::kChainMaxPhases], Ns[mtl::kChainMaxPhases];
  for (int i = 0; i < nphases; ++i) {
    const mtl_chain_phase& P = phases[i];
    if (!P.tiles || !P.x || !P.y) return fail(MTL_E_INVALID, "mtl_w4_chain: phase %d: NULL tiles / x / y", i);
    if (P.K <= 0 || P.N <= 0 || P.K % group_size || P.N % 16 || P.K > mtl::kChainMaxK)
      return fail(MTL_E_INVALID, "mtl_w4_chain: phase %d: K=%d (multiple of %d, <= %d), N=%d (multiple of 16)", i,
                  P.K, group_size, mtl::kChainMaxK, P.N);
    if (P.epilogue != MTL_EPI_STORE && P.epilogue != MTL_EPI_RESIDUAL && P.epilogue != MTL_EPI_SWIGLU)
      return fail(MTL_E_INVALID, "mtl_w4_chain: phase %d: unknown epilogue %d", i, P.epilogue);
    if (P.epilogue == MTL_EPI_RESIDUAL && !P.residual)
      return fail(MTL_E_INVALID, "mtl_w4_chain: phase %d: residual epilogue needs residual", i);
    if (!aligned(P.tiles, 16) || !aligned(P.x, 16) || (P.norm_w && !aligned(P.norm_w, 16)) || !aligned(P.y, 2) ||
        (P.residual && !aligned(P.residual, 2)))
      return fail(MTL_E_ALIGN, "mtl_w4_chain: phase %d: tiles / x / norm_w 16-byte, y / residual 2-byte aligned", i);
    // every CTA reads all of x while others write their strips of y
    const uintptr_t yb = reinterpret_cast<uintptr_t>(P.y), xb = reinterpret_cast<uintptr_t>(P.x);
    const size_t ybytes = (size_t)(P.epilogue == MTL_EPI_SWIGLU ? P.N / 2 : P.N) * 2;
    if (yb < xb + (size_t)P.K * 2 && xb < yb + ybytes)
      return fail(MTL_E_INVALID, "mtl_w4_chain: phase %d: y overlaps its own x", i);
    a.ph[i].tiles = static_cast<const uint8_t*>(P.tiles);
    a.ph[i].x = P.x;
    a.ph[i].norm_w = P.norm_w;
    a.ph[i].residual = P.residual;
    a.ph[i].y = P.y;
    a.ph[i].K = P.K;
    a.ph[i].N = P.N;
    a.ph[i].epi = P.epilogue;
    Ks[i] = P.K;
    Ns[i] = P.N;
  }
  a.nphases = nphases;
  a.eps = norm_eps;
  a.barrier = barrier;
  mtl::ChainPlan plan;
  {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int, int, int, int, int, int, int, int>, mtl::ChainPlan> cache;
    int kk[4] = {0, 0, 0, 0}, nn[4] = {0, 0, 0, 0};
    for (int i = 0; i < nphases; ++i) {
      kk[i] = Ks[i];
      nn[i] = Ns[i];
    }
    const int sms = num_sms();
    auto key = std::make_tuple(nphases, group_size, sms, kk[0], kk[1], kk[2], kk[3], nn[0], nn[1], nn[2], nn[3]);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      plan = it->second;
    } else {
      if (mtl::w4_chain_plan(Ks, Ns, nphases, group_size, sms, &plan) != 0)
        return fail(MTL_E_UNSUPPORTED, "mtl_w4_chain: no plan fits these phases");
      cache[key] = plan;
    }
  }
  cudaError_t e = mtl::w4_chain_launch(a, group_size, plan, stream, use_pdl() ? 1 : 0);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_chain");
}

int mtl_w4_chain_rows(const mtl_chain_phase_rows* phases, int nphases, int M, int group_size, float norm_eps,
                      uint32_t* barrier, mtl_stream_t stream) {
  if (!phases || nphases < 1 || nphases > mtl::kChainMaxPhases)
    return fail(MTL_E_INVALID, "mtl_w4_chain_rows: %d phases (1..%d)", nphases, mtl::kChainMaxPhases);
  if (M < 1 || M > 16) return fail(MTL_E_INVALID, "mtl_w4_chain_rows: M=%d (1..16)", M);
  if (group_size != 64 && group_size != 128 && group_size != 256)
    return fail(MTL_E_UNSUPPORTED, "mtl_w4_chain_rows: group_size %d (64/128/256 served)", group_size);
  if (!barrier || !aligned(barrier, 4)) return fail(MTL_E_INVALID, "mtl_w4_chain_rows: barrier word NULL or misaligned");
  if (!(norm_eps > 0.f)) return fail(MTL_E_INVALID, "mtl_w4_chain_rows: norm_eps must be > 0");
  mtl::ChainBArgs a{};
  int Ks[mtl::kChainMaxPhases], Ns[mtl::kChainMaxPhases], norm[mtl::kChainMaxPhases], epis[mtl::kChainMaxPhases];
  for (int i = 0; i < nphases; ++i) {
    const mtl_chain_phase_rows& P = phases[i];
    if (!P.tiles || !P.x || !P.y) return fail(MTL_E_INVALID, "mtl_w4_chain_rows: phase %d: NULL tiles / x / y", i);
    if (P.K <= 0 || P.N <= 0 || P.K % group_size || P.N % 16)
      return fail(MTL_E_INVALID, "mtl_w4_chain_rows: phase %d: K=%d (multiple of %d), N=%d (multiple of 16)", i,
                  P.K, group_size, P.N);
    if (P.norm_w && P.K > 4096)
      return fail(MTL_E_UNSUPPORTED, "mtl_w4_chain_rows: phase %d: RMSNorm with K=%d > 4096", i, P.K);
    if (P.epilogue != MTL_EPI_STORE && P.epilogue != MTL_EPI_RESIDUAL && P.epilogue != MTL_EPI_SWIGLU)
      return fail(MTL_E_INVALID, "mtl_w4_chain_rows: phase %d: unknown epilogue %d", i, P.epilogue);
    const int nout = P.epilogue == MTL_EPI_SWIGLU ? P.N / 2 : P.N;
    if (P.ldx < P.K || P.ldx % 8 || P.ldy < nout || (P.epilogue == MTL_EPI_RESIDUAL && (!P.residual || P.ldr < P.N)))
      return fail(MTL_E_INVALID, "mtl_w4_chain_rows: phase %d: ldx=%d ldy=%d ldr=%d", i, P.ldx, P.ldy, P.ldr);
    if (!aligned(P.tiles, 16) || !aligned(P.x, 16) || (P.norm_w && !aligned(P.norm_w, 16)) || !aligned(P.y, 2) ||
        (P.residual && !aligned(P.residual, 2)))
      return fail(MTL_E_ALIGN, "mtl_w4_chain_rows: phase %d: tiles / x / norm_w 16-byte, y / residual 2-byte", i);
    // every CTA reads all of x while others write their strips of y
    const uintptr_t yb = reinterpret_cast<uintptr_t>(P.y), xb = reinterpret_cast<uintptr_t>(P.x);
    const size_t xbytes = ((size_t)(M - 1) * P.ldx + P.K) * 2, ybytes = ((size_t)(M - 1) * P.ldy + nout) * 2;
    if (yb < xb + xbytes && xb < yb + ybytes)
      return fail(MTL_E_INVALID, "mtl_w4_chain_rows: phase %d: y overlaps its own x", i);
    mtl::ChainBPhase& Q = a.ph[i];
    Q.tiles = static_cast<const uint8_t*>(P.tiles);
    Q.x = P.x;
    Q.norm_w = P.norm_w;
    Q.residual = P.residual;
    Q.y = P.y;
    Q.ldx = P.ldx;
    Q.ldr = P.ldr;
    Q.ldy = P.ldy;
    Q.K = P.K;
    Q.N = P.N;
    Q.epi = P.epilogue;
    Ks[i] = P.K;
    Ns[i] = P.N;
    norm[i] = P.norm_w != nullptr;
    epis[i] = P.epilogue;
  }
  a.nphases = nphases;
  a.M = M;
  a.eps = norm_eps;
  a.barrier = barrier;
  mtl::ChainPlan plan;
  if (mtl::w4_chainb_plan(Ks, Ns, norm, epis, nphases, M, group_size, num_sms(), &plan) != 0)
    return fail(MTL_E_UNSUPPORTED, "mtl_w4_chain_rows: no plan fits these phases");
  cudaError_t e = mtl::w4_chainb_launch(a, group_size, plan, stream, use_pdl() ? 1 : 0);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_chain_rows");
}

int mtl_attn_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                     long long cache_stream_stride, int max_seq, int n_heads, int n_kv, int head_dim,
                     int rows_per_stream, int streams, int p0, uint16_t* out, mtl_stream_t stream) {
  if (!q || !k_cache || !v_cache || !out) return fail(MTL_E_INVALID, "mtl_attn_prefill: NULL pointer");
  if (head_dim != 128) return fail(MTL_E_UNSUPPORTED, "head_dim %d (only 128)", head_dim);
  if (n_kv <= 0 || n_heads % n_kv) return fail(MTL_E_INVALID, "n_heads=%d n_kv=%d", n_heads, n_kv);
  const int rep = n_heads / n_kv;
  if (rep != 1 && rep != 2 && rep != 4 && rep != 8)
    return fail(MTL_E_UNSUPPORTED, "mtl_attn_prefill: %d query heads per KV head (1/2/4/8 served)", rep);
  if (rows_per_stream < 1 || streams < 1 || p0 < 0 || p0 + rows_per_stream > max_seq)
    return fail(MTL_E_INVALID, "rows_per_stream=%d streams=%d p0=%d max_seq=%d", rows_per_stream, streams, p0,
                max_seq);
  if (streams > 1 && cache_stream_stride < (long long)n_kv * max_seq * 128)
    return fail(MTL_E_INVALID, "cache_stream_stride %lld below one stream's cache", cache_stream_stride);
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 4))
    return fail(MTL_E_ALIGN, "mtl_attn_prefill: q / caches 16-byte, out 4-byte aligned");
  if (streams > 1 && (cache_stream_stride % 8)) return fail(MTL_E_ALIGN, "cache_stream_stride %% 8 != 0");
  mtl::PrefillAttnArgs a{};
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.cache_stream_stride = streams > 1 ? cache_stream_stride : 0;
  a.max_seq = max_seq;
  a.nh = n_heads;
  a.nkv = n_kv;
  a.rows_per_stream = rows_per_stream;
  a.p0 = p0;
  a.scale = 1.0f / sqrtf(128.0f);
  a.out = out;
  cudaError_t e = mtl::launch_attn_prefill(a, streams, stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_attn_prefill");
}

int mtl_embed_sum(const int64_t* ids, int M, const uint16_t* emb_text, int text_vocab, const uint16_t* emb_audio,
                  int hidden, uint16_t* out, mtl_stream_t stream) {
  if (!ids || !emb_text || !emb_audio || !out) return fail(MTL_E_INVALID, "mtl_embed_sum: NULL pointer");
  if (M < 1 || hidden <= 0 || hidden % 8 || text_vocab <= 0)
    return fail(MTL_E_INVALID, "mtl_embed_sum: M=%d hidden=%d text_vocab=%d", M, hidden, text_vocab);
  if (!aligned(emb_text, 16) || !aligned(emb_audio, 16) || !aligned(out, 16))
    return fail(MTL_E_ALIGN, "mtl_embed_sum: tables and out must be 16-byte aligned");
  cudaError_t e = mtl::launch_embed_sum(ids, M, emb_text, text_vocab, emb_audio, hidden, out, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_embed_sum");
}

static size_t attn_partial_floats(int streams, int n_heads, int n_kv, int splits) {
  return (size_t)streams * n_kv * splits * (n_heads / n_kv) * mtl::kAttnRec;
}
static size_t attn_counter_bytes(int streams, int n_kv) { return ((size_t)streams * n_kv * 4 + 255) / 256 * 256; }

int mtl_attn_scratch_bytes(int streams, int n_heads, int n_kv, int splits, size_t* out) {
  if (!out || streams < 1 || n_kv < 1 || n_heads < n_kv || n_heads % n_kv || splits < 1)
    return fail(MTL_E_INVALID, "mtl_attn_scratch_bytes: bad arguments");
  *out = attn_counter_bytes(streams, n_kv) + attn_partial_floats(streams, n_heads, n_kv, splits) * 4;
  return MTL_OK;
}

int mtl_attn_decode(const uint16_t* qkv, const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                    const uint16_t* rope_cos, const uint16_t* rope_sin, uint16_t* k_cache, uint16_t* v_cache,
                    long long cache_stream_stride, int max_seq, const int64_t* pos, int streams, int n_heads,
                    int n_kv, int head_dim, int splits, int flags, uint16_t* out, void* scratch,
                    size_t scratch_bytes, mtl_stream_t stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !rope_cos || !rope_sin || !k_cache || !v_cache || !pos || !out || !scratch)
    return fail(MTL_E_INVALID, "mtl_attn_decode: NULL pointer");
  if (head_dim != mtl::kHeadDim) return fail(MTL_E_UNSUPPORTED, "head_dim %d (only 128)", head_dim);
  if (n_kv < 1 || n_heads % n_kv || n_heads / n_kv > mtl::kAttnMaxRep)
    return fail(MTL_E_UNSUPPORTED, "n_heads=%d n_kv=%d (n_heads/n_kv must divide and be <= 8)", n_heads, n_kv);
  if (streams < 1 || max_seq < 1 || splits < 1 || splits > 64)
    return fail(MTL_E_INVALID, "streams=%d max_seq=%d splits=%d", streams, max_seq, splits);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || cache_stream_stride % 8)
    return fail(MTL_E_ALIGN, "KV cache must be 16-byte aligned");
  if (flags & ~MTL_ATTN_KV_STABLE) return fail(MTL_E_INVALID, "mtl_attn_decode: unknown flags 0x%x", flags);
  size_t need = 0;
  mtl_attn_scratch_bytes(streams, n_heads, n_kv, splits, &need);
  if (scratch_bytes < need) return fail(MTL_E_SCRATCH, "attention scratch %zu < %zu", scratch_bytes, need);
  if (!aligned(scratch, 256)) return fail(MTL_E_ALIGN, "scratch must be 256-byte aligned");
  mtl::AttnArgs a{};
  a.qkv = qkv;
  a.q_norm_w = q_norm_w;
  a.k_norm_w = k_norm_w;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.cache_stream_stride = cache_stream_stride;
  a.max_seq = max_seq;
  a.pos = pos;
  a.nh = n_heads;
  a.nkv = n_kv;
  a.splits = splits;
  a.flags = (flags & MTL_ATTN_KV_STABLE) ? mtl::kAttnKvStable : 0u;
  a.out = out;
  a.counters = static_cast<int*>(scratch);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + attn_counter_bytes(streams, n_kv));
  a.scale = 1.0f / sqrtf((float)head_dim);
  cudaError_t e = mtl::launch_attn_decode(a, streams, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_attn_decode");
}

int mtl_attn_append(const uint16_t* qkv, const uint16_t* q_norm_w, const uint16_t* k_norm_w, const uint16_t* rope_cos,
                    const uint16_t* rope_sin, uint16_t* k_cache, uint16_t* v_cache, long long cache_stream_stride,
                    int max_seq, const int64_t* pos, int streams, int n_heads, int n_kv, int head_dim, uint16_t* q_out,
                    mtl_stream_t stream) {
  if (!qkv || !k_norm_w || !rope_cos || !rope_sin || !k_cache || !v_cache || !pos || (q_out && !q_norm_w))
    return fail(MTL_E_INVALID, "mtl_attn_append: NULL pointer");
  if (head_dim != mtl::kHeadDim) return fail(MTL_E_UNSUPPORTED, "head_dim %d (only 128)", head_dim);
  if (n_kv < 1 || n_heads % n_kv || streams < 1 || streams > 65535 || max_seq < 1 || cache_stream_stride < 0)
    return fail(MTL_E_INVALID, "mtl_attn_append: n_heads=%d n_kv=%d streams=%d", n_heads, n_kv, streams);
  mtl::AttnArgs a{};
  a.qkv = qkv;
  a.k_norm_w = k_norm_w;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.cache_stream_stride = cache_stream_stride;
  a.max_seq = max_seq;
  a.pos = pos;
  a.nh = n_heads;
  a.nkv = n_kv;
  a.q_norm_w = q_norm_w;
  a.out = q_out;
  cudaError_t e = mtl::launch_attn_append(a, streams, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_attn_append");
}

int mtl_bf16_linear(const uint16_t* x, int M, int K, int N, const uint16_t* W, const uint16_t* norm_w, float eps,
                    uint16_t* x_normed, int pad_period, int pad_col, int epilogue, const uint16_t* residual,
                    uint16_t* y, int ldy, mtl_stream_t stream) {
  if (!x || !W || !y) return fail(MTL_E_INVALID, "mtl_bf16_linear: NULL pointer");
  if (epilogue < 0 || epilogue > 2) return fail(MTL_E_INVALID, "mtl_bf16_linear: unknown epilogue %d", epilogue);
  if (epilogue == 1 && !residual) return fail(MTL_E_INVALID, "mtl_bf16_linear: residual epilogue needs residual");
  if (epilogue == 2 && (N % 2)) return fail(MTL_E_INVALID, "mtl_bf16_linear: SwiGLU needs an even N");
  const int nout = epilogue == 2 ? N / 2 : N;
  // 5..16 rows with the store epilogue: the tensor-core kernel (up to 4 rows
  // the CUDA-core kernel, whose rows equal one-row calls bit for bit)
  const bool rows = M > mtl::kGemvMaxM && M <= 16 && epilogue == 0 && K % 32 == 0 && K <= mtl::kGemvMaxK &&
                    mtl::bf16_rows_smem(M, K) <= 227 * 1024;
  if (M < 1 || (M > mtl::kGemvMaxM && !rows) || K <= 0 || K > mtl::kGemvMaxK || K % 8 || N <= 0 || ldy < nout)
    return fail(MTL_E_INVALID,
                "mtl_bf16_linear: M=%d K=%d N=%d ldy=%d (M<=4, or M<=16 with the store epilogue and K%%32==0; "
                "K<=8192, K%%8==0)", M, K, N, ldy);
  if (pad_period < 0 || (pad_period > 0 && (pad_col < 0 || pad_col >= pad_period)))
    return fail(MTL_E_INVALID, "mtl_bf16_linear: pad_period=%d pad_col=%d", pad_period, pad_col);
  if (!aligned(W, 16)) return fail(MTL_E_ALIGN, "mtl_bf16_linear: W must be 16-byte aligned");
  mtl::Bf16GemvArgs a{};
  a.x = x;
  a.M = M;
  a.K = K;
  a.N = N;
  a.W = W;
  a.norm_w = norm_w;
  a.eps = eps;
  a.x_normed = x_normed;
  a.pad_period = pad_period;
  a.pad_col = pad_col;
  a.epi = epilogue;
  a.residual = residual;
  a.y = y;
  a.ldy = ldy;
  cudaError_t e = rows ? mtl::launch_bf16_rows(a, num_sms(), stream, use_pdl())
                       : mtl::launch_bf16_gemv(a, num_sms(), stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_bf16_linear");
}

int mtl_argmax_rows(const uint16_t* x, int rows, int cols, int ld, int64_t* out, mtl_stream_t stream) {
  if (!x || !out || rows < 1 || cols < 1 || ld < cols) return fail(MTL_E_INVALID, "mtl_argmax_rows: bad arguments");
  cudaError_t e = mtl::launch_argmax_rows(x, rows, cols, ld, out, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_argmax_rows");
}

int mtl_argmax_masked(const uint16_t* x, int cols, const int32_t* excluded, int n_excluded, int64_t* out,
                      void* scratch, mtl_stream_t stream) {
  if (!x || !out || cols < 1 || n_excluded < 0 || n_excluded > 8 || (n_excluded && !excluded))
    return fail(MTL_E_INVALID, "mtl_argmax_masked: bad arguments");
  if (scratch && !aligned(scratch, 16)) return fail(MTL_E_ALIGN, "mtl_argmax_masked: scratch must be 16-byte aligned");
  cudaError_t e = mtl::launch_argmax_masked(x, cols, excluded, n_excluded, out, scratch, num_sms(), stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_argmax_masked");
}

int mtl_greedy_feed(const uint16_t* audio_logits, const uint16_t* two_logits, int64_t* ids_row, int64_t* pos,
                    int streams, int gen_slot_id, int delay_slot_id, mtl_stream_t stream) {
  if (!audio_logits || !two_logits || !ids_row || !pos) return fail(MTL_E_INVALID, "mtl_greedy_feed: NULL pointer");
  if (streams < 1 || streams > 65535) return fail(MTL_E_INVALID, "mtl_greedy_feed: streams=%d", streams);
  cudaError_t e = mtl::launch_greedy_feed(audio_logits, two_logits, ids_row, pos, streams, gen_slot_id,
                                          delay_slot_id, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_greedy_feed");
}

int mtl_feed_row(const int64_t* dec, int text_mode, long long text_const, long long gen_slot_id,
                 long long delay_slot_id, unsigned int audio_mask, int audio_compact, long long pad_code,
                 int64_t* ids_row, int64_t* pos, long long pos_value, uint32_t* seen_bits, int seen_words,
                 mtl_stream_t stream) {
  if (!dec || !ids_row || !pos) return fail(MTL_E_INVALID, "mtl_feed_row: NULL pointer");
  if (text_mode < 0 || text_mode > 2 || (seen_bits && seen_words < 1) || pos_value < 0)
    return fail(MTL_E_INVALID, "mtl_feed_row: text_mode %d seen_words %d pos %lld", text_mode, seen_words, pos_value);
  mtl::FeedArgs f{};
  f.dec = dec;
  f.ids = ids_row;
  f.pos_dev = pos;
  f.seen = seen_bits;
  f.pos = pos_value;
  f.text_const = text_const;
  f.gen_slot = gen_slot_id;
  f.delay_slot = delay_slot_id;
  f.pad_code = pad_code;
  f.audio_mask = audio_mask;
  f.text_mode = text_mode;
  f.audio_compact = audio_compact;
  f.seen_words = seen_words;
  cudaError_t e = mtl::launch_feed_row(f, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_feed_row");
}

// Threads per row (log2) of PyTorch's shared-memory cumsum of a [num_rows,
// row_size] tensor (get_log_num_threads_x_inner_scan, ATen ScanUtils.cuh):
// about 512 threads per block split in the ratio of row_size to num_rows,
// clamped to [2^4, 2^9].
static int inner_scan_log_threads_x(int num_rows, int row_size) {
  int lx = 0, ly = 0;
  while ((1 << lx) < row_size) ++lx;
  while ((1 << ly) < num_rows) ++ly;
  int l = (9 + lx - ly) / 2;
  return l < 4 ? 4 : (l > 9 ? 9 : l);
}

size_t mtl_sample_scratch_bytes(int cols, int n_rows, int top_k) {
  int slice_len = 0;
  const int slices = mtl::sample_slice_count(cols, top_k, &slice_len);
  return slices > 0 && n_rows > 0 ? (size_t)n_rows * slices * top_k * 8 : 0;
}

int mtl_sample_rows(const uint16_t* logits, int ld, int cols, int n_rows, const int32_t* row_index,
                    float temperature, int top_k, float top_p, float repetition_penalty, const uint32_t* seen_bits,
                    int words_per_set, const int32_t* seen_set_of_row, const int32_t* excluded, int n_excluded,
                    const int32_t* scan_rows, uint64_t seed, uint64_t offset, int64_t out_add, int64_t* out,
                    void* scratch, size_t scratch_bytes, mtl_stream_t stream) {
  if (!logits || !out || !row_index) return fail(MTL_E_INVALID, "mtl_sample_rows: NULL pointer");
  if (n_rows < 1 || n_rows > mtl::kSampleMaxRows || cols < 1 || ld < cols)
    return fail(MTL_E_INVALID, "mtl_sample_rows: n_rows=%d (1..%d) cols=%d ld=%d", n_rows, mtl::kSampleMaxRows, cols, ld);
  if (!(temperature > 0.f)) return fail(MTL_E_INVALID, "mtl_sample_rows: temperature must be > 0");
  if (n_excluded < 0 || n_excluded > mtl::kSampleMaxExcl || (n_excluded && !excluded))
    return fail(MTL_E_INVALID, "mtl_sample_rows: n_excluded=%d (<= %d)", n_excluded, mtl::kSampleMaxExcl);
  const int k = (top_k > 0 && top_k < cols) ? top_k : cols;
  if (k > mtl::kSampleMaxCand)
    return fail(MTL_E_UNSUPPORTED, "mtl_sample_rows: %d candidates (top_k=%d, cols=%d) exceed %d", k, top_k, cols,
                mtl::kSampleMaxCand);
  if (repetition_penalty != 1.0f && seen_bits && (!seen_set_of_row || words_per_set < (cols + 31) / 32))
    return fail(MTL_E_INVALID, "mtl_sample_rows: seen bitmap needs words_per_set >= %d", (cols + 31) / 32);
  mtl::SampleArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.cols = cols;
  a.n_rows = n_rows;
  const bool pen = repetition_penalty != 1.0f && seen_bits != nullptr;
  for (int r = 0; r < n_rows; ++r) {
    a.row_index[r] = row_index[r];
    a.seen_set[r] = pen ? seen_set_of_row[r] : -1;
    const int sr = scan_rows ? scan_rows[r] : 1;
    if (sr < 1) return fail(MTL_E_INVALID, "mtl_sample_rows: scan_rows[%d]=%d (>= 1)", r, sr);
    a.scan_lognx[r] = sr == 1 ? 0 : inner_scan_log_threads_x(sr, cols);
  }
  a.seen_bits = pen ? seen_bits : nullptr;
  a.words_per_set = words_per_set;
  // PyTorch on CUDA divides by a Python scalar as a multiply by its float reciprocal
  a.inv_temp = 1.0f / temperature;
  a.penalty = repetition_penalty;
  a.inv_penalty = 1.0f / repetition_penalty;
  a.top_k = top_k;
  // `cumulative_probs > top_p` compares bf16 against the scalar rounded to bf16
  a.top_p_bf = top_p >= 1.0f ? 2.0f : __bfloat162float(__float2bfloat16_rn(top_p));
  a.n_excl = n_excluded;
  for (int e = 0; e < n_excluded; ++e) a.excl[e] = excluded[e];
  a.seed_lo = (uint32_t)seed;
  a.seed_hi = (uint32_t)(seed >> 32);
  a.off_lo = (uint32_t)offset;
  a.off_hi = (uint32_t)(offset >> 32);
  a.out = out;
  a.out_add = out_add;
  int slice_len = 0;
  const int slices = scratch ? mtl::sample_slice_count(cols, top_k, &slice_len) : 0;
  if (slices > 0) {
    const size_t per = (size_t)n_rows * slices * top_k;
    if (scratch_bytes < per * 8) return fail(MTL_E_SCRATCH, "mtl_sample_rows: scratch %zu < %zu bytes", scratch_bytes, per * 8);
    if (!aligned(scratch, 16)) return fail(MTL_E_ALIGN, "mtl_sample_rows: scratch must be 16-byte aligned");
    a.slices = slices;
    a.slice_len = slice_len;
    a.cand_val = static_cast<float*>(scratch);
    a.cand_id = reinterpret_cast<int32_t*>(static_cast<float*>(scratch) + per);
  }
  cudaError_t e = mtl::launch_sample_rows(a, stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_sample_rows");
}

int mtl_rmsnorm(const uint16_t* x, int rows, int K, int ldx, const uint16_t* weight, float eps, uint16_t* y,
                int ldy, mtl_stream_t stream) {
  if (!x || !weight || !y || rows < 1 || K < 1 || ldx < K || ldy < K)
    return fail(MTL_E_INVALID, "mtl_rmsnorm: bad arguments");
  cudaError_t e = mtl::launch_rmsnorm_rows(x, rows, K, ldx, weight, eps, y, ldy, stream, use_pdl());
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_rmsnorm");
}

int mtl_w4_rtn_quantize(const uint16_t* w, int N, int K, int group_size, uint8_t* q, uint16_t* qsz,
                        mtl_stream_t stream) {
  if (!w || !q || !qsz) return fail(MTL_E_INVALID, "mtl_w4_rtn_quantize: NULL pointer");
  if (!valid_group(group_size) || K % group_size || N < 1)
    return fail(MTL_E_INVALID, "mtl_w4_rtn_quantize: N=%d K=%d group_size=%d", N, K, group_size);
  cudaError_t e = mtl::launch_rtn_quantize(w, N, K, group_size, q, qsz, stream);
  return e == cudaSuccess ? MTL_OK : cuda_fail(e, "mtl_w4_rtn_quantize");
}

}  // extern "C"
