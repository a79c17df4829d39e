// Shared device helpers for the moss-tts-lite B200 kernels (sm_100a only).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "moss_tts_lite_b200 kernels are written for sm_100a (B200) only"
#endif

namespace mtl {

// ---------------------------------------------------------------- status ---
// Device-side error word. Kernels never trap: a bounded wait that gives up,
// or an index that fails a check, ORs a code in here and the kernel returns.
// The host reads it with mtl_device_status().
enum DeviceError : uint32_t {
  kDevOk = 0,
  kDevWaitTimeout = 1u << 0,      // an mbarrier wait exceeded its spin bound
  kDevBadIndex = 1u << 1,         // an id / position failed its bound check
  kDevCopyDrainTimeout = 1u << 2  // in-flight bulk copies did not land at exit
};
// Defined here: the library is built as one translation unit (mtl_all.cu).
__device__ uint32_t g_device_status = 0;

__device__ __forceinline__ void flag_error(uint32_t code) { atomicOr(&g_device_status, code); }

// Every wait in these kernels is bounded in wall time (%globaltimer, ns):
// a wait that has not completed after kWaitNs flags the device status and
// returns false instead of spinning forever.
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------ bf16 / f32 ---
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }
// Two floats rounded to bf16 (nearest even) by one packed conversion: lo in
// bits 0-15, hi in bits 16-31.
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&r);
}

// --------------------------------------------------------------- mbarrier ---
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait until `deadline` (globaltimer ns); false on timeout.
__device__ __forceinline__ bool mbar_wait_until(uint64_t* bar, uint32_t parity, uint64_t deadline) {
  if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 0 && globaltimer_ns() > deadline) return false;
  }
}
// Bounded wait of at most kWaitNs; flags the device status on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  if (mbar_wait_until(bar, parity, globaltimer_ns() + kWaitNs)) return true;
  flag_error(kDevWaitTimeout);
  return false;
}

// 1-D bulk copy global -> shared completing on an mbarrier (no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Programmatic dependent launch: wait for the upstream grid's memory to be
// visible (no-op when the launch was not programmatic), and allow the
// downstream grid to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ int4 unpack ---
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

// bf16x2 fused multiply-add, one rounding per half (fma.rn.bf16x2).
__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Reference-format dequantisation of two codes, as torch's int4 GEMM
// (_weight_int4pack_mm, called at moss_tts_lite/fast.py:118) forms its
// operand: w = bf16((q - 8) * scale + zero), one rounding.  `biased` is the
// bf16 pair (128 + q_lo, 128 + q_hi) from lop3_and_or(..., 0x43004300);
// 128 + q - 136 = q - 8 is exact in bf16, then one bf16 FMA with the
// column's (scale, scale) and (zero, zero) pairs.
__device__ __forceinline__ uint32_t w4_ref_pair(uint32_t biased, uint32_t scale2, uint32_t zero2) {
  const uint32_t q8 = bf16x2_fma(biased, 0x3F803F80u, 0xC308C308u);  // * 1.0 + (-136)
  return bf16x2_fma(q8, scale2, zero2);
}

// m16n8k16 fp16 MMA with fp32 accumulate (register-sourced operands).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace mtl
