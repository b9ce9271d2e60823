// Shared device/host helpers for libpcb200: dtypes, the device error word,
// bounded mbarrier waits and the fp8 conversions used by every kernel.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pcb200.h"

namespace pcb {

// ----------------------------------------------------------------------------
// Device error word: {code, site, info}.  The first failure sticks (CAS on
// code); pcb_get_device_error() reads and clears it.
// ----------------------------------------------------------------------------
__device__ unsigned int g_device_error[3];

enum ErrorSite : int {
  SITE_GEMM_PRODUCER = 1,
  SITE_GEMM_MMA = 2,
  SITE_GEMM_EPILOGUE = 3,
  SITE_GEMM_INJECTED = 4,
  SITE_FUSED_PRODUCER = 5,
  SITE_FUSED_MMA = 6,
  SITE_FUSED_EPILOGUE = 7,
  SITE_QUANT_TILE = 8,
};

__device__ __forceinline__ void report_error(int code, int site) {
  if (atomicCAS(&g_device_error[0], 0u, (unsigned)code) == 0u) {
    g_device_error[1] = (unsigned)site;
    g_device_error[2] = blockIdx.x;
  }
}

// A bounded wait gives up after kWaitLimitNs of wall time (read from
// %globaltimer every 64 polls), far above any legitimate wait in these kernels.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------------------
// Shared-memory / mbarrier primitives (inline PTX, sm_90+/sm_100).
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait that polls with the non-blocking test_wait (no suspend): used
// where the arrival comes from the other CTA of a pair.
__device__ __forceinline__ bool mbar_spin_bounded(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
  }
  report_error(PCB_ERR_TIMEOUT, site);
  *abort_flag = 1;
  return false;
}

// Warp-collective form of mbar_spin_bounded: every lane of the warp polls and
// the loop exits on a vote, so the result and the control flow stay uniform
// across the warp.
__device__ __forceinline__ bool mbar_spin_bounded_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                       int site) {
  if (__all_sync(0xffffffffu, mbar_test_wait(bar, parity))) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (__all_sync(0xffffffffu, mbar_test_wait(bar, parity))) return true;
    if ((i & 255u) == 0u) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) return false;
      if (__any_sync(0xffffffffu, global_timer_ns() - t0 > kWaitLimitNs)) break;
    }
  }
  if ((threadIdx.x & 31) == 0) report_error(PCB_ERR_TIMEOUT, site);
  *abort_flag = 1;
  return false;
}

// Bounded wait on phase `parity` of an mbarrier.  Returns false (after
// recording an error and raising the CTA abort flag) when the wait runs out
// or when another warp of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
  }
  report_error(PCB_ERR_TIMEOUT, site);
  *abort_flag = 1;
  return false;
}

// ----------------------------------------------------------------------------
// Conversions.
// ----------------------------------------------------------------------------
template <int DT>
struct InType;
template <>
struct InType<PCB_DTYPE_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f32(T v) { return v; }
};
template <>
struct InType<PCB_DTYPE_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f32(T v) { return __half2float(v); }
};
template <>
struct InType<PCB_DTYPE_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f32(T v) { return __bfloat162float(v); }
};

// Two fp32 values -> two saturated fp8 bytes (RNE, |v| > max -> +-max, NaN -> NaN),
// element 0 in the low byte.  Equals clamp(v, -max, max) followed by an RNE cast.
template <int YT>
__device__ __forceinline__ uint16_t cvt2_fp8(float v0, float v1) {
  const __nv_fp8_interpretation_t kind = (YT == PCB_DTYPE_E4M3) ? __NV_E4M3 : __NV_E5M2;
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(v0, v1), __NV_SATFINITE, kind);
}

template <int YT>
__device__ __forceinline__ uint8_t cvt1_fp8(float v) {
  const __nv_fp8_interpretation_t kind = (YT == PCB_DTYPE_E4M3) ? __NV_E4M3 : __NV_E5M2;
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, kind);
}

template <int YT>
struct Fp8Max;
template <>
struct Fp8Max<PCB_DTYPE_E4M3> {
  static constexpr float value = 448.0f;
};
template <>
struct Fp8Max<PCB_DTYPE_E5M2> {
  static constexpr float value = 57344.0f;
};

// |x| as ordered bits: for non-negative floats the unsigned order is the float
// order, and any NaN compares above +inf, so max() over these propagates NaN
// like torch.amax does.
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7fffffffu; }

// torch's `fp8_max / amax` (python scalar / tensor) is reciprocal(amax) * fp8_max.
__device__ __forceinline__ float quant_scale_from_amax(float safe_amax, float fp8_max) {
  return __fmul_rn(__frcp_rn(safe_amax), fp8_max);
}

// Power-of-two (E8M0) quantization scale: 2^-e with e the smallest integer
// such that 2^e >= RN(safe_amax / fp8_max), so the dequant scale 2^e is exact
// in an 8-bit exponent.  A zero or subnormal ratio r (eps = 0 and an all-zero
// or tiny tile) is clamped up to the smallest normal power of two, 2^-126, so
// its scale is still an E8M0 value; a non-finite r (inf / NaN input) gives
// 1/r (0 or NaN), whose dequant scale (inf / NaN) packs to the E8M0 NaN byte.
__device__ __forceinline__ float pow2_quant_scale(float safe_amax, float fp8_max) {
  const float r = __fdiv_rn(safe_amax, fp8_max);
  const uint32_t bits = __float_as_uint(r);
  const int ef = (int)((bits >> 23) & 0xffu);
  if (ef == 0xff) return __frcp_rn(r);
  if (ef == 0) return __uint_as_float((uint32_t)(127 + 126) << 23);  // 2^126
  const int e = ef - 127 + ((bits & 0x7fffffu) != 0u ? 1 : 0);
  return __uint_as_float((uint32_t)(127 - e) << 23);
}

// amax.clamp_min(eps), keeping NaN.
__device__ __forceinline__ float clamp_min_eps(float amax, float eps) {
  return (amax < eps) ? eps : amax;
}

}  // namespace pcb
