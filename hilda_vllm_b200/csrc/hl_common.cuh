// Shared helpers for the sm_100a kernels: error reporting, mbarrier + bulk-copy PTX,
// element conversions.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "hilda_b200.h"

namespace hl {

// ---------------------------------------------------------------- host-side errors
void set_error(const char* fmt, ...);
void clear_error();

#define HL_CHECK_ARG(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      ::hl::set_error(__VA_ARGS__);             \
      return HL_ERR_INVALID;                    \
    }                                           \
  } while (0)

#define HL_CHECK_LAUNCH(name)                                                   \
  do {                                                                          \
    cudaError_t _e = cudaGetLastError();                                        \
    if (_e != cudaSuccess) {                                                    \
      ::hl::set_error("%s: launch failed: %s", name, cudaGetErrorString(_e));   \
      return HL_ERR_CUDA;                                                       \
    }                                                                           \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- device helpers
// Bounded waits: every spin on an mbarrier gives up after this many polls (each poll
// suspends the thread for up to the hardware time limit), records an error bit and lets
// the kernel return instead of hanging the GPU.
constexpr uint32_t kMaxWaitPolls = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Returns true once the phase with the given parity has completed; false after
// kMaxWaitPolls unsuccessful polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxWaitPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 1-D bulk copy global -> shared (TMA engine), completion signalled on `bar` as tx bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_evict_first(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                     uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bf16 pair (packed in a u32, low element first) -> two floats.  Exact.
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Two e4m3 values (low byte first) -> two floats.  Exact (every e4m3 value is an f16 value).
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(v), __NV_E4M3);
  __half2 hh = *reinterpret_cast<__half2*>(&h);
  return __half22float2(hh);
}

// float -> e4m3 with round-to-nearest-even and saturation to +-448 (NaN stays NaN).
__device__ __forceinline__ uint8_t float_to_e4m3_sat(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// 8 bf16 (one 16-byte vector) -> 8 e4m3 bytes (one 8-byte store), all divided by `scale`.
// IEEE division (not a reciprocal multiply) so the bytes match x / scale exactly.
__device__ __forceinline__ uint2 quant8_e4m3(uint4 v, float scale) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t out[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t qa = float_to_e4m3_sat(__fdiv_rn(bf16lo(w[i]), scale));
    const uint32_t qb = float_to_e4m3_sat(__fdiv_rn(bf16hi(w[i]), scale));
    out[i >> 1] |= (qa | (qb << 8)) << ((i & 1) * 16);
  }
  return make_uint2(out[0], out[1]);
}

}  // namespace hl
