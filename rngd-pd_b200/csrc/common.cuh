// Shared helpers for the rngd-pd B200 kernels: status codes, last-error text,
// bf16 bit helpers and bounded-wait constants.  Every extern "C" entry point
// returns an int status (0 ok, negative on failure) and records a message that
// rngd_last_error() hands back, mirroring the reference's "no silent fallback"
// rule (src/rngd_pd/connector/transport.py:330-338).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <stdio.h>

#include "../../include/rngd_b200.h"

// Per-CTA %globaltimer stamps in the decode and prefill GEMMs (rngd_tc_gemv_trace,
// rngd_trace_decode_gemms) are diagnostics: compiled in only by `make TRACE=1`.  In the product
// build the stamps fold away and those two entries return RNGD_ERR_UNSUPPORTED for a non-NULL buffer.
#ifndef RNGD_TRACE
#define RNGD_TRACE 0
#endif

namespace rngd {

void set_error(const char* fmt, ...);
unsigned long long* gemm_trace();      // the buffer set by rngd_tc_gemv_trace (null unless tracing)
unsigned long long* next_seq_trace();  // next block of rngd_trace_decode_gemms' sequence, or null

// Returns RNGD_ERR_CUDA and records the message when a launch or call failed.
inline int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RNGD_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return RNGD_ERR_CUDA;
}
inline int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

#define RNGD_REQUIRE(cond, ...)          \
  do {                                   \
    if (!(cond)) {                       \
      ::rngd::set_error(__VA_ARGS__);    \
      return RNGD_ERR_ARG;               \
    }                                    \
  } while (0)

#define RNGD_TRY(expr)          \
  do {                          \
    int _st = (expr);           \
    if (_st != RNGD_OK) return _st; \
  } while (0)

// Raise a kernel's dynamic shared-memory limit on the current device once.  The
// attribute belongs to (kernel, device), so `mask` keeps one bit per device ordinal;
// a process driving several GPUs sets it on each before its first launch there.
inline int set_smem_limit_once(const void* func, int bytes, std::atomic<unsigned long long>* mask,
                               const char* what) {
  int dev = 0;
  RNGD_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  const unsigned long long bit = 1ull << (dev & 63);
  if (mask->load(std::memory_order_acquire) & bit) return RNGD_OK;
  RNGD_TRY(check_cuda(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what));
  mask->fetch_or(bit, std::memory_order_acq_rel);
  return RNGD_OK;
}

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }

// Round-to-nearest-even fp32 -> bf16 bits (finite inputs).  The host uses the same
// integer rule as the oracle; the device uses the hardware RNE convert, which gives
// the same bits for every finite input, so host and device roundings agree.
__host__ __device__ __forceinline__ uint16_t f2bf_bits(float f) {
#ifdef __CUDA_ARCH__
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
  return r;
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
#endif
}

// 8 bf16 (one 16-byte vector) -> 8 fp32
__device__ __forceinline__ void unpack8(const uint4 v, float* f) {
  f[0] = bf_lo(v.x); f[1] = bf_hi(v.x);
  f[2] = bf_lo(v.y); f[3] = bf_hi(v.y);
  f[4] = bf_lo(v.z); f[5] = bf_hi(v.z);
  f[6] = bf_lo(v.w); f[7] = bf_hi(v.w);
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
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

constexpr int kNumSMs = 148;

}  // namespace rngd
