// Last-error bookkeeping and the synthetic-input generators.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace rngd {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// splitmix64 finaliser, the hash of the synthetic-input recipe (see rngd_b200.h)
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_gauss_kernel(uint16_t* __restrict__ dst, uint64_t n, uint64_t key, uint64_t start,
                                   float scale) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t h = mix64(key + start + i);
    int64_t s = (int64_t)((h & 0xFFFF) + ((h >> 16) & 0xFFFF) + ((h >> 32) & 0xFFFF) + (h >> 48)) - 131070;
    // __fmul_rn: no contraction, correctly rounded like the host's fp32 multiply
    dst[i] = f2bf_bits(__fmul_rn((float)s, scale));
  }
}

__global__ void synth_uniform_kernel(int32_t* __restrict__ dst, uint64_t n, uint64_t key, uint64_t start,
                                     uint32_t hi) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = (int32_t)((mix64(key + start + i) >> 32) % hi);
}

}  // namespace rngd

using namespace rngd;

extern "C" int rngd_last_error(char* buf, size_t n) {
  if (!buf || n == 0) return RNGD_ERR_ARG;
  strncpy(buf, g_err, n - 1);
  buf[n - 1] = 0;
  return RNGD_OK;
}

extern "C" int rngd_abi_version(void) { return 5; }

extern "C" int rngd_synth_gauss_bf16(void* dst, uint64_t n, uint64_t seed, uint64_t tid, uint64_t start,
                                     float scale, rngd_stream_t stream) {
  RNGD_REQUIRE(dst != nullptr || n == 0, "synth_gauss: null destination");
  if (n == 0) return RNGD_OK;
  uint64_t key = mix64(mix64(seed) ^ tid);
  int blocks = (int)((n + 255) / 256 < 148 * 64 ? (n + 255) / 256 : 148 * 64);
  synth_gauss_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((uint16_t*)dst, n, key, start, scale);
  return check_launch("synth_gauss_kernel");
}

extern "C" int rngd_synth_uniform_i32(int32_t* dst, uint64_t n, uint64_t seed, uint64_t tid, uint64_t start,
                                      uint32_t hi, rngd_stream_t stream) {
  RNGD_REQUIRE(dst != nullptr || n == 0, "synth_uniform: null destination");
  RNGD_REQUIRE(hi > 0, "synth_uniform: hi must be positive");
  if (n == 0) return RNGD_OK;
  uint64_t key = mix64(mix64(seed) ^ tid);
  int blocks = (int)((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
  synth_uniform_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(dst, n, key, start, hi);
  return check_launch("synth_uniform_kernel");
}
