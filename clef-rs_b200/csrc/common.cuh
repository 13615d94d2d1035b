// common.cuh — shared helpers of libclef_b200: status handling, BF16
// conversion, bounded mbarrier waits and the device error flag.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/clef_b200.h"

namespace clef {

// Last error message of the calling host thread (clef_last_error()).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define CLEF_CUDA(call)                                                                  \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return ::clef::fail(CLEF_ERR_CUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
  } while (0)

#define CLEF_CHECK(cond, code, msg)                 \
  do {                                              \
    if (!(cond)) return ::clef::fail((code), (msg)); \
  } while (0)

// Launch status of the most recent kernel on this thread.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CLEF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return CLEF_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// Device error flag. Kernels that wait on a barrier give up after a bounded
// time, record a nonzero code in their translation unit's flag and return;
// the host reads the flags after the work it issued has completed
// (clef::device_errors()).
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kDevOk = 0,
  kDevGemmTimeout = 1,
  kDevAttentionTimeout = 2,
  kDevScanTimeout = 3,
  kDevProbeTimeout = 4,
};
static __device__ int g_device_error = 0;  // one flag per translation unit

__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// Reads and clears this translation unit's flag on the current device.
static inline int read_device_error(int* code) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return CLEF_ERR_CUDA;
  if (v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return CLEF_ERR_CUDA;
  }
  *code = v;
  return CLEF_OK;
}
// Synchronises the current device and collects every kernel family's flag.
int device_errors(int* code);
int gemm_device_error(int* code);
int attention_tc_device_error(int* code);
int scan_device_error(int* code);

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// BF16 helpers (round to nearest even, as __float2bfloat16_rn).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ uint16_t f2bf(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&b);
}
__device__ __forceinline__ float bf2f(uint16_t u) {
  return __uint_as_float(((uint32_t)u) << 16);
}
// Two round-to-nearest-even BF16 conversions in one instruction; `lo` lands
// in the low half (lower address).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Split BF16 pair of two floats: hi = bf16(x), lo = bf16(x - hi) (x - hi is
// exact in F32), so hi + lo carries x to about 2^-17 relative.
__device__ __forceinline__ uint32_t split_lo_bf16x2(float a, float b, uint32_t hi) {
  return pack_bf16x2(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
}

// Candle's CPU definitions: sigmoid = 1 / (1 + exp(-x)), silu = x / (1 + exp(-x)).
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x / (1.f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int num_sms(int device);
// CTAs a persistent kernel (one CTA per SM) launched from this host thread may
// use: all SMs, or fewer while a cap is set for the thread (an engine that
// shares the GPU with another stream's work sets one around its prefill).
int persistent_ctas(int device);
void set_persistent_cap(int ctas);  // 0 = no cap

}  // namespace clef
