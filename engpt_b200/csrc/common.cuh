// Shared helpers for the engpt_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/engpt_b200.h"

namespace engpt {

// ---------------------------------------------------------------- host errors
int set_error(int code, const char* fmt, ...);
void clear_error();
int check_launch(const char* what);
// Mean of row_loss over the rows whose target is not -100 (F.cross_entropy's reduction) into loss_out[0].
int launch_mean_loss(const float* row_loss, const int64_t* targets, int64_t rows, float* loss_out, cudaStream_t st);

#define ENGPT_REQUIRE(cond, code, ...)            \
  do {                                            \
    if (!(cond)) return ::engpt::set_error((code), __VA_ARGS__); \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// --------------------------------------------------------- device status word
// First failure recorded by any kernel of this library on this device.
// Bits 0..7: engpt_status code; bits 8..31: site id of the failing wait.
extern __device__ int g_device_status;

__device__ __forceinline__ void record_device_error(int code, int site) {
  atomicCAS(&g_device_status, 0, (code & 0xff) | (site << 8));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded waits give up after this long and record ENGPT_ERR_TIMEOUT.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ------------------------------------------------------------------ numerics
__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

struct alignas(16) bf16x8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const uint4& raw, float* out) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    out[2 * i] = f.x;
    out[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* in) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(in[2 * i], in[2 * i + 1]);
  return raw;
}

// Streaming (read-once) 16-byte load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// 16-byte load through the coherent path (for buffers the same kernel also writes), not kept in L1.
__device__ __forceinline__ uint4 ld_once(const void* p) {
  uint4 r;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

template <int N>
__device__ __forceinline__ float warp_sum_xor(float v) {
#pragma unroll
  for (int o = N / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Number of SMs of the current device (cached per device).
int num_sms();

}  // namespace engpt
