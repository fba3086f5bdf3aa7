// Shared device/host helpers for the tssm_b200 kernels (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>

#include "../../include/tssm.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tssm_b200 kernels target sm_100a (B200) only"
#endif

namespace tssm {

// ---------------------------------------------------------------- errors
// Host-side status reporting: the last error message is kept per host thread.
void set_error(const char* fmt, ...);
int check_launch(const char* what);
// Device address of this device's status word (0 = fine); kernels with bounded
// waits store a non-zero code there when a wait gives up.
int* device_status_ptr();
// Streaming multiprocessors of the current device (148 on B200; 1 if the query fails).
int num_sms();

#define TSSM_REQUIRE(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      ::tssm::set_error(__VA_ARGS__);           \
      return TSSM_ERR_INVALID;                  \
    }                                           \
  } while (0)

// ---------------------------------------------------------------- dtypes
template <typename T> struct io;
template <> struct io<float> {
  __device__ __forceinline__ static float ld(const float* p) { return *p; }
  __device__ __forceinline__ static void st(float* p, float v) { *p = v; }
};
template <> struct io<__nv_bfloat16> {
  __device__ __forceinline__ static float ld(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ __forceinline__ static void st(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct io<__half> {
  __device__ __forceinline__ static float ld(const __half* p) { return __half2float(*p); }
  __device__ __forceinline__ static void st(__half* p, float v) { *p = __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return io<T>::ld(p); }
// v rounded to T and back (what a T tensor holds after storing v).
template <typename T>
__device__ __forceinline__ float io_round(float v) {
  if constexpr (std::is_same<T, float>::value) return v;
  else { T t; io<T>::st(&t, v); return io<T>::ld(&t); }
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) { io<T>::st(p, v); }

// The reference's guarded exp(x)-1 (discretize_kernel.py:51-53 and :88).
// `e` is exp(x), already computed by the caller.
__device__ __forceinline__ float expm1_guard_f32(float x, float e) {
  return fabsf(x) > 1e-5f ? e - 1.0f : x * (1.0f + x * 0.5f);
}
__device__ __forceinline__ float expm1_guard_bf16(float x, float e) {
  return fabsf(x) > 1e-5f ? e - 1.0f : x + x * x * 0.5f;
}

// ZOH input coefficient (exp(x)-1)/(a+1e-12) with x = dt*a (discretize_kernel.py:50-54).
__device__ __forceinline__ float zoh_coeff(float x, float e, float a) {
  return expm1_guard_f32(x, e) / (a + 1e-12f);
}

// Streaming (evict-first) 128-bit accesses for data touched once.
__device__ __forceinline__ float4 ld_stream_f4(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream_f4(float4* p, float4 v) { __stcs(p, v); }

// Packed two-lane f32 arithmetic (one instruction, two IEEE-rounded results).
__device__ __forceinline__ unsigned long long f2_bits(float2 v) { return *reinterpret_cast<unsigned long long*>(&v); }
__device__ __forceinline__ float2 f2_from(unsigned long long r) { return *reinterpret_cast<float2*>(&r); }
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_from(r);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(r);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(r);
}

__host__ __device__ constexpr inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kNumSMs = 148;

}  // namespace tssm
