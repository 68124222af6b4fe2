// hokv_common.cuh -- shared device helpers and host error plumbing.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "hokv.h"
#include "hokv_math.cuh"

namespace hokv {

// ---- host-side error reporting -------------------------------------------
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);

#define HOKV_REQUIRE(cond, ...) \
  do { if (!(cond)) return ::hokv::fail(HOKV_ERR_INVALID, __VA_ARGS__); } while (0)

// ---- device-side status flag (first non-zero code wins) -------------------
// Defined here: the library is built as one translation unit (hokv_lib.cu).
__device__ int g_dev_status = 0;
__device__ __forceinline__ void dev_flag(int code) { atomicCAS(&g_dev_status, 0, code); }

// ---- loads ----------------------------------------------------------------
__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == HOKV_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  if (dtype == HOKV_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_from_f32(void* p, int dtype, int64_t i, float v) {
  if (dtype == HOKV_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else if (dtype == HOKV_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// 4 consecutive 16-bit storage values -> float4 (8-byte aligned load).
template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  uint2 r = *reinterpret_cast<const uint2*>(p);
  __half2 a = *reinterpret_cast<__half2*>(&r.x), b = *reinterpret_cast<__half2*>(&r.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 r = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&r.x), b = *reinterpret_cast<__nv_bfloat162*>(&r.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

// ---- phase stamps (profiling build only) ----------------------------------
// Built with -DHOKV_STAMPS, the decode kernels record %globaltimer at their
// phase boundaries (thread 0 of each CTA) into g_stamps[kernel][cta][phase]
// (kernel 0: candidate stage, 1: attention, 2: reserved);
// hokv_phase_stamps() copies them out.  The product build compiles no stamp.
constexpr int STAMP_CTAS = 4096;
constexpr int STAMP_N = 16;
#ifdef HOKV_STAMPS
__device__ unsigned long long g_stamps[3][STAMP_CTAS][STAMP_N];
__device__ __forceinline__ void stamp(int kernel, int cta, int phase) {
  if (threadIdx.x == 0 && cta < STAMP_CTAS) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)::"memory");
    g_stamps[kernel][cta][phase] = t;
  }
}
#else
__device__ __forceinline__ void stamp(int, int, int) {}
#endif

}  // namespace hokv
