// Shared host/device helpers of the flash_attn_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "flash_attn_b200.h"

namespace fab {

// ---------------------------------------------------------------- host errors
std::string& last_error();
int fail(int code, const char* fmt, ...);

#define FAB_CHECK_ARG(cond, ...)                                    \
  do {                                                              \
    if (!(cond)) return ::fab::fail(FA_ERR_INVALID, __VA_ARGS__);   \
  } while (0)

#define FAB_LAUNCH_CHECK(what)                                                   \
  do {                                                                           \
    cudaError_t e_ = cudaGetLastError();                                         \
    if (e_ != cudaSuccess)                                                       \
      return ::fab::fail(FA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e_));   \
  } while (0)

inline bool present(const fa_tensor* t) { return t != nullptr && t->ptr != nullptr; }
inline bool present(const fa_tensor& t) { return t.ptr != nullptr; }
inline bool is_float(int dt) { return dt == FA_F16 || dt == FA_BF16 || dt == FA_F32; }
inline int elem_size(int dt) {
  switch (dt) {
    case FA_F16: case FA_BF16: return 2;
    case FA_F32: case FA_I32: return 4;
    case FA_I64: return 8;
    case FA_E4M3: case FA_BOOL: case FA_U8: return 1;
    default: return 0;
  }
}
int sm_count();  // cached per device

// --------------------------------------------------------------- device side
// Generic element load (any supported float storage -> float). FP8 E4M3FN
// decoding follows the format definition: exponent field 0 is subnormal with
// step 2^-9, bytes 0x7F/0xFF are NaN.
__device__ __forceinline__ float e4m3_to_float(uint8_t bits) {
  const uint32_t e = (bits >> 3) & 15u, m = bits & 7u;
  float x;
  if (e == 0) {
    x = (float)m * 0.001953125f;
  } else {
    x = __uint_as_float(((e + 120u) << 23) | (m << 20));
  }
  if (e == 15 && m == 7) x = __uint_as_float(0x7fc00000u);
  return (bits & 128u) ? -x : x;
}

__device__ __forceinline__ float load_float(const void* p, int dtype, int64_t off) {
  switch (dtype) {
    case FA_F16: return __half2float(reinterpret_cast<const __half*>(p)[off]);
    case FA_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off]);
    case FA_F32: return reinterpret_cast<const float*>(p)[off];
    case FA_E4M3: return e4m3_to_float(reinterpret_cast<const uint8_t*>(p)[off]);
    default: return 0.f;
  }
}

__device__ __forceinline__ void store_float(void* p, int dtype, int64_t off, float v) {
  switch (dtype) {
    case FA_F16: reinterpret_cast<__half*>(p)[off] = __float2half_rn(v); break;
    case FA_BF16: reinterpret_cast<__nv_bfloat16*>(p)[off] = __float2bfloat16_rn(v); break;
    case FA_F32: reinterpret_cast<float*>(p)[off] = v; break;
    default: break;
  }
}

__device__ __forceinline__ int64_t load_index(const void* p, int dtype, int64_t off) {
  return dtype == FA_I64 ? reinterpret_cast<const int64_t*>(p)[off]
                         : (int64_t) reinterpret_cast<const int32_t*>(p)[off];
}

// Saturating round-to-nearest-even float -> E4M3FN code: |x| beyond 448
// (inf included) saturates to 0x7E with the sign of x, NaN keeps its sign
// with payload 0x7F. The conversion itself is the sm_89+ hardware
// cvt.rn.satfinite.e4m3x2.f32 instruction.
__device__ __forceinline__ uint8_t float_to_e4m3_sat(float v) {
  if (isnan(v)) return (uint8_t)(((__float_as_uint(v) >> 24) & 128u) | 127u);
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Host-side count of kernel launches issued by the library; every launch
// site calls this right after its <<<...>>> (defined in attention.cu).
void note_launch();

}  // namespace fab
