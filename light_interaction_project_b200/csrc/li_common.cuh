// Shared host/device helpers of the li_b200 C ABI library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "li_b200.h"

namespace li {

// Records `fmt` as this host thread's last error and returns `code`.
li_status fail(li_status code, const char* fmt, ...);
// LI_OK when `e` is cudaSuccess, else records the CUDA error string.
li_status cuda_status(cudaError_t e, const char* what);

inline int dtype_size(int dt) { return dt == LI_DTYPE_FP32 ? 4 : 2; }
inline bool valid_dtype(int dt) { return dt == LI_DTYPE_BF16 || dt == LI_DTYPE_FP16 || dt == LI_DTYPE_FP32; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// A 16-byte-vectorisable [.., D] view: D contiguous, every other stride a
// multiple of 16 bytes, base 16-byte aligned.
li_status check_vec_view(const void* data, const int64_t* stride, int rank, int dtype,
                         int64_t D, const char* name);

// ---------------------------------------------------------------------------
// Device-side rounding helpers (exact IEEE round-to-nearest-even).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float round_dt(float x, int dt) {
  if (dt == LI_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dt == LI_DTYPE_FP16) return __half2float(__float2half_rn(x));
  return x;
}

// Element `i` of a 16-byte chunk as float (exact widening).
__device__ __forceinline__ float chunk_elem(const uint4& v, int i, int dt) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if (dt == LI_DTYPE_FP32) return __uint_as_float(w[i]);
  uint32_t word = w[i >> 1];
  uint16_t h = (i & 1) ? (uint16_t)(word >> 16) : (uint16_t)(word & 0xFFFF);
  if (dt == LI_DTYPE_BF16) return __uint_as_float(((uint32_t)h) << 16);
  return __half2float(__ushort_as_half(h));
}

// Store a dtype-representable float as the dtype at p.
__device__ __forceinline__ void store_dt(void* p, int64_t i, float x, int dt) {
  if (dt == LI_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else if (dt == LI_DTYPE_FP16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
  else reinterpret_cast<float*>(p)[i] = x;
}

__device__ __forceinline__ float load_dt(const void* p, int64_t i, int dt) {
  if (dt == LI_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == LI_DTYPE_FP16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

}  // namespace li
