// Shared host/device helpers of the li_b200 C ABI library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

#include "li_b200.h"

namespace li {

// Records `fmt` as this host thread's last error and returns `code`.
li_status fail(li_status code, const char* fmt, ...);
// LI_OK when `e` is cudaSuccess, else records the CUDA error string.
li_status cuda_status(cudaError_t e, const char* what);
// Checks the launch just issued (cudaGetLastError) and, when it was accepted,
// adds one to the process-wide count li_kernel_launches() reports.
li_status launched(const char* what);

inline int dtype_size(int dt) { return dt == LI_DTYPE_FP32 ? 4 : 2; }
inline bool valid_dtype(int dt) { return dt == LI_DTYPE_BF16 || dt == LI_DTYPE_FP16 || dt == LI_DTYPE_FP32; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// A 16-byte-vectorisable [.., D] view: D contiguous, every other stride a
// multiple of 16 bytes, base 16-byte aligned.
li_status check_vec_view(const void* data, const int64_t* stride, int rank, int dtype,
                         int64_t D, const char* name);

// Kernel attributes (the dynamic shared-memory limit) belong to one device's
// context. `done` holds one bit per device ordinal below 64 for one call site;
// `setup` runs on the current device until it has succeeded there once.
template <class F>
li_status once_per_device(std::atomic<uint64_t>& done, F&& setup) {
  int dev = 0;
  if (li_status st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t{1} << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return LI_OK;
  if (li_status st = setup()) return st;
  done.fetch_or(bit, std::memory_order_release);
  return LI_OK;
}

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

// Exact widening of a 16-bit float (bf16 / fp16 bits) or an fp32 to double,
// built from the bit fields with integer operations (no float-to-double
// conversion instruction). Zero, subnormal, infinite and NaN inputs take the
// conversion path.
__device__ __forceinline__ double bf16_bits_to_f64(uint32_t b) {
  const uint32_t e = (b >> 7) & 0xFFu;
  if (e - 1u < 0xFEu)
    return __longlong_as_double((long long)(((uint64_t)(b >> 15) << 63) | ((uint64_t)(e + 896u) << 52) |
                                            ((uint64_t)(b & 0x7Fu) << 45)));
  if ((b & 0x7FFFu) == 0u) return __longlong_as_double((long long)((uint64_t)(b >> 15) << 63));
  return (double)__uint_as_float(b << 16);
}
__device__ __forceinline__ double fp16_bits_to_f64(uint32_t h) {
  const uint32_t e = (h >> 10) & 0x1Fu;
  if (e - 1u < 0x1Eu)
    return __longlong_as_double((long long)(((uint64_t)(h >> 15) << 63) | ((uint64_t)(e + 1008u) << 52) |
                                            ((uint64_t)(h & 0x3FFu) << 42)));
  if ((h & 0x7FFFu) == 0u) return __longlong_as_double((long long)((uint64_t)(h >> 15) << 63));
  return (double)__half2float(__ushort_as_half((unsigned short)h));
}
__device__ __forceinline__ double fp32_bits_to_f64(uint32_t f) {
  const uint32_t e = (f >> 23) & 0xFFu;
  if (e - 1u < 0xFEu)
    return __longlong_as_double((long long)(((uint64_t)(f >> 31) << 63) | ((uint64_t)(e + 896u) << 52) |
                                            ((uint64_t)(f & 0x7FFFFFu) << 29)));
  if ((f & 0x7FFFFFFFu) == 0u) return __longlong_as_double((long long)((uint64_t)(f >> 31) << 63));
  return (double)__uint_as_float(f);
}
// Element `i` of a 16-byte chunk as double (exact).
__device__ __forceinline__ double chunk_elem_f64(const uint4& v, int i, int dt) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if (dt == LI_DTYPE_FP32) return fp32_bits_to_f64(w[i]);
  const uint32_t word = w[i >> 1];
  const uint32_t h = (i & 1) ? (word >> 16) : (word & 0xFFFFu);
  return dt == LI_DTYPE_BF16 ? bf16_bits_to_f64(h) : fp16_bits_to_f64(h);
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
