// Library-level entry points (version, last error) and host helpers.
#include <cstdarg>
#include <cstdio>
#include <string>

#include "li_common.cuh"

namespace {
thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
}

namespace li {

li_status fail(li_status code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

li_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return LI_OK;
  return fail(LI_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

li_status launched(const char* what) {
  if (li_status st = cuda_status(cudaGetLastError(), what)) return st;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return LI_OK;
}

li_status check_vec_view(const void* data, const int64_t* stride, int rank, int dtype,
                         int64_t D, const char* name) {
  if (!data) return fail(LI_ERR_INVALID_ARG, "%s: null data pointer", name);
  if (!valid_dtype(dtype)) return fail(LI_ERR_INVALID_ARG, "%s: unknown dtype %d", name, dtype);
  const int es = dtype_size(dtype);
  if (stride[rank - 1] != 1) return fail(LI_ERR_STRIDE, "%s: head dim must be contiguous", name);
  if ((D * es) % 16) return fail(LI_ERR_SHAPE, "%s: D*elem_size must be a multiple of 16", name);
  for (int i = 0; i < rank - 1; ++i)
    if ((stride[i] * es) % 16)
      return fail(LI_ERR_ALIGNMENT, "%s: stride %d (%lld elements) is not a multiple of 16 bytes",
                  name, i, (long long)stride[i]);
  if (!aligned16(data)) return fail(LI_ERR_ALIGNMENT, "%s: base pointer not 16-byte aligned", name);
  return LI_OK;
}

}  // namespace li

extern "C" const char* li_version(void) { return "li_b200 0.1.0 (sm_100a)"; }

extern "C" const char* li_last_error(void) { return g_last_error.c_str(); }

extern "C" uint64_t li_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }
