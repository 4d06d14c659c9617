// Status plumbing for the C ABI: thread-local last-error message and launch checks.
#pragma once
#include <cstdarg>
#include <cstdio>
#include <string>
#include <cuda_runtime.h>
#include "../../include/b3r.h"

namespace b3r {

std::string& last_error_ref();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error_ref() = buf;
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B3R_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return B3R_OK;
}

inline int check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(B3R_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return B3R_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  return (int)(g < 1 ? 1 : g);
}

#define B3R_TRY(expr)              \
  do {                             \
    int _rc = (expr);              \
    if (_rc != B3R_OK) return _rc; \
  } while (0)

#define B3R_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) return ::b3r::fail(B3R_E_INVALID, __VA_ARGS__); \
  } while (0)

}  // namespace b3r
