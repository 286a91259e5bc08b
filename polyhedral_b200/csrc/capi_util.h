// Host-side helpers shared by the C-ABI entry points: per-thread error message,
// argument checks that fail before any launch, and CUDA error translation.
#pragma once
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <cuda_runtime.h>
#include "polyattn.h"

namespace pa {

void set_error(const char* fmt, ...);
void clear_error();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(PA_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  return PA_OK;
}

#define PA_CHECK_ARG(cond, ...)                   \
  do {                                            \
    if (!(cond)) return ::pa::fail(PA_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define PA_CUDA(call, what)                                                      \
  do {                                                                           \
    cudaError_t _e = (call);                                                     \
    if (_e != cudaSuccess)                                                       \
      return ::pa::fail(PA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(_e));    \
  } while (0)

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

namespace attn {
// Status of the last attention forward on a workspace (device memory), read
// stream-ordered and synchronising `stream` (csrc/attn.cu).
int read_status(const void* ws, int32_t* status_host, cudaStream_t stream, const char* who);
}  // namespace attn

}  // namespace pa
