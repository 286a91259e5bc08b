// pa_attn_fwd_noalloc: the block-sparse attention forward for callers that cannot
// allocate device memory.
//
// Some callers of this library may not call cudaMalloc at all: code running
// inside another framework's memory pool or a fixed-budget serving process, code
// that must not allocate between warm-up and steady state, or a host language
// binding with no device allocator of its own.  pa_attn_fwd needs a workspace for
// its work list (pa_attn_workspace_size bytes); this entry point takes that
// workspace from a fixed array compiled into the library instead, so the caller
// passes only inputs and outputs.
//
// The array is kNoAllocScratchBytes (4 MiB) of device memory that every GPU which
// loads the library keeps until the process exits.  Requests whose workspace
// would exceed it are rejected with PA_ERR_ARG (about N <= 36096 at A = 16,
// 51200 at A = 32, larger for wider tiles).  All calls share the one array and each call rebuilds
// everything in it that the kernels read, so nothing carries over between calls;
// two calls whose work overlaps on the GPU (different streams, or several host
// threads without ordering) race on the array and must not be issued.
#include <mutex>
#include "capi_util.h"
#include "common.cuh"

namespace pa {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_attn_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device, looked up once per
// device (the host-side name is only a stand-in for the symbol).
int scratch_for_current_device(void** out) {
  int dev = 0;
  PA_CUDA(cudaGetDevice(&dev), "pa_attn_fwd_noalloc");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(PA_ERR_UNSUPPORTED, "pa_attn_fwd_noalloc: device %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    PA_CUDA(cudaGetSymbolAddress(&p, g_attn_scratch), "pa_attn_fwd_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return PA_OK;
}

}  // namespace
}  // namespace pa

extern "C" int pa_attn_fwd_noalloc(const pa_attn_args* args, pa_stream_t stream) {
  using namespace pa;
  PA_CHECK_ARG(args != nullptr, "pa_attn_fwd_noalloc: null args");
  const size_t need = pa_attn_workspace_size(args);
  PA_CHECK_ARG(need > 0, "pa_attn_fwd_noalloc: invalid N=%d / A=%d", args->N, args->A);
  if (need > kNoAllocScratchBytes)
    return fail(PA_ERR_ARG,
                "pa_attn_fwd_noalloc: work list needs %zu bytes, more than the %zu-byte static "
                "scratch (N=%d, A=%d); use pa_attn_plan/pa_attn_fwd with a caller workspace",
                need, kNoAllocScratchBytes, args->N, args->A);
  void* ws = nullptr;
  int rc = scratch_for_current_device(&ws);
  if (rc) return rc;
  rc = pa_attn_plan(args, ws, kNoAllocScratchBytes, stream);
  if (rc) return rc;
  return pa_attn_fwd(args, ws, kNoAllocScratchBytes, stream);
}
