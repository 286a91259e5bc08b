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
// pa_attn_noalloc_status reads the device status the last call left in the array.
#include <cuda.h>
#include <mutex>
#include "capi_util.h"
#include "common.cuh"

namespace pa {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_attn_scratch[kNoAllocScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of g_attn_scratch, per device and per CUDA context: the host-side
// name is only a stand-in for the symbol, and a context created after a device
// reset loads the module afresh, possibly at another address.
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

int scratch_for_current_device(void** out, const char* who) {
  int dev = 0;
  PA_CUDA(cudaGetDevice(&dev), who);
  if (dev < 0 || dev >= kMaxDevices)
    return fail(PA_ERR_UNSUPPORTED, "%s: device %d beyond %d", who, dev, kMaxDevices);
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return fail(PA_ERR_CUDA, "%s: cuCtxGetCurrent unavailable", who);
  CUcontext ctx = nullptr;   // NULL until the runtime binds a context to this thread
  if (get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (ctx && g_scratch_ptr[dev] && g_scratch_ctx[dev] == ctx) {
    *out = g_scratch_ptr[dev];
    return PA_OK;
  }
  // the lookup binds the device's primary context to this thread if none was
  void* p = nullptr;
  PA_CUDA(cudaGetSymbolAddress(&p, g_attn_scratch), who);
  if (get(&ctx) != CUDA_SUCCESS || !ctx)
    return fail(PA_ERR_CUDA, "%s: no current CUDA context after the symbol lookup", who);
  g_scratch_ptr[dev] = p;
  g_scratch_ctx[dev] = ctx;
  *out = p;
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
  int rc = scratch_for_current_device(&ws, "pa_attn_fwd_noalloc");
  if (rc) return rc;
  rc = pa_attn_plan(args, ws, kNoAllocScratchBytes, stream);
  if (rc) return rc;
  return pa_attn_fwd(args, ws, kNoAllocScratchBytes, stream);
}

extern "C" int pa_attn_noalloc_status(int32_t* status_host, pa_stream_t stream) {
  using namespace pa;
  PA_CHECK_ARG(status_host != nullptr, "pa_attn_noalloc_status: null status_host");
  void* ws = nullptr;
  int rc = scratch_for_current_device(&ws, "pa_attn_noalloc_status");
  if (rc) return rc;
  return attn::read_status(ws, status_host, (cudaStream_t)stream, "pa_attn_noalloc_status");
}
