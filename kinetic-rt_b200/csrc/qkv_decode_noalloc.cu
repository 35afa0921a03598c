// Decode entry point for callers that cannot allocate device memory.
//
// krt_qkv_rope_decode needs a workspace (status word, normalised activations,
// per-token slots) that the caller allocates.  Some callers have no way to do
// that: a plugin whose host application owns every device allocation through
// its own arena and rejects outside cudaMalloc calls, or a serving loop that
// must not allocate after start-up because allocation can block, fragment
// memory or break its memory accounting.  They can still hand over the
// inputs and outputs.  krt_qkv_rope_decode_noalloc serves them: it runs the
// same decode kernels with the workspace placed in a fixed array of this
// library's own device memory.
//
// The array is a file-scope static __device__ object of 4 MiB.  Every GPU on
// which the library is loaded reserves it until the process exits.  Host
// code only sees a host-side stand-in for its name, so the device address is
// looked up once per device (cudaGetSymbolAddress, with that device current)
// the first time the entry point runs there, and cached.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/krt.h"
#include "capi_internal.h"
#include "qkv_paged.cuh"

namespace krt {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

// Identity of the current CUDA context (cuCtxGetId), or 0 when the driver
// cannot tell.  A device reset destroys the primary context and the module
// with it; the next context gets a new id, so a cached array address is
// looked up again instead of pointing into freed memory.
unsigned long long current_context_id() {
  typedef CUresult (*GetCurrentFn)(CUcontext*);
  typedef CUresult (*GetIdFn)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

std::mutex g_scratch_mu;
void* g_scratch_addr[kNoAllocMaxDevices] = {};
unsigned long long g_scratch_ctx[kNoAllocMaxDevices] = {};

// Device address of g_decode_scratch on the current device: looked up with
// cudaGetSymbolAddress the first time per device (and again after the
// device's context was replaced), then cached.
int scratch_for_current_device(const char* name, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, name);
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: device %d beyond %d", name, dev, kNoAllocMaxDevices);
  const unsigned long long ctx = current_context_id();  // 0 until the runtime bound a context here
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr || ctx == 0 || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);  // binds the device's primary context
    if (e != cudaSuccess) return cuda_error(e, name);
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = current_context_id();
  }
  *out = g_scratch_addr[dev];
  return KRT_OK;
}

}  // namespace
}  // namespace krt

using namespace krt;

extern "C" int krt_qkv_rope_decode_noalloc(const krt_qkv_paged_args* args, void* stream) {
  const char* name = "krt_qkv_rope_decode_noalloc";
  // Every argument check comes first: a rejected call touches neither the
  // GPU nor the shared array.
  int rc = decode_args_check(args, name);
  if (rc) return rc;
  const size_t need = krt_qkv_rope_decode_workspace_size(args->num_tokens, args->d_model, args->n_heads,
                                                         args->n_kv_heads, args->head_dim);
  if (need == 0 || need > kNoAllocScratchBytes)
    return set_error(KRT_ERR_UNSUPPORTED,
                     "%s: this call needs %zu bytes of scratch (num_tokens %d, d_model %d); "
                     "the library's fixed scratch holds %zu bytes",
                     name, need, args->num_tokens, args->d_model, kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = scratch_for_current_device(name, &scratch);
  if (rc) return rc;
  // The status word and the header must start at zero; the rest of the
  // scratch is fully rewritten by every call.
  cudaError_t e = cudaMemsetAsync(scratch, 0, kWsHeaderBytes, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_error(e, name);
  krt_qkv_paged_args a;
  std::memcpy(&a, args, sizeof(a));
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  rc = krt_qkv_rope_decode(&a, stream);
  if (rc) {
    // keep the failing call's message but name this entry point
    char msg[1024];
    std::snprintf(msg, sizeof(msg), "%s", krt_last_error());
    return set_error(rc, "%s: %s", name, msg);
  }
  return KRT_OK;
}

extern "C" int krt_qkv_rope_decode_noalloc_status(void* stream, int32_t* bits) {
  const char* name = "krt_qkv_rope_decode_noalloc_status";
  if (!bits) return set_error(KRT_ERR_INVALID, "%s: bits is NULL", name);
  void* scratch = nullptr;
  int rc = scratch_for_current_device(name, &scratch);
  if (rc) return rc;
  return krt_read_status(scratch, stream, bits);
}
