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
#include <cuda_runtime.h>

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

std::mutex g_scratch_mu;
void* g_scratch_addr[kNoAllocMaxDevices] = {};

// Device address of g_decode_scratch on the current device.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(KRT_ERR_UNSUPPORTED, "krt_qkv_rope_decode_noalloc: device %d beyond %d", dev,
                     kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_decode_noalloc: cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return KRT_OK;
}

}  // namespace
}  // namespace krt

using namespace krt;

extern "C" int krt_qkv_rope_decode_noalloc(const krt_qkv_paged_args* args, void* stream) {
  if (!args) return set_error(KRT_ERR_INVALID, "krt_qkv_rope_decode_noalloc: args is NULL");
  const size_t need = krt_qkv_rope_decode_workspace_size(args->num_tokens, args->d_model, args->n_heads,
                                                         args->n_kv_heads, args->head_dim);
  if (need > kNoAllocScratchBytes)
    return set_error(KRT_ERR_UNSUPPORTED,
                     "krt_qkv_rope_decode_noalloc: this call needs %zu bytes of scratch (num_tokens %d, d_model %d); "
                     "the library's fixed scratch holds %zu bytes",
                     need, args->num_tokens, args->d_model, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // The status word and the header must start at zero; the rest of the
  // scratch is fully rewritten by every call.
  cudaError_t e = cudaMemsetAsync(scratch, 0, kWsHeaderBytes, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_decode_noalloc: clearing the scratch header");
  krt_qkv_paged_args a;
  std::memcpy(&a, args, sizeof(a));
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  return krt_qkv_rope_decode(&a, stream);
}
