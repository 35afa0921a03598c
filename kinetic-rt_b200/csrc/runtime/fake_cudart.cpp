// Host-only CUDA runtime test double (KRT_MOCK_CUDA builds only).
#if defined(KRT_MOCK_CUDA)
#include "fake_cudart.h"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <string>

namespace {
std::mutex g_mu;
FakeCudaState g_state;
std::set<void*> g_exec_in_flight;  // execs launched and not yet synchronised

struct FakeEvent {
  bool recorded = false;
};
struct FakeLibrary {
  std::string image_magic;
};
int g_kernel_tag = 0;
}  // namespace

void FakeCudaState::reset() { *this = FakeCudaState(); }
FakeCudaState& fake_cuda_state() { return g_state; }

const char* cudaGetErrorString(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return "no error";
    case cudaErrorInvalidValue: return "invalid argument (fake runtime)";
    case cudaErrorNotReady: return "not ready (fake runtime)";
    case cudaErrorIllegalState: return "illegal state (fake runtime)";
    case cudaErrorNoDevice: return "no CUDA-capable device (fake runtime)";
    default: return "unknown error (fake runtime)";
  }
}
cudaError_t cudaGetLastError() { return cudaSuccess; }
cudaError_t cudaGetDevice(int* dev) {
  *dev = 0;
  return cudaSuccess;
}
cudaError_t cudaSetDevice(int) { return cudaSuccess; }
cudaError_t cudaGetDeviceCount(int* n) {
  *n = 1;
  return cudaSuccess;
}
cudaError_t cudaGetDeviceProperties(cudaDeviceProp* prop, int) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.get_device_properties++;
  std::memset(prop, 0, sizeof(*prop));
  std::strncpy(prop->name, "Fake CUDA device", sizeof(prop->name) - 1);
  prop->major = 0;
  prop->minor = 0;
  prop->multiProcessorCount = 148;
  prop->sharedMemPerBlock = 48 * 1024;
  prop->totalGlobalMem = size_t(1) << 30;
  return cudaSuccess;
}
cudaError_t cudaMalloc(void** p, size_t bytes) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.malloc_calls++;
  *p = std::calloc(1, bytes ? bytes : 1);
  return *p ? cudaSuccess : cudaErrorInvalidValue;
}
cudaError_t cudaFree(void* p) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.free_calls++;
  std::free(p);
  return cudaSuccess;
}
cudaError_t cudaMemset(void* p, int v, size_t bytes) {
  std::memset(p, v, bytes);
  return cudaSuccess;
}
cudaError_t cudaMemsetAsync(void* p, int v, size_t bytes, cudaStream_t) { return cudaMemset(p, v, bytes); }
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind) {
  std::memmove(dst, src, bytes);
  return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes, cudaMemcpyKind k, cudaStream_t) {
  return cudaMemcpy(dst, src, bytes, k);
}
cudaError_t cudaEventCreate(cudaEvent_t* e) { return cudaEventCreateWithFlags(e, 0); }
cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.event_create++;
  *e = new FakeEvent();
  return cudaSuccess;
}
cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.event_record++;
  static_cast<FakeEvent*>(e)->recorded = true;
  // Work on the fake device completes immediately: everything launched
  // before this record is no longer in flight.
  g_exec_in_flight.clear();
  g_state.graphs_in_flight = 0;
  return cudaSuccess;
}
cudaError_t cudaEventQuery(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaEventSynchronize(cudaEvent_t) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.event_synchronize++;
  g_exec_in_flight.clear();
  g_state.graphs_in_flight = 0;
  return cudaSuccess;
}
cudaError_t cudaEventDestroy(cudaEvent_t e) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.event_destroy++;
  delete static_cast<FakeEvent*>(e);
  return cudaSuccess;
}
cudaError_t cudaEventElapsedTime(float* ms, cudaEvent_t, cudaEvent_t) {
  *ms = 1.0f;
  return cudaSuccess;
}
cudaError_t cudaStreamSynchronize(cudaStream_t) {
  std::lock_guard<std::mutex> l(g_mu);
  g_exec_in_flight.clear();
  g_state.graphs_in_flight = 0;
  return cudaSuccess;
}
cudaError_t cudaStreamBeginCapture(cudaStream_t, cudaStreamCaptureMode) {
  std::lock_guard<std::mutex> l(g_mu);
  if (g_state.capturing) return cudaErrorIllegalState;
  g_state.stream_begin_capture++;
  g_state.capturing = true;
  return cudaSuccess;
}
cudaError_t cudaStreamEndCapture(cudaStream_t, cudaGraph_t* g) {
  std::lock_guard<std::mutex> l(g_mu);
  if (!g_state.capturing) return cudaErrorIllegalState;
  g_state.stream_end_capture++;
  g_state.capturing = false;
  *g = new int(1);
  return cudaSuccess;
}
cudaError_t cudaGraphInstantiate(cudaGraphExec_t* exec, cudaGraph_t g, unsigned long long) {
  std::lock_guard<std::mutex> l(g_mu);
  if (!g) return cudaErrorInvalidValue;
  g_state.graph_instantiate++;
  *exec = new int(2);
  return cudaSuccess;
}
cudaError_t cudaGraphLaunch(cudaGraphExec_t exec, cudaStream_t) {
  std::lock_guard<std::mutex> l(g_mu);
  if (!exec) return cudaErrorInvalidValue;
  g_state.graph_launch++;
  g_exec_in_flight.insert(exec);
  g_state.graphs_in_flight = (int)g_exec_in_flight.size();
  return cudaSuccess;
}
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t exec) {
  std::lock_guard<std::mutex> l(g_mu);
  if (g_exec_in_flight.count(exec)) return cudaErrorIllegalState;  // destroying an exec still in flight
  g_state.graph_exec_destroy++;
  delete static_cast<int*>(exec);
  return cudaSuccess;
}
cudaError_t cudaGraphDestroy(cudaGraph_t g) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.graph_destroy++;
  delete static_cast<int*>(g);
  return cudaSuccess;
}
cudaError_t cudaLibraryLoadData(cudaLibrary_t* lib, const void* image, void*, void*, unsigned, void*, void*,
                                unsigned) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.library_load++;
  const unsigned char* b = static_cast<const unsigned char*>(image);
  if (!b || b[0] != 0x7f || b[1] != 'E' || b[2] != 'L' || b[3] != 'F') return cudaErrorInvalidValue;
  *lib = new FakeLibrary();
  return cudaSuccess;
}
cudaError_t cudaLibraryUnload(cudaLibrary_t lib) {
  delete static_cast<FakeLibrary*>(lib);
  return cudaSuccess;
}
cudaError_t cudaLibraryGetKernel(cudaKernel_t* k, cudaLibrary_t, const char* name) {
  const std::string n(name);
  if (n != "fused_rmsnorm_qkv_rope" && n != "fused_rmsnorm_qkv_rope_bf16") return cudaErrorInvalidValue;
  *k = &g_kernel_tag;
  return cudaSuccess;
}
cudaError_t cudaLaunchKernel(const void*, dim3, dim3, void**, size_t, cudaStream_t) {
  std::lock_guard<std::mutex> l(g_mu);
  g_state.kernel_launch++;
  return cudaSuccess;
}
cudaError_t cudaFuncSetAttribute(const void*, int, int) { return cudaSuccess; }
#endif
