// Host-only test double of the CUDA runtime calls used by the host runtime
// (compiled only with KRT_MOCK_CUDA; see cuda_shim.h).  It keeps call
// counters and a little state so tests can assert on the runtime's
// bookkeeping: capture state, graph instantiation, launches in flight, and a
// refusal to destroy a graph exec that is still in flight (the behaviour the
// reference's tests/mock_hip.h checks).  Allocation is host malloc.
#pragma once
#include <cstddef>
#include <cstdint>

typedef int cudaError_t;
enum : int {
  cudaSuccess = 0,
  cudaErrorInvalidValue = 1,
  cudaErrorNotReady = 600,
  cudaErrorIllegalState = 401,
  cudaErrorNoDevice = 100,
};
typedef void* cudaStream_t;
typedef void* cudaEvent_t;
typedef void* cudaGraph_t;
typedef void* cudaGraphExec_t;
typedef void* cudaLibrary_t;
typedef void* cudaKernel_t;
typedef int cudaStreamCaptureMode;
constexpr int cudaStreamCaptureModeGlobal = 0;
constexpr int cudaStreamCaptureModeThreadLocal = 1;
constexpr unsigned cudaEventDisableTiming = 2;
constexpr unsigned cudaIpcMemLazyEnablePeerAccess = 1;

enum cudaMemcpyKind { cudaMemcpyHostToDevice = 1, cudaMemcpyDeviceToHost = 2, cudaMemcpyDeviceToDevice = 3 };

struct cudaDeviceProp {
  char name[256];
  int major;
  int minor;
  int multiProcessorCount;
  size_t sharedMemPerBlock;
  size_t totalGlobalMem;
};

struct dim3 {
  unsigned x, y, z;
  dim3(unsigned a = 1, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {}
};

struct cudaIpcMemHandle_t {
  char reserved[64];
};

// Counters and state, readable from tests through the mock module.
struct FakeCudaState {
  int stream_begin_capture = 0;
  int stream_end_capture = 0;
  int graph_instantiate = 0;
  int graph_launch = 0;
  int graph_exec_destroy = 0;
  int graph_destroy = 0;
  int event_create = 0;
  int event_record = 0;
  int event_synchronize = 0;
  int event_destroy = 0;
  int library_load = 0;
  int kernel_launch = 0;
  int get_device_properties = 0;
  int malloc_calls = 0;
  int free_calls = 0;
  bool capturing = false;
  int graphs_in_flight = 0;
  void reset();
};
FakeCudaState& fake_cuda_state();

const char* cudaGetErrorString(cudaError_t e);
cudaError_t cudaGetLastError();
cudaError_t cudaGetDevice(int* dev);
cudaError_t cudaSetDevice(int dev);
cudaError_t cudaGetDeviceCount(int* n);
cudaError_t cudaGetDeviceProperties(cudaDeviceProp* prop, int dev);
cudaError_t cudaMalloc(void** p, size_t bytes);
cudaError_t cudaFree(void* p);
cudaError_t cudaMemset(void* p, int v, size_t bytes);
cudaError_t cudaMemsetAsync(void* p, int v, size_t bytes, cudaStream_t s);
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind);
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t s);
cudaError_t cudaEventCreate(cudaEvent_t* e);
cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned flags);
cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t s);
cudaError_t cudaEventQuery(cudaEvent_t e);
cudaError_t cudaEventSynchronize(cudaEvent_t e);
cudaError_t cudaEventDestroy(cudaEvent_t e);
cudaError_t cudaEventElapsedTime(float* ms, cudaEvent_t a, cudaEvent_t b);
cudaError_t cudaStreamSynchronize(cudaStream_t s);
cudaError_t cudaStreamBeginCapture(cudaStream_t s, cudaStreamCaptureMode mode);
cudaError_t cudaStreamEndCapture(cudaStream_t s, cudaGraph_t* g);
cudaError_t cudaGraphInstantiate(cudaGraphExec_t* exec, cudaGraph_t g, unsigned long long flags);
cudaError_t cudaGraphLaunch(cudaGraphExec_t exec, cudaStream_t s);
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t exec);
cudaError_t cudaGraphDestroy(cudaGraph_t g);
cudaError_t cudaLibraryLoadData(cudaLibrary_t* lib, const void* image, void*, void*, unsigned, void*, void*,
                                unsigned);
cudaError_t cudaLibraryUnload(cudaLibrary_t lib);
cudaError_t cudaLibraryGetKernel(cudaKernel_t* k, cudaLibrary_t lib, const char* name);
cudaError_t cudaLaunchKernel(const void* func, dim3 grid, dim3 block, void** args, size_t smem, cudaStream_t s);
cudaError_t cudaFuncSetAttribute(const void* func, int attr, int value);
constexpr int cudaFuncAttributeMaxDynamicSharedMemorySize = 8;
