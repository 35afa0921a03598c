// Selects the CUDA runtime the host runtime is built against.
//
// Production builds use the real CUDA runtime.  Builds with KRT_MOCK_CUDA
// use fake_cudart.h, a host-only test double of the handful of runtime calls
// the host runtime makes (events, stream capture, graphs, allocation, module
// loading).  The double exists so that the host-side bookkeeping (graph
// lifetime, event pools, block allocation, .kin validation, the host
// rendezvous of Communicator) can be tested on machines without a GPU, the
// way the reference tests its runtime against tests/mock_hip.h.  It runs no
// kernels: a kernel launch through it computes nothing.
#pragma once

#if defined(KRT_MOCK_CUDA)
#include "fake_cudart.h"
#else
#include <cuda_runtime.h>
#endif

#include <stdexcept>
#include <string>

#define KRT_CHECK_CUDA(cmd)                                                                         \
  do {                                                                                              \
    cudaError_t krt_err_ = (cmd);                                                                   \
    if (krt_err_ != cudaSuccess) {                                                                  \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(krt_err_) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                          \
    }                                                                                               \
  } while (0)
