// HardwareRouter (interface of the reference's include/Router.h:9-58).
//
// The reference routes "sm" targets to TensorRT and everything else to the
// HIP AOT engine.  This build has one backend for sm_100a, the AOTEngine over
// its own kernels, so every call goes there; KINETIC_TARGET is still read and
// reported.
#pragma once

#include <cstdlib>
#include <string>

#include "AOTEngine.h"

class HardwareRouter {
 public:
  HardwareRouter() {
    const char* t = std::getenv("KINETIC_TARGET");
    target_ = t ? t : "";
  }
  void load_model(const std::string& filepath) { engine_.load_model(filepath); }
  void launch(void* input_ptr, void* output_ptr, int seq_len, size_t byte_size = 0) {
    engine_.launch_ptr(input_ptr, output_ptr, seq_len, byte_size);
  }
  void launch_py(void* input_ptr, void* output_ptr, int seq_len, uintptr_t stream_ptr, size_t byte_size = 0) {
    engine_.launch(input_ptr, output_ptr, seq_len, stream_ptr, byte_size);
  }
  std::string backend() const { return "CUDA_AOT"; }
  const std::string& target() const { return target_; }
  AOTEngine& engine() { return engine_; }

 private:
  std::string target_;
  AOTEngine engine_;
};
