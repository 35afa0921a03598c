// AOT artifact (.kin) serializer and the engine that loads and launches the
// fused RMSNorm + QKV + RoPE kernel.
//
// Interface of the reference's include/AOTEngine.h:19-151: KinHeader (packed,
// magic 0x4B494E00), KernelLaunchDescriptor (the 33 fields bound in
// bindings/python_bindings.cpp:300-334, plus paged-cache extensions),
// Serializer (save/load/TP degree, hardware "poison pill") and AOTEngine
// (compile_ahead_of_time, load_model, launch, synchronize_and_clear).
//
// The .kin artifact carries this build's own nvcc cubin of the kernel with the
// reference's 24-parameter signature (aot_kernel.cu); paged launches go to
// libkrt's tcgen05 kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "cuda_shim.h"

class HardwareMismatchError : public std::runtime_error {
 public:
  explicit HardwareMismatchError(const std::string& msg) : std::runtime_error(msg) {}
};

constexpr uint32_t kKinMagic = 0x4B494E00u;  // "KIN\0"

#pragma pack(push, 1)
struct KinHeader {
  uint32_t magic_number;
  uint32_t version;
  char device_id[256];
  char kinetic_target[256];
  uint64_t weights_hash;
  uint64_t op_graph_data_offset;
  uint64_t op_graph_data_size;
  uint64_t kernel_binaries_offset;
  uint64_t kernel_binaries_size;
  uint32_t tensor_parallel_degree;
};
#pragma pack(pop)
static_assert(sizeof(KinHeader) == 564, "KinHeader must stay 564 bytes (on-disk format)");

struct KernelLaunchDescriptor {
  // reference fields
  uintptr_t input_ptr = 0;
  uintptr_t output_ptr = 0;
  uintptr_t qkv_weight_ptr = 0;
  uintptr_t qkv_bias_ptr = 0;
  uintptr_t rms_weight_ptr = 0;
  uintptr_t freqs_cos_ptr = 0;
  uintptr_t freqs_sin_ptr = 0;
  uintptr_t k_output_ptr = 0;
  uintptr_t v_output_ptr = 0;
  int seq_len = 0;
  int d_model = 0;
  int n_heads = 0;
  int head_dim = 0;
  float eps = 1.0e-5f;
  int stride_x_seq = 0;
  int stride_x_dim = 0;
  int stride_w_out = 0;
  int stride_w_in = 0;
  int stride_q_seq = 0;
  int stride_q_dim = 0;
  int stride_k_seq = 0;
  int stride_k_dim = 0;
  int stride_v_seq = 0;
  int stride_v_dim = 0;
  size_t byte_size = 0;
  std::string kernel_name;
  unsigned int grid_x = 0;
  unsigned int grid_y = 1;
  unsigned int grid_z = 1;
  unsigned int block_x = 256;
  unsigned int block_y = 1;
  unsigned int block_z = 1;
  unsigned int shared_mem_bytes = 0;
  // extensions: the paged decode/prefill path (used when kv_pool_ptr != 0)
  int dtype = 0;  // DataType code; 0 = float32
  int n_kv_heads = 0;
  uintptr_t positions_ptr = 0;
  uintptr_t token_seq_ptr = 0;
  uintptr_t block_table_ptr = 0;
  uintptr_t kv_pool_ptr = 0;
  int num_seqs = 0;
  int block_table_stride = 0;
  int num_blocks = 0;
  int tokens_per_block = 16;
  int max_position = 0;
  uintptr_t workspace_ptr = 0;
  size_t workspace_bytes = 0;
};

class Serializer {
 public:
  Serializer();
  void save_kin_file(const std::string& filepath, const std::string& device_id, const std::string& kinetic_target,
                     uint64_t weights_hash, const std::vector<uint8_t>& op_graph_data,
                     const std::vector<uint8_t>& kernel_binaries);
  std::vector<uint8_t> load_kin_file(const std::string& filepath);
  uint32_t get_tensor_parallel_degree(const std::string& filepath);
  const std::string& get_device_id() const { return device_id_; }
  const std::string& get_loaded_kinetic_target() const { return loaded_kinetic_target_; }

 private:
  std::string device_id_;
  std::string loaded_kinetic_target_;
};

class AOTEngine {
 public:
  AOTEngine();
  ~AOTEngine();
  AOTEngine(const AOTEngine&) = delete;
  AOTEngine& operator=(const AOTEngine&) = delete;

  void compile_ahead_of_time(const std::string& output_filepath, uintptr_t stream_ptr,
                             const std::string& kinetic_target);
  void load_model(const std::string& filepath);
  void launch(const KernelLaunchDescriptor& descriptor, uintptr_t stream_ptr);
  void launch(void* input_ptr, void* output_ptr, int seq_len, uintptr_t stream_ptr, size_t byte_size = 0);
  void launch_ptr(void* input_ptr, void* output_ptr, int seq_len, size_t byte_size = 0);
  void synchronize_and_clear(uintptr_t stream_ptr);

  static uint64_t compute_fnv1a_hash(const std::vector<uint8_t>& data);
  // Directory holding the kernel cubin packed into .kin files.
  static std::string kernel_dir();

 private:
  void load_kernel(const std::vector<uint8_t>& binary, const std::string& kinetic_target);
  void validate_elf_structure(const std::vector<uint8_t>& binary, const std::string& kinetic_target) const;
  void launch_paged(const KernelLaunchDescriptor& d, uintptr_t stream_ptr);

  Serializer serializer_;
  cudaLibrary_t library_ = nullptr;
  std::unordered_map<std::string, cudaKernel_t> kernels_;
  std::string default_kernel_name_;
  std::recursive_mutex mutex_;
};
