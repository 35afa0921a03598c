// Paged KV-cache pool: one device allocation cut into fixed-size blocks.
//
// Same contract as the reference's include/BlockManager.h:29-95:
//   * pool = num_blocks * tokens_per_block * token_byte_size bytes, allocated
//     once in the constructor and freed in the destructor;
//   * block i starts at pool + i * tokens_per_block * token_byte_size;
//   * allocate_block() pops the most recently freed id (the free list starts
//     as 0..N-1, so the first id handed out is N-1); free_block() pushes it
//     back (LIFO reuse); both are mutex-protected;
//   * an empty pool and an out-of-range id raise std::runtime_error with the
//     reference's messages.
// Additions: block_ptr(id) and num_free().
//
// The fused QKV kernels write a token's K and V heads at
//   pool + (block * tokens_per_block + offset) * token_byte_size
// as [K | V][kv_head][head_dim] bf16 (token_byte_size = 2 * kv_heads * 128 * 2).
#pragma once

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "cuda_shim.h"

class BlockManager {
 public:
  BlockManager(int num_blocks, int tokens_per_block, int token_byte_size)
      : tokens_per_block_(tokens_per_block), token_byte_size_(token_byte_size), num_blocks_(num_blocks) {
    if (num_blocks <= 0 || tokens_per_block <= 0 || token_byte_size <= 0)
      throw std::invalid_argument("BlockManager: num_blocks, tokens_per_block and token_byte_size must be positive");
    const size_t bytes = pool_bytes();
    cudaError_t e = cudaMalloc(&pool_, bytes);
    if (e != cudaSuccess) throw std::runtime_error("CUDA memory error in BlockManager");
    free_blocks_.reserve(num_blocks);
    for (int i = 0; i < num_blocks; ++i) free_blocks_.push_back(i);
  }

  ~BlockManager() {
    if (pool_) cudaFree(pool_);
    pool_ = nullptr;
  }

  BlockManager(const BlockManager&) = delete;
  BlockManager& operator=(const BlockManager&) = delete;

  int allocate_block() {
    std::lock_guard<std::mutex> lock(mutex_);
    if (free_blocks_.empty()) throw std::runtime_error("Out of KV Cache blocks! Massive pool exhausted.");
    const int id = free_blocks_.back();
    free_blocks_.pop_back();
    return id;
  }

  void free_block(int id) {
    std::lock_guard<std::mutex> lock(mutex_);
    if (id < 0 || id >= num_blocks_)
      throw std::runtime_error("BlockManager::free_block: block ID " + std::to_string(id) + " out of range [0, " +
                               std::to_string(num_blocks_) + ")");
    // Any in-range id goes back on the free list, as the reference does
    // (include/BlockManager.h:73-82): freeing an id twice lists it twice.
    free_blocks_.push_back(id);
  }

  void* get_pool_ptr() const { return pool_; }
  void* block_ptr(int id) const {
    if (id < 0 || id >= num_blocks_) throw std::runtime_error("BlockManager::block_ptr: block ID out of range");
    return static_cast<char*>(pool_) + static_cast<size_t>(id) * block_bytes();
  }
  size_t block_bytes() const { return static_cast<size_t>(tokens_per_block_) * token_byte_size_; }
  size_t pool_bytes() const { return static_cast<size_t>(num_blocks_) * block_bytes(); }
  int num_blocks() const { return num_blocks_; }
  int tokens_per_block() const { return tokens_per_block_; }
  int token_byte_size() const { return token_byte_size_; }
  int num_free() const {
    std::lock_guard<std::mutex> lock(mutex_);
    return static_cast<int>(free_blocks_.size());
  }

 private:
  int tokens_per_block_;
  int token_byte_size_;
  int num_blocks_;
  void* pool_ = nullptr;
  std::vector<int> free_blocks_;
  mutable std::mutex mutex_;
};
