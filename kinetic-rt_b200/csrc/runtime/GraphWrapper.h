// CUDA-graph capture and replay of the per-step kernel sequence, with the
// paged KV pool it feeds.
//
// Interface of the reference's include/GraphWrapper.h:143-193 /
// src/GraphWrapper.cpp: begin_capture(stream, batch, seq) invalidates and
// re-allocates when the shape changes, allocates ceil(seq / tokens_per_block)
// blocks from the BlockManager (src/GraphWrapper.cpp:139-145) and starts a
// global-mode capture; end_capture instantiates; launch(streams, buffers)
// replays the exec on each stream with the GIL released and keeps the Python
// buffer references alive until an event recorded after the replay has
// completed; invalidate() waits for in-flight replays, destroys the graph and
// returns the blocks.  Events come from a pre-allocated pool (2047 entries).
// One GraphWrapper per device: a graph exec belongs to one device.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include <pybind11/pybind11.h>

#include "BlockManager.h"
#include "cuda_shim.h"

// Bounded multi-producer / multi-consumer ring of trivially copyable items.
template <typename T, size_t Size>
class LockFreeRingBuffer {
 public:
  bool push(const T& item) {
    size_t tail = tail_.load(std::memory_order_relaxed);
    for (;;) {
      const size_t next = (tail + 1) % Size;
      if (next == head_.load(std::memory_order_acquire)) return false;  // full
      if (tail_.compare_exchange_weak(tail, next, std::memory_order_acq_rel, std::memory_order_relaxed)) {
        slots_[tail].value = item;
        slots_[tail].ready.store(true, std::memory_order_release);
        return true;
      }
    }
  }

  bool pop(T& item) {
    size_t head = head_.load(std::memory_order_relaxed);
    for (;;) {
      if (head == tail_.load(std::memory_order_acquire)) return false;  // empty
      if (!slots_[head].ready.load(std::memory_order_acquire)) {
        std::this_thread::yield();  // claimed by a producer that is still writing
        head = head_.load(std::memory_order_relaxed);
        continue;
      }
      T copy = slots_[head].value;
      if (head_.compare_exchange_weak(head, (head + 1) % Size, std::memory_order_acq_rel,
                                      std::memory_order_relaxed)) {
        slots_[head].ready.store(false, std::memory_order_release);
        item = copy;
        return true;
      }
    }
  }

  bool empty() const { return head_.load(std::memory_order_acquire) == tail_.load(std::memory_order_acquire); }

 private:
  struct Slot {
    T value{};
    std::atomic<bool> ready{false};
  };
  Slot slots_[Size];
  std::atomic<size_t> head_{0};
  std::atomic<size_t> tail_{0};
};

struct InFlightState {
  cudaEvent_t event;
  std::vector<pybind11::object> refs;
};

class GraphWrapper {
 public:
  GraphWrapper();
  ~GraphWrapper();
  GraphWrapper(const GraphWrapper&) = delete;
  GraphWrapper& operator=(const GraphWrapper&) = delete;

  void begin_capture(uintptr_t stream_ptr, int batch_size, int seq_len);
  void end_capture(uintptr_t stream_ptr);
  void launch(std::vector<pybind11::object> stream_objs, std::vector<pybind11::object> buffers);
  bool is_valid(int batch_size, int seq_len) const;
  void invalidate();

  // Additions for the paged kernels: the pool and the blocks of the capture.
  BlockManager& block_manager() { return *block_manager_; }
  std::vector<int> block_table() const;
  size_t in_flight() const;

  static constexpr size_t kEventPool = 2048;

 private:
  void reap_completed();

  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t exec_ = nullptr;
  bool instantiated_ = false;
  int batch_size_ = -1;
  int seq_len_ = -1;
  std::deque<InFlightState> in_flight_;
  LockFreeRingBuffer<cudaEvent_t, kEventPool> event_pool_;
  std::unique_ptr<BlockManager> block_manager_;
  std::vector<int> block_table_;
  int tokens_per_block_ = 16;
  mutable std::recursive_mutex mutex_;
};
