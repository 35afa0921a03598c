// Tensor-parallel communicator (interface of the reference's
// include/Communicator.h:15-26: Communicator(rank, world_size) and
// all_reduce_async(send, recv, count, datatype, op, stream)).
//
// CUDA build: backed by libkrt's peer-buffer communicator (krt_comm_*): the
// allreduce and the fused row-parallel GEMM + allreduce run as kernels that
// store into peers' buffers over NVLink.  One process per GPU; after
// construction every rank calls ipc_handle(), exchanges the handles and calls
// open_peers(handles) (world_size 1 needs neither).
//
// Host-only test build: an in-process rendezvous that reduces host float32
// buffers across the Communicator objects of one process (one thread per
// rank), with a 5 s timeout -- the behaviour the reference's mock backend
// gives its tests (tests/mock_rccl.h:27-76).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

struct krt_comm;

class Communicator {
 public:
  Communicator(int rank, int world_size);
  ~Communicator();
  Communicator(const Communicator&) = delete;
  Communicator& operator=(const Communicator&) = delete;

  void all_reduce_async(void* sendbuff, void* recvbuff, size_t count, int datatype, int op, uintptr_t stream_ptr);

  std::string ipc_handle();
  void open_peers(const std::vector<std::string>& handles);
  void rowparallel_gemm_ar(uintptr_t x, uintptr_t weight, uintptr_t y, int num_tokens, int k_local, int n_out,
                           int x_stride, int y_stride, uintptr_t stream_ptr);
  // Device status word of this communicator's collectives (0 = no error).
  int read_status(uintptr_t stream_ptr);
  int rank() const { return rank_; }
  int world_size() const { return world_size_; }

 private:
  int rank_;
  int world_size_;
  krt_comm* comm_ = nullptr;
  void* status_ = nullptr;  // device workspace header (status word)
};
