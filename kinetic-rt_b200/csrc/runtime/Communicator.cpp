#include "Communicator.h"

#include <chrono>
#include <condition_variable>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>

#include "cuda_shim.h"

#if !defined(KRT_MOCK_CUDA)
#include "krt.h"
#endif

namespace {
void check_rank(int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world)
    throw std::invalid_argument("Communicator: rank " + std::to_string(rank) + " outside world of " +
                                std::to_string(world));
}
}  // namespace

#if defined(KRT_MOCK_CUDA)
// ------------------------------------------------------- host rendezvous
namespace {
struct Rendezvous {
  std::mutex mu;
  std::condition_variable cv;
  std::vector<float*> recv;
  int arrived = 0;
  unsigned long long generation = 0;
};
std::mutex g_registry_mu;
std::map<int, Rendezvous> g_registry;  // keyed by world size
}  // namespace

Communicator::Communicator(int rank, int world_size) : rank_(rank), world_size_(world_size) {
  check_rank(rank, world_size);
}
Communicator::~Communicator() = default;

void Communicator::all_reduce_async(void* sendbuff, void* recvbuff, size_t count, int datatype, int op,
                                    uintptr_t stream_ptr) {
  (void)stream_ptr;
  if ((datatype != 0 && datatype != 1) || op != 0)
    throw std::runtime_error("host allreduce supports float32 sum only");
  const float* send = static_cast<const float*>(sendbuff);
  float* recv = static_cast<float*>(recvbuff);
  if (recv != send) std::memmove(recv, send, count * sizeof(float));
  if (world_size_ == 1) return;
  Rendezvous* rv;
  {
    std::lock_guard<std::mutex> l(g_registry_mu);
    rv = &g_registry[world_size_];
  }
  std::unique_lock<std::mutex> lock(rv->mu);
  const unsigned long long gen = rv->generation;
  rv->recv.push_back(recv);
  if (++rv->arrived == world_size_) {
    for (size_t i = 0; i < count; ++i) {
      float s = 0.f;
      for (float* b : rv->recv) s += b[i];
      for (float* b : rv->recv) b[i] = s;
    }
    rv->recv.clear();
    rv->arrived = 0;
    ++rv->generation;
    rv->cv.notify_all();
  } else if (!rv->cv.wait_for(lock, std::chrono::seconds(5), [&] { return rv->generation != gen; })) {
    throw std::runtime_error("allreduce timed out waiting for ranks");
  }
}

std::string Communicator::ipc_handle() { return std::string(); }
void Communicator::open_peers(const std::vector<std::string>&) {}
void Communicator::rowparallel_gemm_ar(uintptr_t, uintptr_t, uintptr_t, int, int, int, int, int, uintptr_t) {
  throw std::runtime_error("rowparallel_gemm_ar needs the CUDA build");
}
int Communicator::read_status(uintptr_t) { return 0; }

#else
// ------------------------------------------------------- libkrt backend
namespace {
void krt_check(int rc, const char* what) {
  if (rc != KRT_OK) throw std::runtime_error(std::string(what) + ": " + krt_last_error());
}
}  // namespace

Communicator::Communicator(int rank, int world_size) : rank_(rank), world_size_(world_size) {
  check_rank(rank, world_size);
  krt_check(krt_comm_create(rank, world_size, 8192, &comm_), "Communicator");
  KRT_CHECK_CUDA(cudaMalloc(&status_, 8192));
  KRT_CHECK_CUDA(cudaMemset(status_, 0, 8192));
}

Communicator::~Communicator() {
  if (comm_) krt_comm_destroy(comm_);
  if (status_) cudaFree(status_);
}

void Communicator::all_reduce_async(void* sendbuff, void* recvbuff, size_t count, int datatype, int op,
                                    uintptr_t stream_ptr) {
  if (op != 0) throw std::runtime_error("Communicator::all_reduce_async supports op 0 (sum) only");
  if (datatype == 0) datatype = KRT_DTYPE_FLOAT32;
  krt_check(krt_allreduce(comm_, sendbuff, recvbuff, count, datatype, status_, reinterpret_cast<void*>(stream_ptr)),
            "Communicator::all_reduce_async");
}

std::string Communicator::ipc_handle() {
  std::string h(krt_comm_handle_size(), '\0');
  krt_check(krt_comm_ipc_handle(comm_, &h[0]), "Communicator::ipc_handle");
  return h;
}

void Communicator::open_peers(const std::vector<std::string>& handles) {
  if (static_cast<int>(handles.size()) != world_size_)
    throw std::invalid_argument("Communicator::open_peers: one handle per rank expected");
  std::string blob;
  for (const auto& h : handles) {
    if (h.size() != krt_comm_handle_size()) throw std::invalid_argument("Communicator::open_peers: bad handle size");
    blob += h;
  }
  krt_check(krt_comm_open_peers(comm_, blob.data()), "Communicator::open_peers");
}

void Communicator::rowparallel_gemm_ar(uintptr_t x, uintptr_t weight, uintptr_t y, int num_tokens, int k_local,
                                       int n_out, int x_stride, int y_stride, uintptr_t stream_ptr) {
  krt_gemm_ar_args a;
  std::memset(&a, 0, sizeof(a));
  a.x = reinterpret_cast<const void*>(x);
  a.weight = reinterpret_cast<const void*>(weight);
  a.y = reinterpret_cast<void*>(y);
  a.num_tokens = num_tokens;
  a.k_local = k_local;
  a.n_out = n_out;
  a.x_stride = x_stride > 0 ? x_stride : k_local;
  a.y_stride = y_stride > 0 ? y_stride : n_out;
  a.workspace = status_;
  a.workspace_bytes = 8192;
  krt_check(krt_rowparallel_gemm_ar(comm_, &a, reinterpret_cast<void*>(stream_ptr)),
            "Communicator::rowparallel_gemm_ar");
}

int Communicator::read_status(uintptr_t stream_ptr) {
  int32_t bits = 0;
  krt_read_status(status_, reinterpret_cast<void*>(stream_ptr), &bits);
  return bits;
}
#endif
