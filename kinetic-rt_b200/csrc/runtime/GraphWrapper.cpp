#include "GraphWrapper.h"

#include <cstdlib>
#include <cstring>
#include <iostream>
#include <string>

namespace {

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  return std::stoi(v);
}

// Accept a raw stream handle (int) or an object exposing `cuda_stream`
// (torch.cuda.Stream).
uintptr_t stream_handle(const pybind11::object& o) {
  if (pybind11::hasattr(o, "cuda_stream")) return o.attr("cuda_stream").cast<uintptr_t>();
  return o.cast<uintptr_t>();
}

}  // namespace

GraphWrapper::GraphWrapper() {
  // KV pool geometry: KINETIC_KV_POOL_SIZE blocks (default 64 per SM) of
  // KINETIC_BLOCK_SIZE tokens (default 16), 4096 bytes per token
  // (src/GraphWrapper.cpp:17-41 of the reference).
  int pool = env_int("KINETIC_KV_POOL_SIZE", 0);
  if (pool <= 0) {
    int dev = 0;
    cudaDeviceProp prop;
    pool = (cudaGetDevice(&dev) == cudaSuccess && cudaGetDeviceProperties(&prop, dev) == cudaSuccess)
               ? prop.multiProcessorCount * 64
               : 4096;
    if (pool <= 0) pool = 4096;
  }
  tokens_per_block_ = env_int("KINETIC_BLOCK_SIZE", 16);
  block_manager_ = std::make_unique<BlockManager>(pool, tokens_per_block_, 4096);
  for (size_t i = 0; i + 1 < kEventPool; ++i) {
    cudaEvent_t e;
    KRT_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    event_pool_.push(e);
  }
}

GraphWrapper::~GraphWrapper() {
  try {
    invalidate();
  } catch (const std::exception& e) {
    std::cerr << "GraphWrapper: " << e.what() << std::endl;
  }
  cudaEvent_t e;
  while (event_pool_.pop(e)) cudaEventDestroy(e);
}

void GraphWrapper::reap_completed() {
  while (!in_flight_.empty()) {
    const cudaError_t s = cudaEventQuery(in_flight_.front().event);
    if (s == cudaErrorNotReady) break;
    KRT_CHECK_CUDA(s);
    if (!event_pool_.push(in_flight_.front().event)) cudaEventDestroy(in_flight_.front().event);
    in_flight_.pop_front();
  }
}

bool GraphWrapper::is_valid(int batch_size, int seq_len) const {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  return instantiated_ && batch_size_ == batch_size && seq_len_ == seq_len;
}

void GraphWrapper::invalidate() {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  for (auto& st : in_flight_) KRT_CHECK_CUDA(cudaEventSynchronize(st.event));
  for (auto& st : in_flight_)
    if (!event_pool_.push(st.event)) cudaEventDestroy(st.event);
  in_flight_.clear();
  if (exec_) {
    KRT_CHECK_CUDA(cudaGraphExecDestroy(exec_));
    exec_ = nullptr;
  }
  if (graph_) {
    KRT_CHECK_CUDA(cudaGraphDestroy(graph_));
    graph_ = nullptr;
  }
  instantiated_ = false;
  batch_size_ = -1;
  seq_len_ = -1;
  for (int id : block_table_) block_manager_->free_block(id);
  block_table_.clear();
}

void GraphWrapper::begin_capture(uintptr_t stream_ptr, int batch_size, int seq_len) {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  if (is_valid(batch_size, seq_len)) return;  // already captured for these shapes
  if (batch_size <= 0 || seq_len <= 0) throw std::invalid_argument("begin_capture: batch_size and seq_len must be positive");
  invalidate();
  batch_size_ = batch_size;
  seq_len_ = seq_len;
  const int blocks = (seq_len + tokens_per_block_ - 1) / tokens_per_block_;
  while (static_cast<int>(block_table_.size()) < blocks) block_table_.push_back(block_manager_->allocate_block());
  KRT_CHECK_CUDA(cudaStreamBeginCapture(reinterpret_cast<cudaStream_t>(stream_ptr), cudaStreamCaptureModeGlobal));
}

void GraphWrapper::end_capture(uintptr_t stream_ptr) {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  KRT_CHECK_CUDA(cudaStreamEndCapture(reinterpret_cast<cudaStream_t>(stream_ptr), &graph_));
  KRT_CHECK_CUDA(cudaGraphInstantiate(&exec_, graph_, 0));
  instantiated_ = true;
}

void GraphWrapper::launch(std::vector<pybind11::object> stream_objs, std::vector<pybind11::object> buffers) {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  reap_completed();
  if (!instantiated_) throw std::runtime_error("Cannot launch graph: not instantiated.");
  std::vector<uintptr_t> streams;
  streams.reserve(stream_objs.size());
  for (auto& o : stream_objs) streams.push_back(stream_handle(o));
  {
    pybind11::gil_scoped_release release;
    for (uintptr_t s : streams) KRT_CHECK_CUDA(cudaGraphLaunch(exec_, reinterpret_cast<cudaStream_t>(s)));
  }
  for (size_t i = 0; i < streams.size(); ++i) {
    cudaEvent_t ev = nullptr;
    if (!event_pool_.pop(ev)) KRT_CHECK_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    const cudaError_t rec = cudaEventRecord(ev, reinterpret_cast<cudaStream_t>(streams[i]));
    if (rec != cudaSuccess) {
      cudaEventDestroy(ev);
      KRT_CHECK_CUDA(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(streams[i])));
      continue;
    }
    InFlightState st;
    st.event = ev;
    st.refs.reserve(buffers.size() + 1);
    st.refs.push_back(stream_objs[i]);
    st.refs.insert(st.refs.end(), buffers.begin(), buffers.end());
    in_flight_.push_back(std::move(st));
  }
}

std::vector<int> GraphWrapper::block_table() const {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  return block_table_;
}

size_t GraphWrapper::in_flight() const {
  std::lock_guard<std::recursive_mutex> lock(mutex_);
  return in_flight_.size();
}
