// Request queue and worker thread (interface of the reference's
// include/AsyncAPI.h:12-124): submit() enqueues a request, a worker thread
// drives HardwareRouter::launch once per output token and pushes one response
// per token, poll() returns the next response or None.  Launch failures are
// reported in the response instead of being dropped.
#pragma once

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include <pybind11/pybind11.h>

#include "GraphWrapper.h"
#include "Router.h"

struct InferenceRequest {
  uintptr_t input_ptr = 0;
  size_t input_len = 0;
  int max_tokens = 0;
  char request_id[64] = {};
};

struct InferenceResponse {
  char request_id[64] = {};
  char token[8] = {};
  char error[120] = {};
  bool is_finished = false;
};

class InferenceQueue {
 public:
  void submit(uintptr_t input_ptr, size_t input_len, int max_tokens, const std::string& request_id) {
    InferenceRequest r;
    r.input_ptr = input_ptr;
    r.input_len = input_len;
    r.max_tokens = max_tokens;
    request_id.copy(r.request_id, sizeof(r.request_id) - 1);
    const auto t0 = std::chrono::steady_clock::now();
    while (!requests_.push(r)) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(5))
        throw std::runtime_error("InferenceQueue.submit: request queue full");
      std::this_thread::yield();
    }
  }

  pybind11::object poll() {
    InferenceResponse r;
    if (!responses_.pop(r)) return pybind11::none();
    pybind11::dict d;
    d["request_id"] = std::string(r.request_id);
    d["token"] = std::string(r.token);
    d["is_finished"] = r.is_finished;
    if (r.error[0]) d["error"] = std::string(r.error);
    return d;
  }

  bool fetch_request(InferenceRequest& r) { return requests_.pop(r); }
  void push_response(const InferenceResponse& r) {
    while (!responses_.push(r)) std::this_thread::yield();
  }

 private:
  LockFreeRingBuffer<InferenceRequest, 1024> requests_;
  LockFreeRingBuffer<InferenceResponse, 4096> responses_;
};

class InferenceWorker {
 public:
  InferenceWorker(InferenceQueue& queue, HardwareRouter& router) : queue_(queue), router_(router) {
    thread_ = std::thread([this] { run(); });
  }
  ~InferenceWorker() {
    stop_ = true;
    if (thread_.joinable()) thread_.join();
  }

 private:
  void run() {
    while (!stop_) {
      InferenceRequest req;
      if (!queue_.fetch_request(req)) {
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
        continue;
      }
      int32_t token = 0;
      void* input = reinterpret_cast<void*>(req.input_ptr);
      size_t len = req.input_len;
      for (int i = 0; i < req.max_tokens; ++i) {
        InferenceResponse resp;
        std::memcpy(resp.request_id, req.request_id, sizeof(resp.request_id));
        try {
          router_.launch(input, &token, static_cast<int>(len), len * sizeof(int32_t));
        } catch (const std::exception& e) {
          std::strncpy(resp.error, e.what(), sizeof(resp.error) - 1);
          resp.is_finished = true;
          queue_.push_response(resp);
          break;
        }
        const char c = (token > 0 && token < 256) ? static_cast<char>(token) : static_cast<char>('A' + (token + i) % 26);
        resp.token[0] = c;
        resp.is_finished = (i == req.max_tokens - 1);
        queue_.push_response(resp);
        input = &token;
        len = 1;
      }
    }
  }

  InferenceQueue& queue_;
  HardwareRouter& router_;
  std::atomic<bool> stop_{false};
  std::thread thread_;
};
