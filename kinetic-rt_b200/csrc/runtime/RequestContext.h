// Per-request lifecycle of the serving path around the decode hot path
// (include/RequestContext.h, src/RequestContext.cpp:45-393 of the
// reference): the request's immutable parameters, its lifecycle state
// machine, two-phase cancellation, an optional deadline, the handoff of
// ownership between the ingress, scheduler, executor and backend, the tokens
// generated so far, its KV block ids and device buffers, and cleanup
// callbacks run once the request is over.
//
// The decode driver (python/kinetic_rt/orchestrator.py, KineticRuntime
// .generate_ids) walks a context through RECEIVED -> VALIDATED -> TOKENIZED
// -> ENQUEUED -> PREFILL -> DECODE <-> STREAMING -> COMPLETE, checks the
// cancellation flag and the deadline between decode steps, and frees the
// sequence's KV blocks from a cleanup callback.
//
// The class and method names, the states, the legal transitions and the
// phrases of the error messages are the reference's (its tests match them by
// substring); the implementation is this build's own.
#pragma once

#include <atomic>
#include <chrono>
#include <cstdint>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

enum class RequestState : uint8_t {
  RECEIVED = 0,
  VALIDATED,
  TOKENIZED,
  ENQUEUED,
  PREFILL,
  DECODE,
  STREAMING,
  COMPLETE,
  CANCELLED,
  TIMED_OUT,
  FAILED
};
const char* to_string(RequestState state);

enum class CompletionReason : uint8_t { STREAMING = 0, EOS, STOP_TOKEN, LENGTH, CANCELLED, TIMEOUT, ERROR };
const char* to_string(CompletionReason reason);

enum class Owner : uint8_t { Ingress = 0, Scheduler, Executor, Backend };
const char* to_string(Owner owner);

// Opaque handles the serving layer attaches to a request.
class Tokenizer;
struct LogicalDecodeState;
struct KVBlockTable;

class RequestContextError : public std::runtime_error {
 public:
  explicit RequestContextError(const std::string& what) : std::runtime_error(what) {}
};
class InvalidStateTransitionError : public RequestContextError {
 public:
  explicit InvalidStateTransitionError(const std::string& what) : RequestContextError(what) {}
};
class RequestOwnershipError : public RequestContextError {
 public:
  explicit RequestOwnershipError(const std::string& what) : RequestContextError(what) {}
};

class RequestContext {
 public:
  using Clock = std::chrono::steady_clock;

  struct Config {
    std::string request_id;
    std::string prompt_text;
    std::vector<int32_t> prompt_tokens;
    int max_new_tokens = 0;
    float temperature = 1.0f;
    float top_p = 1.0f;
    int top_k = 0;
    std::vector<int32_t> stop_token_ids;
    std::string backend_hint;
    Clock::duration timeout{Clock::duration::zero()};  // zero: no deadline
    Owner initial_owner{Owner::Ingress};
  };

  // Throws RequestContextError for an empty request_id, a negative
  // max_new_tokens / temperature / top_k / timeout, or top_p outside [0, 1].
  explicit RequestContext(Config config);
  RequestContext(const RequestContext&) = delete;
  RequestContext& operator=(const RequestContext&) = delete;
  RequestContext(RequestContext&&) = delete;
  RequestContext& operator=(RequestContext&&) = delete;
  // Runs the cleanup callbacks not run yet; the state is left as it is.
  ~RequestContext();

  const std::string& request_id() const noexcept { return cfg_.request_id; }
  const std::string& prompt_text() const noexcept { return cfg_.prompt_text; }
  const std::vector<int32_t>& prompt_tokens() const noexcept { return cfg_.prompt_tokens; }
  int max_new_tokens() const noexcept { return cfg_.max_new_tokens; }
  float temperature() const noexcept { return cfg_.temperature; }
  float top_p() const noexcept { return cfg_.top_p; }
  int top_k() const noexcept { return cfg_.top_k; }
  const std::vector<int32_t>& stop_token_ids() const noexcept { return cfg_.stop_token_ids; }
  const std::string& backend_hint() const noexcept { return cfg_.backend_hint; }

  // Not terminal, not cleaned up; ensure_executable() throws otherwise.
  bool is_valid() const noexcept;
  void ensure_executable() const;

  // Lifecycle: each state has one successor (STREAMING two: back to DECODE
  // for the next token, or COMPLETE); CANCELLED, TIMED_OUT and FAILED are
  // reachable from every non-terminal state; terminal states have none.
  RequestState state() const;
  bool can_transition_to(RequestState to) const;
  void transition_to(RequestState to);  // InvalidStateTransitionError when illegal
  static bool is_terminal(RequestState state) noexcept;
  bool is_terminal() const noexcept;

  // Two-phase cancellation: any thread raises the flag (lock-free); the
  // owner of the request acknowledges it at a safe point, which moves the
  // request to CANCELLED.
  void request_cancellation() noexcept;
  bool is_cancellation_requested() const noexcept;
  void acknowledge_cancellation();

  // Deadline = construction time + timeout (none when the timeout is zero).
  bool has_deadline() const noexcept;
  int64_t deadline_ns() const noexcept;  // steady-clock nanoseconds, 0 without a deadline
  bool is_expired(Clock::time_point now = Clock::now()) const noexcept;
  void acknowledge_timeout(Clock::time_point now = Clock::now());  // -> TIMED_OUT

  Owner current_owner() const;
  // Compare-and-set: throws RequestOwnershipError when the current owner is
  // not `expected_current_owner` or the request is over.
  void transfer_ownership(Owner new_owner, Owner expected_current_owner);

  void append_generated_token(int32_t token_id);
  std::vector<int32_t> generated_tokens() const;

  void set_input_device_ptr(uintptr_t ptr);   // a null pointer is rejected
  void set_output_device_ptr(uintptr_t ptr);  // a null pointer is rejected
  uintptr_t input_device_ptr() const noexcept;
  uintptr_t output_device_ptr() const noexcept;

  void add_kv_block_id(int block_id);
  void set_kv_block_ids(std::vector<int> block_ids);
  std::vector<int> kv_block_ids() const;
  void set_kv_block_table_handle(KVBlockTable* handle);
  KVBlockTable* kv_block_table_handle() const noexcept;

  // Binding a different tokenizer than the one already bound is an error.
  void set_tokenizer_ref(Tokenizer* tokenizer_ref);
  Tokenizer* tokenizer_ref() const noexcept;
  void set_logical_decode_state(LogicalDecodeState* state);
  LogicalDecodeState* logical_decode_state() const noexcept;
  void set_session_sequence(uint64_t sequence) noexcept;
  uint64_t session_sequence() const noexcept;

  void set_finish_reason(CompletionReason reason);
  CompletionReason finish_reason() const;
  void set_error_code(int code) noexcept;
  int error_code() const noexcept;

  // Cleanup callbacks run once, newest first, outside the lock (they may call
  // back into the context), exceptions swallowed.  cleanup() is allowed only
  // in a terminal state and returns false when it already ran.
  void register_cleanup_callback(std::function<void()> callback);
  bool is_cleaned_up() const noexcept;
  bool cleanup();

 private:
  struct Dynamic {  // everything behind mu_
    RequestState state = RequestState::RECEIVED;
    Owner owner = Owner::Ingress;
    std::vector<int32_t> generated;
    uintptr_t input_ptr = 0, output_ptr = 0;
    std::vector<int> kv_blocks;
    KVBlockTable* kv_table = nullptr;
    Tokenizer* tokenizer = nullptr;
    LogicalDecodeState* decode_state = nullptr;
    uint64_t session_sequence = 0;
    CompletionReason reason = CompletionReason::STREAMING;
    int error_code = 0;
    std::vector<std::function<void()>> callbacks;
    bool cleaned = false;
  };

  static Config checked(Config config);
  void move_to(RequestState to);                       // mu_ held
  std::vector<std::function<void()>> take_callbacks();  // mu_ held; marks the context cleaned
  static void run_newest_first(std::vector<std::function<void()>>& callbacks);

  const Config cfg_;
  const Clock::time_point deadline_;
  std::atomic<bool> cancel_{false};
  mutable std::mutex mu_;
  Dynamic d_;
};
