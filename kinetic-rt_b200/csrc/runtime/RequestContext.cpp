// RequestContext: see RequestContext.h.
#include "RequestContext.h"

#include <utility>

namespace {

constexpr const char* kStateNames[] = {"RECEIVED", "VALIDATED", "TOKENIZED", "ENQUEUED", "PREFILL",  "DECODE",
                                       "STREAMING", "COMPLETE", "CANCELLED", "TIMED_OUT", "FAILED"};
constexpr const char* kReasonNames[] = {"STREAMING", "EOS", "STOP_TOKEN", "LENGTH", "CANCELLED", "TIMEOUT", "ERROR"};
constexpr const char* kOwnerNames[] = {"Ingress", "Scheduler", "Executor", "Backend"};

constexpr uint32_t bit(RequestState s) { return 1u << static_cast<unsigned>(s); }

// Successors of every state in the normal flow (one bit per state); the
// abort states are added for every non-terminal state in allowed().
constexpr uint32_t kNext[] = {
    bit(RequestState::VALIDATED),                               // RECEIVED
    bit(RequestState::TOKENIZED),                               // VALIDATED
    bit(RequestState::ENQUEUED),                                // TOKENIZED
    bit(RequestState::PREFILL),                                 // ENQUEUED
    bit(RequestState::DECODE),                                  // PREFILL
    bit(RequestState::STREAMING),                               // DECODE
    bit(RequestState::DECODE) | bit(RequestState::COMPLETE),    // STREAMING: next token, or done
    0, 0, 0, 0,                                                 // terminal
};
constexpr uint32_t kAbort = bit(RequestState::CANCELLED) | bit(RequestState::TIMED_OUT) | bit(RequestState::FAILED);

bool allowed(RequestState from, RequestState to) {
  if (RequestContext::is_terminal(from)) return false;
  return ((kNext[static_cast<unsigned>(from)] | kAbort) & bit(to)) != 0;
}

template <size_t N>
const char* name_of(const char* const (&names)[N], unsigned i) {
  return i < N ? names[i] : "UNKNOWN";
}

}  // namespace

const char* to_string(RequestState state) { return name_of(kStateNames, static_cast<unsigned>(state)); }
const char* to_string(CompletionReason reason) { return name_of(kReasonNames, static_cast<unsigned>(reason)); }
const char* to_string(Owner owner) { return name_of(kOwnerNames, static_cast<unsigned>(owner)); }

RequestContext::Config RequestContext::checked(Config c) {
  const char* bad = nullptr;
  if (c.request_id.empty())
    bad = "request_id cannot be empty";
  else if (c.max_new_tokens < 0)
    bad = "max_new_tokens cannot be negative";
  else if (c.temperature < 0.0f)
    bad = "temperature cannot be negative";
  else if (!(c.top_p >= 0.0f && c.top_p <= 1.0f))
    bad = "top_p must be in range [0.0, 1.0]";
  else if (c.top_k < 0)
    bad = "top_k cannot be negative";
  else if (c.timeout < Clock::duration::zero())
    bad = "timeout cannot be negative";
  if (bad) throw RequestContextError(std::string("RequestContext ") + bad);
  return c;
}

RequestContext::RequestContext(Config config)
    : cfg_(checked(std::move(config))),
      deadline_(cfg_.timeout > Clock::duration::zero() ? Clock::now() + cfg_.timeout : Clock::time_point{}) {
  d_.owner = cfg_.initial_owner;
}

RequestContext::~RequestContext() {
  std::vector<std::function<void()>> cbs;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (!d_.cleaned) cbs = take_callbacks();
  }
  run_newest_first(cbs);
}

bool RequestContext::is_valid() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return !cfg_.request_id.empty() && !is_terminal(d_.state) && !d_.cleaned;
}

void RequestContext::ensure_executable() const {
  std::lock_guard<std::mutex> g(mu_);
  if (is_terminal(d_.state))
    throw RequestContextError(std::string("RequestContext is in terminal state: ") + to_string(d_.state));
  if (d_.cleaned) throw RequestContextError("RequestContext has already been cleaned up");
}

RequestState RequestContext::state() const {
  std::lock_guard<std::mutex> g(mu_);
  return d_.state;
}

bool RequestContext::can_transition_to(RequestState to) const {
  std::lock_guard<std::mutex> g(mu_);
  return allowed(d_.state, to);
}

void RequestContext::move_to(RequestState to) {
  if (!allowed(d_.state, to))
    throw InvalidStateTransitionError(std::string("Invalid lifecycle transition from ") + to_string(d_.state) + " to " +
                                      to_string(to) + " for request_id " + cfg_.request_id);
  d_.state = to;
}

void RequestContext::transition_to(RequestState to) {
  std::lock_guard<std::mutex> g(mu_);
  move_to(to);
}

bool RequestContext::is_terminal(RequestState s) noexcept {
  return s == RequestState::COMPLETE || s == RequestState::CANCELLED || s == RequestState::TIMED_OUT ||
         s == RequestState::FAILED;
}

bool RequestContext::is_terminal() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return is_terminal(d_.state);
}

void RequestContext::request_cancellation() noexcept { cancel_.store(true, std::memory_order_release); }

bool RequestContext::is_cancellation_requested() const noexcept { return cancel_.load(std::memory_order_acquire); }

void RequestContext::acknowledge_cancellation() {
  std::lock_guard<std::mutex> g(mu_);
  if (!cancel_.load(std::memory_order_acquire))
    throw RequestContextError("Cannot acknowledge cancellation: cancel flag is not set for request_id " +
                              cfg_.request_id);
  if (is_terminal(d_.state))
    throw InvalidStateTransitionError("Cannot acknowledge cancellation on terminal request_id " + cfg_.request_id);
  move_to(RequestState::CANCELLED);
  d_.reason = CompletionReason::CANCELLED;
}

bool RequestContext::has_deadline() const noexcept { return cfg_.timeout > Clock::duration::zero(); }

int64_t RequestContext::deadline_ns() const noexcept {
  if (!has_deadline()) return 0;
  return std::chrono::duration_cast<std::chrono::nanoseconds>(deadline_.time_since_epoch()).count();
}

bool RequestContext::is_expired(Clock::time_point now) const noexcept { return has_deadline() && now >= deadline_; }

void RequestContext::acknowledge_timeout(Clock::time_point now) {
  std::lock_guard<std::mutex> g(mu_);
  if (!has_deadline())
    throw RequestContextError("Cannot acknowledge timeout: no deadline configured for request_id " + cfg_.request_id);
  if (now < deadline_)
    throw RequestContextError("Cannot acknowledge timeout: deadline has not passed for request_id " + cfg_.request_id);
  if (is_terminal(d_.state))
    throw InvalidStateTransitionError("Cannot acknowledge timeout on terminal request_id " + cfg_.request_id);
  move_to(RequestState::TIMED_OUT);
  d_.reason = CompletionReason::TIMEOUT;
}

Owner RequestContext::current_owner() const {
  std::lock_guard<std::mutex> g(mu_);
  return d_.owner;
}

void RequestContext::transfer_ownership(Owner new_owner, Owner expected_current_owner) {
  std::lock_guard<std::mutex> g(mu_);
  if (is_terminal(d_.state))
    throw RequestOwnershipError("Cannot transfer ownership of terminal request_id " + cfg_.request_id);
  if (d_.owner != expected_current_owner)
    throw RequestOwnershipError("Ownership transfer failed for request_id " + cfg_.request_id + ": expected owner " +
                                to_string(expected_current_owner) + " but actual owner is " + to_string(d_.owner));
  d_.owner = new_owner;
}

void RequestContext::append_generated_token(int32_t token_id) {
  std::lock_guard<std::mutex> g(mu_);
  d_.generated.push_back(token_id);
}

std::vector<int32_t> RequestContext::generated_tokens() const {
  std::lock_guard<std::mutex> g(mu_);
  return d_.generated;
}

void RequestContext::set_input_device_ptr(uintptr_t ptr) {
  if (!ptr) throw RequestContextError("Null device pointer rejected for input_device_ptr");
  std::lock_guard<std::mutex> g(mu_);
  d_.input_ptr = ptr;
}

void RequestContext::set_output_device_ptr(uintptr_t ptr) {
  if (!ptr) throw RequestContextError("Null device pointer rejected for output_device_ptr");
  std::lock_guard<std::mutex> g(mu_);
  d_.output_ptr = ptr;
}

uintptr_t RequestContext::input_device_ptr() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.input_ptr;
}

uintptr_t RequestContext::output_device_ptr() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.output_ptr;
}

void RequestContext::add_kv_block_id(int block_id) {
  std::lock_guard<std::mutex> g(mu_);
  d_.kv_blocks.push_back(block_id);
}

void RequestContext::set_kv_block_ids(std::vector<int> block_ids) {
  std::lock_guard<std::mutex> g(mu_);
  d_.kv_blocks = std::move(block_ids);
}

std::vector<int> RequestContext::kv_block_ids() const {
  std::lock_guard<std::mutex> g(mu_);
  return d_.kv_blocks;
}

void RequestContext::set_kv_block_table_handle(KVBlockTable* handle) {
  std::lock_guard<std::mutex> g(mu_);
  d_.kv_table = handle;
}

KVBlockTable* RequestContext::kv_block_table_handle() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.kv_table;
}

void RequestContext::set_tokenizer_ref(Tokenizer* tokenizer_ref) {
  std::lock_guard<std::mutex> g(mu_);
  if (d_.tokenizer && d_.tokenizer != tokenizer_ref)
    throw RequestContextError("Tokenizer reference already bound to a different instance");
  d_.tokenizer = tokenizer_ref;
}

Tokenizer* RequestContext::tokenizer_ref() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.tokenizer;
}

void RequestContext::set_logical_decode_state(LogicalDecodeState* state) {
  std::lock_guard<std::mutex> g(mu_);
  d_.decode_state = state;
}

LogicalDecodeState* RequestContext::logical_decode_state() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.decode_state;
}

void RequestContext::set_session_sequence(uint64_t sequence) noexcept {
  std::lock_guard<std::mutex> g(mu_);
  d_.session_sequence = sequence;
}

uint64_t RequestContext::session_sequence() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.session_sequence;
}

void RequestContext::set_finish_reason(CompletionReason reason) {
  std::lock_guard<std::mutex> g(mu_);
  d_.reason = reason;
}

CompletionReason RequestContext::finish_reason() const {
  std::lock_guard<std::mutex> g(mu_);
  return d_.reason;
}

void RequestContext::set_error_code(int code) noexcept {
  std::lock_guard<std::mutex> g(mu_);
  d_.error_code = code;
}

int RequestContext::error_code() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.error_code;
}

void RequestContext::register_cleanup_callback(std::function<void()> callback) {
  std::lock_guard<std::mutex> g(mu_);
  if (d_.cleaned) throw RequestContextError("Cannot register cleanup callback on already cleaned up RequestContext");
  d_.callbacks.push_back(std::move(callback));
}

bool RequestContext::is_cleaned_up() const noexcept {
  std::lock_guard<std::mutex> g(mu_);
  return d_.cleaned;
}

std::vector<std::function<void()>> RequestContext::take_callbacks() {
  d_.cleaned = true;
  std::vector<std::function<void()>> cbs;
  cbs.swap(d_.callbacks);
  return cbs;
}

void RequestContext::run_newest_first(std::vector<std::function<void()>>& cbs) {
  while (!cbs.empty()) {
    std::function<void()> f = std::move(cbs.back());
    cbs.pop_back();
    if (!f) continue;
    try {
      f();
    } catch (...) {
      // a failing callback must not stop the others, nor escape teardown
    }
  }
}

bool RequestContext::cleanup() {
  std::vector<std::function<void()>> cbs;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (!is_terminal(d_.state))
      throw RequestContextError(
          std::string("Cannot cleanup RequestContext before reaching terminal state (current state: ") +
          to_string(d_.state) + ")");
    if (d_.cleaned) return false;
    cbs = take_callbacks();
  }
  run_newest_first(cbs);
  return true;
}
