"""RequestContext (kinetic-rt_b200/csrc/runtime/RequestContext.cpp) through the
Python binding of the host runtime, and its wiring into the decode driver
(KineticRuntime.generate_ids) with a scripted stand-in for the GPU decoder.
The lifecycle semantics follow the reference's include/RequestContext.h
(src/RequestContext.cpp:45-393); its own C++ test runs unmodified through
tests/run_reference_suite.py --cpp."""
import time
import types

import pytest
import torch

import python.kinetic_rt._core_mock as krt


def test_lifecycle_and_errors():
    r = krt.RequestContext("req", max_new_tokens=4, top_k=5, timeout_s=0.0)
    assert r.state() == krt.RequestState.RECEIVED and r.current_owner() == krt.Owner.Ingress
    assert not r.has_deadline() and r.is_valid()
    with pytest.raises(krt.InvalidStateTransitionError, match="Invalid lifecycle transition"):
        r.transition_to(krt.RequestState.PREFILL)  # skips stages
    for st in ("VALIDATED", "TOKENIZED", "ENQUEUED", "PREFILL", "DECODE", "STREAMING", "DECODE", "STREAMING",
               "COMPLETE"):
        r.transition_to(getattr(krt.RequestState, st))
    assert r.is_terminal() and not r.is_valid()
    with pytest.raises(krt.InvalidStateTransitionError):
        r.transition_to(krt.RequestState.FAILED)  # nothing leaves a terminal state
    with pytest.raises(krt.RequestOwnershipError, match="terminal"):
        r.transfer_ownership(krt.Owner.Executor, krt.Owner.Ingress)
    for bad, msg in ((dict(request_id=""), "request_id cannot be empty"),
                     (dict(request_id="x", top_p=1.5), "top_p"),
                     (dict(request_id="x", max_new_tokens=-1), "max_new_tokens")):
        with pytest.raises(krt.RequestContextError, match=msg):
            krt.RequestContext(**bad)


def test_cancellation_timeout_ownership_cleanup():
    r = krt.RequestContext("c")
    with pytest.raises(krt.RequestContextError, match="cancel flag is not set"):
        r.acknowledge_cancellation()
    r.request_cancellation()
    assert r.state() == krt.RequestState.RECEIVED  # two-phase: nothing moves until acknowledged
    r.acknowledge_cancellation()
    assert r.state() == krt.RequestState.CANCELLED and r.finish_reason() == krt.CompletionReason.CANCELLED

    t = krt.RequestContext("t", timeout_s=0.02)
    assert t.has_deadline() and not t.is_expired()
    with pytest.raises(krt.RequestContextError, match="deadline has not passed"):
        t.acknowledge_timeout()
    time.sleep(0.03)
    assert t.is_expired()
    t.acknowledge_timeout()
    assert t.state() == krt.RequestState.TIMED_OUT and t.finish_reason() == krt.CompletionReason.TIMEOUT

    o = krt.RequestContext("o")
    o.transfer_ownership(krt.Owner.Scheduler, krt.Owner.Ingress)
    with pytest.raises(krt.RequestOwnershipError, match="Ownership transfer failed"):
        o.transfer_ownership(krt.Owner.Backend, krt.Owner.Ingress)
    order = []
    o.register_cleanup_callback(lambda: order.append(1))
    o.register_cleanup_callback(lambda: order.append(2))
    with pytest.raises(krt.RequestContextError, match="before reaching terminal state"):
        o.cleanup()
    o.transition_to(krt.RequestState.FAILED)
    assert o.cleanup() and order == [2, 1]  # newest first
    assert not o.cleanup() and order == [2, 1]  # once


class FakeDecoder:
    """The parts of PagedDecoder that generate_ids uses; each replay 'chooses'
    the next scripted token.  on_step(i) runs inside replay i."""

    def __init__(self, script, on_step=None):
        self.torch = torch
        self.B, self.max_seq_len = 1, 64
        self.block_table = torch.tensor([[7, 3, 9]], dtype=torch.int32)
        self.next_input = torch.full((1,), -1, dtype=torch.int32)
        self.tokens = torch.zeros(1, dtype=torch.int32)
        self.script, self.on_step, self.replays = list(script), on_step, 0

    def start(self, toks, pos):
        pass

    def capture(self):
        def replay():
            if self.on_step:
                self.on_step(self.replays)
            self.tokens[0] = self.script[self.replays % len(self.script)]
            self.replays += 1
        return types.SimpleNamespace(replay=replay)

    def check_status(self):
        pass


def _runtime(dec):
    import python.kinetic_rt.orchestrator as orch
    rt = orch.KineticRuntime.__new__(orch.KineticRuntime)
    rt.attach_decoder(dec)
    return rt


@pytest.fixture
def mock_package(monkeypatch):
    """The package's runtime names resolve to the host-only module."""
    import python.kinetic_rt as pkg
    for name in ("RequestState", "Owner", "CompletionReason"):
        monkeypatch.setattr(pkg, name, getattr(krt, name))


def test_generate_ids_drives_the_request_to_length(mock_package):
    dec = FakeDecoder([11, 12, 13, 14, 15, 16])
    req = krt.RequestContext("g", max_new_tokens=3)
    freed = []
    req.register_cleanup_callback(lambda: freed.append(True))
    out = _runtime(dec).generate_ids([1, 2, 3], max_new_tokens=10, request=req)
    # 2 prompt steps then 3 generated tokens (the context's max_new_tokens wins)
    assert out == [13, 14, 15] and req.generated_tokens() == out
    assert req.state() == krt.RequestState.COMPLETE and req.finish_reason() == krt.CompletionReason.LENGTH
    assert req.current_owner() == krt.Owner.Executor and req.kv_block_ids() == [7, 3, 9]
    assert req.is_cleaned_up() and freed == [True]


def test_generate_ids_stops_on_a_stop_token(mock_package):
    dec = FakeDecoder([5, 6, 42, 7])
    req = krt.RequestContext("s", stop_token_ids=[42])
    out = _runtime(dec).generate_ids([1], max_new_tokens=8, request=req)
    assert out == [5, 6, 42]
    assert req.state() == krt.RequestState.COMPLETE and req.finish_reason() == krt.CompletionReason.STOP_TOKEN


def test_generate_ids_honours_cancellation_between_steps(mock_package):
    req = krt.RequestContext("x")
    dec = FakeDecoder([21, 22, 23, 24], on_step=lambda i: req.request_cancellation() if i == 1 else None)
    out = _runtime(dec).generate_ids([1], max_new_tokens=8, request=req)
    assert out == [21, 22]  # the step in flight finishes; the next one does not start
    assert req.state() == krt.RequestState.CANCELLED and req.is_cleaned_up()


def test_generate_ids_honours_the_deadline(mock_package):
    req = krt.RequestContext("d", timeout_s=0.05)
    dec = FakeDecoder([31, 32, 33, 34, 35], on_step=lambda i: time.sleep(0.03))
    out = _runtime(dec).generate_ids([1], max_new_tokens=5, request=req)
    assert 1 <= len(out) < 5
    assert req.state() == krt.RequestState.TIMED_OUT and req.finish_reason() == krt.CompletionReason.TIMEOUT


def test_generate_ids_marks_a_failure(mock_package):
    req = krt.RequestContext("f")

    def boom(i):
        if i == 2:
            raise RuntimeError("kernel status 0x10")
    dec = FakeDecoder([1, 2, 3, 4], on_step=boom)
    with pytest.raises(RuntimeError, match="kernel status"):
        _runtime(dec).generate_ids([1], max_new_tokens=4, request=req)
    assert req.state() == krt.RequestState.FAILED and req.error_code() == 1 and req.is_cleaned_up()
