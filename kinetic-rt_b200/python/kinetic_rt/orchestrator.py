"""Host-side helpers around the hot path (python/kinetic_rt/orchestrator.py of
the reference, reduced to what callers of the hot path use): the zero-copy and
device-residency checks applied before pointers cross into native code, the
stream context, and a runtime that loads .kin artifacts, checks their TP
degree and generates tokens through an attached paged decoder
(decoder.PagedDecoder): the reference's loop (orchestrator.py:419-448)
re-runs the whole model per token; here every token is one graph-replayed
decode step that reuses the cached K/V.
"""
import glob
import os


class DeviceMismatchError(ValueError):
    pass


class TensorValidationError(ValueError):
    pass


class RuntimeConfigurationError(ValueError):
    pass


class ContextWindowExceededError(RuntimeConfigurationError):
    pass


def _env_flag_enabled(name):
    return os.environ.get(name, "").strip().lower() in ("1", "true", "yes", "on")


def allows_mock_device_residency():
    return _env_flag_enabled("KINETIC_ALLOW_MOCKS") or _env_flag_enabled("KINETIC_MOCK_CUDA")


def validate_tensor_device_residency(tensor, *, name="tensor", allow_mock=None):
    """The tensor must live on a CUDA device (unless mocks are allowed)."""
    try:
        import torch
    except ImportError as e:
        raise RuntimeError("PyTorch is required to validate tensor device residency.") from e
    if not isinstance(tensor, torch.Tensor):
        raise DeviceMismatchError(f"{name}: expected torch.Tensor for device residency validation.")
    if allow_mock is None:
        allow_mock = allows_mock_device_residency()
    if not tensor.is_cuda and not allow_mock:
        raise DeviceMismatchError(f"{name}: tensor must reside on a CUDA device, found {tensor.device}.")
    return tensor


def validate_tensor_for_zero_copy(tensor, *, expected_dtype, name="tensor"):
    """Contiguous, offset-free, dtype-checked, non-empty; returns data_ptr()."""
    try:
        import torch
    except ImportError as e:
        raise RuntimeError("PyTorch is required for zero-copy validation.") from e
    if not isinstance(tensor, torch.Tensor):
        raise TensorValidationError(f"{name}: expected torch.Tensor, got {type(tensor).__name__}.")
    if tensor.dtype != expected_dtype:
        raise TensorValidationError(f"{name}: expected dtype {expected_dtype}, got {tensor.dtype}.")
    if not tensor.is_contiguous():
        raise TensorValidationError(f"{name}: tensor must be contiguous (call .contiguous()).")
    if tensor.storage_offset() != 0:
        raise TensorValidationError(f"{name}: storage_offset must be 0, got {tensor.storage_offset()}.")
    if tensor.numel() == 0:
        raise TensorValidationError(f"{name}: empty tensors cannot cross the zero-copy boundary.")
    ptr = tensor.data_ptr()
    if ptr == 0:
        raise TensorValidationError(f"{name}: data_ptr() returned 0 (null).")
    return ptr


class StreamContext:
    """Runs a block on a dedicated CUDA stream (or a no-op without CUDA)."""

    def __init__(self):
        self.stream = None
        try:
            import torch
            if torch.cuda.is_available():
                self.stream = torch.cuda.Stream()
        except ImportError:
            pass
        self._ctx = None

    def __enter__(self):
        if self.stream is not None:
            import torch
            self._ctx = torch.cuda.stream(self.stream)
            self._ctx.__enter__()
        return self

    def __exit__(self, exc_type, exc, tb):
        if self._ctx is not None:
            self._ctx.__exit__(exc_type, exc, tb)
        return False


class KineticRuntime:
    """Loads .kin artifacts and checks the tensor-parallel degree."""

    def __init__(self, max_seq_len=2048):
        from . import AOTEngine, Serializer
        self.engine = AOTEngine()
        self.serializer = Serializer()
        self.max_seq_len = int(max_seq_len)
        self.model_path = None
        self.decoder, self.tokenizer, self._graph = None, None, None

    def load_model(self, model_dir, tensor_parallel_degree=1):
        kins = sorted(glob.glob(os.path.join(model_dir, "*.kin")))
        if not kins:
            raise FileNotFoundError(f"no .kin artifact in {model_dir}")
        tp = self.serializer.get_tensor_parallel_degree(kins[0])
        if tp != tensor_parallel_degree:
            raise RuntimeConfigurationError(f"artifact built for TP={tp}, runtime configured for TP={tensor_parallel_degree}")
        self.engine.load_model(kins[0])
        self.model_path = kins[0]
        return kins[0]

    def attach_decoder(self, decoder, tokenizer=None):
        """A decoder.PagedDecoder (batch 1) that generate() drives; `tokenizer`
        is any object with encode(str) -> ids and decode(ids) -> str."""
        if decoder.B != 1:
            raise RuntimeConfigurationError("generate() drives a decoder of batch 1")
        self.decoder, self.tokenizer = decoder, tokenizer
        self._graph = None

    def encode_prompt(self, prompt):
        """Token ids of the prompt: the tokenizer's, else its UTF-8 bytes (the
        reference's fallback, orchestrator.py:303-313)."""
        ids = self.tokenizer.encode(prompt) if getattr(self, "tokenizer", None) else list(prompt.encode("utf-8"))
        return [int(t) for t in ids]

    def generate_ids(self, prompt_ids, max_new_tokens=10, request=None):
        """Greedy continuation of `prompt_ids` (a list of ints): the prompt is
        fed one token per decode step (its K/V cached as it goes), then each
        step's argmax (orchestrator.py:442-444) becomes the next input.
        Returns the new token ids.

        With `request` (a RequestContext of the runtime module) the call drives
        its lifecycle: RECEIVED -> VALIDATED -> TOKENIZED -> ENQUEUED (ownership
        to the executor) -> PREFILL while the prompt is fed -> DECODE <->
        STREAMING per generated token (each appended to the context) ->
        COMPLETE with reason LENGTH (the context's max_new_tokens, when set,
        replaces the argument) or STOP_TOKEN (a token in its stop_token_ids).
        Between steps it honours a cancellation request (acknowledged ->
        CANCELLED) and the deadline (-> TIMED_OUT), returning the tokens made
        so far; an exception moves the context to FAILED.  The context records
        the sequence's KV block ids and is cleaned up when it ends."""
        dec = getattr(self, "decoder", None)
        if dec is None:
            raise RuntimeConfigurationError("no decoder attached (KineticRuntime.attach_decoder)")
        if request is not None and request.max_new_tokens > 0:
            max_new_tokens = request.max_new_tokens
        if not prompt_ids:
            raise RuntimeConfigurationError("empty prompt")
        if len(prompt_ids) + max_new_tokens > dec.max_seq_len:
            raise ContextWindowExceededError("prompt and new tokens exceed the decoder's max_seq_len")
        if request is None:
            return self._generate(dec, prompt_ids, max_new_tokens, None)
        from . import RequestState as S, Owner, CompletionReason
        try:
            for st in (S.VALIDATED, S.TOKENIZED, S.ENQUEUED):
                request.transition_to(st)
            request.transfer_ownership(Owner.Executor, request.current_owner())
            request.set_kv_block_ids([int(b) for b in dec.block_table[0].tolist()])
            request.transition_to(S.PREFILL)
            out = self._generate(dec, prompt_ids, max_new_tokens, request)
        except Exception:
            if not request.is_terminal():
                request.set_error_code(1)
                request.set_finish_reason(CompletionReason.ERROR)
                request.transition_to(S.FAILED)
            request.cleanup()
            raise
        request.cleanup()
        return out

    def _generate(self, dec, prompt_ids, max_new_tokens, request):
        torch = dec.torch
        dec.start([prompt_ids[0]], [0])
        if self._graph is None:
            self._graph = dec.capture()
        steps = len(prompt_ids) - 1 + max_new_tokens
        # one pinned slot per step: a slot is not rewritten while its copy may still be queued
        feed = torch.tensor([prompt_ids[i + 1] if i + 1 < len(prompt_ids) else -1 for i in range(steps)],
                            dtype=torch.int32)
        if torch.cuda.is_available():
            feed = feed.pin_memory()
        stop = set(request.stop_token_ids) if request is not None else set()
        out = []
        for i in range(steps):
            if request is not None and self._request_over(request):
                break
            dec.next_input.copy_(feed[i:i + 1], non_blocking=True)
            self._graph.replay()
            if i + 1 >= len(prompt_ids):
                tok = int(dec.tokens[0].item())
                out.append(tok)
                if request is not None:
                    from . import RequestState as S, CompletionReason
                    if request.state() == S.PREFILL:
                        request.transition_to(S.DECODE)
                    request.append_generated_token(tok)
                    request.transition_to(S.STREAMING)
                    if tok in stop or len(out) == max_new_tokens:
                        request.set_finish_reason(CompletionReason.STOP_TOKEN if tok in stop
                                                  else CompletionReason.LENGTH)
                        request.transition_to(S.COMPLETE)
                        break
                    request.transition_to(S.DECODE)
        dec.check_status()
        return out

    @staticmethod
    def _request_over(request):
        """Cancellation and deadline checks between decode steps."""
        if request.is_cancellation_requested():
            request.acknowledge_cancellation()
            return True
        if request.is_expired():
            request.acknowledge_timeout()
            return True
        return False

    def generate(self, prompt, max_new_tokens=10):
        """Text in, text out (the reference's generate, orchestrator.py:419-448)."""
        ids = self.encode_prompt(prompt)
        ids = ids + self.generate_ids(ids, max_new_tokens)
        if getattr(self, "tokenizer", None):
            return self.tokenizer.decode(ids)
        return bytes(t % 256 for t in ids).decode("utf-8", errors="replace")
