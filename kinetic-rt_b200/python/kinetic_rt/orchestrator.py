"""Host-side helpers around the hot path (python/kinetic_rt/orchestrator.py of
the reference, reduced to what callers of the hot path use): the zero-copy and
device-residency checks applied before pointers cross into native code, the
stream context, and a runtime that loads .kin artifacts and checks their TP
degree.  The reference's token-generation loop re-runs a full model that it
does not have; that loop is outside this build (generate() says so).
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

    def generate(self, prompt, max_tokens=16):
        raise NotImplementedError("token generation over a full decoder stack is outside this build's hot path")
