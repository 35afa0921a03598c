"""kinetic_rt -- B200-native decoder hot path behind Kinetic-RT's API.

Same public names as the reference package (python/kinetic_rt/__init__.py:1-23).
The native module is `_core` (CUDA).  Setting KINETIC_MOCK_CUDA=1 selects
`_core_mock`, the same host runtime built over a host-only test double of the
CUDA runtime, for headless tests of host-side logic; it runs no kernels.
"""
import os

from .hardware_probe import get_topology_string

try:
    if os.environ.get("KINETIC_MOCK_CUDA") == "1":
        from . import _core_mock as _native
    else:
        from . import _core as _native
except ImportError as e:  # pragma: no cover - exercised only on broken installs
    raise ImportError("Unable to load the kinetic_rt native module; build it with kinetic-rt_b200/build.py") from e

AOTEngine = _native.AOTEngine
GraphWrapper = _native.GraphWrapper
Serializer = _native.Serializer
Communicator = _native.Communicator
HardwareMismatchError = _native.HardwareMismatchError
HardwareRouter = _native.HardwareRouter
InferenceQueue = _native.InferenceQueue
InferenceWorker = _native.InferenceWorker
TensorDescriptor = _native.TensorDescriptor
DataType = _native.DataType
KernelLaunchDescriptor = _native.KernelLaunchDescriptor
BlockManager = _native.BlockManager
RequestContext = _native.RequestContext
RequestState = _native.RequestState
CompletionReason = _native.CompletionReason
Owner = _native.Owner
RequestContextError = _native.RequestContextError
InvalidStateTransitionError = _native.InvalidStateTransitionError
RequestOwnershipError = _native.RequestOwnershipError
MOCK_CUDA = _native.MOCK_CUDA


class TopologyMismatchError(Exception):
    pass


from .orchestrator import KineticRuntime, StreamContext, validate_tensor_for_zero_copy, TensorValidationError  # noqa: E402
from .serve import serve  # noqa: E402
