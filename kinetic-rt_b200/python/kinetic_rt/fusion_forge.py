"""Fused RMSNorm + QKV + RoPE launcher and the .kin AOT bridge.

Same public surface as the reference's python/kinetic_rt/fusion_forge.py:
  * `fused_rmsnorm_qkv_rope[grid](x, W, b, gamma, cos, sin, q, k, v, seq_len,
    d_model, n_heads, head_dim, eps, <10 strides>, BLOCK_DIM=...)` -- the
    Triton kernel's call shape (fusion_forge.py:21-31), here forwarded to the
    CUDA kernel in libkrt (krt_fused_rmsnorm_qkv_rope).  Any d_model (the
    Triton kernel silently breaks above 128); RoPE is applied per head, which
    is the reference computation exactly when n_heads == 1.  Host tensors are
    staged to the current CUDA device with their strides and results copied
    back; without a CUDA device the call raises -- there is no CPU fallback.
  * validate_compilation / _validate_ir and their exception types
    (fusion_forge.py:165-259), KernelRegistry and the kernel signature
    (264-325), the test-only mock ELF (332-344), compile_and_serialize
    (538-575), native_triton_compile and get_op_graph_data (479-598).
The .kin artifacts carry this build's own sm_100a cubin of the kernel
(aot_kernel.cu) instead of a Triton binary.
"""
import functools
import hashlib
import json
import logging
import os
import struct

from .hardware_probe import probe_hardware

logger = logging.getLogger(__name__)

_artifact_kind = "production"
KERNEL_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kernels")
KERNEL_CUBIN = os.path.join(KERNEL_DIR, "fused_rmsnorm_qkv_rope.sm_100a.cubin")

SUPPORTED_FX_OPS = {"placeholder", "call_function", "call_method", "call_module", "get_attr", "output"}


# ------------------------------------------------------------------ launcher
class _FusedLauncher:
    """`fused_rmsnorm_qkv_rope[grid](...)`.  The grid is accepted for call
    compatibility; the CUDA kernel strides over tokens itself."""

    def __getitem__(self, grid):
        return functools.partial(self._launch, grid)

    @staticmethod
    def _launch(grid, x_ptr, qkv_weight_ptr, qkv_bias_ptr, rms_weight_ptr, freqs_cos_ptr, freqs_sin_ptr,
                q_out_ptr, k_out_ptr, v_out_ptr, seq_len, d_model, n_heads, head_dim, eps,
                stride_x_seq, stride_x_dim, stride_w_out, stride_w_in, stride_q_seq, stride_q_dim,
                stride_k_seq, stride_k_dim, stride_v_seq, stride_v_dim, BLOCK_DIM=None, **_):
        import torch
        from . import _lib
        if not torch.cuda.is_available():
            raise RuntimeError("fused_rmsnorm_qkv_rope runs on a CUDA device and none is available")
        dev = torch.device("cuda", torch.cuda.current_device())

        def stage(t):
            if t is None or (t.is_cuda and t.device == dev):
                return t
            s = torch.empty_strided(t.size(), t.stride(), dtype=t.dtype, device=dev)
            s.copy_(t)
            return s

        ins = [stage(t) for t in (x_ptr, qkv_weight_ptr, qkv_bias_ptr, rms_weight_ptr, freqs_cos_ptr, freqs_sin_ptr)]
        outs = [stage(t) for t in (q_out_ptr, k_out_ptr, v_out_ptr)]
        strides = (stride_x_seq, stride_x_dim, stride_w_out, stride_w_in, stride_q_seq, stride_q_dim,
                   stride_k_seq, stride_k_dim, stride_v_seq, stride_v_dim)
        _lib.fused_rmsnorm_qkv_rope(*ins, *outs, seq_len, d_model, n_heads, head_dim, eps, strides)
        for host, devt in zip((q_out_ptr, k_out_ptr, v_out_ptr), outs):
            if devt is not host:
                host.copy_(devt)
        if any(t is not None and not t.is_cuda for t in (q_out_ptr, k_out_ptr, v_out_ptr)):
            torch.cuda.current_stream().synchronize()


fused_rmsnorm_qkv_rope = _FusedLauncher()


# --------------------------------------------------------------- validation
class TritonCompilationError(Exception):
    """Compilation or binary-validation failure (name kept for callers)."""

    def __init__(self, message, context=None):
        self.message = message
        self.context = context or {}
        full = message + (f" | Context: {json.dumps(self.context, default=str)}" if self.context else "")
        logger.error("TritonCompilationError: %s", full)
        super().__init__(full)


class IRValidationError(Exception):
    def __init__(self, message, context=None):
        self.message = message
        self.context = context or {}
        full = f"IRValidationError: {message}" + (
            f" | Context: {json.dumps(self.context, default=str)}" if self.context else "")
        logger.error(full)
        super().__init__(full)


def _validate_ir(ir):
    """Structural checks of an op-graph descriptor dict or a torch.fx graph."""
    if isinstance(ir, dict):
        if not isinstance(ir.get("artifact_kind"), str):
            raise IRValidationError("Missing or invalid 'artifact_kind' in IR dictionary.", {"ir_keys": list(ir)})
        if not isinstance(ir.get("graph"), list):
            raise IRValidationError("Missing or invalid 'graph' list in IR dictionary.", {"ir_keys": list(ir)})
        if not isinstance(ir.get("version"), int):
            raise IRValidationError("Missing or invalid 'version' integer in IR dictionary.", {"ir_keys": list(ir)})
        if ir["version"] != 1:
            raise IRValidationError(f"Unsupported IR version: {ir['version']}. Expected 1.", {"version": ir["version"]})
        if not ir["graph"]:
            raise IRValidationError("Graph structure is empty.", {})
        for node in ir["graph"]:
            if not isinstance(node, str) or not node.strip():
                raise IRValidationError(f"Malformed or empty node entry in graph: {node}", {"node": node})
        return True
    try:
        import torch.fx as fx
    except ImportError as e:
        raise IRValidationError(f"Unsupported IR type for validation: {type(ir)}", {"type": str(type(ir))}) from e
    if isinstance(ir, (fx.Graph, fx.GraphModule)):
        graph = ir if isinstance(ir, fx.Graph) else ir.graph
        nodes = list(graph.nodes)
        if not nodes:
            raise IRValidationError("torch.fx.Graph contains no nodes.", {})
        node_set = set(nodes)
        for node in nodes:
            if not node.name:
                raise IRValidationError("Node is missing a valid name.", {"node": str(node)})
            if node.op not in SUPPORTED_FX_OPS:
                raise IRValidationError(
                    f"Un-fusable or unsupported operation breaking compilation boundaries: {node.op}",
                    {"node": node.name, "op": node.op})

            def check(arg, node=node):
                if isinstance(arg, fx.Node) and arg not in node_set:
                    raise IRValidationError(
                        f"Dangling reference detected: node '{node.name}' references missing node '{arg.name}'.",
                        {"node": node.name, "dangling_ref": arg.name})
            fx.node.map_arg(node.args, check)
            fx.node.map_arg(node.kwargs, check)
        return True
    raise IRValidationError(f"Unsupported IR type for validation: {type(ir)}", {"type": str(type(ir))})


def validate_compilation(compiled_binary, backend):
    """ELF sanity checks of a kernel image (messages as the reference)."""
    if not compiled_binary:
        raise TritonCompilationError("Triton compilation yielded an empty binary.")
    if not compiled_binary.startswith(b"\x7fELF"):
        raise TritonCompilationError("Triton binary lacks the standard ELF magic header.")
    if len(compiled_binary) < 20:
        raise TritonCompilationError("Triton binary is too short to be a valid ELF.")
    if compiled_binary[4] != 2:
        raise TritonCompilationError("Triton binary is not a 64-bit ELF.")
    machine = compiled_binary[18:20]
    if backend == "CUDA" and machine != b"\xBE\x00":
        raise TritonCompilationError("Triton binary architecture is not CUDA.")
    if backend == "ROCm" and machine != b"\xE0\x00":
        raise TritonCompilationError("Triton binary architecture is not AMDGPU.")


# ---------------------------------------------------------------- registry
class KernelRegistry:
    _kernels = {}

    @classmethod
    def register(cls, name, kernel_fn, signature, constants=None, grid=None):
        cls._kernels[name] = {"fn": kernel_fn, "signature": signature, "constants": constants or {}, "grid": grid}

    @classmethod
    def get_all(cls):
        return cls._kernels

    @classmethod
    def get(cls, name):
        return cls._kernels.get(name)


_FUSED_KERNEL_SIGNATURE = {
    "x_ptr": "*fp32", "qkv_weight_ptr": "*fp32", "qkv_bias_ptr": "*fp32", "rms_weight_ptr": "*fp32",
    "freqs_cos_ptr": "*fp32", "freqs_sin_ptr": "*fp32", "q_out_ptr": "*fp32", "k_out_ptr": "*fp32",
    "v_out_ptr": "*fp32", "seq_len": "i32", "d_model": "i32", "n_heads": "i32", "head_dim": "i32", "eps": "fp32",
    "stride_x_seq": "i32", "stride_x_dim": "i32", "stride_w_out": "i32", "stride_w_in": "i32",
    "stride_q_seq": "i32", "stride_q_dim": "i32", "stride_k_seq": "i32", "stride_k_dim": "i32",
    "stride_v_seq": "i32", "stride_v_dim": "i32",
}

KernelRegistry.register("fused_rmsnorm_qkv_rope", fused_rmsnorm_qkv_rope, _FUSED_KERNEL_SIGNATURE,
                        constants={"BLOCK_DIM": 128}, grid=(1,))


def _build_test_only_mock_elf(backend):
    """A structurally valid 64-byte ELF header for tests (never loadable)."""
    elf = bytearray(64)
    elf[0:4] = b"\x7fELF"
    elf[4] = 2
    elf[5] = 1
    elf[6] = 1
    elf[18:20] = b"\xBE\x00" if backend == "CUDA" else b"\xE0\x00"
    return bytes(elf)


def _compute_weights_hash(model, kwargs):
    """uint64 from a SHA-256 over a model's state dict (or the kwargs)."""
    if model is None and "weights_hash" in kwargs:
        return int(kwargs["weights_hash"])
    h = hashlib.sha256()
    if model is not None:
        try:
            sd = model.state_dict()
            for name in sorted(sd):
                h.update(name.encode())
                h.update(sd[name].detach().cpu().numpy().tobytes())
        except Exception:
            h.update(repr(model).encode())
    else:
        h.update(repr(sorted(kwargs.items())).encode())
    return struct.unpack("<Q", h.digest()[:8])[0]


def _compile_kernel_binary(kinetic_target, backend):
    """The kernel image for `kinetic_target`: this build's sm_100a cubin for
    CUDA targets, a mock ELF (artifact kind "mock") for anything else."""
    global _artifact_kind
    if backend == "CUDA" and os.path.exists(KERNEL_CUBIN):
        with open(KERNEL_CUBIN, "rb") as f:
            binary = f.read()
        _artifact_kind = "production"
        return binary
    logger.warning("no sm_100a kernel image for %s; producing a mock ELF", kinetic_target)
    _artifact_kind = "mock"
    return _build_test_only_mock_elf(backend)


def _build_op_graph_data(model):
    if model is None:
        return {"artifact_kind": _artifact_kind, "graph": ["placeholder"], "version": 1}
    try:
        import torch
        gm = torch.fx.symbolic_trace(model)
        _validate_ir(gm)
        return {"artifact_kind": _artifact_kind, "graph": [n.name for n in gm.graph.nodes], "version": 1}
    except IRValidationError:
        raise
    except Exception as exc:
        logger.warning("torch.fx tracing failed (%s); minimal op graph", exc)
        return {"artifact_kind": _artifact_kind, "graph": ["fallback"], "version": 1}


def native_triton_compile(kinetic_target, kernel_fn=None):
    """Kernel image bytes for `kinetic_target` (name kept for callers)."""
    backend = "CUDA" if "CUDA" in kinetic_target or "sm" in kinetic_target else "ROCm"
    return _compile_kernel_binary(kinetic_target, backend)


def compile_and_serialize(engine, serializer, output_filepath, device_id=None, model=None, **kwargs):
    """Write a .kin file holding the fused kernel image for the probed target."""
    topology, backend, target = probe_hardware()
    kinetic_target = f"{backend}_{target}" if backend != "CPU" else "CPU_CPU"
    if device_id is None:
        device_id = target
    weights_hash = _compute_weights_hash(model, kwargs)
    binary = _compile_kernel_binary(kinetic_target, backend)
    op_graph = _build_op_graph_data(model)
    _validate_ir(op_graph)
    serializer.save_kin_file(output_filepath, device_id, kinetic_target, weights_hash,
                             list(json.dumps(op_graph).encode()), list(binary))
    logger.info("compiled and serialized %s", output_filepath)


def get_op_graph_data(kinetic_target):
    return json.dumps({"target": kinetic_target, "kernels": list(KernelRegistry.get_all()), "version": 1,
                       "artifact_kind": _artifact_kind}).encode()
