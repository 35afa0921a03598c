"""Argument validation of the C ABI (include/krt.h), exercised on the CPU.

Every case below is rejected by host-side checks before any CUDA call, so the
test runs without a GPU: the status code and the krt_last_error() message
follow the reference's conventions (std::invalid_argument -> ValueError for
malformed descriptors, bindings/python_bindings.cpp; "unsupported" for shapes
the kernels do not cover).  Pointers are fake, 16-byte-aligned integers that
are never dereferenced.
"""
import ctypes
import os

import pytest

from python.kinetic_rt import _lib

pytestmark = pytest.mark.skipif(not os.path.exists(_lib.LIB_PATH), reason="libkrt.so not built")

FAKE = 0x10000  # aligned, never dereferenced


def _paged(**over):
    a = _lib.QkvPagedArgs()
    for name in ("x", "qkv_weight", "rms_weight", "rope_cos", "rope_sin", "positions", "token_seq",
                 "block_table", "kv_pool", "q_out", "workspace"):
        setattr(a, name, FAKE)
    a.num_tokens, a.d_model, a.n_heads, a.n_kv_heads, a.head_dim = 64, 4096, 32, 8, 128
    a.x_stride, a.q_stride, a.max_position = 4096, 4096, 2048
    a.num_seqs, a.block_table_stride, a.num_blocks, a.tokens_per_block = 64, 128, 8192, 16
    a.eps, a.workspace_bytes = 1e-5, 1 << 30
    for k, v in over.items():
        setattr(a, k, v)
    return a


def _call(fn, *args):
    h = _lib.lib()
    rc = getattr(h, fn)(*args)
    return rc, h.krt_last_error().decode()


@pytest.mark.parametrize("fn", ["krt_qkv_rope_decode", "krt_qkv_rope_prefill", "krt_qkv_rope_decode_noalloc"])
def test_paged_entry_points_reject_null_args(fn):
    rc, msg = _call(fn, None, None)
    assert rc == _lib.KRT_ERR_INVALID and "NULL" in msg


@pytest.mark.parametrize("over,code,text", [
    (dict(x=None), _lib.KRT_ERR_INVALID, "required pointer"),
    (dict(num_tokens=0), _lib.KRT_ERR_INVALID, "must be positive"),
    (dict(head_dim=64), _lib.KRT_ERR_UNSUPPORTED, "head_dim"),
    (dict(d_model=4000), _lib.KRT_ERR_UNSUPPORTED, "multiple of 64"),
    (dict(x_stride=4092), _lib.KRT_ERR_INVALID, "x_stride"),
    (dict(q_stride=100), _lib.KRT_ERR_INVALID, "q_stride"),
    (dict(x=FAKE + 4), _lib.KRT_ERR_INVALID, "16-byte aligned"),
    (dict(num_blocks=0), _lib.KRT_ERR_INVALID, "geometry"),
    (dict(workspace=None), _lib.KRT_ERR_WORKSPACE, "workspace"),
    (dict(num_tokens=257), _lib.KRT_ERR_UNSUPPORTED, "prefill path"),
    (dict(workspace_bytes=1024), _lib.KRT_ERR_WORKSPACE, "needed"),
])
def test_decode_rejects_bad_arguments(over, code, text):
    a = _paged(**over)
    rc, msg = _call("krt_qkv_rope_decode", ctypes.byref(a), None)
    assert rc == code, msg
    assert text in msg and msg.startswith("krt_qkv_rope_decode")


@pytest.mark.parametrize("over,code,text", [
    (dict(x=None), _lib.KRT_ERR_INVALID, "required pointer"),
    (dict(num_tokens=0), _lib.KRT_ERR_INVALID, "must be positive"),
    (dict(head_dim=64), _lib.KRT_ERR_UNSUPPORTED, "head_dim"),
    (dict(d_model=4000), _lib.KRT_ERR_UNSUPPORTED, "multiple of 64"),
    (dict(x_stride=4092), _lib.KRT_ERR_INVALID, "x_stride"),
    (dict(q_stride=100), _lib.KRT_ERR_INVALID, "q_stride"),
    (dict(x=FAKE + 4), _lib.KRT_ERR_INVALID, "16-byte aligned"),
    (dict(num_blocks=0), _lib.KRT_ERR_INVALID, "geometry"),
    (dict(num_tokens=257), _lib.KRT_ERR_UNSUPPORTED, "prefill path"),
    (dict(num_tokens=256, d_model=8192, x_stride=8192), _lib.KRT_ERR_UNSUPPORTED, "scratch"),
])
def test_decode_noalloc_rejects_bad_arguments_before_any_gpu_call(over, code, text):
    """The no-allocation entry point checks every argument (its workspace
    fields are ignored) before it looks up or clears the shared scratch, so
    these rejections need no GPU and report its own name."""
    a = _paged(workspace=None, workspace_bytes=0, **over)
    rc, msg = _call("krt_qkv_rope_decode_noalloc", ctypes.byref(a), None)
    assert rc == code, msg
    assert text in msg and msg.startswith("krt_qkv_rope_decode_noalloc")


def test_decode_noalloc_status_rejects_null():
    rc, msg = _call("krt_qkv_rope_decode_noalloc_status", None, None)
    assert rc == _lib.KRT_ERR_INVALID and msg.startswith("krt_qkv_rope_decode_noalloc_status")


def test_prefill_rejects_a_small_workspace():
    a = _paged(num_tokens=4096, workspace_bytes=4096)
    rc, msg = _call("krt_qkv_rope_prefill", ctypes.byref(a), None)
    assert rc == _lib.KRT_ERR_WORKSPACE and "needed" in msg


def test_workspace_sizes():
    h = _lib.lib()
    assert h.krt_qkv_rope_decode_workspace_size(64, 4096, 32, 8, 128) > 64 * 4096 * 2
    assert h.krt_qkv_rope_decode_workspace_size(257, 4096, 32, 8, 128) == 0   # decode takes <= 256 tokens
    assert h.krt_qkv_rope_decode_workspace_size(64, 4096, 32, 8, 64) == 0     # head_dim 128 only
    assert h.krt_qkv_rope_prefill_workspace_size(16384, 4096, 32, 8, 128) >= 16384 * 4096 * 2
    assert h.krt_rowparallel_gemm_ar_workspace_size() > 0


def _gemm(**over):
    a = _lib.GemmArArgs()
    a.x, a.weight, a.y, a.workspace = FAKE, FAKE, FAKE, FAKE
    a.num_tokens, a.k_local, a.n_out, a.x_stride, a.y_stride = 64, 512, 4096, 512, 4096
    a.workspace_bytes = _lib.gemm_ar_workspace_bytes()
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,code,text", [
    (dict(weight=None), _lib.KRT_ERR_INVALID, "NULL"),
    (dict(num_tokens=0), _lib.KRT_ERR_INVALID, "positive"),
    (dict(k_local=500, x_stride=504), _lib.KRT_ERR_UNSUPPORTED, "k_local"),
    (dict(n_out=4000, y_stride=4000), _lib.KRT_ERR_UNSUPPORTED, "n_out"),
    (dict(x_stride=100), _lib.KRT_ERR_INVALID, "strides"),
    (dict(y=FAKE + 2), _lib.KRT_ERR_INVALID, "16-byte aligned"),
    (dict(workspace_bytes=16), _lib.KRT_ERR_WORKSPACE, "workspace"),
])
def test_gemm_ar_rejects_bad_arguments(over, code, text):
    a = _gemm(**over)
    rc, msg = _call("krt_rowparallel_gemm_ar", None, ctypes.byref(a), None)
    assert rc == code, msg
    assert text in msg


def test_gemm_ar_rejects_null_args():
    rc, msg = _call("krt_rowparallel_gemm_ar", None, None, None)
    assert rc == _lib.KRT_ERR_INVALID and "NULL" in msg


@pytest.mark.parametrize("rank,world,max_n", [(0, 0, 4096), (2, 2, 4096), (-1, 2, 4096), (0, 9, 4096),
                                              (0, 2, 100), (0, 2, 0)])
def test_comm_create_rejects_bad_geometry(rank, world, max_n):
    out = ctypes.c_void_p()
    rc, msg = _call("krt_comm_create", rank, world, max_n, ctypes.byref(out))
    assert rc == _lib.KRT_ERR_INVALID and msg.startswith("krt_comm_create")
    assert not out.value


def test_collectives_need_a_communicator():
    rc, msg = _call("krt_allreduce", None, FAKE, FAKE, 16, _lib.KRT_DTYPE_FLOAT32, FAKE, None)
    assert rc == _lib.KRT_ERR_INVALID and "communicator" in msg
    rc, msg = _call("krt_comm_ipc_handle", None, None)
    assert rc == _lib.KRT_ERR_INVALID
    assert _call("krt_comm_destroy", None)[0] == _lib.KRT_OK


def test_read_status_rejects_null():
    bits = ctypes.c_int32(0)
    rc, msg = _call("krt_read_status", None, None, ctypes.byref(bits))
    assert rc == _lib.KRT_ERR_INVALID and "NULL" in msg


def _prefill_attn(**over):
    a = _lib.PagedPrefillAttentionArgs()
    for name in ("q", "out", "kv_pool", "block_table", "q_start", "q_pos0", "workspace"):
        setattr(a, name, FAKE)
    a.num_seqs, a.n_heads, a.n_kv_heads, a.head_dim = 8, 32, 8, 128
    a.q_stride, a.out_stride = 4096, 4096
    a.block_table_stride, a.num_blocks, a.tokens_per_block = 128, 1024, 16
    a.max_q_len, a.workspace_bytes = 2048, 1 << 20
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,code,text", [
    (dict(q=0), _lib.KRT_ERR_INVALID, "NULL"),
    (dict(head_dim=64), _lib.KRT_ERR_UNSUPPORTED, "head_dim"),
    (dict(n_heads=24, n_kv_heads=8), _lib.KRT_ERR_UNSUPPORTED, "1, 2, 4, 8 or 16"),
    (dict(n_heads=30, n_kv_heads=8), _lib.KRT_ERR_INVALID, "n_kv_heads"),
    (dict(tokens_per_block=8), _lib.KRT_ERR_UNSUPPORTED, "multiple of 16"),
    (dict(q_stride=1000), _lib.KRT_ERR_INVALID, "strides"),
    (dict(max_q_len=0), _lib.KRT_ERR_INVALID, "positive"),
    (dict(workspace_bytes=16), _lib.KRT_ERR_WORKSPACE, "workspace"),
])
def test_prefill_attention_rejects_bad_arguments(over, code, text):
    a = _prefill_attn(**over)
    rc, msg = _call("krt_paged_attention_prefill", ctypes.byref(a), None)
    assert rc == code and text in msg and "krt_paged_attention_prefill" in msg, (rc, msg)
