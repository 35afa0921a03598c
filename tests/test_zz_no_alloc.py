"""The decode entry point for callers that cannot allocate device memory.

Such callers (a plugin inside a host application that owns all device
memory through its own allocator, or a serving loop that must not allocate
after start-up) can pass inputs and outputs but no workspace.
krt_qkv_rope_decode_noalloc uses the library's fixed device scratch instead.
These tests call it through the C ABI and check that two calls in a row give
the same results as krt_qkv_rope_decode with a caller-owned workspace, within
the bf16 tolerance of the other parity tests (max-abs 2e-2 + rel 1e-2), with
K/V placed in the same pool slots.

This file is named to be collected last, so a run that stops at its first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from tests.paged_cases import PagedCase, check_outputs, check_pool

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _args(krt, d, case, workspace):
    return krt.paged_args(d["x"], d["w"], d["bias"], d["gamma"], d["cos"], d["sin"], d["positions"],
                          d["token_seq"], d["block_table"], d["pool"], d["q"], case.n_heads, case.n_kv_heads,
                          case.num_blocks, case.tokens_per_block, workspace, k_out=d["k"], v_out=d["v"])


def _call_noalloc(krt, args):
    stream = ctypes.c_void_p(__import__("torch").cuda.current_stream().cuda_stream)
    return krt.lib().krt_qkv_rope_decode_noalloc(ctypes.byref(args), stream)


@pytest.mark.parametrize("num_seqs,ctx,bias", [(64, 2048, False), (5, 77, True)])
def test_noalloc_matches_workspace_entry_point(torch_cuda, num_seqs, ctx, bias):
    torch = torch_cuda
    from python.kinetic_rt import _lib as krt
    case = PagedCase(num_seqs, 1, 4096, 32, 8, seed=21 + num_seqs, ctx=ctx, bias=bias)

    # reference run: the existing entry point with a caller-owned workspace
    ref = case.to_device(torch)
    ws = torch.zeros(krt.decode_workspace_bytes(case.T, 4096, 32, 8), dtype=torch.uint8, device="cuda")
    krt.qkv_rope_decode(_args(krt, ref, case, ws))
    rc, bits = krt.read_status(ws)
    assert rc == 0 and bits == 0
    torch.cuda.synchronize()

    # two no-alloc calls in a row, each into fresh outputs and a fresh pool
    for call in range(2):
        d = case.to_device(torch)
        rc = _call_noalloc(krt, _args(krt, d, case, None))
        assert rc == 0, krt.lib().krt_last_error().decode()
        torch.cuda.synchronize()
        for name in ("q", "k", "v"):
            np.testing.assert_allclose(d[name].float().cpu().numpy(), ref[name].float().cpu().numpy(),
                                       atol=2e-2, rtol=1e-2, err_msg=f"call {call}: {name}")
        check_outputs(case, d, torch)
        check_pool(case, d, torch)


def test_noalloc_rejects_oversized_calls(torch_cuda):
    """256 tokens at d_model 8192 would need more than the 4 MiB scratch."""
    torch = torch_cuda
    from python.kinetic_rt import _lib as krt
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    a = krt.QkvPagedArgs()
    a.x = a.qkv_weight = a.rms_weight = a.rope_cos = a.rope_sin = dummy.data_ptr()
    a.positions = a.token_seq = a.block_table = a.kv_pool = a.q_out = dummy.data_ptr()
    a.num_tokens, a.d_model, a.n_heads, a.n_kv_heads, a.head_dim = 256, 8192, 8, 1, 128
    a.x_stride, a.q_stride = 8192, 1024
    a.max_position, a.num_seqs, a.block_table_stride, a.num_blocks, a.tokens_per_block = 1, 1, 1, 1, 16
    rc = _call_noalloc(krt, a)
    assert rc == krt.KRT_ERR_UNSUPPORTED
    assert b"scratch" in krt.lib().krt_last_error()


def test_noalloc_status_reports_a_bad_block(torch_cuda):
    """The status word lives in the shared scratch; the caller reads it with
    krt_qkv_rope_decode_noalloc_status.  A token whose block id lies outside
    the pool sets bit 8, the other tokens still land, and reading clears it."""
    torch = torch_cuda
    from python.kinetic_rt import _lib as krt
    case = PagedCase(4, 1, 512, 4, 2, seed=3, ctx=40)
    d = case.to_device(torch)
    bt = d["block_table"].clone()
    bt[2, :] = case.num_blocks + 5  # outside the pool
    d["block_table"] = bt
    assert _call_noalloc(krt, _args(krt, d, case, None)) == 0, krt.lib().krt_last_error().decode()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bits = ctypes.c_int32(0)
    rc = krt.lib().krt_qkv_rope_decode_noalloc_status(stream, ctypes.byref(bits))
    assert rc == krt.KRT_ERR_DEVICE and bits.value & 8
    pool = d["pool"].view(torch.int16).cpu().numpy().reshape(case.num_blocks * 16, 2, -1)
    kd = d["k"].view(torch.int16).cpu().numpy()
    slots = case.slots()
    for t in (0, 1, 3):
        np.testing.assert_array_equal(pool[slots[t], 0], kd[t])
    assert krt.lib().krt_qkv_rope_decode_noalloc_status(stream, ctypes.byref(bits)) == 0 and bits.value == 0
