"""GPU parity of the fused RMSNorm + QKV + RoPE kernels against the oracle.

Tolerances: fp32 paths atol = rtol = 1e-5 (known-answer, as the reference's
tests/test_fusion.py:119-121) or 1e-4 (config 1); bf16 paths max-abs 2e-2 +
rel 1e-2; KV placement and indices bit-exact.
"""
import os

import numpy as np
import pytest

from oracle.bf16 import bf16_bits_to_f32
from tests.golden import inputs as golden_inputs
from tests.paged_cases import PagedCase, check_outputs, check_pool

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def krt():
    from python.kinetic_rt import _lib
    _lib.lib()
    return _lib


def test_generic_known_answer(torch_cuda, krt):
    torch = torch_cuda
    g = np.load(os.path.join(GOLDEN, "known_answer_d128.npz"))
    dev = {n: torch.from_numpy(g[n]).cuda() for n in ("x", "w", "rms_w", "cos", "sin")}
    q = torch.empty(1, 1, 128, device="cuda")
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    x, w = dev["x"], dev["w"]
    krt.fused_rmsnorm_qkv_rope(x, w, None, dev["rms_w"], dev["cos"], dev["sin"], q, k, v, 1, 128, 1, 128, 1e-5,
                               (x.stride(1), x.stride(2), w.stride(0), w.stride(1), q.stride(1), q.stride(2),
                                k.stride(1), k.stride(2), v.stride(1), v.stride(2)))
    torch.cuda.synchronize()
    for out, name in ((q, "q"), (k, "k"), (v, "v")):
        np.testing.assert_allclose(out.cpu().numpy(), g["ref_" + name], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(out.cpu().numpy(), g["triton_" + name], atol=1e-5, rtol=1e-5)


def test_generic_config1_fp32(torch_cuda, krt):
    torch = torch_cuda
    c = golden_inputs.config1_inputs()
    g = np.load(os.path.join(GOLDEN, "config1_fp32.npz"))
    x = torch.from_numpy(c["x"]).cuda().reshape(64, 512)
    w = torch.from_numpy(c["w"]).cuda()
    gamma = torch.from_numpy(c["gamma"]).cuda()
    cos = torch.from_numpy(c["cos"][0]).cuda()   # [32, 64], one row per position
    sin = torch.from_numpy(c["sin"][0]).cuda()
    pos = torch.arange(32, dtype=torch.int32, device="cuda").repeat(2)
    q = torch.empty(64, 512, device="cuda")
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    krt.fused_rmsnorm_qkv_rope(x, w, None, gamma, cos, sin, q, k, v, 64, 512, 8, 64, 1e-5,
                               (512, 1, 512, 1, 512, 1, 512, 1, 512, 1), n_kv_heads=8,
                               freqs_strides=(64, 1), freqs_head_stride=0, positions=pos)
    torch.cuda.synchronize()
    np.testing.assert_allclose(q.cpu().numpy().reshape(2, 32, 8, 64), g["q"], atol=1e-4, rtol=1e-4)
    np.testing.assert_allclose(k.cpu().numpy().reshape(2, 32, 8, 64), g["k"], atol=1e-4, rtol=1e-4)
    np.testing.assert_allclose(v.cpu().numpy().reshape(2, 32, 8, 64), g["v"], atol=1e-4, rtol=1e-4)


def _run_paged(krt, torch, case, d, kind, workspace=None):
    if workspace is None:
        nbytes = (krt.decode_workspace_bytes if kind == "decode" else krt.prefill_workspace_bytes)(
            case.T, case.d_model, case.n_heads, case.n_kv_heads)
        workspace = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    a = krt.paged_args(d["x"], d["w"], d["bias"], d["gamma"], d["cos"], d["sin"], d["positions"], d["token_seq"],
                       d["block_table"], d["pool"], d["q"], case.n_heads, case.n_kv_heads, case.num_blocks,
                       case.tokens_per_block, workspace, k_out=d["k"], v_out=d["v"])
    (krt.qkv_rope_decode if kind == "decode" else krt.qkv_rope_prefill)(a)
    rc, bits = krt.read_status(workspace)
    assert rc == 0 and bits == 0, f"kernel status 0x{bits:x}"
    return workspace


@pytest.mark.parametrize("kind", ["decode", "prefill"])
def test_paged_gqa_golden(torch_cuda, krt, kind):
    """The golden GQA bf16 case (bias, ragged positions, permuted block table)."""
    torch = torch_cuda
    from oracle.fused_layer import rope_tables
    c = golden_inputs.gqa_bf16_inputs()
    g = np.load(os.path.join(GOLDEN, "gqa_bf16.npz"))
    case = PagedCase(6, 1, 512, 4, 2, seed=1, bias=True, ctx=160)
    case.x, case.w, case.gamma, case.bias = c["x"], c["w"], c["gamma"], c["bias"]
    case.positions, case.token_seq = c["positions"], np.arange(6, dtype=np.int32)
    case.block_table, case.num_blocks = c["block_table"], 64
    case.cos, case.sin = rope_tables(np.arange(160), 128, 5e5)
    np.testing.assert_array_equal(case.cos[case.positions], c["cos"])   # same table rows as the golden run
    d = case.to_device(torch)
    _run_paged(krt, torch, case, d, kind)
    torch.cuda.synchronize()
    for name in ("q", "k", "v"):
        got = d[name].float().cpu().numpy().reshape(g[name].shape)
        np.testing.assert_allclose(got, g[name], atol=2e-2, rtol=1e-2)
        # the literal bf16 run of the reference is also within tolerance
        lit = bf16_bits_to_f32(g["bf16_" + name]).reshape(got.shape)
        np.testing.assert_allclose(got, lit, atol=3e-2, rtol=2e-2)
    check_pool(case, d, torch)


@pytest.mark.parametrize("kind,num_seqs,tokens_per_seq,ctx", [
    ("decode", 64, 1, 2048),      # Llama-3-8B decode batch 64 at context 2048
    ("decode", 5, 1, 77),         # ragged small batch
    ("decode", 128, 1, 300),      # decode batch 128 (half-head tiles)
    ("decode", 200, 1, 90),       # decode batch 200 (whole-head tiles)
    ("prefill", 1, 300, None),    # one sequence, two token blocks, ragged tail
    ("prefill", 3, 100, None),    # three sequences
])
def test_paged_llama_shapes(torch_cuda, krt, kind, num_seqs, tokens_per_seq, ctx):
    torch = torch_cuda
    case = PagedCase(num_seqs, tokens_per_seq, 4096, 32, 8, seed=num_seqs, ctx=ctx)
    d = case.to_device(torch)
    ws = _run_paged(krt, torch, case, d, kind)
    torch.cuda.synchronize()
    check_outputs(case, d, torch)
    check_pool(case, d, torch)
    if kind == "decode":
        # split-K counters were reset: a second call gives bit-identical output
        q1 = d["q"].clone()
        _run_paged(krt, torch, case, d, kind, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(q1, d["q"])


@pytest.mark.parametrize("num_seqs,d_model,n_heads,n_kv_heads", [
    (256, 8192, 8, 1),   # Llama-3-70B TP=8 shard at decode batch 256 (half-head tiles above 128 tokens)
    (200, 1024, 16, 2),  # 20 heads at 200 tokens
    (144, 512, 32, 8),   # 48 heads above 128 tokens: whole-head tiles
])
def test_paged_decode_above_128_tokens(torch_cuda, krt, num_seqs, d_model, n_heads, n_kv_heads):
    torch = torch_cuda
    case = PagedCase(num_seqs, 1, d_model, n_heads, n_kv_heads, seed=num_seqs + n_heads, ctx=400)
    d = case.to_device(torch)
    _run_paged(krt, torch, case, d, "decode")
    torch.cuda.synchronize()
    check_outputs(case, d, torch)
    check_pool(case, d, torch)


@pytest.mark.parametrize("num_seqs,tokens_per_seq", [(1, 300), (3, 100)])
def test_prefill_persistent_kernel(torch_cuda, krt, monkeypatch, num_seqs, tokens_per_seq):
    """KRT_PREFILL_KERNEL=1: the persistent projection kernel's QKV epilogue
    instead of the dedicated prefill kernel; the same oracle checks."""
    monkeypatch.setenv("KRT_PREFILL_KERNEL", "1")
    test_paged_llama_shapes(torch_cuda, krt, "prefill", num_seqs, tokens_per_seq, None)
    test_paged_gqa_golden(torch_cuda, krt, "prefill")


def test_prefill_full_size_sampled(torch_cuda, krt):
    """8 sequences x 2048 tokens (the full prefill configuration): sampled
    rows against the oracle, every token's K/V placement bit-exact."""
    torch = torch_cuda
    case = PagedCase(8, 2048, 4096, 32, 8, seed=11)
    d = case.to_device(torch)
    _run_paged(krt, torch, case, d, "prefill")
    torch.cuda.synchronize()
    rows = np.random.Generator(np.random.PCG64(5)).choice(case.T, 48, replace=False)
    check_outputs(case, d, torch, rows=rows)
    check_pool(case, d, torch)


def test_decode_bad_block_sets_status(torch_cuda, krt):
    torch = torch_cuda
    case = PagedCase(4, 1, 512, 4, 2, seed=3, ctx=40)
    d = case.to_device(torch)
    bt = d["block_table"].clone()
    bt[2, :] = case.num_blocks + 5        # outside the pool
    d["block_table"] = bt
    ws = torch.zeros(krt.decode_workspace_bytes(case.T, 512, 4, 2), dtype=torch.uint8, device="cuda")
    a = krt.paged_args(d["x"], d["w"], None, d["gamma"], d["cos"], d["sin"], d["positions"], d["token_seq"],
                       d["block_table"], d["pool"], d["q"], 4, 2, case.num_blocks, 16, ws, k_out=d["k"], v_out=d["v"])
    krt.qkv_rope_decode(a)
    rc, bits = krt.read_status(ws)
    assert rc == krt.KRT_ERR_DEVICE and bits & 8
    # the other tokens still landed, and nothing outside the pool was touched
    pool = d["pool"].view(torch.int16).cpu().numpy().reshape(case.num_blocks * 16, 2, -1)
    slots = case.slots()
    kd = d["k"].view(torch.int16).cpu().numpy()
    for t in (0, 1, 3):
        np.testing.assert_array_equal(pool[slots[t], 0], kd[t])


def test_paged_rejects_bad_arguments(torch_cuda, krt):
    torch = torch_cuda
    case = PagedCase(2, 1, 512, 4, 2, seed=4, ctx=20)
    d = case.to_device(torch)
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    a = krt.paged_args(d["x"], d["w"], None, d["gamma"], d["cos"], d["sin"], d["positions"], d["token_seq"],
                       d["block_table"], d["pool"], d["q"], 4, 2, case.num_blocks, 16, ws)
    with pytest.raises(ValueError, match="workspace"):
        krt.qkv_rope_decode(a)
    a.head_dim = 64
    with pytest.raises(ValueError, match="head_dim"):
        krt.qkv_rope_decode(a)
