"""GPU parity of paged decode attention (krt_paged_attention_decode).

The oracle is oracle/attention.py: float64 scaled-dot-product attention with
grouped KV heads over the pool layout [block][token][K|V][kv_head][128].
Inputs are bf16 (q and the pool); the kernel accumulates in fp32.  bf16
output tolerance: max-abs 2e-2 + rel 1e-2.
"""
import numpy as np
import pytest

from oracle import attention as orc
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def to_dev(torch, bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def run_case(torch, seq_lens, n_heads, n_kv_heads, seed, tokens_per_block=16, spare=5, q_pad=0):
    from python.kinetic_rt import _lib
    rng = np.random.Generator(np.random.PCG64(seed))
    S = len(seq_lens)
    max_len = max(max(seq_lens), 1)
    bps = -(-max_len // tokens_per_block)
    num_blocks = S * bps + spare
    perm = rng.permutation(num_blocks).astype(np.int32)
    table = perm[:S * bps].reshape(S, bps)
    pool_f = rng.standard_normal((num_blocks, tokens_per_block, 2, n_kv_heads, 128), dtype=np.float32)
    pool = f32_to_bf16_bits(pool_f)
    q_f = rng.standard_normal((S, n_heads, 128), dtype=np.float32)
    qb = f32_to_bf16_bits(q_f)
    q_dev = torch.zeros(S, n_heads * 128 + q_pad, dtype=torch.bfloat16, device="cuda")
    q_dev[:, :n_heads * 128] = to_dev(torch, qb.reshape(S, -1))
    out = torch.full((S, n_heads * 128), 9.0, dtype=torch.bfloat16, device="cuda")
    lens = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    ws = torch.zeros(_lib.attention_workspace_bytes(S, n_heads, n_kv_heads, max_len), dtype=torch.uint8,
                     device="cuda")
    pool_dev = to_dev(torch, pool)
    table_dev = torch.from_numpy(table).cuda()
    a = _lib.attention_args(q_dev, pool_dev, table_dev, lens, out, n_heads, n_kv_heads, num_blocks,
                            tokens_per_block, max_len, ws)
    ref = orc.paged_decode_attention(bf16_bits_to_f32(qb), bf16_bits_to_f32(pool), table, seq_lens, n_heads,
                                     n_kv_heads, tokens_per_block)
    for _ in range(2):  # a second call reuses the split counters the first one left at zero
        out.fill_(9.0)
        _lib.paged_attention_decode(a)
        rc, bits = _lib.read_status(ws)
        assert rc == 0 and bits == 0, f"status {bits:#x}"
        got = out.float().cpu().numpy().reshape(S, n_heads, 128)
        np.testing.assert_allclose(got, ref, atol=2e-2, rtol=1e-2)
    return got, ref


@pytest.mark.parametrize("n_heads,n_kv_heads", [(32, 8), (4, 1), (8, 8), (64, 8), (16, 1)])
def test_attention_ragged(torch_cuda, n_heads, n_kv_heads):
    # lengths across chunk (16) and split boundaries, one empty sequence
    lens = [1, 15, 16, 17, 100, 257, 0, 1030]
    run_case(torch_cuda, lens, n_heads, n_kv_heads, seed=n_heads + n_kv_heads)


def test_attention_forced_splits(torch_cuda, monkeypatch):
    """Small splits (2 chunks per CTA): the last-CTA merge of many partials."""
    monkeypatch.setenv("KRT_ATTN_SPLIT_CHUNKS", "2")
    run_case(torch_cuda, [33, 64, 700, 5, 2048], 32, 8, seed=3)


@pytest.mark.parametrize("lens,n_heads,n_kv_heads", [
    ([8192], 4, 1),                     # one pair in many splits
    ([1] * 300, 32, 8),                 # many one-token sequences
    ([0] * 40 + [3000] * 2 + [17] * 30, 8, 1),  # long, short and empty sequences together
], ids=["one_long", "many_short", "mixed"])
def test_attention_shapes(torch_cuda, lens, n_heads, n_kv_heads):
    run_case(torch_cuda, lens, n_heads, n_kv_heads, seed=len(lens))


def test_attention_block_size_32_and_q_stride(torch_cuda):
    run_case(torch_cuda, [31, 32, 33, 500], 8, 2, seed=4, tokens_per_block=32, q_pad=64)


def test_attention_decode_batch_llama(torch_cuda):
    """Llama-3-8B heads at TP=1, batch 32 at context ~4096."""
    rng = np.random.Generator(np.random.PCG64(11))
    lens = list(rng.integers(3900, 4353, size=32))
    run_case(torch_cuda, lens, 32, 8, seed=12)


def test_attention_bad_block_sets_status(torch_cuda):
    torch = torch_cuda
    from python.kinetic_rt import _lib
    S, H, KV = 2, 4, 1
    pool = torch.zeros(4, 16, 2, KV, 128, dtype=torch.bfloat16, device="cuda")
    table = torch.tensor([[0, 1], [2, 99]], dtype=torch.int32, device="cuda")  # 99 is outside the pool
    lens = torch.tensor([20, 20], dtype=torch.int32, device="cuda")
    q = torch.ones(S, H * 128, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(S, H * 128, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.attention_workspace_bytes(S, H, KV, 32), dtype=torch.uint8, device="cuda")
    _lib.paged_attention_decode(_lib.attention_args(q, pool, table, lens, out, H, KV, 4, 16, 32, ws))
    rc, bits = _lib.read_status(ws)
    assert bits & 8
    assert torch.isfinite(out.float()).all()


def test_attention_length_beyond_max_is_clamped(torch_cuda):
    """A sequence longer than max_seq_len attends over its first max_seq_len
    tokens and reports status bit 8; the split counters stay consistent, so
    the next call is exact."""
    torch = torch_cuda
    from python.kinetic_rt import _lib
    rng = np.random.Generator(np.random.PCG64(21))
    S, H, KV, max_len = 3, 8, 2, 300
    bps = -(-max_len // 16) + 2
    nb = S * bps
    table = rng.permutation(nb).astype(np.int32).reshape(S, bps)
    pool = f32_to_bf16_bits(rng.standard_normal((nb, 16, 2, KV, 128), dtype=np.float32))
    qb = f32_to_bf16_bits(rng.standard_normal((S, H, 128), dtype=np.float32))
    q, pool_d = to_dev(torch, qb.reshape(S, -1)), to_dev(torch, pool)
    out = torch.empty(S, H * 128, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.attention_workspace_bytes(S, H, KV, max_len), dtype=torch.uint8, device="cuda")
    table_d = torch.from_numpy(table).cuda()
    for lens, bad in (([100, max_len + 25, 7], True), ([100, 250, 7], False)):
        lens_d = torch.tensor(lens, dtype=torch.int32, device="cuda")  # referenced while the kernel runs
        a = _lib.attention_args(q, pool_d, table_d, lens_d, out, H, KV, nb, 16, max_len, ws)
        _lib.paged_attention_decode(a)
        rc, bits = _lib.read_status(ws)
        assert bool(bits & 8) == bad
        ref = orc.paged_decode_attention(bf16_bits_to_f32(qb), bf16_bits_to_f32(pool), table,
                                         [min(n, max_len) for n in lens], H, KV, 16)
        np.testing.assert_allclose(out.float().cpu().numpy().reshape(S, H, 128), ref, atol=2e-2, rtol=1e-2)
