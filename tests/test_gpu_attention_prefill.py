"""GPU parity of causal paged prefill attention (krt_paged_attention_prefill).

The oracle is oracle/attention.py's paged_prefill_attention: every query row
is float64 scaled-dot-product attention over its sequence's pool tokens
0 .. its position, with grouped KV heads, over the pool layout
[block][token][K|V][kv_head][128].  Inputs are bf16; the kernel accumulates in
fp32.  bf16 output tolerance: max-abs 2e-2 + rel 1e-2.
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


def run_case(torch, q_lens, pos0, n_heads, n_kv_heads, seed, tokens_per_block=16, spare=3, q_pad=0, rows=None):
    """q_lens[s] query tokens of sequence s at positions pos0[s] ..; the pool
    holds random K/V for every position up to the last query's."""
    from python.kinetic_rt import _lib
    rng = np.random.Generator(np.random.PCG64(seed))
    S = len(q_lens)
    ctx = [p + n for p, n in zip(pos0, q_lens)]
    bps = -(-max(max(ctx), 1) // tokens_per_block)
    num_blocks = S * bps + spare
    table = rng.permutation(num_blocks).astype(np.int32)[:S * bps].reshape(S, bps)
    pool = f32_to_bf16_bits(rng.standard_normal((num_blocks, tokens_per_block, 2, n_kv_heads, 128), dtype=np.float32))
    T = sum(q_lens)
    qb = f32_to_bf16_bits(rng.standard_normal((T, n_heads, 128), dtype=np.float32))
    q_start = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q_dev = torch.zeros(T, n_heads * 128 + q_pad, dtype=torch.bfloat16, device="cuda")
    q_dev[:, :n_heads * 128] = to_dev(torch, qb.reshape(T, -1))
    out = torch.full((T, n_heads * 128), 9.0, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.prefill_attention_workspace_bytes(), dtype=torch.uint8, device="cuda")
    pool_dev, table_dev = to_dev(torch, pool), torch.from_numpy(table).cuda()
    qs_dev = torch.from_numpy(q_start).cuda()
    p0_dev = torch.tensor(pos0, dtype=torch.int32, device="cuda")
    a = _lib.prefill_attention_args(q_dev, pool_dev, table_dev, qs_dev, p0_dev, out, n_heads, n_kv_heads,
                                    num_blocks, tokens_per_block, max(q_lens), ws)
    _lib.paged_attention_prefill(a)
    rc, bits = _lib.read_status(ws)
    assert rc == 0 and bits == 0, f"status {bits:#x}"
    got = out.float().cpu().numpy().reshape(T, n_heads, 128)
    if rows is None:
        ref = orc.paged_prefill_attention(bf16_bits_to_f32(qb), bf16_bits_to_f32(pool), table, q_start, pos0,
                                          n_heads, n_kv_heads, tokens_per_block)
        np.testing.assert_allclose(got, ref, atol=2e-2, rtol=1e-2)
    else:
        # sampled rows (long prompts): each row is the decode case at its position
        pool_f, q_f = bf16_bits_to_f32(pool), bf16_bits_to_f32(qb)
        seq_of = np.searchsorted(q_start, rows, side="right") - 1
        lens = [int(pos0[s]) + int(r - q_start[s]) + 1 for r, s in zip(rows, seq_of)]
        ref = orc.paged_decode_attention(q_f[rows], pool_f, table[seq_of], lens, n_heads, n_kv_heads,
                                         tokens_per_block)
        np.testing.assert_allclose(got[rows], ref, atol=2e-2, rtol=1e-2)
    return out


@pytest.mark.parametrize("n_heads,n_kv_heads", [(32, 8), (64, 8), (8, 8), (16, 1), (4, 2)])
def test_prefill_attention_ragged_prompts(torch_cuda, n_heads, n_kv_heads):
    """Prompts of 1, 15, 16, 17, 40 and 130 tokens (tile and chunk edges)."""
    run_case(torch_cuda, [1, 15, 16, 17, 40, 130], [0] * 6, n_heads, n_kv_heads, seed=n_heads * 3 + n_kv_heads)


def test_prefill_attention_after_a_prefix(torch_cuda):
    """q_pos0 > 0: query tokens continue after a prefix already in the pool."""
    run_case(torch_cuda, [20, 33, 5], [7, 64, 200], 32, 8, seed=5)


def test_prefill_attention_block_size_32_and_q_stride(torch_cuda):
    run_case(torch_cuda, [45, 70], [0, 3], 8, 2, seed=6, tokens_per_block=32, q_pad=64)


def test_prefill_attention_long_prompt_sampled(torch_cuda):
    """Two 2048-token prompts (Llama-3-8B heads): sampled rows across the
    causal range, the rest only run."""
    rows = np.array([0, 1, 15, 16, 31, 32, 511, 1024, 2047, 2048, 2049, 3000, 4095])
    run_case(torch_cuda, [2048, 2048], [0, 0], 32, 8, seed=7, rows=rows)


def test_prefill_attention_bad_block_sets_status(torch_cuda):
    """A block-table entry out of range: status bit 8, the chunk masked."""
    torch = torch_cuda
    from python.kinetic_rt import _lib
    n_heads, n_kv = 8, 2
    q = torch.randn(20, n_heads * 128, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    pool = torch.randn(8, 16, 2 * n_kv * 128, device="cuda").to(torch.bfloat16)
    table = torch.tensor([[3, 99]], dtype=torch.int32, device="cuda")  # block 99 > num_blocks
    ws = torch.zeros(_lib.prefill_attention_workspace_bytes(), dtype=torch.uint8, device="cuda")
    a = _lib.prefill_attention_args(q, pool, table, torch.tensor([0, 20], dtype=torch.int32, device="cuda"),
                                    torch.tensor([0], dtype=torch.int32, device="cuda"), out, n_heads, n_kv, 8, 16,
                                    20, ws)
    _lib.paged_attention_prefill(a)
    rc, bits = _lib.read_status(ws)
    assert bits == 8  # the bad-block bit alone (krt_read_status also returns an error code for it)
    assert torch.isfinite(out.float()).all()
