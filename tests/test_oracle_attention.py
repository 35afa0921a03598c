"""CPU check of the attention oracle against torch's scaled_dot_product_attention
(float64, GQA expanded by repeat_interleave) on a small paged case."""
import numpy as np
import pytest

from oracle import attention as orc


def test_oracle_matches_torch_sdpa():
    torch = pytest.importorskip("torch")
    rng = np.random.Generator(np.random.PCG64(0))
    S, H, KV, B = 3, 8, 2, 16
    lens = [5, 16, 40]
    bps = 3
    nb = S * bps + 2
    table = rng.permutation(nb)[:S * bps].reshape(S, bps).astype(np.int32)
    pool = rng.standard_normal((nb, B, 2, KV, 128))
    q = rng.standard_normal((S, H, 128))
    got = orc.paged_decode_attention(q, pool, table, lens, H, KV, B)
    for s, n in enumerate(lens):
        k, v = orc.gather_kv(pool, table[s], n, B)
        kt = torch.from_numpy(k).permute(1, 0, 2).repeat_interleave(H // KV, 0)  # [H, n, 128]
        vt = torch.from_numpy(v).permute(1, 0, 2).repeat_interleave(H // KV, 0)
        qt = torch.from_numpy(q[s])[:, None, :]  # [H, 1, 128]
        ref = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)[:, 0, :].numpy()
        np.testing.assert_allclose(got[s], ref, atol=1e-10, rtol=1e-9)


def test_oracle_empty_sequence_is_zero():
    pool = np.ones((2, 16, 2, 1, 128))
    out = orc.paged_decode_attention(np.ones((1, 2, 128)), pool, np.array([[0]]), [0], 2, 1, 16)
    assert not out.any()


def test_prefill_oracle_matches_sdpa_with_causal_mask():
    """paged_prefill_attention equals torch SDPA with a causal mask (and the
    prefix offset) on gathered K/V."""
    torch = pytest.importorskip("torch")
    rng = np.random.Generator(np.random.PCG64(9))
    n_heads, n_kv, B = 4, 2, 16
    pos0, q_len = 5, 27
    ctx = pos0 + q_len
    table = np.array([[2, 0, 3]], dtype=np.int32)
    pool = rng.standard_normal((4, B, 2, n_kv, 128))
    q = rng.standard_normal((q_len, n_heads, 128))
    got = orc.paged_prefill_attention(q, pool, table, np.array([0, q_len]), np.array([pos0]), n_heads, n_kv, B)
    k, v = orc.gather_kv(pool, table[0], ctx, B)
    kt = torch.from_numpy(np.repeat(k, n_heads // n_kv, axis=1)).permute(1, 0, 2)
    vt = torch.from_numpy(np.repeat(v, n_heads // n_kv, axis=1)).permute(1, 0, 2)
    qt = torch.from_numpy(q).permute(1, 0, 2)
    mask = torch.from_numpy(np.arange(ctx)[None, :] <= (pos0 + np.arange(q_len))[:, None])
    ref = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask).permute(1, 0, 2).numpy()
    np.testing.assert_allclose(got, ref, atol=1e-10, rtol=1e-9)
