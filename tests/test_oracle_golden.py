"""Pin the oracle against the golden vectors made from the reference itself
(tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest

from oracle import fused_layer, gemm_ar, paged_kv
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16
from tests.golden import inputs as golden_inputs
from tests.golden.make_golden import sha

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.Generator(np.random.PCG64(7))
    a = np.concatenate([rng.standard_normal(10000, dtype=np.float32) * 100,
                        np.array([0.0, -0.0, 1e-40, 3.0e38, -3.0e38, 1.00390625, 1.01171875], np.float32)])
    ref = torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(f32_to_bf16_bits(a), ref)
    assert np.array_equal(bf16_bits_to_f32(ref), torch.from_numpy(ref.view(np.int16)).view(torch.bfloat16).float().numpy())


def test_known_answer_reference_and_triton():
    """tests/test_fusion.py:65-121: seed 42, B=S=1, d=128, one head, atol=rtol=1e-5."""
    g = load("known_answer_d128.npz")
    q, k, v = fused_layer.literal_reference(g["x"], g["w"], g["rms_w"], g["cos"], g["sin"], 128)
    for mine, ref, tri in ((q, g["ref_q"], g["triton_q"]), (k, g["ref_k"], g["triton_k"]), (v, g["ref_v"], g["triton_v"])):
        np.testing.assert_allclose(mine, ref, atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(mine, tri, atol=1e-5, rtol=1e-5)
    # One head of width d_model: per-head RoPE is the literal call.
    pq, pk, pv = fused_layer.fused_layer(g["x"], g["w"], g["rms_w"], g["cos"], g["sin"], 1, 1, 128)
    np.testing.assert_allclose(pq.reshape(q.shape), q, atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(pk.reshape(k.shape), k, atol=1e-6, rtol=1e-6)


def test_config1_fp32_per_head():
    g = load("config1_fp32.npz")
    c = golden_inputs.config1_inputs()
    assert str(g["inputs_sha256"]) == sha(*(c[n] for n in sorted(c))), "input generator changed"
    q, k, v = fused_layer.fused_layer(c["x"], c["w"], c["gamma"], c["cos"], c["sin"], 8, 8, 64)
    np.testing.assert_allclose(q, g["q"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(k, g["k"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(v, g["v"], atol=1e-5, rtol=1e-5)


def test_gqa_bf16_oracle():
    g = load("gqa_bf16.npz")
    c = golden_inputs.gqa_bf16_inputs()
    assert str(g["inputs_sha256"]) == sha(*(c[n] for n in sorted(c)))
    nh, nkv, hd = c["dims"].tolist()
    f = {n: bf16_bits_to_f32(c[n]) for n in ("x", "w", "gamma", "bias")}
    q, k, v = fused_layer.fused_layer(f["x"], f["w"], f["gamma"], c["cos"], c["sin"], nh, nkv, hd,
                                      bias=f["bias"], act_dtype="bf16")
    np.testing.assert_allclose(q, g["q"], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(k, g["k"], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(v, g["v"], atol=2e-5, rtol=1e-5)
    # The bf16 tolerance of the product path also covers the literal bf16 run.
    for name, ref in (("q", q), ("k", k), ("v", v)):
        lit = bf16_bits_to_f32(g["bf16_" + name])
        np.testing.assert_allclose(lit, ref, atol=2e-2, rtol=1e-2)


def test_blockmanager_model_lifo():
    bm = paged_kv.BlockManagerModel(4, 16, 4096)
    assert bm.pool_bytes == 4 * 16 * 4096
    assert [bm.allocate_block() for _ in range(3)] == [3, 2, 1]
    bm.free_block(2)
    assert bm.allocate_block() == 2
    with pytest.raises(RuntimeError, match="out of range"):
        bm.free_block(4)
    assert bm.allocate_block() == 0
    with pytest.raises(RuntimeError, match="exhausted"):
        bm.allocate_block()
    table = paged_kv.block_table_for_capture(paged_kv.BlockManagerModel(8, 16, 4096), 33)
    assert table == [7, 6, 5]


def test_scatter_places_rows():
    pool = np.full((8, 16, 2, 2, 4), 0xFFFF, np.uint16)
    k = np.arange(3 * 2 * 4, dtype=np.uint16).reshape(3, 2, 4)
    v = k + 100
    bt = np.array([[5, 2], [1, 7]], np.int32)
    slots = paged_kv.scatter_kv(pool, k, v, bt, [0, 0, 1], [3, 17, 0])
    assert slots == [5 * 16 + 3, 2 * 16 + 1, 1 * 16 + 0]
    assert np.array_equal(pool[5, 3, 0], k[0]) and np.array_equal(pool[2, 1, 1], v[1])
    assert (pool == 0xFFFF).sum() == pool.size - 3 * 2 * 2 * 4


def test_rowparallel_shards_sum_to_full():
    rng = np.random.Generator(np.random.PCG64(3))
    x = rng.standard_normal((5, 40)).astype(np.float32)
    w = rng.standard_normal((12, 40)).astype(np.float32)
    for world in (1, 2, 3, 4, 8):
        parts = [gemm_ar.partial_gemm(xr, wr) for xr, wr in gemm_ar.shard_rows(x, w, world)]
        outs = gemm_ar.allreduce_sum(parts)
        for o in outs:
            np.testing.assert_allclose(o, gemm_ar.rowparallel_reference(x, w), rtol=1e-5, atol=1e-5)
    assert gemm_ar.chunk_bounds(14336, 8)[-1] == (12544, 14336)


def test_chunk_bounds_match_torch():
    torch = pytest.importorskip("torch")
    for k, world in ((14336, 8), (4096, 3), (10, 4), (7, 8)):
        t = torch.zeros(1, k)
        sizes = [c.shape[1] for c in torch.chunk(t, world, dim=1)]
        assert [hi - lo for lo, hi in gemm_ar.chunk_bounds(k, world)] == sizes


def test_round_bf16_idempotent():
    a = np.linspace(-5, 5, 1001, dtype=np.float32)
    r = round_bf16(a)
    assert np.array_equal(round_bf16(r), r)
