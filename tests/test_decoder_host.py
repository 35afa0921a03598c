"""Host-side logic of the decode driver (no GPU): block allocation order,
vocabulary shards, the gate/up interleave and the RoPE tables."""
import numpy as np
import pytest

from oracle import fused_layer, paged_kv


def test_block_allocator_matches_blockmanager_order():
    from python.kinetic_rt.decoder import BlockAllocator
    a, m = BlockAllocator(7), paged_kv.BlockManagerModel(7, 16, 4096)
    got = [a.allocate_block() for _ in range(4)]
    assert got == [m.allocate_block() for _ in range(4)] == [6, 5, 4, 3]
    a.free_block(5)
    m.free_block(5)
    assert a.allocate_block() == m.allocate_block() == 5
    with pytest.raises(RuntimeError):
        a.free_block(7)
    for _ in range(3):
        a.allocate_block()
    with pytest.raises(RuntimeError, match="Out of KV Cache blocks"):
        a.allocate_block()


def test_vocab_shards_cover_the_vocabulary():
    from python.kinetic_rt.decoder import vocab_shard
    for world in (1, 2, 4, 8):
        spans = [vocab_shard(128256, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 128256
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_interleave_gate_up_layout():
    torch = pytest.importorskip("torch")
    from python.kinetic_rt import _lib
    gate = torch.arange(128 * 3, dtype=torch.float32).view(128, 3)
    up = -gate
    gu = _lib.interleave_gate_up(gate, up)
    assert gu.shape == (256, 3)
    assert torch.equal(gu[0:64], gate[0:64]) and torch.equal(gu[64:128], up[0:64])
    assert torch.equal(gu[128:192], gate[64:128]) and torch.equal(gu[192:256], up[64:128])


def test_rope_cache_matches_oracle_tables():
    torch = pytest.importorskip("torch")
    from python.kinetic_rt.decoder import rope_cache
    cos, sin = rope_cache(torch, 300, 128, 5e5, device="cpu")
    oc, os_ = fused_layer.rope_tables(np.arange(300), 128, 5e5)
    np.testing.assert_array_equal(cos.numpy(), oc)
    np.testing.assert_array_equal(sin.numpy(), os_)


def test_argmax_key_orders_logits_then_first_index():
    from python.kinetic_rt import _lib
    k = _lib.argmax_key
    assert k(1.0, 5) > k(0.5, 0) > k(-0.5, 0) > k(-1.0, 0)
    assert k(2.0, 3) > k(2.0, 4)  # equal logits: the lower index wins
    assert k(0.0, 0) > k(-0.0, 0) or k(0.0, 0) >= k(-1e-30, 0)
