"""Seeded paged-QKV cases shared by the GPU parity tests and bench.py's checks.

A case is generated with numpy's PCG64 (bf16 values carried as uint16 bit
patterns), moved to the device, and checked against the oracle
(oracle.fused_layer / oracle.paged_kv) on the CPU.
"""
import numpy as np

from oracle import fused_layer, paged_kv
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits


class PagedCase:
    def __init__(self, num_seqs, tokens_per_seq, d_model, n_heads, n_kv_heads, *, seed=0, ctx=None,
                 tokens_per_block=16, theta=5e5, bias=False, max_position=None, spare_blocks=7):
        """num_seqs sequences contribute tokens_per_seq consecutive tokens each,
        ending at position ctx-1 (decode: tokens_per_seq=1, ctx=context length;
        prefill: positions 0..tokens_per_seq-1)."""
        rng = np.random.Generator(np.random.PCG64(seed))
        hd = 128
        self.hd, self.d_model, self.n_heads, self.n_kv_heads = hd, d_model, n_heads, n_kv_heads
        self.tokens_per_block = tokens_per_block
        ctx = tokens_per_seq if ctx is None else ctx
        T = num_seqs * tokens_per_seq
        self.T = T
        n_out = (n_heads + 2 * n_kv_heads) * hd
        self.x = f32_to_bf16_bits(rng.standard_normal((T, d_model), dtype=np.float32))
        self.w = f32_to_bf16_bits(rng.standard_normal((n_out, d_model), dtype=np.float32) * np.float32(0.02))
        self.gamma = f32_to_bf16_bits(1.0 + 0.1 * rng.standard_normal(d_model, dtype=np.float32))
        self.bias = f32_to_bf16_bits(0.1 * rng.standard_normal(n_out, dtype=np.float32)) if bias else None
        self.positions = np.concatenate(
            [np.arange(ctx - tokens_per_seq, ctx, dtype=np.int32) for _ in range(num_seqs)])
        self.token_seq = np.repeat(np.arange(num_seqs, dtype=np.int32), tokens_per_seq)
        self.max_position = max_position or ctx
        blocks_per_seq = -(-ctx // tokens_per_block)
        self.num_blocks = num_seqs * blocks_per_seq + spare_blocks
        perm = rng.permutation(self.num_blocks).astype(np.int32)
        self.block_table = perm[:num_seqs * blocks_per_seq].reshape(num_seqs, blocks_per_seq)
        cos, sin = fused_layer.rope_tables(np.arange(self.max_position), hd, theta)
        self.cos, self.sin = cos, sin

    # ---------------------------------------------------------------- oracle
    def oracle(self, rows=None):
        """fp32 (q [T,Hq,hd], k, v [T,Hkv,hd]) for all tokens or the given rows."""
        idx = np.arange(self.T) if rows is None else np.asarray(rows)
        x = bf16_bits_to_f32(self.x[idx])
        w = bf16_bits_to_f32(self.w)
        g = bf16_bits_to_f32(self.gamma)
        b = None if self.bias is None else bf16_bits_to_f32(self.bias)
        pos = self.positions[idx]
        return fused_layer.fused_layer(x, w, g, self.cos[pos], self.sin[pos], self.n_heads, self.n_kv_heads,
                                       self.hd, bias=b, act_dtype="bf16")

    def slots(self):
        B = self.tokens_per_block
        return np.array([paged_kv.slot_of(self.block_table, s, p, B) for s, p in zip(self.token_seq, self.positions)])

    # ---------------------------------------------------------------- device
    def to_device(self, torch, device="cuda"):
        def bf(a):
            return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
        d = {
            "x": bf(self.x), "w": bf(self.w), "gamma": bf(self.gamma),
            "bias": None if self.bias is None else bf(self.bias),
            "cos": torch.from_numpy(self.cos).to(device), "sin": torch.from_numpy(self.sin).to(device),
            "positions": torch.from_numpy(self.positions).to(device),
            "token_seq": torch.from_numpy(self.token_seq).to(device),
            "block_table": torch.from_numpy(self.block_table).to(device),
        }
        tok_elems = 2 * self.n_kv_heads * self.hd
        d["pool"] = torch.full((self.num_blocks, self.tokens_per_block, tok_elems), -7.0,
                               dtype=torch.bfloat16, device=device)
        d["q"] = torch.empty((self.T, self.n_heads * self.hd), dtype=torch.bfloat16, device=device)
        d["k"] = torch.empty((self.T, self.n_kv_heads * self.hd), dtype=torch.bfloat16, device=device)
        d["v"] = torch.empty((self.T, self.n_kv_heads * self.hd), dtype=torch.bfloat16, device=device)
        return d


def check_outputs(case, d, torch, rows=None, atol=2e-2, rtol=1e-2):
    """Compare device q/k/v with the oracle (bf16 tolerance written here:
    max-abs 2e-2 + rel 1e-2) and check the pool placement bit-exactly."""
    idx = np.arange(case.T) if rows is None else np.asarray(rows)
    q, k, v = case.oracle(idx)
    T = len(idx)
    gq = d["q"][torch.as_tensor(idx, device=d["q"].device)].float().cpu().numpy().reshape(T, case.n_heads, case.hd)
    gk = d["k"][torch.as_tensor(idx, device=d["k"].device)].float().cpu().numpy().reshape(T, case.n_kv_heads, case.hd)
    gv = d["v"][torch.as_tensor(idx, device=d["v"].device)].float().cpu().numpy().reshape(T, case.n_kv_heads, case.hd)
    np.testing.assert_allclose(gq, q, atol=atol, rtol=rtol)
    np.testing.assert_allclose(gk, k, atol=atol, rtol=rtol)
    np.testing.assert_allclose(gv, v, atol=atol, rtol=rtol)


def check_pool(case, d, torch):
    """Every token's K and V rows sit at BlockManager's address for its slot,
    bit-identical to the dense outputs; every other pool element still holds
    the sentinel."""
    pool = d["pool"].view(torch.int16).cpu().numpy().reshape(case.num_blocks * case.tokens_per_block, 2, -1)
    kd = d["k"].view(torch.int16).cpu().numpy()
    vd = d["v"].view(torch.int16).cpu().numpy()
    slots = case.slots()
    assert len(set(slots.tolist())) == len(slots), "test case maps two tokens to one slot"
    np.testing.assert_array_equal(pool[slots, 0], kd)
    np.testing.assert_array_equal(pool[slots, 1], vd)
    sentinel = np.int16(torch.tensor(-7.0, dtype=torch.bfloat16).view(torch.int16).item())
    mask = np.ones(pool.shape[0], bool)
    mask[slots] = False
    assert (pool[mask] == sentinel).all()
