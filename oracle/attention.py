"""Oracle for paged decode attention (test infrastructure, never shipped).

The reference has no attention kernel: its generation loop re-runs the whole
model per token (python/kinetic_rt/orchestrator.py:419-448) and its KV blocks
are only allocated (include/BlockManager.h:29-95).  The decode path that
consumes those blocks is standard scaled-dot-product attention with Llama's
grouped KV heads (query head h reads KV head h // (n_heads / n_kv_heads)),
which this module restates in float64 numpy over the pool layout the fused
QKV kernel writes: [block][token_in_block][K|V][kv_head][128].

Parity for this function is unpinned by reference vectors (there are none);
the GPU tests compare against this restatement within the bf16 tolerance.
"""
import numpy as np


def gather_kv(pool, block_table_row, seq_len, tokens_per_block):
    """K, V of one sequence's first seq_len tokens: two [seq_len, n_kv_heads, 128]
    arrays.  pool is float [num_blocks, tokens_per_block, 2, n_kv_heads, 128]."""
    pos = np.arange(seq_len)
    blocks = np.asarray(block_table_row)[pos // tokens_per_block]
    rows = pool[blocks, pos % tokens_per_block]  # [seq_len, 2, n_kv_heads, 128]
    return rows[:, 0], rows[:, 1]


def paged_decode_attention(q, pool, block_table, seq_lens, n_heads, n_kv_heads, tokens_per_block, scale=None):
    """q [num_seqs, n_heads, 128] (float); returns [num_seqs, n_heads, 128]
    float64; sequences with seq_len <= 0 give zeros."""
    q = np.asarray(q, dtype=np.float64)
    hd = q.shape[-1]
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    group = n_heads // n_kv_heads
    out = np.zeros(q.shape, dtype=np.float64)
    for s, n in enumerate(seq_lens):
        if n <= 0:
            continue
        k, v = gather_kv(pool, block_table[s], int(n), tokens_per_block)
        for h in range(n_heads):
            kv = h // group
            logits = (k[:, kv].astype(np.float64) @ q[s, h]) * scale
            w = np.exp(logits - logits.max())
            w /= w.sum()
            out[s, h] = w @ v[:, kv].astype(np.float64)
    return out


def paged_prefill_attention(q, pool, block_table, q_start, q_pos0, n_heads, n_kv_heads, tokens_per_block,
                            scale=None):
    """Causal attention of prompt tokens over the pool: sequence s's query rows
    q_start[s] .. q_start[s + 1] - 1 sit at positions q_pos0[s] + i and attend
    to the sequence's pool tokens 0 .. q_pos0[s] + i.  q [T, n_heads, 128];
    returns [T, n_heads, 128] float64.  Each query row is the decode case with
    seq_len = its position + 1 (paged_decode_attention)."""
    q = np.asarray(q, dtype=np.float64)
    out = np.zeros(q.shape, dtype=np.float64)
    for s in range(len(q_pos0)):
        rows = list(range(int(q_start[s]), int(q_start[s + 1])))
        if not rows:
            continue
        lens = [int(q_pos0[s]) + i + 1 for i in range(len(rows))]
        tables = np.repeat(np.asarray(block_table)[s:s + 1], len(rows), axis=0)
        out[rows] = paged_decode_attention(q[rows], pool, tables, lens, n_heads, n_kv_heads, tokens_per_block, scale)
    return out
