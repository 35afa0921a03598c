"""Oracle of one Llama decode step over the paged KV cache (test infrastructure).

The reference has no decoder forward (its generation loop,
python/kinetic_rt/orchestrator.py:419-448, re-runs a whole model per token
and picks the next token with argmax at 442-444).  This module composes the
pieces the B200 path implements, each already restated elsewhere in
oracle/, in Llama's layer order and with the same rounding points as the
kernels (fp32/fp64 arithmetic, bf16 at every tensor the kernels store):

  x_hat = bf16(rms_norm(h, g_attn))                    fused_layer.rms_norm
  q, k, v = per-head RoPE projection of x_hat           fused_layer.fused_layer
  K/V of the token -> pool slot of its position        paged_kv layout
  a = bf16(attention(q, pool))                          attention.paged_decode_attention
  h = bf16(h + a @ W_o^T)                               gemm_ar (with the residual)
  x_hat = bf16(rms_norm(h, g_mlp))
  act = bf16(silu(x_hat W_gate^T) * (x_hat W_up^T))
  h = bf16(h + act @ W_down^T)
after the last layer: logits = bf16(rms_norm(h, g_final)) @ W_lm^T, the next
token is the first index of the maximum, and h of the next step is that
token's embedding row.

Weights are float32 arrays holding bf16 values; the pool is a float32 array
[num_blocks, tokens_per_block, 2, n_kv_heads, 128] of bf16 values.
"""
import numpy as np

from . import attention, fused_layer
from .bf16 import round_bf16


def silu(x):
    return x / (1.0 + np.exp(-x))


def decode_step(w, h, positions, block_table, pools, cos, sin, n_heads, n_kv_heads, tokens_per_block, eps=1e-5):
    """One decode step for all sequences (one token each).

    w: dict with lists per layer 'qkv', 'g_attn', 'o', 'g_mlp', 'gate', 'up',
       'down' and 'g_final', 'lm_head', 'embed'.
    h: [S, D] float32 (bf16 values), the input hidden state.
    positions: [S] position of each sequence's token (its K/V slot and RoPE row).
    pools: list per layer of the pool (updated in place with the new K/V).
    cos, sin: RoPE tables [max_position, 128].
    Returns (logits [S, V] float64, next tokens [S], h_next [S, D]).
    """
    hd = 128
    S = h.shape[0]
    h = np.asarray(h, np.float32).copy()
    pos = np.asarray(positions)
    for li in range(len(w["qkv"])):
        q, k, v = fused_layer.fused_layer(h, w["qkv"][li], w["g_attn"][li], cos[pos], sin[pos], n_heads, n_kv_heads,
                                          hd, eps=eps, act_dtype="bf16")
        q, k, v = round_bf16(q), round_bf16(k), round_bf16(v)
        pool = pools[li]
        for s in range(S):
            blk = block_table[s][pos[s] // tokens_per_block]
            pool[blk, pos[s] % tokens_per_block, 0] = k[s]
            pool[blk, pos[s] % tokens_per_block, 1] = v[s]
        a = attention.paged_decode_attention(q, pool, block_table, pos + 1, n_heads, n_kv_heads, tokens_per_block)
        a = round_bf16(a.reshape(S, n_heads * hd).astype(np.float32))
        h = round_bf16((h.astype(np.float64) + a.astype(np.float64) @ w["o"][li].astype(np.float64).T)
                       .astype(np.float32))
        xm = round_bf16(fused_layer.rms_norm(h, w["g_mlp"][li], eps))
        g = xm.astype(np.float64) @ w["gate"][li].astype(np.float64).T
        u = xm.astype(np.float64) @ w["up"][li].astype(np.float64).T
        act = round_bf16((silu(g) * u).astype(np.float32))
        h = round_bf16((h.astype(np.float64) + act.astype(np.float64) @ w["down"][li].astype(np.float64).T)
                       .astype(np.float32))
    xf = round_bf16(fused_layer.rms_norm(h, w["g_final"], eps))
    logits = xf.astype(np.float64) @ w["lm_head"].astype(np.float64).T
    tokens = np.argmax(logits, axis=-1)
    return logits, tokens, np.asarray(w["embed"], np.float32)[tokens]
