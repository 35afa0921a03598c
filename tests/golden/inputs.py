"""Seeded input generators shared by the golden-vector script and the tests.

Inputs come from numpy's PCG64 so they are identical on every machine; the
golden fixtures store a sha256 of them, which tests/test_oracle_golden.py
checks before trusting a fixture.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle.bf16 import f32_to_bf16_bits  # noqa: E402
from oracle.fused_layer import rope_tables  # noqa: E402


def config1_inputs():
    """Batch 2, seq 32, hidden 512, 8 Q / 8 KV heads x 64, fp32.
    x ~ N(0,1); Wq, Wk, Wv ~ N(0, 0.02) fused as [Q; K; V]; gamma = 1 + N(0, 0.1);
    RoPE theta 1e4 at positions 0..31, one table row per token."""
    rng = np.random.Generator(np.random.PCG64(0))
    x = rng.standard_normal((2, 32, 512), dtype=np.float32)
    w = (rng.standard_normal((3 * 512, 512), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(512, dtype=np.float32)).astype(np.float32)
    cos, sin = rope_tables(np.arange(32), 64, 1e4)
    return {"x": x, "w": w, "gamma": gamma, "cos": cos[None], "sin": sin[None]}


def gqa_bf16_inputs():
    """6 tokens of 6 sequences at ragged positions, hidden 512, 4 Q / 2 KV
    heads x 128, bf16, with bias; Llama RoPE theta 5e5; a paged cache of
    16-token blocks whose tables are a seeded permutation of 64 blocks."""
    rng = np.random.Generator(np.random.PCG64(1))
    T, D, nh, nkv, hd = 6, 512, 4, 2, 128
    n_out = (nh + 2 * nkv) * hd
    x = f32_to_bf16_bits(rng.standard_normal((T, D), dtype=np.float32))
    w = f32_to_bf16_bits(rng.standard_normal((n_out, D), dtype=np.float32) * np.float32(0.02))
    gamma = f32_to_bf16_bits(1.0 + 0.1 * rng.standard_normal(D, dtype=np.float32))
    bias = f32_to_bf16_bits(0.1 * rng.standard_normal(n_out, dtype=np.float32))
    positions = np.array([0, 5, 17, 31, 100, 159], dtype=np.int32)
    cos, sin = rope_tables(positions, hd, 5e5)
    block_table = rng.permutation(64).astype(np.int32)[:60].reshape(6, 10)
    return {"x": x, "w": w, "gamma": gamma, "bias": bias, "cos": cos, "sin": sin,
            "positions": positions, "block_table": block_table,
            "dims": np.array([nh, nkv, hd], dtype=np.int32)}
