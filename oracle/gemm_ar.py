"""Oracle for the row-parallel GEMM fused with the allreduce (test infrastructure).

shard_rows follows scripts/export_hf.py:62-65: o_proj / down_proj weights of
shape [N, K] are split with torch.chunk(dim=1), so rank r holds W[:, K_r] and
the matching activation slice X[:, K_r].  Each rank computes the partial
Y_r = X[:, K_r] @ W[:, K_r]^T and the allreduce-sum (tests/mock_rccl.h:51-62:
every rank's recv buffer ends up holding the elementwise sum of all ranks'
send buffers) yields Y = X @ W^T on every rank.  torch.chunk gives
ceil(K / world) columns to every rank but the last.
"""
import numpy as np


def chunk_bounds(k, world):
    """Column ranges of torch.chunk(t, world, dim=1) for a dimension of size k."""
    step = -(-k // world)
    bounds = []
    for r in range(world):
        lo = min(r * step, k)
        hi = min(lo + step, k)
        if lo < hi:
            bounds.append((lo, hi))
    return bounds


def shard_rows(x, w, world):
    """Return [(x_r, w_r)] for each rank (export_hf.py:64)."""
    return [(x[:, lo:hi], w[:, lo:hi]) for lo, hi in chunk_bounds(w.shape[1], world)]


def partial_gemm(x_r, w_r):
    return np.asarray(x_r, np.float64) @ np.asarray(w_r, np.float64).T


def allreduce_sum(parts):
    """tests/mock_rccl.h:51-62: every rank receives the sum of all sends."""
    total = np.zeros_like(np.asarray(parts[0], np.float64))
    for p in parts:
        total = total + np.asarray(p, np.float64)
    return [total.copy() for _ in parts]


def rowparallel_reference(x, w):
    """The unsharded fp32 product the sharded result must match."""
    return (np.asarray(x, np.float64) @ np.asarray(w, np.float64).T).astype(np.float32)
