"""GPU parity of the row-parallel GEMM fused with the allreduce.

The oracle is the unsharded fp32 product X W^T (oracle/gemm_ar.py; shards
follow torch.chunk(dim=1), scripts/export_hf.py:62-65).  bf16 output
tolerance: max-abs 2e-2 + rel 1e-2.  Multi-GPU cases run one process per GPU
and are skipped with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

from oracle import gemm_ar as orc
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def make_case(T, K, N, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = f32_to_bf16_bits(rng.standard_normal((T, K), dtype=np.float32))
    w = f32_to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    return x, w


def to_dev(torch, bits, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.parametrize("T,K,N", [
    (1, 4096, 4096),      # o_proj, one token
    (64, 4096, 4096),     # o_proj, decode batch 64
    (8, 14336, 4096),     # down_proj, unsharded K
    (300, 1792, 4096),    # down_proj shard at TP8, 3 blocks of 128 tokens (persistent, ragged last block)
    (17, 512, 256),       # small ragged case
])
def test_gemm_single_gpu(torch_cuda, T, K, N):
    torch = torch_cuda
    from python.kinetic_rt import _lib
    x, w = make_case(T, K, N, seed=T + K)
    xd, wd = to_dev(torch, x), to_dev(torch, w)
    y = torch.full((T, N), 7.0, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    _lib.rowparallel_gemm_ar(None, _lib.gemm_ar_args(xd, wd, y, ws))
    rc, bits = _lib.read_status(ws)
    assert rc == 0 and bits == 0
    ref = orc.rowparallel_reference(bf16_bits_to_f32(x), bf16_bits_to_f32(w))
    np.testing.assert_allclose(y.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("T,K,N,residual,large", [
    (512, 7168, 4096, False, "1"),    # down_proj shard at TP2: 128 tiles of 128 x 128 (persistent)
    (512, 7168, 4096, True, "0"),     # the same through the 256-token slices (KRT_GEMM_LARGE_T=0)
    (4096, 4096, 4096, True, "1"),    # o_proj unsharded: 512 tiles of 128 x 256 (persistent)
    (8192, 1792, 4096, False, "1"),   # down_proj shard at TP8
    (8192, 14336, 4096, True, "1"),   # down_proj unsharded
    (4700, 512, 4096, True, "1"),     # o_proj shard at TP8, last token block ragged
    (4700, 512, 4096, True, "0"),     # the same through the slices (KRT_GEMM_LARGE_T=0)
])
def test_gemm_large_token_counts(torch_cuda, monkeypatch, T, K, N, residual, large):
    """Config-3 token counts on one GPU: y = x W^T (+ residual) against the
    fp64 product of the same bf16 values on a sample of rows that covers
    the first and last rows of every 128-token block (so of every 256-token
    block too) and the ragged tail."""
    torch = torch_cuda
    from python.kinetic_rt import _lib
    monkeypatch.setenv("KRT_GEMM_LARGE_T", large)
    g = torch.Generator(device="cuda").manual_seed(T + K)
    xd = torch.randn(T, K, generator=g, device="cuda").to(torch.bfloat16)
    wd = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    res = (torch.randn(T, N, generator=g, device="cuda")).to(torch.bfloat16) if residual else None
    y = torch.full((T, N), 7.0, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    _lib.rowparallel_gemm_ar(None, _lib.gemm_ar_args(xd, wd, y, ws, residual=res))
    rc, bits = _lib.read_status(ws)
    assert rc == 0 and bits == 0
    rows = sorted({t for b in range(0, T, 128) for t in (b, b + 1, min(b + 127, T - 1))} | {T - 1})
    idx = torch.tensor(rows, device="cuda")
    xs = xd[idx].float().cpu().numpy().astype(np.float64)
    ref = xs @ wd.float().cpu().numpy().astype(np.float64).T
    if res is not None:
        ref = ref + res[idx].float().cpu().numpy()
    np.testing.assert_allclose(y[idx].float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("T,K,N", [(33, 1536, 384), (200, 640, 256)])
def test_gemm_half_height_tiles(torch_cuda, monkeypatch, T, K, N):
    """KRT_GEMM_TILE_M=64 selects 64-row weight tiles (read when a shape is
    first configured; these shapes are used nowhere else in the suite)."""
    monkeypatch.setenv("KRT_GEMM_TILE_M", "64")
    test_gemm_single_gpu(torch_cuda, T, K, N)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp_worker(rank, world, port, cases):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from python.kinetic_rt import _lib
    from python.kinetic_rt.dist import TPComm
    comm = TPComm(rank, world, max_n_out=4096)
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    try:
        for (T, K, N) in cases:
            x, w = make_case(T, K, N, seed=1000 + T + K)
            lo, hi = orc.chunk_bounds(K, world)[rank]
            xd = to_dev(torch, x[:, lo:hi])
            wd = to_dev(torch, w[:, lo:hi])
            y = torch.full((T, N), 7.0, dtype=torch.bfloat16, device="cuda")
            for rep in range(3):  # replays reuse the exchange buffers and flags
                comm.gemm_ar(xd, wd, y, ws)
                rc, bits = _lib.read_status(ws)
                assert rc == 0 and bits == 0, f"rank {rank} status {bits:#x}"
            ref = orc.rowparallel_reference(bf16_bits_to_f32(x), bf16_bits_to_f32(w))
            got = y.float().cpu().numpy()
            np.testing.assert_allclose(got, ref, atol=2e-2, rtol=1e-2)
            all_y = [None] * world
            dist.all_gather_object(all_y, y.view(torch.int16).cpu().numpy())
            for other in all_y:
                assert np.array_equal(other, all_y[0]), "ranks disagree"
        # standalone allreduce: tests/test_distributed.py:8-48 (1 + 2 = 3) and random bf16
        send = torch.full((100,), float(rank + 1), device="cuda")
        recv = torch.zeros_like(send)
        comm.allreduce(send, recv, ws)
        torch.cuda.synchronize()
        assert torch.all(recv == float(sum(range(1, world + 1)))).item()
        rng = np.random.Generator(np.random.PCG64(77))
        full = rng.standard_normal((world, 100003), dtype=np.float32)
        send = to_dev(torch, f32_to_bf16_bits(full[rank]))
        recv = torch.empty_like(send)
        comm.allreduce(send, recv, ws)
        ref = bf16_bits_to_f32(f32_to_bf16_bits(full)).astype(np.float64).sum(0)
        np.testing.assert_allclose(recv.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
        rc, bits = _lib.read_status(ws)
        assert rc == 0 and bits == 0
    finally:
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemm_ar_multi_gpu(torch_cuda, world):
    torch = torch_cuda
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    cases = [(1, 4096, 4096), (64, 14336, 4096), (300, 4096, 4096)]
    mp.spawn(_tp_worker, args=(world, _free_port(), cases), nprocs=world, join=True)


def _timeout_worker(rank, world, port):
    """Rank 1 skips one fused call (between steps, nothing in flight); rank 0's
    bounded peer wait runs out and reports status bit 16; both ranks reset the
    communicator (drain, barrier, krt_comm_reset, barrier); the next call
    matches the fp32 product on both ranks."""
    import datetime
    import time
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from python.kinetic_rt import _lib
    from python.kinetic_rt.dist import TPComm
    comm = TPComm(rank, world, max_n_out=4096)
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    try:
        T, K, N = 64, 4096, 4096
        x, w = make_case(T, K, N, seed=55)
        lo, hi = orc.chunk_bounds(K, world)[rank]
        xd, wd = to_dev(torch, x[:, lo:hi]), to_dev(torch, w[:, lo:hi])
        y = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        ref = orc.rowparallel_reference(bf16_bits_to_f32(x), bf16_bits_to_f32(w))
        comm.gemm_ar(xd, wd, y, ws)  # a good call first
        assert _lib.read_status(ws) == (0, 0)
        dist.barrier()
        t0 = time.time()
        if rank == 0:
            comm.gemm_ar(xd, wd, y, ws)  # its peer never joins this one
            rc, bits = _lib.read_status(ws)
            elapsed = time.time() - t0
            assert rc == _lib.KRT_ERR_DEVICE and bits & 16, bits
            assert elapsed < 6.0, elapsed
        comm.reset()
        y.fill_(0)
        comm.gemm_ar(xd, wd, y, ws)
        rc, bits = _lib.read_status(ws)
        assert rc == 0 and bits == 0, f"rank {rank} status {bits:#x} after the reset"
        np.testing.assert_allclose(y.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
    finally:
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def test_gemm_ar_peer_timeout_then_reset(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_timeout_worker, args=(2, _free_port()), nprocs=2, join=True)


def _nccl_worker(rank, world, port):
    """The size-selected NCCL route (threshold 0: every call): GEMM without the
    fused exchange, then ncclAllReduce in place; with a residual (added once,
    by rank 0) and without; plus krt_allreduce through NCCL."""
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from python.kinetic_rt import _lib
    from python.kinetic_rt.dist import TPComm
    comm = TPComm(rank, world, max_n_out=4096)
    comm.attach_nccl(0)
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    try:
        for (T, K, N, with_res) in [(1, 4096, 4096, False), (64, 14336, 4096, True), (300, 4096, 4096, True),
                                    (512, 1792 * world, 4096, False)]:
            x, w = make_case(T, K, N, seed=2000 + T + K)
            rng = np.random.Generator(np.random.PCG64(T))
            res = f32_to_bf16_bits(rng.standard_normal((T, N), dtype=np.float32))
            lo, hi = orc.chunk_bounds(K, world)[rank]
            xd, wd = to_dev(torch, x[:, lo:hi]), to_dev(torch, w[:, lo:hi])
            y = to_dev(torch, res) if with_res else torch.full((T, N), 7.0, dtype=torch.bfloat16, device="cuda")
            comm.gemm_ar(xd, wd, y, ws) if not with_res else _lib.rowparallel_gemm_ar(
                comm.handle, _lib.gemm_ar_args(xd, wd, y, ws, residual=y))
            rc, bits = _lib.read_status(ws)
            assert rc == 0 and bits == 0
            ref = orc.rowparallel_reference(bf16_bits_to_f32(x), bf16_bits_to_f32(w))
            if with_res:
                ref = ref + bf16_bits_to_f32(res)
            np.testing.assert_allclose(y.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
            all_y = [None] * world
            dist.all_gather_object(all_y, y.view(torch.int16).cpu().numpy())
            for other in all_y:
                assert np.array_equal(other, all_y[0]), "ranks disagree"
        send = torch.full((1000,), float(rank + 1), device="cuda")
        recv = torch.zeros_like(send)
        comm.allreduce(send, recv, ws)
        torch.cuda.synchronize()
        assert torch.all(recv == float(sum(range(1, world + 1)))).item()
    finally:
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 8])
def test_gemm_ar_nccl_route(torch_cuda, world):
    torch = torch_cuda
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_nccl_worker, args=(world, _free_port()), nprocs=world, join=True)
