"""The drop-in runtime (python.kinetic_rt._core) on the GPU.

Mirrors the reference's tests/test_fusion.py (bridge + known-answer math
through the `fused_rmsnorm_qkv_rope[grid](...)` call shape with CPU tensors,
atol = rtol = 1e-5) and exercises the .kin compile -> load -> launch path,
the paged launch through KernelLaunchDescriptor, GraphWrapper capture and
replay on a real stream, BlockManager's pool as the KV cache, and
Communicator at world size 1.
"""
import os

import numpy as np
import pytest

from oracle import gemm_ar as orc
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
from tests.paged_cases import PagedCase, check_outputs, check_pool

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="module")
def kinetic_rt():
    import python.kinetic_rt as k
    assert not k.MOCK_CUDA
    return k


def _known_answer(torch):
    """tests/test_fusion.py:70-90 inputs (seed 42, B=S=1, d_model=128)."""
    torch.manual_seed(42)
    d = 128
    x = torch.randn(1, 1, d, dtype=torch.float32)
    rms_w = torch.ones(d, dtype=torch.float32)
    w = torch.randn(3 * d, d, dtype=torch.float32)
    cos = torch.randn(1, 1, d, dtype=torch.float32)
    sin = torch.randn(1, 1, d, dtype=torch.float32)
    return x, rms_w, w, cos, sin


def test_fusion_math(torch_cuda, kinetic_rt):
    torch = torch_cuda
    from python.kinetic_rt.fusion_forge import fused_rmsnorm_qkv_rope
    g = np.load(os.path.join(GOLDEN, "known_answer_d128.npz"))
    x, rms_w, w, cos, sin = _known_answer(torch)
    assert np.array_equal(x.numpy(), g["x"]) and np.array_equal(w.numpy(), g["w"])
    q, k, v = (torch.empty(1, 1, 128) for _ in range(3))
    fused_rmsnorm_qkv_rope[(1,)](
        x, w, None, rms_w, cos, sin, q, k, v, 1, 128, 1, 128, 1e-5,
        x.stride(1), x.stride(2), w.stride(0), w.stride(1), q.stride(1), q.stride(2),
        k.stride(1), k.stride(2), v.stride(1), v.stride(2), BLOCK_DIM=128)
    for out, name in ((q, "q"), (k, "k"), (v, "v")):
        torch.testing.assert_close(out, torch.from_numpy(g["ref_" + name]), atol=1e-5, rtol=1e-5)


def test_fusion_bridge_kin_round_trip(torch_cuda, kinetic_rt, tmp_path):
    """compile_and_serialize -> AOTEngine.load_model -> launch_descriptor runs
    this build's cubin with the reference's 24-argument signature."""
    torch = torch_cuda
    from python.kinetic_rt.fusion_forge import compile_and_serialize
    path = str(tmp_path / "fused_kernel.kin")
    engine = kinetic_rt.AOTEngine()
    compile_and_serialize(engine, kinetic_rt.Serializer(), path)
    assert os.path.exists(path)
    engine.load_model(path)
    g = np.load(os.path.join(GOLDEN, "known_answer_d128.npz"))
    dev = {n: torch.from_numpy(g[n]).cuda() for n in ("x", "w", "rms_w", "cos", "sin")}
    bias = torch.zeros(384, device="cuda")
    q, k, v = (torch.empty(1, 1, 128, device="cuda") for _ in range(3))
    d = kinetic_rt.KernelLaunchDescriptor()
    d.input_ptr, d.output_ptr = dev["x"].data_ptr(), q.data_ptr()
    d.qkv_weight_ptr, d.qkv_bias_ptr, d.rms_weight_ptr = dev["w"].data_ptr(), bias.data_ptr(), dev["rms_w"].data_ptr()
    d.freqs_cos_ptr, d.freqs_sin_ptr = dev["cos"].data_ptr(), dev["sin"].data_ptr()
    d.k_output_ptr, d.v_output_ptr = k.data_ptr(), v.data_ptr()
    d.seq_len, d.d_model, d.n_heads, d.head_dim = 1, 128, 1, 128
    d.stride_x_seq, d.stride_x_dim, d.stride_w_out, d.stride_w_in = 128, 1, 128, 1
    d.stride_q_seq = d.stride_k_seq = d.stride_v_seq = 128
    d.stride_q_dim = d.stride_k_dim = d.stride_v_dim = 1
    engine.launch_descriptor(d, torch.cuda.current_stream().cuda_stream)
    engine.synchronize_and_clear(torch.cuda.current_stream().cuda_stream)
    for out, name in ((q, "q"), (k, "k"), (v, "v")):
        np.testing.assert_allclose(out.cpu().numpy(), g["ref_" + name], atol=1e-5, rtol=1e-5)
    d.qkv_bias_ptr = 0   # the reference's launch contract requires a bias buffer (src/AOTEngine.cpp:530-535)
    with pytest.raises(RuntimeError, match="missing required weight"):
        engine.launch_descriptor(d, 0)


def _paged_descriptor(kinetic_rt, case, d, ws, pool_ptr=None):
    desc = kinetic_rt.KernelLaunchDescriptor()
    desc.input_ptr, desc.output_ptr = d["x"].data_ptr(), d["q"].data_ptr()
    desc.qkv_weight_ptr, desc.rms_weight_ptr = d["w"].data_ptr(), d["gamma"].data_ptr()
    desc.qkv_bias_ptr = 0 if d["bias"] is None else d["bias"].data_ptr()
    desc.freqs_cos_ptr, desc.freqs_sin_ptr = d["cos"].data_ptr(), d["sin"].data_ptr()
    desc.k_output_ptr, desc.v_output_ptr = d["k"].data_ptr(), d["v"].data_ptr()
    desc.positions_ptr, desc.token_seq_ptr = d["positions"].data_ptr(), d["token_seq"].data_ptr()
    desc.block_table_ptr = d["block_table"].data_ptr()
    desc.kv_pool_ptr = pool_ptr if pool_ptr is not None else d["pool"].data_ptr()
    desc.seq_len, desc.d_model, desc.n_heads, desc.n_kv_heads, desc.head_dim = case.T, case.d_model, case.n_heads, case.n_kv_heads, 128
    desc.dtype = 3
    desc.num_seqs, desc.block_table_stride = case.block_table.shape
    desc.num_blocks, desc.tokens_per_block, desc.max_position = case.num_blocks, 16, case.max_position
    desc.workspace_ptr, desc.workspace_bytes = ws.data_ptr(), ws.numel()
    return desc


def test_launch_descriptor_paged_path(torch_cuda, kinetic_rt):
    torch = torch_cuda
    from python.kinetic_rt import _lib
    case = PagedCase(8, 1, 512, 4, 2, seed=31, ctx=100, bias=True)
    d = case.to_device(torch)
    ws = torch.zeros(_lib.decode_workspace_bytes(case.T, 512, 4, 2), dtype=torch.uint8, device="cuda")
    kinetic_rt.AOTEngine().launch_descriptor(_paged_descriptor(kinetic_rt, case, d, ws),
                                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    check_outputs(case, d, torch)
    check_pool(case, d, torch)


def test_graphwrapper_replays_decode_on_a_real_stream(torch_cuda, kinetic_rt):
    torch = torch_cuda
    from python.kinetic_rt import _lib
    case = PagedCase(16, 1, 4096, 32, 8, seed=41, ctx=512)
    d = case.to_device(torch)
    ws = torch.zeros(_lib.decode_workspace_bytes(case.T, 4096, 32, 8), dtype=torch.uint8, device="cuda")
    args = _lib.paged_args(d["x"], d["w"], None, d["gamma"], d["cos"], d["sin"], d["positions"], d["token_seq"],
                           d["block_table"], d["pool"], d["q"], 32, 8, case.num_blocks, 16, ws, k_out=d["k"],
                           v_out=d["v"])
    stream = torch.cuda.Stream()
    _lib.qkv_rope_decode(args, stream=stream.cuda_stream)   # first call outside capture
    torch.cuda.synchronize()
    gw = kinetic_rt.GraphWrapper()
    gw.begin_capture(stream.cuda_stream, 16, 512)
    _lib.qkv_rope_decode(args, stream=stream.cuda_stream)
    gw.end_capture(stream.cuda_stream)
    assert gw.is_valid(16, 512) and len(gw.block_table()) == 32
    d["q"].zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        gw.launch([stream], [d["q"]])
    stream.synchronize()
    check_outputs(case, d, torch)
    gw.invalidate()
    assert gw.in_flight() == 0 and _lib.read_status(ws) == (0, 0)


def test_blockmanager_pool_is_the_kv_cache(torch_cuda, kinetic_rt):
    """K/V land in a BlockManager-owned pool at block_ptr(b) + offset."""
    torch = torch_cuda
    from cuda.bindings import runtime as cudart
    from python.kinetic_rt import _lib
    case = PagedCase(4, 1, 512, 4, 2, seed=51, ctx=40)
    token_bytes = 2 * 2 * 128 * 2
    bm = kinetic_rt.BlockManager(case.num_blocks, 16, token_bytes)
    d = case.to_device(torch)
    ws = torch.zeros(_lib.decode_workspace_bytes(case.T, 512, 4, 2), dtype=torch.uint8, device="cuda")
    kinetic_rt.AOTEngine().launch_descriptor(_paged_descriptor(kinetic_rt, case, d, ws, pool_ptr=bm.get_pool_ptr()),
                                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    kd = d["k"].view(torch.int16).cpu().numpy()
    for t, slot in enumerate(case.slots()):
        blk, off = divmod(int(slot), 16)
        host = np.empty(token_bytes // 2, np.int16)
        err, = cudart.cudaMemcpy(host.ctypes.data, bm.block_ptr(blk) + off * token_bytes, token_bytes,
                                 cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert err == cudart.cudaError_t.cudaSuccess
        np.testing.assert_array_equal(host[:256], kd[t])


def test_communicator_world_one(torch_cuda, kinetic_rt):
    torch = torch_cuda
    c = kinetic_rt.Communicator(0, 1)
    send = torch.arange(1000, dtype=torch.float32, device="cuda")
    recv = torch.zeros_like(send)
    c.all_reduce_async(send.data_ptr(), recv.data_ptr(), 1000, 0, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(recv, send)
    rng = np.random.Generator(np.random.PCG64(61))
    x = f32_to_bf16_bits(rng.standard_normal((24, 1024), dtype=np.float32))
    w = f32_to_bf16_bits(rng.standard_normal((512, 1024), dtype=np.float32) * np.float32(0.02))
    to_dev = lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda()
    xd, wd = to_dev(x), to_dev(w)
    y = torch.empty(24, 512, dtype=torch.bfloat16, device="cuda")
    c.rowparallel_gemm_ar(xd.data_ptr(), wd.data_ptr(), y.data_ptr(), 24, 1024, 512,
                          stream_obj=torch.cuda.current_stream().cuda_stream)
    assert c.read_status(torch.cuda.current_stream().cuda_stream) == 0
    ref = orc.rowparallel_reference(bf16_bits_to_f32(x), bf16_bits_to_f32(w))
    np.testing.assert_allclose(y.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)


def _core_comm_worker(rank, world, port):
    """python.kinetic_rt.Communicator(rank, world) as the reference constructs
    it (include/Communicator.h:15-26), one process per GPU: the peers' buffers
    are mapped with ipc_handle() / open_peers() (handles exchanged here over
    gloo), then all_reduce_async sums 1.0 + 2.0 (tests/test_distributed.py:47-48)
    and the fused row-parallel GEMM + allreduce matches the fp32 product."""
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import python.kinetic_rt as k
    c = k.Communicator(rank, world)
    handles = [None] * world
    dist.all_gather_object(handles, c.ipc_handle())
    c.open_peers(handles)
    stream = torch.cuda.current_stream().cuda_stream
    count = 100
    send = torch.full((count,), float(rank + 1), dtype=torch.float32, device="cuda")
    recv = torch.zeros_like(send)
    c.all_reduce_async(send.data_ptr(), recv.data_ptr(), count, 0, 0, stream)
    torch.cuda.synchronize()
    assert torch.all(recv == 3.0).item()
    rng = np.random.Generator(np.random.PCG64(62))
    x = f32_to_bf16_bits(rng.standard_normal((24, 1024), dtype=np.float32))
    w = f32_to_bf16_bits(rng.standard_normal((512, 1024), dtype=np.float32) * np.float32(0.02))
    lo, hi = orc.chunk_bounds(1024, world)[rank]
    to_dev = lambda b: torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).cuda()
    xd, wd = to_dev(x[:, lo:hi]), to_dev(w[:, lo:hi])
    y = torch.empty(24, 512, dtype=torch.bfloat16, device="cuda")
    c.rowparallel_gemm_ar(xd.data_ptr(), wd.data_ptr(), y.data_ptr(), 24, hi - lo, 512, stream_obj=stream)
    assert c.read_status(stream) == 0
    ref = orc.rowparallel_reference(bf16_bits_to_f32(x), bf16_bits_to_f32(w))
    np.testing.assert_allclose(y.float().cpu().numpy(), ref, atol=2e-2, rtol=1e-2)
    torch.cuda.synchronize()
    dist.barrier()
    del c
    dist.barrier()
    dist.destroy_process_group()


def test_core_communicator_two_gpus(torch_cuda, kinetic_rt):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_core_comm_worker, args=(2, port), nprocs=2, join=True)
