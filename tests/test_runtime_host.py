"""Host-side logic of the runtime, on CPU, against _core_mock (the runtime
built over a host-only test double of the CUDA runtime).  Mirrors the
reference's tests/test_graph.py, tests/test_distributed.py, tests/test_aot.py,
tests/test_validation.py and tests/test_serializer_errors.cpp."""
import ctypes
import os
import struct
import threading

import pytest

import python.kinetic_rt._core_mock as krt
from oracle.paged_kv import BlockManagerModel

KIN_HEADER = 564


@pytest.fixture(autouse=True)
def _env(monkeypatch, tmp_path):
    monkeypatch.delenv("KINETIC_TARGET", raising=False)
    monkeypatch.delenv("KINETIC_ALLOW_MOCKS", raising=False)
    monkeypatch.setenv("KINETIC_KV_POOL_SIZE", "64")
    monkeypatch.chdir(tmp_path)
    krt.reset_fake_cuda_state()


# ------------------------------------------------------------ GraphWrapper
def test_graph_capture_and_launch():
    w = krt.GraphWrapper()
    s = 1234
    assert not w.is_valid(batch_size=1, seq_len=128)
    w.begin_capture(s, batch_size=1, seq_len=128)
    w.end_capture(s)
    assert w.is_valid(batch_size=1, seq_len=128)
    w.begin_capture(s, batch_size=1, seq_len=128)          # redundant: no new capture
    assert krt.fake_cuda_state()["stream_begin_capture"] == 1
    w.launch([s], [])
    assert not w.is_valid(batch_size=2, seq_len=128)
    w.begin_capture(s, batch_size=2, seq_len=128)
    w.end_capture(s)
    assert w.is_valid(batch_size=2, seq_len=128) and not w.is_valid(batch_size=1, seq_len=128)
    w.launch([s], [])
    st = krt.fake_cuda_state()
    assert st["graph_instantiate"] == 2 and st["graph_launch"] == 2 and st["graph_exec_destroy"] == 1


def test_uninstantiated_launch():
    with pytest.raises(RuntimeError, match="(?i)not instantiated"):
        krt.GraphWrapper().launch([1234], [])


def test_async_stress_holds_buffers():
    w = krt.GraphWrapper()
    w.begin_capture(1234, batch_size=1, seq_len=128)
    w.end_capture(1234)
    for i in range(1000):
        w.launch([1234], [[i]])
    w.invalidate()
    assert w.in_flight() == 0


def test_capture_allocates_blocks_like_blockmanager():
    """ceil(seq / 16) blocks per capture, handed out LIFO from the top
    (src/GraphWrapper.cpp:139-145, include/BlockManager.h:63-82)."""
    w = krt.GraphWrapper()
    w.begin_capture(1234, batch_size=1, seq_len=33)
    w.end_capture(1234)
    model = BlockManagerModel(64, 16, 4096)
    expect = [model.allocate_block() for _ in range(3)]
    assert w.block_table() == expect == [63, 62, 61]
    w.invalidate()
    assert w.block_table() == []
    w.begin_capture(1234, batch_size=1, seq_len=16)        # freed blocks come back LIFO
    assert w.block_table() == [61]


# ------------------------------------------------------------ BlockManager
def test_blockmanager_matches_model():
    bm = krt.BlockManager(5, 16, 4096)
    model = BlockManagerModel(5, 16, 4096)
    assert bm.pool_bytes == model.pool_bytes and bm.block_bytes == 16 * 4096
    got = [bm.allocate_block() for _ in range(3)]
    assert got == [model.allocate_block() for _ in range(3)]
    bm.free_block(got[1])
    model.free_block(got[1])
    assert bm.allocate_block() == model.allocate_block()
    assert bm.block_ptr(3) - bm.get_pool_ptr() == model.block_offset(3)
    with pytest.raises(RuntimeError, match=r"out of range \[0, 5\)"):
        bm.free_block(5)
    # freeing an id twice lists it twice (include/BlockManager.h:73-82 takes any in-range id)
    n = bm.num_free()
    bm.free_block(got[0])
    bm.free_block(got[0])
    model.free_block(got[0])
    model.free_block(got[0])
    assert bm.num_free() == n + 2 == len(model.free)
    assert bm.allocate_block() == model.allocate_block() == got[0]
    while bm.num_free():
        bm.allocate_block()
    with pytest.raises(RuntimeError, match="exhausted"):
        bm.allocate_block()


# ------------------------------------------------------------ Communicator
def test_distributed_sharding():
    """tests/test_distributed.py:8-48: two ranks, 1.0 + 2.0 == 3.0."""
    n = 100
    arr = ctypes.c_float * n
    t0, t1 = arr(*([1.0] * n)), arr(*([2.0] * n))
    r0, r1 = arr(*([0.0] * n)), arr(*([0.0] * n))
    c0, c1 = krt.Communicator(0, 2), krt.Communicator(1, 2)
    w = krt.GraphWrapper()
    w.begin_capture(0x1000, 1, 1)
    th = [threading.Thread(target=lambda: c0.all_reduce_async(ctypes.addressof(t0), ctypes.addressof(r0), n, 0, 0, 0x1000)),
          threading.Thread(target=lambda: c1.all_reduce_async(ctypes.addressof(t1), ctypes.addressof(r1), n, 0, 0, 0x2000))]
    [t.start() for t in th]
    [t.join() for t in th]
    w.end_capture(0x1000)
    w.launch([0x1000, 0x2000], [])
    w.invalidate()
    assert list(r0) == [3.0] * n and list(r1) == [3.0] * n


def test_allreduce_rejects_other_ops_and_bad_ranks():
    arr = (ctypes.c_float * 4)()
    c = krt.Communicator(0, 1)
    with pytest.raises(RuntimeError, match="sum"):
        c.all_reduce_async(ctypes.addressof(arr), ctypes.addressof(arr), 4, 0, 1, 0)
    with pytest.raises(ValueError):
        krt.Communicator(2, 2)


def test_allreduce_times_out_when_a_rank_never_joins():
    arr = (ctypes.c_float * 4)()
    c = krt.Communicator(0, 3)
    with pytest.raises(RuntimeError, match="timed out"):
        c.all_reduce_async(ctypes.addressof(arr), ctypes.addressof(arr), 4, 0, 0, 0)


# ------------------------------------------------------------ .kin files
def _kernel_bytes(machine=b"\xBE\x00"):
    b = bytearray(64)
    b[0:4] = b"\x7fELF"
    b[4] = 2
    b[18:20] = machine
    return list(b)


def test_serializer_round_trip_and_poison_pill(monkeypatch):
    monkeypatch.setenv("KINETIC_TARGET", "sm100")
    s = krt.Serializer()
    bins = _kernel_bytes()
    s.save_kin_file("m.kin", "sm100", "CUDA_sm100", 123456789, [1, 2, 3], bins)
    assert s.load_kin_file("m.kin") == bins
    assert s.get_tensor_parallel_degree("m.kin") == 1
    raw = open("m.kin", "rb").read()
    assert len(raw) == KIN_HEADER + 3 + 64
    magic, version = struct.unpack_from("<II", raw, 0)
    assert (magic, version) == (0x4B494E00, 1)
    s.save_kin_file("bad.kin", "gfx1100", "ROCm_gfx1100", 1, [1, 2, 3], _kernel_bytes(b"\xE0\x00"))
    with pytest.raises(krt.HardwareMismatchError, match="expected Kinetic target gfx1100 but got sm100"):
        s.load_kin_file("bad.kin")


def test_serializer_error_handling(tmp_path):
    s = krt.Serializer()
    with pytest.raises(RuntimeError, match="Failed to open file for reading"):
        s.load_kin_file("non_existent_file.kin")
    with pytest.raises(RuntimeError, match="Failed to open file for writing"):
        s.save_kin_file(str(tmp_path / "no_dir" / "x.kin"), "CPU", "CPU_CPU", 1, [], [])


def _header(magic=0x4B494E00, device=b"CPU", og=(KIN_HEADER, 0), kb=(KIN_HEADER, 0)):
    h = struct.pack("<II", magic, 1) + device.ljust(256, b"\0") + b"CPU_CPU".ljust(256, b"\0")
    h += struct.pack("<QQQQQI", 0, og[0], og[1], kb[0], kb[1], 1)
    assert len(h) == KIN_HEADER
    return h


@pytest.mark.parametrize("content,message", [
    (b"\0" * 10, "file too small for header"),
    (_header(magic=0x12345678), "bad magic number"),
    (_header(magic=0xDEADBEEF), "bad magic number"),
    (_header(og=(2**64 - 1, 10)), "offset overflow"),
    (_header(og=(100, 10), kb=(2**64 - 1, 10)), "offset overflow"),
    (_header(og=(KIN_HEADER, 100)), "sizes exceed file bounds"),
    (_header(kb=(KIN_HEADER, 10000)), "sizes exceed file bounds"),
])
def test_serializer_hardening(content, message):
    """tests/test_serializer_errors.cpp:16-222."""
    open("f.kin", "wb").write(content)
    with pytest.raises(RuntimeError, match=message):
        krt.Serializer().load_kin_file("f.kin")


def test_serializer_hardware_mismatch_header():
    open("f.kin", "wb").write(_header(device=b"wrong_hw"))
    with pytest.raises(krt.HardwareMismatchError, match="Hardware mismatch"):
        krt.Serializer().load_kin_file("f.kin")


def test_aot_engine_compile_and_load(monkeypatch):
    e = krt.AOTEngine()
    e.compile_ahead_of_time("aot.kin", 1234, "CUDA_sm100")
    raw = open("aot.kin", "rb").read()
    kb_off, kb_size = struct.unpack_from("<QQ", raw, 4 + 4 + 512 + 8 + 16)
    image = raw[kb_off:kb_off + kb_size]
    assert image[:4] == b"\x7fELF" and image[18:20] == b"\xBE\x00"
    assert b'"artifact_kind": "mock"' in raw[KIN_HEADER:kb_off]
    with pytest.raises(RuntimeError, match="Refusing to load mock artifact"):
        e.load_model("aot.kin")
    monkeypatch.setenv("KINETIC_ALLOW_MOCKS", "1")
    e.load_model("aot.kin")
    assert krt.fake_cuda_state()["library_load"] == 1


def test_hardware_mismatch_propagates_from_engine(monkeypatch):
    monkeypatch.setenv("KINETIC_ALLOW_MOCKS", "1")
    s = krt.Serializer()
    s.save_kin_file("mm.kin", "gfx942", "ROCm_gfx942", 12345, list(b'{"artifact_kind": "mock"}'), [])
    with pytest.raises(krt.HardwareMismatchError, match="Hardware mismatch"):
        krt.AOTEngine().load_model("mm.kin")


def test_launch_without_module_and_descriptor_checks():
    e = krt.AOTEngine()
    with pytest.raises(RuntimeError, match="not loaded"):
        e.launch(1, 2, 4, 0, 0)
    d = krt.KernelLaunchDescriptor()
    assert (d.block_x, d.grid_y, d.eps) == (256, 1, pytest.approx(1e-5))
    d.kv_pool_ptr = 0x1000
    with pytest.raises(RuntimeError, match="host-only"):
        e.launch_descriptor(d, 0)


# ------------------------------------------------------------ TensorDescriptor
def test_tensor_descriptor_contract():
    torch = pytest.importorskip("torch")
    t = torch.arange(12, dtype=torch.float32).view(3, 4)
    d = krt.TensorDescriptor.from_tensor(t, "t")
    assert (d.shape, d.strides, d.byte_size, d.dtype) == ([3, 4], [4, 1], 48, krt.DataType.FLOAT32)
    with pytest.raises(ValueError, match="not C-contiguous"):
        krt.TensorDescriptor.from_tensor(t.t(), "tt")
    with pytest.raises(ValueError, match="storage_offset"):
        krt.TensorDescriptor.from_tensor(t[1:], "off")
    with pytest.raises(ValueError, match="unsupported dtype"):
        krt.TensorDescriptor.from_tensor(t.to(torch.float64), "f64")
    bad = krt.TensorDescriptor()
    with pytest.raises(ValueError, match="null data_ptr"):
        bad.validate("bad")


# ------------------------------------------------------------ fusion_forge
def test_validate_compilation_messages():
    from python.kinetic_rt.fusion_forge import TritonCompilationError, validate_compilation
    ok = bytearray(64)
    ok[0:4], ok[4], ok[18:20] = b"\x7fELF", 2, b"\xE0\x00"
    validate_compilation(bytes(ok), "ROCm")
    cases = [(b"", "Triton compilation yielded an empty binary."),
             (b"NOT_AN_ELF_BINARY", "Triton binary lacks the standard ELF magic header."),
             (b"\x7fELF", "Triton binary is too short to be a valid ELF.")]
    b32 = bytearray(ok)
    b32[4] = 1
    cases.append((bytes(b32), "Triton binary is not a 64-bit ELF."))
    for mach in (b"\x3E\x00", b"\xE0\xFF"):
        bad = bytearray(ok)
        bad[18:20] = mach
        cases.append((bytes(bad), "Triton binary architecture is not AMDGPU."))
    for blob, msg in cases:
        with pytest.raises(TritonCompilationError) as ei:
            validate_compilation(blob, "ROCm")
        assert str(ei.value) == msg


def test_fusion_bridge_writes_kin(monkeypatch):
    from python.kinetic_rt.fusion_forge import compile_and_serialize
    monkeypatch.setenv("KINETIC_TARGET", "sm100")
    compile_and_serialize(krt.AOTEngine(), krt.Serializer(), "fused_kernel.kin")
    assert os.path.exists("fused_kernel.kin")
    assert krt.Serializer().load_kin_file("fused_kernel.kin")[:4] == list(b"\x7fELF")
