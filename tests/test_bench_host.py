"""Host-side helpers of bench.py (no GPU): the NUMA-local CPU set that the
end-to-end measurement binds to while it allocates pinned buffers and
launches its graphs."""
import os
import types

import bench


def test_parse_cpulist():
    assert bench.parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert bench.parse_cpulist("5") == {5}
    assert bench.parse_cpulist("") == set()


def _fake_torch(domain, bus, dev):
    props = types.SimpleNamespace(pci_domain_id=domain, pci_bus_id=bus, pci_device_id=dev)
    return types.SimpleNamespace(cuda=types.SimpleNamespace(get_device_properties=lambda d: props))


def test_gpu_local_cpus_reads_the_gpu_pci_function(tmp_path):
    allowed = sorted(os.sched_getaffinity(0))
    fn = tmp_path / "0000:1b:00.0"
    fn.mkdir()
    # a node holding only the first allowed CPU (plus one that is not allowed)
    (fn / "local_cpulist").write_text(f"{allowed[0]},{max(allowed) + 1000}\n")
    got = bench.gpu_local_cpus(_fake_torch(0, 0x1B, 0), 0, sysfs=str(tmp_path))
    if len(allowed) == 1:
        assert got is None            # the node covers every allowed CPU: nothing to bind
    else:
        assert got == {allowed[0]}


def test_gpu_local_cpus_unknown_device(tmp_path):
    assert bench.gpu_local_cpus(_fake_torch(0, 0x2A, 0), 0, sysfs=str(tmp_path)) is None


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` (the CPU path, no GPU) prints one JSON line
    with the keys the driver reads, on the same metric and config as the
    GPU arm's default (stack) workload."""
    import json
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["value"] > 0
    assert d["config"] == bench.stack_config(1)
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"
    assert d["cpu_baseline"]["cores"] == os.cpu_count()


def test_stack_kernel_bytes_cover_the_step():
    """Per-GPU algorithmic bytes of one decode step at TP=1 and context 4224:
    the weights (about 15 GB without the embedding) plus the KV cache read
    (about 71 GB)."""
    kb = bench.stack_kernel_bytes(1, 4224)
    per_step = sum(v[0] * (bench.LAYERS if k not in ("lm_head_argmax", "greedy_step") else 1) for k, v in kb.items())
    assert 85e9 < per_step < 88e9
    kb8 = bench.stack_kernel_bytes(8, 4224)
    kv = lambda kb, heads: kb["paged_attention"][0] - 2 * 128 * heads * 128 * 2  # the K/V part
    assert kv(kb, 32) == 8 * kv(kb8, 4)


def test_stack_config_names_the_metric_workload():
    c = bench.stack_config(8)
    assert c["layers"] == 32 and c["global_batch"] == 128 and c["parallelism"] == "tp8"
    assert "per_box" in c and c["vocab"] == 128256


def test_seventy_b_stack_sizes():
    """Config 5's decode half: 80 layers, hidden 8192, batch 256 at context
    2048.  Its weights (141 GB) and KV cache (about 172 GB) need TP >= 4 on
    180 GB GPUs; at TP=8 one step moves about 41 GB per GPU (weight shards
    17.4 GB, K/V 21.5 GB, activations and the residual stream 2.4 GB)."""
    c = bench.stack_config(8, "70b")
    assert c["layers"] == 80 and c["hidden"] == 8192 and c["global_batch"] == 256 and c["seq_len"] == 2048
    assert not bench.stack_fits("70b", 1)[0] and not bench.stack_fits("70b", 2)[0]
    assert bench.stack_fits("70b", 8)[0] and bench.stack_fits("8b", 1)[0]
    kb = bench.stack_kernel_bytes(8, 2048, 256, "70b")
    per_step = sum(v[0] * (80 if k not in ("lm_head_argmax", "greedy_step") else 1) for k, v in kb.items())
    assert 40e9 < per_step < 42.5e9
