"""Benchmark of the decoder hot path on B200.

One step = one Llama-3-8B decoder layer's hot path for a decode batch of 64
sequences at context 2048, tensor-parallel over N GPUs (one process each):

  1. fused RMSNorm + QKV projection + RoPE + paged K/V scatter
     (krt_qkv_rope_decode; Q/K/V heads split over ranks, no collective)
  2. o_proj   row-parallel GEMM fused with the allreduce (K = 4096 / N)
  3. down_proj row-parallel GEMM fused with the allreduce (K = 14336 / N)

Inputs are synthetic (seeded N(0,1) activations, N(0, 0.02) weights,
gamma = 1 + N(0, 0.1), block tables a seeded permutation of the pool).  Each
step uses the weights of a different layer, cycling over enough layers that
the weights touched between two uses of a layer exceed the 126 MB L2.
Steps are CUDA-graph replays (8 steps per graph, the kernels chained by
programmatic dependent launch); the timed region is bracketed by a barrier
and device synchronisation and timed with CUDA events, max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl krt|reference]
  python bench.py --workload prefill     # the fused QKV prefill kernel alone (TFLOP/s)

For N > 1 launch one process per GPU with torch.distributed.run.  Prints one
JSON line on rank 0.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "kinetic-rt_b200"))

METRIC = "decode tokens/s per box at TP=1/2/4/8; fused QKV+RoPE & GEMM+AR % roofline"
HIDDEN, N_HEADS, N_KV, HEAD_DIM, INTER = 4096, 32, 8, 128, 14336
BATCH, CTX, BLOCK = 64, 2048, 16
L2_BYTES = 126 * 1024 * 1024
NVLINK_GBS = 770.0  # measured B200 peer-copy bandwidth per direction over NVLink 5 (900 GB/s nominal)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def workload_config(n):
    return {
        "workload": (f"Llama-3-8B decoder-layer hot path, decode batch {BATCH} at context {CTX}, TP={n}: "
                     "fused RMSNorm+QKV+RoPE+paged-KV scatter, o_proj GEMM+allreduce, down_proj GEMM+allreduce"),
        "global_batch": BATCH, "seq_len": CTX, "parallelism": f"tp{n}", "hidden": HIDDEN,
        "heads": f"{N_HEADS}/{N_KV}x{HEAD_DIM}", "intermediate": INTER, "kv_block": BLOCK,
        "l2": "weights rotated over layers whose total exceeds L2",
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML every
    2 ms while the timed region runs."""
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, gpu_index):
        self.gpu, self.samples, self.reasons, self.stop_evt, self.thread = gpu_index, [], set(), None, None
        self.max_mhz = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:
            return
        self.stop_evt = threading.Event()

        def poll():
            while not self.stop_evt.is_set():
                try:
                    self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for mask, name in self.REASONS.items():
                        if bits & mask:
                            self.reasons.add(name)
                except Exception:
                    pass
                time.sleep(0.002)

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": ["nvml unavailable"]}
        self.stop_evt.set()
        self.thread.join(timeout=2)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": sorted(self.reasons)}


# ------------------------------------------------------------- CPU baseline
def cpu_baseline(seconds=10.0):
    """The reference's CPU path (torch fp32 on all host cores, oracle/torch_ref.py)
    on the full step's shapes, repeated for about `seconds`."""
    import torch
    from oracle import torch_ref
    from oracle.fused_layer import rope_tables
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    x = torch.randn(BATCH, HIDDEN, generator=g)
    w_qkv = torch.randn((N_HEADS + 2 * N_KV) * HEAD_DIM, HIDDEN, generator=g) * 0.02
    gamma = 1 + 0.1 * torch.randn(HIDDEN, generator=g)
    cos, sin = (torch.from_numpy(a) for a in rope_tables([CTX - 1] * BATCH, HEAD_DIM, 5e5))
    attn = torch.randn(BATCH, HIDDEN, generator=g)
    w_o = torch.randn(HIDDEN, HIDDEN, generator=g) * 0.02
    act = torch.randn(BATCH, INTER, generator=g)
    w_d = torch.randn(HIDDEN, INTER, generator=g) * 0.02
    torch_ref.layer_hot_path_ref(x, w_qkv, gamma, cos, sin, attn, w_o, act, w_d, N_HEADS, N_KV, HEAD_DIM)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        torch_ref.layer_hot_path_ref(x, w_qkv, gamma, cos, sin, attn, w_o, act, w_d, N_HEADS, N_KV, HEAD_DIM)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": BATCH / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} steps of the full {BATCH}-token layer hot path in torch fp32 (oracle/torch_ref.py), "
                      f"{dt * 1e3:.1f} ms/step"}


# --------------------------------------------------------------- GPU setup
class Layer:
    """Weights of one decoder layer (this rank's shards)."""

    def __init__(self, torch, rank, world, seed):
        g = torch.Generator(device="cuda").manual_seed(seed)
        hq, hkv = N_HEADS // world, N_KV // world
        rows = (hq + 2 * hkv) * HEAD_DIM
        self.w_qkv = (torch.randn(rows, HIDDEN, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        self.gamma = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device="cuda")).to(torch.bfloat16)
        self.w_o = (torch.randn(HIDDEN, HIDDEN // world, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        self.w_d = (torch.randn(HIDDEN, INTER // world, generator=g, device="cuda") * 0.02).to(torch.bfloat16)

    @property
    def nbytes(self):
        return sum(t.numel() * 2 for t in (self.w_qkv, self.gamma, self.w_o, self.w_d))


class Rig:
    def __init__(self, torch, rank, world, comm):
        from python.kinetic_rt import _lib
        from oracle.fused_layer import rope_tables
        self.torch, self.lib, self.rank, self.world, self.comm = torch, _lib, rank, world, comm
        self.hq, self.hkv = N_HEADS // world, N_KV // world
        g = torch.Generator(device="cuda").manual_seed(1234 + rank)
        probe = Layer(torch, rank, world, 0)
        self.n_layers = max(2, -(-2 * L2_BYTES // probe.nbytes) + 1)
        self.layers = [probe] + [Layer(torch, rank, world, 1 + i) for i in range(self.n_layers - 1)]
        self.x = torch.randn(BATCH, HIDDEN, generator=g, device="cuda").to(torch.bfloat16)
        self.attn = torch.randn(BATCH, HIDDEN // world, generator=g, device="cuda").to(torch.bfloat16)
        self.act = torch.randn(BATCH, INTER // world, generator=g, device="cuda").to(torch.bfloat16)
        cos, sin = rope_tables(range(CTX), HEAD_DIM, 5e5)
        self.cos, self.sin = torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda()
        self.positions = torch.full((BATCH,), CTX - 1, dtype=torch.int32, device="cuda")
        self.token_seq = torch.arange(BATCH, dtype=torch.int32, device="cuda")
        blocks_per_seq = CTX // BLOCK
        self.num_blocks = BATCH * blocks_per_seq
        perm = torch.randperm(self.num_blocks, generator=torch.Generator().manual_seed(7)).to(torch.int32)
        self.block_table = perm.view(BATCH, blocks_per_seq).cuda()
        self.pool = torch.zeros(self.num_blocks, BLOCK, 2 * self.hkv * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
        self.q = torch.empty(BATCH, self.hq * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
        self.y_o = torch.empty(BATCH, HIDDEN, dtype=torch.bfloat16, device="cuda")
        self.y_d = torch.empty(BATCH, HIDDEN, dtype=torch.bfloat16, device="cuda")
        self.ws_qkv = torch.zeros(_lib.decode_workspace_bytes(BATCH, HIDDEN, self.hq, self.hkv), dtype=torch.uint8,
                                  device="cuda")
        self.ws_gemm = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
        self.args = []
        for L in self.layers:
            qa = _lib.paged_args(self.x, L.w_qkv, None, L.gamma, self.cos, self.sin, self.positions, self.token_seq,
                                 self.block_table, self.pool, self.q, self.hq, self.hkv, self.num_blocks, BLOCK,
                                 self.ws_qkv)
            oa = _lib.gemm_ar_args(self.attn, L.w_o, self.y_o, self.ws_gemm)
            da = _lib.gemm_ar_args(self.act, L.w_d, self.y_d, self.ws_gemm)
            self.args.append((qa, oa, da))
        self.comm_handle = comm.handle if comm is not None else None
        self.launches_per_step = 4  # prep + decode, o_proj, down_proj

    def step(self, i, parts=(0, 1, 2), args=None):
        qa, oa, da = (args or self.args)[i % self.n_layers]
        if 0 in parts:
            self.lib.qkv_rope_decode(qa)
        if 1 in parts:
            self.lib.rowparallel_gemm_ar(self.comm_handle, oa)
        if 2 in parts:
            self.lib.rowparallel_gemm_ar(self.comm_handle, da)

    def io_set(self):
        """A second set of step inputs and outputs (and the per-layer call
        arguments that use them), for pipelining host copies across steps."""
        torch, _lib = self.torch, self.lib
        io = {k: torch.empty_like(getattr(self, k)) for k in ("x", "attn", "act", "q", "y_o", "y_d")}
        for k in ("x", "attn", "act"):
            io[k].copy_(getattr(self, k))
        io["ws_qkv"] = torch.zeros_like(self.ws_qkv)
        io["args"] = []
        for L in self.layers:
            qa = _lib.paged_args(io["x"], L.w_qkv, None, L.gamma, self.cos, self.sin, self.positions, self.token_seq,
                                 self.block_table, self.pool, io["q"], self.hq, self.hkv, self.num_blocks, BLOCK,
                                 io["ws_qkv"])
            oa = _lib.gemm_ar_args(io["attn"], L.w_o, io["y_o"], self.ws_gemm)
            da = _lib.gemm_ar_args(io["act"], L.w_d, io["y_d"], self.ws_gemm)
            io["args"].append((qa, oa, da))
        return io

    def graphs(self, parts=(0, 1, 2), per_graph=1):
        """One CUDA graph per starting layer; graph k holds steps
        k*per_graph .. (k+1)*per_graph - 1, so replaying the graphs in order
        walks the layers in order."""
        torch = self.torch
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for i in range(self.n_layers):
                self.step(i, parts)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        gs = []
        for k in range(self.n_layers):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(k * per_graph, (k + 1) * per_graph):
                    self.step(i, parts)
            gs.append(g)
        return gs

    def check_status(self):
        for ws in (self.ws_qkv, self.ws_gemm):
            rc, bits = self.lib.read_status(ws)
            if rc != 0:
                raise RuntimeError(f"kernel status {bits:#x}")


def max_over_ranks(torch, value, world):
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(torch, world):
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def parse_cpulist(text):
    """CPU ids of a sysfs cpulist string ("0-3,8,10-11")."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def gpu_local_cpus(torch, device, sysfs="/sys/bus/pci/devices"):
    """The allowed CPUs on the GPU's own NUMA node (the local_cpulist of its
    PCI function in sysfs), or None when that is unknown or covers them all."""
    try:
        p = torch.cuda.get_device_properties(device)
        path = f"{sysfs}/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/local_cpulist"
        with open(path) as f:
            local = parse_cpulist(f.read())
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None
    allowed = os.sched_getaffinity(0)
    local &= allowed
    return local if local and local != allowed else None


STEPS_PER_GRAPH = 8


def timed_graph_replays(torch, graphs, steps, world):
    """Time exactly `steps` steps: graphs[0] holds STEPS_PER_GRAPH steps per
    replay, graphs[1] one step (the remainder)."""
    multi, single = graphs
    barrier(torch, world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps // STEPS_PER_GRAPH):
        multi[i % len(multi)].replay()
    for i in range(steps % STEPS_PER_GRAPH):
        single[i % len(single)].replay()
    b.record()
    barrier(torch, world)
    return a.elapsed_time(b)  # ms


def run_krt(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    comm = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
        from python.kinetic_rt.dist import TPComm
        comm = TPComm(rank, world, max_n_out=HIDDEN)
    rig = Rig(torch, rank, world, comm)
    graphs = (rig.graphs(per_graph=STEPS_PER_GRAPH), rig.graphs())
    for i in range(args.warmup):
        graphs[1][i % len(graphs[1])].replay()
    rig.check_status()

    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.05)
    ms = timed_graph_replays(torch, graphs, args.steps, world)
    clk = clocks.stop()
    rig.check_status()
    ms = max_over_ranks(torch, ms, world)
    ms_step = ms / args.steps
    value = BATCH / (ms_step * 1e-3)

    # per-kernel durations: graphs of one kernel type, replayed over all layers
    hbm, peak_kind = peaks()
    kernels = []
    hq, hkv = rig.hq, rig.hkv
    kbytes = [
        ("qkv_rope_decode", (hq + 2 * hkv) * HEAD_DIM * HIDDEN * 2 + BATCH * HIDDEN * 2 * 2 + BATCH * hkv * HEAD_DIM * 4,
         "W_qkv + x read, q + K/V written"),
        ("o_proj_gemm_ar", HIDDEN * (HIDDEN // world) * 2 + BATCH * (HIDDEN // world) * 2 + BATCH * HIDDEN * 2,
         "W_o shard + x read, y written"),
        ("down_proj_gemm_ar", HIDDEN * (INTER // world) * 2 + BATCH * (INTER // world) * 2 + BATCH * HIDDEN * 2,
         "W_down shard + x read, y written"),
    ]
    traffic = {}
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            traffic = json.load(f)
    except Exception:
        pass
    reps = max(min(args.steps, 2000), 2 * rig.n_layers)
    for part, (name, nbytes, what) in enumerate(kbytes):
        g = (rig.graphs(parts=(part,), per_graph=STEPS_PER_GRAPH), rig.graphs(parts=(part,)))
        for i in range(3):
            g[0][i % len(g[0])].replay()
        kms = max_over_ranks(torch, timed_graph_replays(torch, g, reps, world), world) / reps
        ach = nbytes / (kms * 1e-3) / 1e9
        entry = {"kernel": name, "bound": "hbm", "us": round(kms * 1e3, 3), "algorithmic_bytes": nbytes,
                 "bytes": what, "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                 "frac": round(ach / hbm, 4), "traffic": traffic.get(f"{name}_tp{world}")}
        if part > 0 and world > 1:
            # fused allreduce of the [64, 4096] output: bus bytes as NCCL counts
            # them (2 (w-1)/w x bf16 message) and the bytes this build puts on
            # NVLink per GPU (4 B per value in each of the two phases)
            msg = BATCH * HIDDEN * 2
            bus = 2 * (world - 1) / world * msg
            wire = 2 * (world - 1) / world * BATCH * HIDDEN * 4
            target_us = max(nbytes / hbm / 1e3, wire / NVLINK_GBS / 1e3)
            entry.update({"allreduce_bus_bytes": int(bus), "allreduce_bus_GBps": round(bus / (kms * 1e-3) / 1e9, 1),
                          "nvlink_wire_bytes_per_gpu": int(wire), "nvlink_peak_GBps": NVLINK_GBS,
                          "roofline_us": round(target_us, 3), "frac_of_roofline": round(target_us / (kms * 1e3), 4)})
        kernels.append(entry)
    rig.check_status()
    dominant = max(kernels, key=lambda k: k["us"])

    # End to end through the C ABI with host buffers: every step copies its
    # activations from pinned host memory, runs the three calls and copies q
    # and both layer outputs back.  Two input/output sets alternate so that a
    # step's copies overlap its neighbours' kernels (H2D and D2H on their own
    # streams).  One CUDA graph holds a whole number of passes over the layers
    # and at least 48 steps, since the pipeline drains where a graph ends (its
    # side streams join the main one).  The pinned buffers are allocated, and
    # the graphs launched, from the CPUs of the GPU's own NUMA node: pinned
    # pages on the far socket cross the inter-socket link on every copy.
    saved_cpus = os.sched_getaffinity(0)
    local_cpus = gpu_local_cpus(torch, local_rank)
    if local_cpus:
        try:
            os.sched_setaffinity(0, local_cpus)
        except OSError:
            local_cpus = None
    ios = [rig.io_set(), rig.io_set()]
    pin = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t.cpu())
    h_in = [{k: pin(io[k]) for k in ("x", "attn", "act")} for io in ios]
    h_out = [{k: torch.empty(io[k].shape, dtype=io[k].dtype, pin_memory=True) for k in ("q", "y_o", "y_d")}
             for io in ios]
    h2d = sum(t.numel() * t.element_size() for t in h_in[0].values())
    d2h = sum(t.numel() * t.element_size() for t in h_out[0].values())
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    passes = -(-48 // rig.n_layers)
    e2e_per_graph = rig.n_layers * passes  # a graph starts at layer 0 and ends at the last layer

    def e2e_steps_captured(first):
        comp = torch.cuda.current_stream()
        ev = lambda: torch.cuda.Event()
        done_in, done_comp, done_out = {}, {}, {}
        fork = ev()
        fork.record(comp)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        for i in range(first, first + e2e_per_graph):
            b = i % 2
            with torch.cuda.stream(s_in):
                if i - 2 in done_comp:
                    s_in.wait_event(done_comp[i - 2])
                for k in ("x", "attn", "act"):
                    ios[b][k].copy_(h_in[b][k], non_blocking=True)
                done_in[i] = ev()
                done_in[i].record(s_in)
            comp.wait_event(done_in[i])
            if i - 2 in done_out:
                comp.wait_event(done_out[i - 2])
            rig.step(i, args=ios[b]["args"])
            done_comp[i] = ev()
            done_comp[i].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done_comp[i])
                for k in ("q", "y_o", "y_d"):
                    h_out[b][k].copy_(ios[b][k], non_blocking=True)
                done_out[i] = ev()
                done_out[i].record(s_out)
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)

    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap):
        e2e_steps_captured(0)  # eager warm-up of the same sequence
    torch.cuda.current_stream().wait_stream(cap)
    torch.cuda.synchronize()
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_steps_captured(0)
    e2e_steps = e2e_per_graph * max(2, min(args.steps, 800) // e2e_per_graph)
    e2e_graph.replay()
    barrier(torch, world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(e2e_steps // e2e_per_graph):
        e2e_graph.replay()
    b.record()
    barrier(torch, world)
    e2e_ms = max_over_ranks(torch, a.elapsed_time(b), world) / e2e_steps
    if local_cpus:
        os.sched_setaffinity(0, saved_cpus)  # the CPU baseline below uses every allowed core
    rig.check_status()
    for io in ios:
        rc, bits = rig.lib.read_status(io["ws_qkv"])
        if rc != 0:
            raise RuntimeError(f"kernel status {bits:#x}")

    base = cpu_baseline() if rank == 0 else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s (one decoder layer's hot path)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights and activations)", "config": workload_config(world),
            "e2e": {"value": round(BATCH / (e2e_ms * 1e-3), 1), "unit": "tokens/s (one decoder layer's hot path)",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "host_cpus": (f"{len(local_cpus)} on the GPU's NUMA node" if local_cpus
                                  else f"all {len(saved_cpus)} allowed")},
            "gpu_launches": rig.launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "kernel": dominant["kernel"], "achieved": dominant["achieved"],
                         "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": dominant["frac"],
                         "traffic": dominant["traffic"]},
            "kernels": kernels,
            "cpu_baseline": base,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        import torch.distributed as dist
        del graphs, e2e_graph
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args, rank, world, local_rank):
    """Prefill of the fused RMSNorm + QKV + RoPE + paged scatter (not the
    decode step): 8 sequences x 2048 tokens, Llama-3-8B heads split over the
    N ranks (each rank its own shard, no collective), bf16 tcgen05 tiles.
    The activations (134 MB) exceed L2.  Reports TFLOP/s against the
    measured dense bf16 peak."""
    import torch
    from python.kinetic_rt import _lib
    from oracle.fused_layer import rope_tables
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
    seqs, seq_len = 8, 2048
    T = seqs * seq_len
    hq, hkv = N_HEADS // world, N_KV // world
    rows = (hq + 2 * hkv) * HEAD_DIM
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    x = torch.randn(T, HIDDEN, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(rows, HIDDEN, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(HIDDEN, generator=g, device="cuda")).to(torch.bfloat16)
    cos, sin = (torch.from_numpy(a).cuda() for a in rope_tables(range(seq_len), HEAD_DIM, 5e5))
    positions = torch.arange(seq_len, dtype=torch.int32, device="cuda").repeat(seqs)
    token_seq = torch.arange(seqs, dtype=torch.int32, device="cuda").repeat_interleave(seq_len)
    nblk = seqs * seq_len // BLOCK
    perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(5)).to(torch.int32)
    table = perm.view(seqs, seq_len // BLOCK).cuda()
    pool = torch.zeros(nblk, BLOCK, 2 * hkv * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(T, hq * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.prefill_workspace_bytes(T, HIDDEN, hq, hkv), dtype=torch.uint8, device="cuda")
    a = _lib.paged_args(x, w, None, gamma, cos, sin, positions, token_seq, table, pool, q, hq, hkv, nblk, BLOCK, ws)
    per_graph = 4
    _lib.qkv_rope_prefill(a)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            _lib.qkv_rope_prefill(a)
    for _ in range(max(1, args.warmup // per_graph)):
        graph.replay()
    reps = max(1, min(args.steps, 40) // per_graph)
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    barrier(torch, world)
    clk = clocks.stop()
    ms = max_over_ranks(torch, e0.elapsed_time(e1), world) / (reps * per_graph)
    rc, bits = _lib.read_status(ws)
    if rc != 0:
        raise RuntimeError(f"kernel status {bits:#x}")
    flops = 2.0 * T * HIDDEN * rows * world
    tflops = flops / (ms * 1e-3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peak, peak_sus, kind = float(pk["bf16_tflops"]), float(pk["bf16_tflops_sustained"]), "measured"
    except Exception:
        peak, peak_sus, kind = 1590.0, 1400.0, "fallback"
    if rank == 0:
        print(json.dumps({
            "metric": "prefill TFLOP/s (fused RMSNorm+QKV+RoPE+paged-KV scatter, 8 x 2048 tokens)",
            "value": round(tflops, 1), "unit": "TFLOP/s", "n_gpus": world, "steps": reps * per_graph,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (seeded random weights and activations)",
            "config": {"workload": f"Llama-3-8B fused QKV prefill, 8 x 2048 tokens, TP={world}",
                       "tokens": T, "hidden": HIDDEN, "heads": f"{N_HEADS}/{N_KV}x{HEAD_DIM}",
                       "l2": "activations (134 MB) exceed L2"},
            "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": peak,
                         "peak_sustained": peak_sus, "peak_kind": kind, "unit": "TFLOP/s per GPU",
                         "frac": round(tflops / world / peak, 4), "frac_of_sustained": round(tflops / world / peak_sus, 4)},
            "clocks": clk,
        }), flush=True)
    if world > 1:
        import torch.distributed as dist
        del graph
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank, world):
    """The reference's own CPU path (torch fp32, every host core), rank 0 only."""
    if rank != 0:
        return
    import torch
    from oracle import torch_ref
    from oracle.fused_layer import rope_tables
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    x = torch.randn(BATCH, HIDDEN, generator=g)
    w_qkv = torch.randn((N_HEADS + 2 * N_KV) * HEAD_DIM, HIDDEN, generator=g) * 0.02
    gamma = 1 + 0.1 * torch.randn(HIDDEN, generator=g)
    cos, sin = (torch.from_numpy(a) for a in rope_tables([CTX - 1] * BATCH, HEAD_DIM, 5e5))
    attn = torch.randn(BATCH, HIDDEN, generator=g)
    w_o = torch.randn(HIDDEN, HIDDEN, generator=g) * 0.02
    act = torch.randn(BATCH, INTER, generator=g)
    w_d = torch.randn(HIDDEN, INTER, generator=g) * 0.02
    f = lambda: torch_ref.layer_hot_path_ref(x, w_qkv, gamma, cos, sin, attn, w_o, act, w_d, N_HEADS, N_KV, HEAD_DIM)
    # Each step is ~10 ms of CPU work: run at most 2000 so the arm ends in minutes.
    steps, warmup = min(args.steps, 2000), min(args.warmup, 10)
    for _ in range(warmup):
        f()
    t0 = time.perf_counter()
    for _ in range(steps):
        f()
    dt = (time.perf_counter() - t0) / steps
    value = BATCH / dt
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 1),
        "unit": "tokens/s (one decoder layer's hot path)", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random weights and activations)",
        "config": workload_config(world),
        "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{steps} steps of the full {BATCH}-token layer hot path in torch fp32 "
                                   "(oracle/torch_ref.py restating tests/test_fusion.py:11-51)"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s (one decoder layer's hot path)",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["krt", "reference"], default="krt")
    ap.add_argument("--workload", choices=["decode", "prefill"], default="decode",
                    help="decode: the decoder-layer step (default); prefill: the fused QKV prefill kernel alone")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}; using WORLD_SIZE", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.workload == "prefill":
        run_prefill(args, rank, world, local_rank)
    else:
        run_krt(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
