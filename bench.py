"""Benchmark of the decoder hot path on B200.

Default workload (``--workload stack``): the metric's own configuration,
decode tokens/s of a Llama-3-8B-shaped stack (random init, bf16): 32 layers,
hidden 4096, 32/8 heads x 128, SwiGLU 14336, vocabulary 128256, decode batch
128 at 4096-token contexts, paged KV blocks of 16, greedy sampling, one CUDA
graph per decode step, tensor-parallel over the N GPUs of the job (one
process each, torch.distributed.run for N > 1).  One step = one new token for
each of the 128 sequences through all 32 layers and the lm_head.  The prompt's
K/V are synthetic (random bf16 written into the paged pools, standing in for
the prefill of the 4096 random prompt tokens); the timed steps sit in the
middle of the 256 greedy steps (contexts 4096 .. 4352).  ``value`` = 128 x K /
device time of K steps (max over ranks); ``config.per_box`` scales it to the
8 GPUs of a box (8 / N replicas).

``--workload layer``: one decoder layer's hot path at decode batch 64 (fused
QKV+RoPE+KV scatter, o_proj and down_proj GEMM+allreduce), the kernels the
scope table names, with their own per-kernel rooflines.
``--workload prefill``: the fused QKV prefill kernel alone (TFLOP/s).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl krt|reference] [--workload stack|layer|prefill]

Prints one JSON line on rank 0.
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
HIDDEN, N_HEADS, N_KV, HEAD_DIM, INTER, VOCAB, LAYERS = 4096, 32, 8, 128, 14336, 128256, 32
BATCH, CTX, BLOCK = 64, 2048, 16              # --workload layer
STACK_BATCH, PROMPT, GEN_STEPS = 128, 4096, 256  # --workload stack
# --workload stack --model: (layers, hidden, heads, kv heads, intermediate,
# decode batch, prompt tokens, greedy steps).  8b = config 4 (the metric's
# workload); 70b = the decode half of config 5 (batch 256 at context 2048).
STACK_MODELS = {
    "8b": (32, 4096, 32, 8, 14336, 128, 4096, 256),
    "70b": (80, 8192, 64, 8, 28672, 256, 2048, 64),
}
L2_BYTES = 126 * 1024 * 1024
NVLINK_GBS = 770.0  # measured B200 peer-copy bandwidth per direction over NVLink 5 (900 GB/s nominal)
# allreduce messages (bf16 bytes) from which the NCCL route is taken, from the
# fused-vs-NCCL config-3 sweep on two B200s (us, o_proj / down_proj): T = 64
# fused 13.0 / 20.3 vs NCCL 29.5 / 40.8; T = 512 (4 MB) 62.4 / 99.8 vs
# 65.8 / 93.2; T = 4096 510.7 / 802.3 vs 247.8 / 380.8.  The decode stack's
# 1 MB messages stay on the fused exchange.
NCCL_THRESHOLD = 8 << 20


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
    return {"value": BATCH / dt, "unit": "tokens/s", "cores": os.cpu_count(), "cpu_model": cpu_model(), "kind": "port",
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

    base = cpu_baseline() if rank == 0 and world == 1 else {"value": None, "note": "timed at N=1 only"}
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


# ------------------------------------------------------------- the stack
def stack_config(n, model="8b"):
    L, D, H, KV, I, B, P, G = STACK_MODELS[model]
    name = "Llama-3-8B" if model == "8b" else "Llama-3-70B"
    return {
        "workload": (f"{name}-shaped decoder stack (random init), decode batch {B} at contexts "
                     f"{P}..{P + G} (prompt K/V synthetic), greedy, TP={n}: per layer fused "
                     "RMSNorm+QKV+RoPE+paged-KV scatter, paged GQA attention, o_proj GEMM+allreduce+residual, "
                     "RMSNorm+gate/up+SwiGLU, down_proj GEMM+allreduce+residual; then RMSNorm+lm_head+argmax and the "
                     "next embedding; one CUDA graph per decode step"),
        "model": f"llama-3-{model}-shaped", "layers": L, "global_batch": B, "seq_len": P,
        "gen_steps": G, "parallelism": f"tp{n}", "hidden": D, "heads": f"{H}/{KV}x{HEAD_DIM}",
        "intermediate": I, "vocab": VOCAB, "kv_block": BLOCK,
        "per_box": f"value x {8 // n} (8 / TP replicas on one 8-GPU box)" if 8 % n == 0 else None,
        "l2": "inputs larger than L2: each step streams every layer's weights and the whole KV cache",
    }


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def cpu_stack_sample(reps=2, attn_seqs=8, ctx=PROMPT + GEN_STEPS // 2):
    """Bounded sample of the reference's CPU path (torch fp32 on every host
    core, oracle/torch_ref.py) for one decode step of the stack: the
    projections of one decoder layer at batch 128 (attention over a 1-token
    context), attention over the full `ctx`-token context for `attn_seqs`
    sequences, and the lm_head + argmax at batch 128.  One step =
    32 x (projections + 128 / attn_seqs x attention) + lm_head."""
    import torch
    from oracle import torch_ref
    from oracle.fused_layer import rope_tables
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(0)
    r = lambda *sz, s=0.02: torch.randn(*sz, generator=g) * s
    B, D, I = STACK_BATCH, HIDDEN, INTER
    w = dict(w_qkv=r((N_HEADS + 2 * N_KV) * HEAD_DIM, D), g_attn=1 + r(D, s=0.1), w_o=r(D, D), g_mlp=1 + r(D, s=0.1),
             w_gate=r(I, D), w_up=r(I, D), w_down=r(D, I))
    cos, sin = (torch.from_numpy(a) for a in rope_tables([ctx] * B, HEAD_DIM, 5e5))
    h = torch.randn(B, D, generator=g)
    empty = torch.zeros(B, 0, N_KV, HEAD_DIM)
    kc = torch.randn(attn_seqs, ctx, N_KV, HEAD_DIM, generator=g)
    vc = torch.randn(attn_seqs, ctx, N_KV, HEAD_DIM, generator=g)
    w_lm, g_f = r(VOCAB, D), 1 + r(D, s=0.1)

    def proj():
        torch_ref.decode_layer_ref(h, w["w_qkv"], w["g_attn"], cos, sin, empty, empty, w["w_o"], w["g_mlp"],
                                   w["w_gate"], w["w_up"], w["w_down"], N_HEADS, N_KV, HEAD_DIM)

    def attn():
        hs = h[:attn_seqs]
        torch_ref.decode_layer_ref(hs, w["w_qkv"], w["g_attn"], cos[:attn_seqs], sin[:attn_seqs], kc, vc, w["w_o"],
                                   w["g_mlp"], w["w_gate"], w["w_up"], w["w_down"], N_HEADS, N_KV, HEAD_DIM)

    def lm():
        torch_ref.lm_head_greedy_ref(h, g_f, w_lm)

    def timed(f):
        f()
        t0 = time.perf_counter()
        for _ in range(reps):
            f()
        return (time.perf_counter() - t0) / reps

    t_proj, t_attn_sub, t_lm = timed(proj), timed(attn), timed(lm)
    # the attention sample also ran the projections for attn_seqs rows: keep only its attention share
    t_attn = max(t_attn_sub - t_proj * attn_seqs / B, 0.0) * (B / attn_seqs)
    step = LAYERS * (t_proj + t_attn) + t_lm
    return {"value": round(B / step, 3), "unit": "tokens/s", "cores": os.cpu_count(), "cpu_model": cpu_model(),
            "kind": "port", "step_s": round(step, 3),
            "sample": (f"torch fp32 (oracle/torch_ref.py), {reps} reps each: one layer's projections at batch {B} "
                       f"({t_proj * 1e3:.1f} ms), attention over {ctx} tokens for {attn_seqs} sequences scaled x"
                       f"{B // attn_seqs} ({t_attn * 1e3:.1f} ms), lm_head+argmax ({t_lm * 1e3:.1f} ms); "
                       f"step = {LAYERS} layers + lm_head")}


def tp_parity_check(torch, comm, rank, world):
    """o_proj / down_proj GEMM + allreduce (+ residual) on seeded inputs against
    the unsharded fp32 product (torch on this GPU), and bit-identity of the
    result across ranks.  Every rank generates the same full X, W and
    residual on the host and keeps its torch.chunk(dim=1) shard
    (scripts/export_hf.py:62-65)."""
    from python.kinetic_rt import _lib
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    worst, ok, same = 0.0, True, True
    for (T, K, with_res) in ((STACK_BATCH, HIDDEN, True), (STACK_BATCH, INTER, True), (BATCH, INTER, False),
                             (1, HIDDEN, False)):
        g = torch.Generator().manual_seed(K + T)
        x = torch.randn(T, K, generator=g).to(torch.bfloat16).cuda()
        w = (torch.randn(HIDDEN, K, generator=g) * 0.02).to(torch.bfloat16).cuda()
        res = torch.randn(T, HIDDEN, generator=g).to(torch.bfloat16).cuda()
        step = -(-K // world)
        lo, hi = rank * step, min((rank + 1) * step, K)
        xs, wsh = x[:, lo:hi].contiguous(), w[:, lo:hi].contiguous()
        y = res.clone() if with_res else torch.empty(T, HIDDEN, dtype=torch.bfloat16, device="cuda")
        args = _lib.gemm_ar_args(xs, wsh, y, ws, residual=y if with_res else None)
        _lib.rowparallel_gemm_ar(comm.handle if comm is not None else None, args)
        rc, bits = _lib.read_status(ws)
        ref = x.float() @ w.float().t() + (res.float() if with_res else 0)
        err = (y.float() - ref).abs()
        worst = max(worst, float(err.max()))
        ok = ok and bool((err <= 2e-2 + 1e-2 * ref.abs()).all()) and rc == 0
        if world > 1:
            import torch.distributed as dist
            allv = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(allv, y)
            same = same and all(torch.equal(a.view(torch.int16), allv[0].view(torch.int16)) for a in allv)
    return {"checked": True, "cases": "o_proj/down_proj at 128 tokens with residual, down_proj at 64, o_proj at 1",
            "max_abs": round(worst, 5), "within_tolerance": ok, "ranks_identical": same,
            "tolerance": "max-abs 2e-2 + rel 1e-2 vs unsharded fp32"}


GEMM_AR_TOKENS = (1, 8, 64, 512, 4096, 8192)


def gemm_ar_sweep(torch, comm, rank, world, tokens=GEMM_AR_TOKENS, reps=5):
    """Config 3: o_proj (K = 4096) and down_proj (K = 14336) row-parallel GEMM +
    allreduce at TP = world for each token count, through the fused exchange
    and through the NCCL route (GEMM, then ncclAllReduce), both timed on the
    device as 5 calls replayed from one CUDA graph (max over ranks; the weight
    shard stays in L2 across the calls when it fits) and checked against the
    unsharded fp32 product
    (torch on this GPU) and for bit-identity across ranks.  roofline_us =
    max(HBM bytes / HBM peak, FLOPs / bf16 peak, allreduce bus bytes / NVLink
    peak) with bus bytes 2 (N-1)/N x T x 4096 x 2 (a bf16 ring)."""
    import torch.distributed as dist
    from python.kinetic_rt import _lib
    hbm, _ = peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tflops = float(json.load(f)["bf16_tflops"])
    except Exception:
        tflops = 1590.0
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    rows = []
    for name, K in (("o_proj", HIDDEN), ("down_proj", INTER)):
        kr = K // world
        g = torch.Generator(device="cuda").manual_seed(K)
        w_full = (torch.randn(HIDDEN, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        w = w_full[:, rank * kr:(rank + 1) * kr].contiguous()
        for T in tokens:
            gx = torch.Generator(device="cuda").manual_seed(T * 7 + K)
            x_full = torch.randn(T, K, generator=gx, device="cuda").to(torch.bfloat16)
            x = x_full[:, rank * kr:(rank + 1) * kr].contiguous()
            ref = x_full.float() @ w_full.float().t()
            y = torch.empty(T, HIDDEN, dtype=torch.bfloat16, device="cuda")
            args = _lib.gemm_ar_args(x, w, y, ws)
            row = {"proj": name, "tokens": T, "tp": world}
            for route in ("fused", "nccl"):
                if route == "nccl" and (world == 1 or not getattr(comm, "has_nccl", False)):
                    continue
                if comm is not None and getattr(comm, "has_nccl", False):
                    comm.set_nccl_threshold(0 if route == "nccl" else (1 << 62))
                call = lambda: _lib.rowparallel_gemm_ar(comm.handle if comm is not None else None, args)
                call()
                torch.cuda.synchronize()
                rc, bits = _lib.read_status(ws)
                err = (y.float() - ref).abs()
                ok = rc == 0 and bool((err <= 2e-2 + 1e-2 * ref.abs()).all())
                same = True
                if world > 1:
                    allv = [torch.empty_like(y) for _ in range(world)]
                    dist.all_gather(allv, y)
                    same = all(torch.equal(a.view(torch.int16), allv[0].view(torch.int16)) for a in allv)
                # device time of `reps` calls replayed from one CUDA graph (no
                # host launch gaps; the graph is released before the next route)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    for _ in range(reps):
                        call()
                gr.replay()
                barrier(torch, world)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                gr.replay()
                e1.record()
                barrier(torch, world)
                us = max_over_ranks(torch, e0.elapsed_time(e1), world) * 1e3 / reps
                torch.cuda.synchronize()
                del gr
                row[f"{route}_us"] = round(us, 2)
                row[f"{route}_max_abs"] = round(float(err.max()), 4)
                row[f"{route}_ok"] = ok and same
            nbytes = HIDDEN * kr * 2 + T * kr * 2 + T * HIDDEN * 2
            flops = 2.0 * T * kr * HIDDEN
            bus = 2 * (world - 1) / world * T * HIDDEN * 2
            target = max(nbytes / hbm / 1e3, flops / tflops / 1e6, bus / NVLINK_GBS / 1e3)
            best = min(row.get("fused_us", 1e30), row.get("nccl_us", 1e30))
            row.update({"roofline_us": round(target, 3), "bound": ("hbm" if target == nbytes / hbm / 1e3 else
                                                                  "tensor" if target == flops / tflops / 1e6 else
                                                                  "nvlink"),
                        "best_route": "fused" if row.get("fused_us", 1e30) <= row.get("nccl_us", 1e30) else "nccl",
                        "frac_of_roofline": round(target / best, 4)})
            rows.append(row)
    if comm is not None and getattr(comm, "has_nccl", False):
        comm.set_nccl_threshold(comm.nccl_threshold)
    return rows


def run_gemm_ar(args, rank, world, local_rank):
    """--workload gemm_ar: the config-3 sweep alone, one JSON line."""
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
        comm.attach_nccl(NCCL_THRESHOLD)
    rows = gemm_ar_sweep(torch, comm, rank, world)
    if rank == 0:
        worst = min(r["frac_of_roofline"] for r in rows)
        print(json.dumps({
            "metric": "row-parallel GEMM + allreduce, % of roofline (config 3)", "value": worst,
            "unit": "min frac_of_roofline over rows", "n_gpus": world, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (N(0,1) activations, N(0,0.02) weights)", "scaling": "strong",
            "config": {"workload": f"o_proj [4096->4096] and down_proj [14336->4096], K sharded over TP={world}, "
                                   f"tokens {list(GEMM_AR_TOKENS)}"},
            "rows": rows, "all_ok": all(r.get("fused_ok", True) and r.get("nccl_ok", True) for r in rows)}),
            flush=True)
    if comm is not None:
        import torch.distributed as dist
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def stack_kernel_bytes(world, ctx, batch=STACK_BATCH, model="8b"):
    """Algorithmic bytes per launch of each kernel of the decode step (this
    rank's share): every input read once, every output written once."""
    _, D, H, KV, I = STACK_MODELS[model][:5]
    B = batch
    hq, hkv, ir = H // world, KV // world, I // world
    vr = -(-VOCAB // world)
    qkv_rows = (hq + 2 * hkv) * HEAD_DIM
    return {
        "qkv_rope_decode": (qkv_rows * D * 2 + B * D * 2 + B * hq * HEAD_DIM * 2 + B * 2 * hkv * HEAD_DIM * 2,
                            "W_qkv shard + x read, q + new K/V written"),
        "paged_attention": (B * ctx * hkv * HEAD_DIM * 2 * 2 + 2 * B * hq * HEAD_DIM * 2,
                            "K/V of every context token read, q read, output written"),
        "o_proj_gemm_ar": (D * hq * HEAD_DIM * 2 + B * hq * HEAD_DIM * 2 + 2 * B * D * 2,
                           "W_o shard + x + residual read, h written"),
        "gate_up_swiglu": (2 * ir * D * 2 + B * D * 2 + B * ir * 2, "W_gate|up shard + x read, act written"),
        "down_proj_gemm_ar": (D * ir * 2 + B * ir * 2 + 2 * B * D * 2, "W_down shard + act + residual read, h written"),
        "lm_head_argmax": (vr * D * 2 + B * D * 2, "lm_head shard + x read"),
        "greedy_step": (B * D * 2 * 2, "embedding rows read, h written"),
    }


def stack_fits(model, world, gpu_bytes=180e9):
    """Weights + KV pools of one rank against one GPU's memory (the 70B
    stack needs TP >= 2)."""
    L, D, H, KV, I, B, P, G = STACK_MODELS[model]
    weights = L * (((H + 2 * KV) * HEAD_DIM * D + D * H * HEAD_DIM + 3 * D * I) * 2 // world) \
        + (VOCAB * D * 2 // world) + VOCAB * D * 2
    kv = L * B * (P + G + 96) * 2 * (KV // world) * HEAD_DIM * 2
    return weights + kv < 0.85 * gpu_bytes, weights + kv


def run_stack(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    fits, need = stack_fits(args.model, world)
    if not fits:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": None, "unit": "decode tokens/s", "n_gpus": world,
                              "config": stack_config(world, args.model),
                              "unavailable": f"weights + KV of one rank ({need / 1e9:.0f} GB) exceed one GPU; "
                                             f"run the {args.model} stack at a higher TP"}), flush=True)
        return
    comm = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=120))
        from python.kinetic_rt.dist import TPComm
        comm = TPComm(rank, world, max_n_out=STACK_MODELS[args.model][1])
        comm.attach_nccl(NCCL_THRESHOLD)
    from python.kinetic_rt.decoder import LLAMA3_8B, LLAMA3_70B, PagedDecoder, RankWeights
    model = args.model
    shape = LLAMA3_8B if model == "8b" else LLAMA3_70B
    n_layers, _, _, _, _, B, prompt, gen_steps = STACK_MODELS[model]
    parity = tp_parity_check(torch, comm, rank, world)
    config3 = gemm_ar_sweep(torch, comm, rank, world) if world > 1 and model == "8b" else None
    K, W = args.steps, args.warmup
    # the position the first warm-up step processes: the timed steps sit in
    # the middle of the greedy steps after the prompt
    first = prompt + max(0, (gen_steps - K) // 2 - W)
    e2e_steps = min(K, 64)
    max_len = max(prompt + gen_steps, first + 1 + W + K + e2e_steps + 8)
    weights = RankWeights.random(torch, shape, rank, world, seed=0)
    dec = PagedDecoder(torch, shape, weights, B, max_len, comm, rank, world)
    g = torch.Generator(device="cuda").manual_seed(7)
    dec.pools[0].copy_(torch.randn(dec.pools[0].shape, generator=g, device="cuda").to(torch.bfloat16))
    for pool in dec.pools[1:]:
        pool.copy_(dec.pools[0])
    start = torch.randint(0, shape.vocab, (B,), generator=torch.Generator().manual_seed(11))
    dec.start(start, [first] * B)
    graph = dec.capture()  # after one eager step (first calls outside the capture), state restored
    dec.check_status()
    for _ in range(W):
        graph.replay()
    dec.check_status()
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.05)
    barrier(torch, world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(K):
        graph.replay()
    b.record()
    barrier(torch, world)
    clk = clocks.stop()
    dec.check_status()
    ms = max_over_ranks(torch, a.elapsed_time(b), world)
    ms_step = ms / K
    value = B * K / (ms * 1e-3)
    if world > 1:
        import torch.distributed as dist
        toks = [torch.empty_like(dec.tokens) for _ in range(world)]
        dist.all_gather(toks, dec.tokens)
        hs = [torch.empty_like(dec.h) for _ in range(world)]
        dist.all_gather(hs, dec.h)
        parity["step_tokens_identical"] = all(torch.equal(t, toks[0]) for t in toks)
        parity["step_hidden_identical"] = all(torch.equal(x.view(torch.int16), hs[0].view(torch.int16)) for x in hs)
    ctx_mid = first + W + K // 2

    # per-kernel device time: one graph per kernel kind over all layers
    hbm, peak_kind = peaks()
    traffic = {}
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            traffic = json.load(f)
    except Exception:
        pass
    kbytes = stack_kernel_bytes(world, ctx_mid, B, model)
    names = ["qkv_rope_decode", "paged_attention", "o_proj_gemm_ar", "gate_up_swiglu", "down_proj_gemm_ar"]
    kernels = []

    def time_graph(fn, launches, reps):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        gr.replay()
        barrier(torch, world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            gr.replay()
        e1.record()
        barrier(torch, world)
        us = max_over_ranks(torch, e0.elapsed_time(e1), world) * 1e3 / (reps * launches)
        del gr
        return us

    saved_pos = dec.positions.clone()
    for part, name in enumerate(names):
        us = time_graph(lambda: [dec.layer(li, parts=(part,)) for li in range(n_layers)], n_layers, 3)
        kernels.append((name, us))
    kernels.append(("lm_head_argmax", time_graph(lambda: _lm(dec), 1, 20)))
    kernels.append(("greedy_step", time_graph(lambda: _greedy(dec), 1, 20)))
    dec.positions.copy_(saved_pos)
    dec.seq_lens.copy_(saved_pos + 1)
    dec.check_status()
    klist = []
    for name, us in kernels:
        nbytes, what = kbytes[name]
        ach = nbytes / (us * 1e-6) / 1e9
        entry = {"kernel": name, "bound": "hbm", "us": round(us, 3), "algorithmic_bytes": int(nbytes), "bytes": what,
                 "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s", "frac": round(ach / hbm, 4),
                 "traffic": traffic.get(f"stack_{name}_tp{world}") if model == "8b" else None,
                 "launches_per_step": n_layers if name in names else 1}
        if name.endswith("gemm_ar") and world > 1:
            wire = 2 * (world - 1) / world * B * shape.d_model * 4
            target = max(nbytes / hbm / 1e3, wire / NVLINK_GBS / 1e3)
            entry.update({"nvlink_wire_bytes_per_gpu": int(wire), "roofline_us": round(target, 3),
                          "frac_of_roofline": round(target / us, 4)})
        klist.append(entry)
    step_bytes = sum(e["algorithmic_bytes"] * e["launches_per_step"] for e in klist)
    dominant = max(klist, key=lambda e: e["us"] * e["launches_per_step"])

    # end to end through the driver's public API: every step the host copies
    # the step's input tokens (pinned) to the device, replays the step and
    # reads the chosen tokens back, waiting for them (a serving loop)
    feed = torch.empty(e2e_steps + 1, B, dtype=torch.int32, pin_memory=True)
    got = torch.empty(e2e_steps, B, dtype=torch.int32, pin_memory=True)
    feed[0].copy_(dec.tokens.cpu())
    torch.cuda.synchronize()
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        dec.next_input.copy_(feed[i], non_blocking=True)
        graph.replay()
        got[i].copy_(dec.tokens, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        feed[i + 1].copy_(got[i])
    e1.record()
    barrier(torch, world)
    e2e_ms = max_over_ranks(torch, e0.elapsed_time(e1), world) / e2e_steps
    dec.check_status()
    prefill = prefill_entry(torch, rank, world) if model == "8b" else None
    del graph
    # whole-model prompt prefill: config 5's 4 x 8192 on the 70b stack; 8 x 2048
    # (config 2's prompts) on the 8b stack at N = 1
    prompt = None
    pf_seqs, pf_len = (4, 8192) if model == "70b" else (8, 2048)
    if model == "70b" or world == 1:
        try:
            prompt = prompt_prefill(torch, shape, weights, comm, rank, world, pf_seqs, pf_len)
        except Exception as exc:  # reported in the line; the decode numbers stand
            prompt = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    base = None
    if world == 1 and model == "8b":
        base = cpu_stack_sample()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "decode tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt ids and prompt K/V)",
            "config": stack_config(world, model),
            "per_box_tokens_per_s": round(value * 8 / world, 1) if 8 % world == 0 else None,
            "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "decode tokens/s",
                    "h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * 4,
                    "how": "per step: pinned-host tokens -> device, graph replay, chosen tokens -> pinned host, "
                           "host waits and feeds them to the next step"},
            "gpu_launches": dec.launches_per_step * K,
            "roofline": {"bound": "hbm", "kernel": dominant["kernel"], "achieved": dominant["achieved"], "peak": hbm,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": dominant["frac"],
                         "traffic": dominant["traffic"]},
            "step": {"algorithmic_bytes_per_gpu": int(step_bytes),
                     "achieved_GBps": round(step_bytes / (ms_step * 1e-3) / 1e9, 1),
                     "frac": round(step_bytes / (ms_step * 1e-3) / 1e9 / hbm, 4), "context_mid": ctx_mid},
            "kernels": klist + ([prefill] if prefill else []),
            "prompt_prefill": prompt,
            "parity": parity,
            "config3_gemm_ar": config3,
            "cpu_baseline": base if base else {"value": None, "note": "timed at N=1 on the 8b stack only (rank 0 "
                                                                      "alone on the host)"},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    bad = not (parity["within_tolerance"] and parity["ranks_identical"] and parity.get("step_tokens_identical", True)
               and parity.get("step_hidden_identical", True)
               and all(r.get("fused_ok", True) and r.get("nccl_ok", True) for r in (config3 or [])))
    if comm is not None:
        import torch.distributed as dist
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
    if bad:
        print("parity check failed", file=sys.stderr)
        sys.exit(3)


def prompt_prefill(torch, shape, weights, comm, rank, world, seqs, prompt_len):
    """A whole-model prefill: `seqs` random prompts of `prompt_len` tokens
    through PagedDecoder.prefill (prefill QKV, causal prefill attention,
    GEMM + allreduce and gate/up over whole prompts, lm_head + greedy on the
    last tokens), timed on the device (max over ranks) after a short untimed
    prefill of the same decoder.  FLOPs: 2 x tokens x (per-layer weights + the
    lm_head on the last tokens only) plus the causal attention, this rank's
    share."""
    from python.kinetic_rt.decoder import PagedDecoder
    dec = PagedDecoder(torch, shape, weights, seqs, prompt_len + 16, comm, rank, world)
    g = torch.Generator().manual_seed(13)
    warm = [torch.randint(0, shape.vocab, (min(prompt_len, 256),), generator=g) for _ in range(seqs)]
    prompts = [torch.randint(0, shape.vocab, (prompt_len,), generator=g) for _ in range(seqs)]
    dec.prefill(warm, group=seqs)
    torch.cuda.synchronize()
    barrier(torch, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    tok = dec.prefill(prompts, group=seqs)
    e1.record()
    torch.cuda.synchronize()
    barrier(torch, world)
    ms = max_over_ranks(torch, e0.elapsed_time(e1), world)
    dec.check_status()
    same = True
    if world > 1:
        import torch.distributed as dist
        toks = [torch.empty_like(tok) for _ in range(world)]
        dist.all_gather(toks, tok)
        same = all(torch.equal(t, toks[0]) for t in toks)
    D, hd = shape.d_model, shape.head_dim
    layer_params = ((shape.n_heads + 2 * shape.n_kv_heads) * hd * D + D * shape.n_heads * hd + 3 * D * shape.inter)
    T = seqs * prompt_len
    flops = (2.0 * T * layer_params * shape.n_layers + 2.0 * seqs * shape.vocab * D
             + shape.n_layers * seqs * shape.n_heads * hd * 4.0 * prompt_len * (prompt_len + 1) / 2) / world
    del dec
    torch.cuda.empty_cache()
    return {"seqs": seqs, "prompt_tokens": prompt_len, "ms": round(ms, 2), "tokens_per_s": round(T / (ms * 1e-3), 1),
            "flops_per_gpu": int(flops), "tflops_per_gpu": round(flops / (ms * 1e-3) / 1e12, 1),
            "first_tokens_identical_across_ranks": same,
            "how": "PagedDecoder.prefill: per layer prefill QKV + causal prefill attention + o_proj GEMM+allreduce "
                   "+ gate/up + down_proj GEMM+allreduce over whole prompts, then lm_head + greedy on the last "
                   "tokens; one run, device time, max over ranks"}


def _lm(dec):
    from python.kinetic_rt import _lib
    _lib.lm_head_argmax(dec.lm_args)


def _greedy(dec):
    from python.kinetic_rt import _lib
    _lib.greedy_step(dec.comm_handle, dec.greedy_args)


def prefill_entry(torch, rank, world, seqs=8, seq_len=2048):
    """The prefill kernel (fused QKV + RoPE + paged scatter) on this rank's
    head shard for 8 x 2048 tokens, as a kernels entry in TFLOP/s."""
    from python.kinetic_rt import _lib
    from python.kinetic_rt.decoder import rope_cache
    T = seqs * seq_len
    hq, hkv = N_HEADS // world, N_KV // world
    rows = (hq + 2 * hkv) * HEAD_DIM
    g = torch.Generator(device="cuda").manual_seed(99 + rank)
    x = torch.randn(T, HIDDEN, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(rows, HIDDEN, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    gamma = torch.ones(HIDDEN, dtype=torch.bfloat16, device="cuda")
    cos, sin = rope_cache(torch, seq_len, HEAD_DIM, 5e5)
    positions = torch.arange(seq_len, dtype=torch.int32, device="cuda").repeat(seqs)
    token_seq = torch.arange(seqs, dtype=torch.int32, device="cuda").repeat_interleave(seq_len)
    nblk = T // BLOCK
    table = torch.randperm(nblk, generator=torch.Generator().manual_seed(5)).to(torch.int32).view(seqs, -1).cuda()
    pool = torch.zeros(nblk, BLOCK, 2 * hkv * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(T, hq * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(_lib.prefill_workspace_bytes(T, HIDDEN, hq, hkv), dtype=torch.uint8, device="cuda")
    a = _lib.paged_args(x, w, None, gamma, cos, sin, positions, token_seq, table, pool, q, hq, hkv, nblk, BLOCK, ws)
    _lib.qkv_rope_prefill(a)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(4):
            _lib.qkv_rope_prefill(a)
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    rc, bits = _lib.read_status(ws)
    if rc != 0:
        raise RuntimeError(f"prefill status {bits:#x}")
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        peak = 1590.0
    tflops = 2.0 * T * HIDDEN * rows / (ms * 1e-3) / 1e12
    return {"kernel": "qkv_rope_prefill", "bound": "tensor", "us": round(ms * 1e3, 1),
            "algorithmic_flops": int(2 * T * HIDDEN * rows), "achieved": round(tflops, 1), "peak": peak,
            "unit": "TFLOP/s", "frac": round(tflops / peak, 4), "launches_per_step": 0,
            "shape": f"{seqs} x {seq_len} tokens, this rank's {hq}/{hkv} heads (not part of the decode step)"}


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
    if args.workload == "stack":
        return run_reference_stack(args, world)
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


def run_kernel(args, rank, world, local_rank):
    """--workload kernel --kernel NAME: one kernel of the decode step alone, at
    the stack's shapes (batch 128, context 4224, the shards of TP = --tp),
    cycling through enough weight copies that they exceed L2 twice over,
    --steps calls per CUDA graph, the graph replayed after --warmup eager
    calls.  A short case for knob sweeps and ncu captures (a few GB on the
    device).  Prints one JSON line with the device time per call."""
    import torch
    from python.kinetic_rt import _lib
    from python.kinetic_rt.decoder import rope_cache
    torch.cuda.set_device(local_rank)
    tp = args.tp or world
    _, D, H, KV, I, B0, P0, G0 = STACK_MODELS[args.model]
    B, ctx = args.batch or B0, P0 + G0 // 2
    H, KV, I, V = H // tp, KV // tp, I // tp, -(-VOCAB // tp)
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(B, D, generator=g, device="cuda").to(torch.bfloat16)
    gam = torch.ones(D, device="cuda", dtype=torch.bfloat16)
    name = args.kernel
    copies = lambda nbytes: max(1, -(-2 * L2_BYTES // nbytes))
    keep = []  # every tensor an argument struct points to stays referenced (the structs hold raw pointers)

    def rnd(*sz):
        t = (torch.randn(*sz, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        keep.append(t)
        return t
    if name == "paged_attention":
        bps = -(-ctx // BLOCK) + 1
        nb = B * bps
        pool = torch.randn(nb, BLOCK, 2 * KV * HEAD_DIM, generator=g, device="cuda").to(torch.bfloat16)
        table = torch.randperm(nb, device="cuda").to(torch.int32).view(B, bps)
        lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(B, H * HEAD_DIM, generator=g, device="cuda").to(torch.bfloat16)
        o = torch.empty_like(q)
        ws = torch.zeros(_lib.attention_workspace_bytes(B, H, KV, ctx), dtype=torch.uint8, device="cuda")
        args_list = [_lib.attention_args(q, pool, table, lens, o, H, KV, nb, BLOCK, ctx, ws)]
        call = _lib.paged_attention_decode
    elif name == "prefill_attention":
        # causal attention of 8 prompts x 2048 tokens (config 2's prefill) over a random pool
        S_, L_ = 8, 2048
        nb = S_ * L_ // BLOCK
        pool = torch.randn(nb, BLOCK, 2 * KV * HEAD_DIM, generator=g, device="cuda").to(torch.bfloat16)
        table = torch.randperm(nb, device="cuda").to(torch.int32).view(S_, -1)
        q = torch.randn(S_ * L_, H * HEAD_DIM, generator=g, device="cuda").to(torch.bfloat16)
        o = torch.empty_like(q)
        q_start = torch.arange(0, S_ * L_ + 1, L_, dtype=torch.int32, device="cuda")
        q_pos0 = torch.zeros(S_, dtype=torch.int32, device="cuda")
        ws = torch.zeros(_lib.prefill_attention_workspace_bytes(), dtype=torch.uint8, device="cuda")
        args_list = [_lib.prefill_attention_args(q, pool, table, q_start, q_pos0, o, H, KV, nb, BLOCK, L_, ws)]
        call = _lib.paged_attention_prefill
        flops = S_ * H * HEAD_DIM * 4.0 * L_ * (L_ + 1) / 2
    elif name == "gate_up_swiglu":
        act = torch.empty(B, I, device="cuda", dtype=torch.bfloat16)
        ws = torch.zeros(_lib.projection_workspace_bytes(B, D), dtype=torch.uint8, device="cuda")
        args_list = [_lib.gate_up_args(x, gam, rnd(2 * I, D), act, ws) for _ in range(copies(2 * I * D * 2))]
        call = _lib.gate_up_swiglu
    elif name == "lm_head_argmax":
        keys = torch.zeros(B, dtype=torch.int64, device="cuda")
        ws = torch.zeros(_lib.projection_workspace_bytes(B, D), dtype=torch.uint8, device="cuda")
        args_list = [_lib.lm_head_args(x, gam, rnd(V, D), keys, ws) for _ in range(copies(V * D * 2))]
        call = _lib.lm_head_argmax
    elif name in ("o_proj_gemm_ar", "down_proj_gemm_ar"):
        K = H * HEAD_DIM if name == "o_proj_gemm_ar" else I
        xx = torch.randn(B, K, generator=g, device="cuda").to(torch.bfloat16)
        y = torch.zeros(B, D, device="cuda", dtype=torch.bfloat16)
        ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
        args_list = [_lib.gemm_ar_args(xx, rnd(D, K), y, ws, residual=y) for _ in range(copies(D * K * 2))]
        call = lambda a: _lib.rowparallel_gemm_ar(None, a)
    elif name == "qkv_rope_decode":
        rows = (H + 2 * KV) * HEAD_DIM
        cos, sin = rope_cache(torch, ctx + 1, HEAD_DIM, 5e5)
        pos = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        seq = torch.arange(B, dtype=torch.int32, device="cuda")
        bps = -(-(ctx + 1) // BLOCK)
        bt = torch.arange(B * bps, dtype=torch.int32, device="cuda").view(B, bps)
        pool = torch.zeros(B * bps, BLOCK, 2 * KV * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
        qq = torch.empty(B, H * HEAD_DIM, dtype=torch.bfloat16, device="cuda")
        ws = torch.zeros(_lib.decode_workspace_bytes(B, D, H, KV), dtype=torch.uint8, device="cuda")
        args_list = [_lib.paged_args(x, rnd(rows, D), None, gam, cos, sin, pos, seq, bt, pool, qq, H, KV, B * bps,
                                     BLOCK, ws) for _ in range(copies(rows * D * 2))]
        call = _lib.qkv_rope_decode
    else:
        raise SystemExit(f"unknown kernel {name}")
    n = len(args_list)
    for i in range(args.warmup):
        call(args_list[i % n])
    torch.cuda.synchronize()
    calls = max(args.steps, n)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(calls):
            call(args_list[i % n])
    graph.replay()
    torch.cuda.synchronize()
    reps = 3
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    rc, bits = _lib.read_status(ws)
    if rc != 0:
        raise RuntimeError(f"{name} status {bits:#x}")
    us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
    del graph, keep
    if rank == 0:
        line = {"workload": "kernel", "kernel": name, "model": args.model, "tp_shapes": tp, "batch": B,
                "calls_per_graph": calls,
                "weight_copies": n, "us": round(us, 2)}
        if name == "prefill_attention":
            line.update({"algorithmic_flops": int(flops), "TFLOPs": round(flops / us / 1e6, 1)})
        else:
            nbytes = stack_kernel_bytes(tp, ctx, B, args.model)[name][0]
            line.update({"algorithmic_bytes": nbytes, "GBps": round(nbytes / us / 1e3, 1)})
        print(json.dumps(line), flush=True)


def run_reference_stack(args, world):
    """The stack's metric on the CPU path: each of min(K, 3) samples is one
    bounded sample (cpu_stack_sample) of a decode step; value = tokens/s."""
    n = max(1, min(args.steps, 3))
    samples = [cpu_stack_sample(reps=1) for _ in range(n)]
    step = sorted(x["step_s"] for x in samples)[len(samples) // 2]
    value = STACK_BATCH / step
    base = dict(samples[0])
    base.update(value=round(value, 3), sample=f"median of {n} samples; each: " + base["sample"])
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "decode tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step * 1e3, 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init weights, random prompt K/V)", "config": stack_config(world),
        "cpu_baseline": base,
        "e2e": {"value": round(value, 3), "unit": "decode tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 64 decode steps of the stack, 20000 layer steps)")
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["krt", "reference"], default="krt")
    ap.add_argument("--kernel", default="paged_attention",
                    help="--workload kernel: paged_attention, qkv_rope_decode, o_proj_gemm_ar, gate_up_swiglu, "
                         "down_proj_gemm_ar, lm_head_argmax, prefill_attention")
    ap.add_argument("--tp", type=int, default=0, help="--workload kernel: TP degree whose shard shapes to use")
    ap.add_argument("--batch", type=int, default=0, help="--workload kernel: tokens per call (default 128)")
    ap.add_argument("--model", choices=sorted(STACK_MODELS), default="8b",
                    help="--workload stack: 8b (config 4, the metric's workload) or 70b (config 5's decode half)")
    ap.add_argument("--workload", choices=["stack", "layer", "prefill", "gemm_ar", "kernel"], default="stack",
                    help="stack: decode steps of the Llama-3-8B-shaped stack (default); layer: one decoder layer's "
                         "hot path; prefill: the fused QKV prefill kernel alone")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"stack": 64, "kernel": 4}.get(args.workload, 20000)
    if args.warmup is None:
        args.warmup = {"stack": 8, "kernel": 1}.get(args.workload, 50)
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
    elif args.workload == "layer":
        run_krt(args, rank, world, local_rank)
    elif args.workload == "gemm_ar":
        run_gemm_ar(args, rank, world, local_rank)
    elif args.workload == "kernel":
        run_kernel(args, rank, world, local_rank)
    else:
        run_stack(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
