"""GPU parity of the decode-step pieces around the hot path and of a whole
decode step (tiny Llama-shaped stack) against oracle/decoder.py.

bf16 tolerance: max-abs 2e-2 + rel 1e-2 (per element, as the other GPU
tests); greedy tokens must match the oracle's argmax unless the oracle's
top two logits are within that tolerance of each other (a near-tie that
bf16 rounding may order either way).
"""
import numpy as np
import pytest

from oracle import decoder as odec
from oracle import fused_layer
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def bf(rng, *shape, scale=1.0, base=0.0):
    return round_bf16((rng.standard_normal(shape, dtype=np.float32) * np.float32(scale) + np.float32(base)))


def dev(torch, a):
    return torch.from_numpy(f32_to_bf16_bits(a).view(np.int16)).view(torch.bfloat16).cuda()


def _projection_kernel(monkeypatch, mode):
    """splitk: the split-K decode kernel; tiles: the persistent kernel on whole
    tiles; streamk: the persistent kernel on equal runs of k-boxes; auto: the
    launcher's choice."""
    if mode == "splitk":
        monkeypatch.setenv("KRT_PROJ_PERSISTENT", "0")
    elif mode in ("tiles", "streamk"):
        monkeypatch.setenv("KRT_PROJ_PERSISTENT", "1")
        monkeypatch.setenv("KRT_PROJ_STREAMK", "1" if mode == "streamk" else "0")


@pytest.mark.parametrize("mode,T,I", [("splitk", 37, 320), ("tiles", 37, 320), ("streamk", 37, 320),
                                      ("auto", 128, 9600), ("tiles", 200, 704), ("streamk", 200, 704),
                                      ("streamk", 64, 9600), ("auto", 700, 704), ("auto", 300, 9600),
                                      ("tiles", 256, 9600)])
def test_gate_up_swiglu(torch_cuda, monkeypatch, mode, T, I):
    """Split-K kernel (few tiles) and the persistent kernel: whole tiles (150
    tiles on 148 SMs gives two tiles to some CTAs, through both TMEM buffers)
    and stream-K (5 tiles of 4 k-boxes on 20 CTAs: every tile is one head
    and three partials; 150 tiles on 148 CTAs: runs of 4-5 boxes crossing
    tile boundaries); prompts of 300 and 700 tokens run in 256-token blocks;
    256 tokens is one full block."""
    torch = torch_cuda
    from python.kinetic_rt import _lib
    _projection_kernel(monkeypatch, mode)
    rng = np.random.Generator(np.random.PCG64(1))
    D = 512
    x, g = bf(rng, T, D), bf(rng, D, scale=0.1, base=1.0)
    wg, wu = bf(rng, I, D, scale=0.05), bf(rng, I, D, scale=0.05)
    act = torch.full((T, I + 16), 5.0, dtype=torch.bfloat16, device="cuda")[:, :I]
    ws = torch.zeros(_lib.projection_workspace_bytes(T, D), dtype=torch.uint8, device="cuda")
    wgu = _lib.interleave_gate_up(dev(torch, wg), dev(torch, wu)).contiguous()
    xd, gd = dev(torch, x), dev(torch, g)  # referenced while the kernels run (the structs hold raw pointers)
    _lib.gate_up_swiglu(_lib.gate_up_args(xd, gd, wgu, act, ws))
    assert _lib.read_status(ws) == (0, 0)
    xm = round_bf16(fused_layer.rms_norm(x, g)).astype(np.float64)
    gg, uu = xm @ wg.astype(np.float64).T, xm @ wu.astype(np.float64).T
    ref = odec.silu(gg) * uu
    np.testing.assert_allclose(act.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def _check_argmax(logits, idx):
    best = logits.max(-1)
    chosen = logits[np.arange(len(idx)), idx]
    assert np.all(chosen >= best - (ATOL + RTOL * np.abs(best))), (chosen, best)
    return np.mean(idx == logits.argmax(-1))


@pytest.mark.parametrize("mode,V0,V1", [("splitk", 1000, 777), ("tiles", 1000, 777), ("streamk", 1000, 777),
                                       ("auto", 40000, 1777), ("tiles", 40000, 1777)])
def test_lm_head_argmax_two_shards(torch_cuda, monkeypatch, mode, V0, V1):
    """Two vocabulary shards (neither a multiple of 128 rows) folded into one
    key array give the argmax over the whole vocabulary; split-K and
    persistent kernels (313 tiles: three tiles for some CTAs on whole tiles;
    runs crossing tile boundaries on stream-K).  The second shard reuses the
    workspace, so stream-K flags left raised would show as wrong sums."""
    torch = torch_cuda
    from python.kinetic_rt import _lib
    _projection_kernel(monkeypatch, mode)
    rng = np.random.Generator(np.random.PCG64(2))
    T, D = 19, 256
    x, g = bf(rng, T, D), bf(rng, D, scale=0.1, base=1.0)
    w = bf(rng, V0 + V1, D, scale=0.05)
    keys = torch.zeros(T, dtype=torch.int64, device="cuda")
    ws = torch.zeros(_lib.projection_workspace_bytes(T, D), dtype=torch.uint8, device="cuda")
    wd, xd, gd = dev(torch, w), dev(torch, x), dev(torch, g)
    for lo, hi in ((0, V0), (V0, V0 + V1)):
        _lib.lm_head_argmax(_lib.lm_head_args(xd, gd, wd[lo:hi], keys, ws, vocab_offset=lo))
    assert _lib.read_status(ws) == (0, 0)
    k = keys.cpu().numpy().view(np.uint64)
    idx = (0xFFFFFFFF - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)
    xm = round_bf16(fused_layer.rms_norm(x, g)).astype(np.float64)
    logits = xm @ w.astype(np.float64).T
    assert _check_argmax(logits, idx) > 0.9
    # the key carries the fp32 logit of the chosen row
    vals = ((k >> np.uint64(32)).astype(np.uint32))
    vals = np.where(vals & 0x80000000, vals & 0x7FFFFFFF, ~vals & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    np.testing.assert_allclose(vals, logits[np.arange(T), idx], atol=ATOL, rtol=RTOL)


def test_greedy_step_single_gpu(torch_cuda):
    torch = torch_cuda
    from python.kinetic_rt import _lib
    B, V, D = 6, 50, 64
    vals = [0.5, -1.0, 3.25, 0.0, -0.0, 7.0]
    idxs = [3, 49, 0, 17, 2, 11]
    keys = torch.tensor([_lib.argmax_key(v, i) - (1 << 64 if _lib.argmax_key(v, i) >= 1 << 63 else 0)
                         for v, i in zip(vals, idxs)], dtype=torch.int64, device="cuda")
    tokens = torch.full((B,), -5, dtype=torch.int32, device="cuda")
    emb = torch.randn(V, D, device="cuda").to(torch.bfloat16)
    hidden = torch.zeros(B, D + 8, dtype=torch.bfloat16, device="cuda")
    pos = torch.arange(B, dtype=torch.int32, device="cuda")
    lens = pos + 1
    forced = torch.tensor([-1, -1, 7, -1, -1, -1], dtype=torch.int32, device="cuda")
    status = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    _lib.greedy_step(None, _lib.greedy_step_args(keys, tokens, status, V, emb, hidden, pos, lens, next_input=forced))
    assert _lib.read_status(status) == (0, 0)
    assert tokens.cpu().tolist() == idxs
    fed = [7 if i == 2 else t for i, t in enumerate(idxs)]
    assert torch.equal(hidden[:, :D], emb[torch.tensor(fed, device="cuda")])
    assert pos.cpu().tolist() == list(range(1, B + 1)) and lens.cpu().tolist() == list(range(2, B + 2))
    assert int(keys.abs().sum()) == 0


def test_gemm_residual_in_place(torch_cuda):
    torch = torch_cuda
    from python.kinetic_rt import _lib
    rng = np.random.Generator(np.random.PCG64(3))
    T, K, N = 21, 640, 384
    x, w, h = bf(rng, T, K), bf(rng, N, K, scale=0.02), bf(rng, T, N)
    hd, xd, wdev = dev(torch, h), dev(torch, x), dev(torch, w)
    ws = torch.zeros(_lib.gemm_ar_workspace_bytes(), dtype=torch.uint8, device="cuda")
    _lib.rowparallel_gemm_ar(None, _lib.gemm_ar_args(xd, wdev, hd, ws, residual=hd))
    assert _lib.read_status(ws) == (0, 0)
    ref = h.astype(np.float64) + x.astype(np.float64) @ w.astype(np.float64).T
    np.testing.assert_allclose(hd.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def tiny_model(rng, L=2, D=256, H=4, KV=2, I=384, V=1000):
    from python.kinetic_rt.decoder import LlamaShape
    shape = LlamaShape(n_layers=L, d_model=D, n_heads=H, n_kv_heads=KV, inter=I, vocab=V, rope_theta=1e4)
    hd = 128
    sc = lambda fan_in: min(0.05, fan_in ** -0.5)  # keeps activations O(1) at wide shapes
    full = {k: [] for k in ("qkv", "g_attn", "o", "g_mlp", "gate", "up", "down")}
    for _ in range(L):
        full["qkv"].append(bf(rng, (H + 2 * KV) * hd, D, scale=sc(D)))
        full["g_attn"].append(bf(rng, D, scale=0.1, base=1.0))
        full["o"].append(bf(rng, D, H * hd, scale=sc(H * hd)))
        full["g_mlp"].append(bf(rng, D, scale=0.1, base=1.0))
        full["gate"].append(bf(rng, I, D, scale=sc(D)))
        full["up"].append(bf(rng, I, D, scale=sc(D)))
        full["down"].append(bf(rng, D, I, scale=sc(I)))
    full["g_final"] = bf(rng, D, scale=0.1, base=1.0)
    full["lm_head"] = bf(rng, V, D, scale=sc(D))
    full["embed"] = bf(rng, V, D)
    return shape, full


def run_decoder_against_oracle(torch, rank=0, world=1, comm=None, steps=3, model=None):
    from python.kinetic_rt.decoder import PagedDecoder, RankWeights
    rng = np.random.Generator(np.random.PCG64(4))
    shape, full = tiny_model(rng, **(model or {}))
    B, max_len = 5, 80
    w = RankWeights.from_full(torch, shape, full, rank, world)
    dec = PagedDecoder(torch, shape, w, B, max_len, comm=comm, rank=rank, world=world)
    start_pos = np.array([0, 5, 16, 33, 70])
    start_tok = rng.integers(0, shape.vocab, size=B)
    # prefix K/V: random bf16 values in the oracle's pools; each rank holds its KV heads
    pools = [bf(rng, dec.num_blocks, 16, 2, shape.n_kv_heads, 128) for _ in range(shape.n_layers)]
    hk = shape.n_kv_heads // world
    for p, pd in zip(pools, dec.pools):
        pd.copy_(dev(torch, np.ascontiguousarray(p[:, :, :, rank * hk:(rank + 1) * hk]).reshape(dec.num_blocks, 16, -1)))
    dec.start(start_tok, start_pos)
    table = dec.block_table.cpu().numpy()
    cos, sin = fused_layer.rope_tables(np.arange(max_len), 128, shape.rope_theta)
    graph = dec.capture()
    h = full["embed"][start_tok]
    pos = start_pos.copy()
    for step in range(steps):
        logits, tok, h_next = odec.decode_step(full, h, pos, table, pools, cos, sin, shape.n_heads,
                                               shape.n_kv_heads, 16)
        dec.next_input.copy_(torch.from_numpy(tok.astype(np.int32)))
        graph.replay()
        dec.check_status()
        got_tok = dec.tokens.cpu().numpy()
        top2 = np.sort(logits, -1)[:, -2:]
        near_tie = top2[:, 1] - top2[:, 0] < ATOL + RTOL * np.abs(top2[:, 1])
        assert np.all((got_tok == tok) | near_tie), (step, got_tok, tok)
        for li in range(shape.n_layers):  # the step's K/V (this rank's heads) landed at each sequence's slot
            got_pool = dec.pools[li].float().cpu().numpy().reshape(dec.num_blocks, 16, 2, hk, 128)
            for s in range(B):
                blk, off = table[s][pos[s] // 16], pos[s] % 16
                np.testing.assert_allclose(got_pool[blk, off], pools[li][blk, off, :, rank * hk:(rank + 1) * hk],
                                           atol=ATOL, rtol=RTOL)
        np.testing.assert_array_equal(dec.h.float().cpu().numpy(), h_next)
        assert dec.positions.cpu().numpy().tolist() == (pos + 1).tolist()
        h, pos = h_next, pos + 1
    del graph
    return dec


def _tp_decoder_worker(rank, world, port):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from python.kinetic_rt.dist import TPComm
    comm = TPComm(rank, world, max_n_out=256)
    try:
        run_decoder_against_oracle(torch, rank, world, comm)
    finally:
        torch.cuda.synchronize()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()


def test_decode_steps_tensor_parallel_match_oracle(torch_cuda):
    """The same three steps with the model split over two GPUs (heads,
    intermediate features and vocabulary; fused allreduce and the greedy
    exchange over NVLink): both ranks match the oracle."""
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    mp.spawn(_tp_decoder_worker, args=(2, port), nprocs=2, join=True)


@pytest.mark.parametrize("mode", ["splitk", "tiles", "streamk"])
def test_decode_steps_match_oracle(torch_cuda, monkeypatch, mode):
    """Three graph-replayed decode steps of a 2-layer model, 5 sequences at
    ragged positions, against the oracle step by step (the oracle's token is
    fed back on both sides, so a near-tie cannot make the runs diverge);
    gate/up and lm_head on each projection kernel."""
    _projection_kernel(monkeypatch, mode)
    run_decoder_against_oracle(torch_cuda)


def test_decode_steps_seventy_b_rank_shapes(torch_cuda):
    """One layer at the shapes one rank of the Llama-3-70B stack holds at
    TP=8 (hidden 8192, 8 Q heads and 1 KV head, 3584 intermediate features):
    10 QKV tiles over 128 k-blocks, a single KV head per pool, 8192-wide
    GEMM outputs; two graph-replayed steps against the oracle."""
    run_decoder_against_oracle(torch_cuda, steps=2, model=dict(L=1, D=8192, H=8, KV=1, I=3584))


@pytest.mark.parametrize("lens", [(37, 37, 37), (5, 300, 64)])
def test_prefill_then_decode_matches_oracle(torch_cuda, lens):
    """PagedDecoder.prefill of a tiny two-layer model (prompt K/V into the
    pools through the prefill QKV and causal prefill attention kernels, the
    MLP over whole prompts) against the oracle fed the prompts token by token:
    the K/V at every prompt position, the first chosen token (near-ties
    excepted), then two graph-replayed decode steps.  A group holding the
    300-token prompt runs gate/up in 256-token blocks and the row-parallel
    GEMMs in 256-token launches."""
    torch = torch_cuda
    from python.kinetic_rt.decoder import PagedDecoder, RankWeights
    rng = np.random.Generator(np.random.PCG64(21))
    shape, full = tiny_model(rng)
    B, max_len = len(lens), max(lens) + 16
    w = RankWeights.from_full(torch, shape, full, 0, 1)
    dec = PagedDecoder(torch, shape, w, B, max_len)
    prompts = [rng.integers(0, shape.vocab, size=n) for n in lens]
    got_tok = dec.prefill(prompts, group=2).cpu().numpy()
    dec.check_status()
    table = dec.block_table.cpu().numpy()
    cos, sin = fused_layer.rope_tables(np.arange(max_len), 128, shape.rope_theta)
    pools = [np.zeros((dec.num_blocks, 16, 2, shape.n_kv_heads, 128), np.float32) for _ in range(shape.n_layers)]
    # the oracle one position at a time; a sequence whose prompt has ended
    # keeps re-running its last token (its K/V slot is rewritten identically)
    last_logits = [None] * B
    for p in range(max(lens)):
        pos = np.array([min(p, n - 1) for n in lens])
        h = np.stack([full["embed"][prompts[b][pos[b]]] for b in range(B)])
        logits, _, _ = odec.decode_step(full, h, pos, table, pools, cos, sin, shape.n_heads, shape.n_kv_heads, 16)
        for b in range(B):
            if p == lens[b] - 1:
                last_logits[b] = logits[b]
    for li in range(shape.n_layers):
        got_pool = dec.pools[li].float().cpu().numpy().reshape(dec.num_blocks, 16, 2, shape.n_kv_heads, 128)
        for b in range(B):
            for p in range(lens[b]):
                blk, off = table[b][p // 16], p % 16
                np.testing.assert_allclose(got_pool[blk, off], pools[li][blk, off], atol=ATOL, rtol=RTOL)
    want = np.array([int(np.argmax(lg)) for lg in last_logits])
    for b in range(B):
        top2 = np.sort(last_logits[b])[-2:]
        assert got_tok[b] == want[b] or top2[1] - top2[0] < ATOL + RTOL * abs(top2[1]), (b, got_tok[b], want[b])
    # continue from the oracle's tokens on both sides
    dec.h.copy_(w.embed.index_select(0, torch.as_tensor(want, device="cuda")))
    graph = dec.capture()
    h, pos = full["embed"][want], np.array(lens)
    for step in range(2):
        logits, tok, h_next = odec.decode_step(full, h, pos, table, pools, cos, sin, shape.n_heads,
                                               shape.n_kv_heads, 16)
        dec.next_input.copy_(torch.from_numpy(tok.astype(np.int32)))
        graph.replay()
        dec.check_status()
        gt = dec.tokens.cpu().numpy()
        top2 = np.sort(logits, -1)[:, -2:]
        near_tie = top2[:, 1] - top2[:, 0] < ATOL + RTOL * np.abs(top2[:, 1])
        assert np.all((gt == tok) | near_tie), (step, gt, tok)
        h, pos = h_next, pos + 1
    del graph


def test_runtime_generate_matches_oracle(torch_cuda):
    """KineticRuntime.generate_ids over an attached batch-1 decoder: the
    prompt is fed token by token, then greedy tokens; equal to the oracle's
    greedy continuation (steps whose top-two logits are a near-tie excepted)."""
    torch = torch_cuda
    from python.kinetic_rt.decoder import PagedDecoder, RankWeights
    from python.kinetic_rt.orchestrator import KineticRuntime
    rng = np.random.Generator(np.random.PCG64(9))
    shape, full = tiny_model(rng)
    dec = PagedDecoder(torch, shape, RankWeights.from_full(torch, shape, full, 0, 1), 1, 48)
    rt = KineticRuntime.__new__(KineticRuntime)
    rt.decoder = rt.tokenizer = rt._graph = None
    rt.attach_decoder(dec)
    prompt = [int(t) for t in rng.integers(0, shape.vocab, size=6)]
    got = rt.generate_ids(prompt, max_new_tokens=5)
    # oracle: the same steps on the CPU
    table = dec.block_table.cpu().numpy()
    pools = [np.zeros((dec.num_blocks, 16, 2, shape.n_kv_heads, 128), np.float32) for _ in range(shape.n_layers)]
    cos, sin = fused_layer.rope_tables(np.arange(48), 128, shape.rope_theta)
    h = full["embed"][[prompt[0]]]
    seq, ref, ties = list(prompt), [], []
    for pos in range(len(prompt) - 1 + 5):
        logits, tok, _ = odec.decode_step(full, h, np.array([pos]), table, pools, cos, sin, shape.n_heads,
                                          shape.n_kv_heads, 16)
        top2 = np.sort(logits[0])[-2:]
        if pos + 1 >= len(prompt):
            ref.append(int(tok[0]))
            ties.append(top2[1] - top2[0] < ATOL + RTOL * abs(top2[1]))
            nxt = got[len(ref) - 1]  # follow the GPU's choice so a near-tie cannot derail the comparison
        else:
            nxt = prompt[pos + 1]
        h = full["embed"][[nxt]]
    assert all(g == r or t for g, r, t in zip(got, ref, ties)), (got, ref, ties)
