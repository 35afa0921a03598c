"""Paged Llama decode driver over libkrt: the caller of the hot path.

The reference's generation loop (python/kinetic_rt/orchestrator.py:419-448)
re-runs the model over the whole token list for every new token and picks
the next token with argmax of the last row (442-444).  This driver keeps the
K/V of every processed token in paged blocks (BlockManager geometry,
include/BlockManager.h:29-95; ceil(len / B) blocks per sequence as
src/GraphWrapper.cpp:139-145 allocates them) and runs one decode step per
new token for a whole batch of sequences, each step one CUDA graph:

  per layer   krt_qkv_rope_decode        RMSNorm + QKV + RoPE, K/V -> pool
              krt_paged_attention_decode  attention over the pool
              krt_rowparallel_gemm_ar     o_proj + allreduce + residual (h in place)
              krt_gate_up_swiglu          RMSNorm + gate/up + SwiGLU
              krt_rowparallel_gemm_ar     down_proj + allreduce + residual
  then        krt_lm_head_argmax         final RMSNorm + lm_head shard + argmax
              krt_greedy_step            argmax over ranks, next embedding,
                                         positions / lengths + 1

Tensor parallelism (one process per GPU, `comm` a TPComm): Q/K/V heads, the
intermediate features and the vocabulary are split over ranks
(column-parallel, scripts/export_hf.py:60), o_proj / down_proj by input
columns (row-parallel, export_hf.py:62-65); the embedding is replicated.
Every rank ends a step with the same tokens and hidden state.
"""
from dataclasses import dataclass

from . import _lib


@dataclass(frozen=True)
class LlamaShape:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    inter: int
    vocab: int
    head_dim: int = 128
    rope_theta: float = 5e5
    eps: float = 1e-5
    tokens_per_block: int = 16


LLAMA3_8B = LlamaShape(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=8, inter=14336, vocab=128256)
LLAMA3_70B = LlamaShape(n_layers=80, d_model=8192, n_heads=64, n_kv_heads=8, inter=28672, vocab=128256)


def rope_cache(torch, max_position, head_dim, theta, device="cuda"):
    """Llama rotary tables, fp32 [max_position, head_dim]:
    emb = cat(pos * inv_freq, pos * inv_freq), inv_freq = theta^(-2i/head_dim),
    evaluated in fp64 on the host (as HF's rotary embedding builds them)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    f = torch.outer(torch.arange(max_position, dtype=torch.float64), inv_freq)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float().to(device), emb.sin().float().to(device)


def vocab_shard(vocab, rank, world):
    """Rows [lo, hi) of the vocabulary on `rank` (torch.chunk along rows)."""
    step = -(-vocab // world)
    lo = min(rank * step, vocab)
    return lo, min(lo + step, vocab)


class BlockAllocator:
    """BlockManager's free list (include/BlockManager.h:63-82): ids 0..N-1,
    allocation pops from the back (the first id handed out is N-1), freeing
    pushes to the back (LIFO reuse).  Only ids are managed here; the pools
    are the decoder's per-layer tensors of the same geometry."""

    def __init__(self, num_blocks):
        self.num_blocks = int(num_blocks)
        self.free = list(range(self.num_blocks))

    def allocate_block(self):
        if not self.free:
            raise RuntimeError("Out of KV Cache blocks! Massive pool exhausted.")
        return self.free.pop()

    def free_block(self, block_id):
        if block_id < 0 or block_id >= self.num_blocks:
            raise RuntimeError(f"block ID {block_id} out of range [0, {self.num_blocks})")
        self.free.append(block_id)


class RankWeights:
    """This rank's bf16 shards of a Llama-shaped stack on the current device.

    Attributes per layer (lists): qkv [(hq + 2 hkv) * 128, D] rows
    [Q heads | K heads | V heads] of this rank; g_attn, g_mlp [D]; o [D, hq * 128];
    gate_up [2 * I / TP, D] in 64-row [gate | up] groups; down [D, I / TP].
    Then g_final [D], lm_head [V_r, D] (vocabulary rows vocab_lo..), embed [V, D].
    """

    @classmethod
    def from_full(cls, torch, shape, full, rank, world, device="cuda"):
        """Shard full-model tensors (float, any device) the way export_hf.py
        does.  full: dict of lists 'qkv' ([Hq*hd + 2*Hkv*hd, D]), 'g_attn', 'o',
        'g_mlp', 'gate', 'up', 'down', and 'g_final', 'lm_head', 'embed'."""
        self = cls.__new__(cls)
        hd = shape.head_dim
        hq, hkv = shape.n_heads // world, shape.n_kv_heads // world
        ir = shape.inter // world
        bf = lambda t: torch.as_tensor(t).to(device=device, dtype=torch.bfloat16).contiguous()
        self.qkv, self.g_attn, self.o, self.g_mlp, self.gate_up, self.down = [], [], [], [], [], []
        for li in range(shape.n_layers):
            w = torch.as_tensor(full["qkv"][li])
            nq, nk = shape.n_heads * hd, shape.n_kv_heads * hd
            q = w[rank * hq * hd:(rank + 1) * hq * hd]
            k = w[nq + rank * hkv * hd:nq + (rank + 1) * hkv * hd]
            v = w[nq + nk + rank * hkv * hd:nq + nk + (rank + 1) * hkv * hd]
            self.qkv.append(bf(torch.cat([q, k, v], 0)))
            self.g_attn.append(bf(full["g_attn"][li]))
            self.o.append(bf(torch.as_tensor(full["o"][li])[:, rank * hq * hd:(rank + 1) * hq * hd]))
            self.g_mlp.append(bf(full["g_mlp"][li]))
            g = bf(torch.as_tensor(full["gate"][li])[rank * ir:(rank + 1) * ir])
            u = bf(torch.as_tensor(full["up"][li])[rank * ir:(rank + 1) * ir])
            self.gate_up.append(_lib.interleave_gate_up(g, u).contiguous())
            self.down.append(bf(torch.as_tensor(full["down"][li])[:, rank * ir:(rank + 1) * ir]))
        self.g_final = bf(full["g_final"])
        self.vocab_lo, self.vocab_hi = vocab_shard(shape.vocab, rank, world)
        self.lm_head = bf(torch.as_tensor(full["lm_head"])[self.vocab_lo:self.vocab_hi])
        self.embed = bf(full["embed"])
        return self

    @classmethod
    def random(cls, torch, shape, rank, world, seed=0, std=0.02, device="cuda"):
        """Random-init shards (weights N(0, std), norm weights 1 + N(0, 0.1)),
        generated per rank directly on the device."""
        self = cls.__new__(cls)
        hd = shape.head_dim
        hq, hkv = shape.n_heads // world, shape.n_kv_heads // world
        ir = shape.inter // world
        g = torch.Generator(device=device).manual_seed(seed * 1000 + rank)

        def rnd(*size, scale=std, base=0.0):
            t = torch.randn(*size, generator=g, device=device) * scale + base
            return t.to(torch.bfloat16)

        # replicated tensors (norm weights, embedding) come from a generator
        # seeded alike on every rank
        gr = torch.Generator(device=device).manual_seed(seed * 1000 + 999)

        def rep(*size, scale, base):
            return (torch.randn(*size, generator=gr, device=device) * scale + base).to(torch.bfloat16)

        D = shape.d_model
        self.qkv = [rnd((hq + 2 * hkv) * hd, D) for _ in range(shape.n_layers)]
        self.g_attn = [rep(D, scale=0.1, base=1.0) for _ in range(shape.n_layers)]
        self.o = [rnd(D, hq * hd) for _ in range(shape.n_layers)]
        self.g_mlp = [rep(D, scale=0.1, base=1.0) for _ in range(shape.n_layers)]
        self.gate_up = [rnd(2 * ir, D) for _ in range(shape.n_layers)]
        self.down = [rnd(D, ir) for _ in range(shape.n_layers)]
        self.g_final = rep(D, scale=0.1, base=1.0)
        self.vocab_lo, self.vocab_hi = vocab_shard(shape.vocab, rank, world)
        self.lm_head = rnd(self.vocab_hi - self.vocab_lo, D)
        self.embed = rep(shape.vocab, D, scale=1.0, base=0.0)
        return self

    def layer_bytes(self, li):
        return sum(t.numel() * 2 for t in (self.qkv[li], self.g_attn[li], self.o[li], self.g_mlp[li],
                                            self.gate_up[li], self.down[li]))


class PagedDecoder:
    """Batched greedy decoding of `batch` sequences over paged KV pools.

    State on the device: hidden h [B, D] (the next step's input embeddings),
    positions [B] (position of the token each sequence processes next),
    seq_lens [B] (= positions + 1 during a step), block tables, one pool per
    layer.  `step()` launches one decode step on the current stream and
    `capture()` records it as a CUDA graph.
    """

    def __init__(self, torch, shape, weights, batch, max_seq_len, comm=None, rank=0, world=1, device="cuda"):
        self.torch, self.shape, self.w = torch, shape, weights
        self.B, self.max_seq_len = int(batch), int(max_seq_len)
        self.comm, self.rank, self.world = comm, rank, world
        hd, tpb = shape.head_dim, shape.tokens_per_block
        self.hq, self.hkv = shape.n_heads // world, shape.n_kv_heads // world
        self.ir = shape.inter // world
        B, D = self.B, shape.d_model
        self.blocks_per_seq = -(-self.max_seq_len // tpb)
        self.num_blocks = B * self.blocks_per_seq
        self.allocator = BlockAllocator(self.num_blocks)
        table = [[self.allocator.allocate_block() for _ in range(self.blocks_per_seq)] for _ in range(B)]
        self.block_table = torch.tensor(table, dtype=torch.int32, device=device)
        self.pools = [torch.zeros(self.num_blocks, tpb, 2 * self.hkv * hd, dtype=torch.bfloat16, device=device)
                      for _ in range(shape.n_layers)]
        i32 = lambda n, v=0: torch.full((n,), v, dtype=torch.int32, device=device)
        self.positions, self.seq_lens = i32(B), i32(B, 1)
        self.token_seq = torch.arange(B, dtype=torch.int32, device=device)
        self.next_input = i32(B, -1)
        self.tokens = i32(B)
        self.keys = torch.zeros(B, dtype=torch.int64, device=device)
        self.h = torch.zeros(B, D, dtype=torch.bfloat16, device=device)
        self.q = torch.empty(B, self.hq * hd, dtype=torch.bfloat16, device=device)
        self.attn = torch.empty(B, self.hq * hd, dtype=torch.bfloat16, device=device)
        self.act = torch.empty(B, self.ir, dtype=torch.bfloat16, device=device)
        self.cos, self.sin = rope_cache(torch, self.max_seq_len, hd, shape.rope_theta, device)
        z = lambda n: torch.zeros(n, dtype=torch.uint8, device=device)
        self.ws_qkv = z(_lib.decode_workspace_bytes(B, D, self.hq, self.hkv))
        self.ws_attn = z(_lib.attention_workspace_bytes(B, self.hq, self.hkv, self.max_seq_len))
        self.ws_proj = z(_lib.projection_workspace_bytes(B, D))
        self.ws_gemm = z(_lib.gemm_ar_workspace_bytes())
        self.ws_greedy = z(_lib.gemm_ar_workspace_bytes())
        self._build_args()

    # ---------------------------------------------------------------- args
    def _build_args(self):
        s, w = self.shape, self.w
        self.layer_args = []
        for li in range(s.n_layers):
            qa = _lib.paged_args(self.h, w.qkv[li], None, w.g_attn[li], self.cos, self.sin, self.positions,
                                 self.token_seq, self.block_table, self.pools[li], self.q, self.hq, self.hkv,
                                 self.num_blocks, s.tokens_per_block, self.ws_qkv, eps=s.eps)
            aa = _lib.attention_args(self.q, self.pools[li], self.block_table, self.seq_lens, self.attn, self.hq,
                                     self.hkv, self.num_blocks, s.tokens_per_block, self.max_seq_len, self.ws_attn)
            oa = _lib.gemm_ar_args(self.attn, w.o[li], self.h, self.ws_gemm, residual=self.h)
            ga = _lib.gate_up_args(self.h, w.g_mlp[li], w.gate_up[li], self.act, self.ws_proj, eps=s.eps)
            da = _lib.gemm_ar_args(self.act, w.down[li], self.h, self.ws_gemm, residual=self.h)
            self.layer_args.append((qa, aa, oa, ga, da))
        self.lm_args = _lib.lm_head_args(self.h, w.g_final, w.lm_head, self.keys, self.ws_proj,
                                         vocab_offset=w.vocab_lo, eps=s.eps)
        self.greedy_args = _lib.greedy_step_args(self.keys, self.tokens, self.ws_greedy, s.vocab, embedding=w.embed,
                                                 hidden=self.h, positions=self.positions, seq_lens=self.seq_lens,
                                                 next_input=self.next_input)

    @property
    def comm_handle(self):
        return None if self.comm is None else self.comm.handle

    # ----------------------------------------------------------- the step
    LAUNCHES_PER_LAYER = 7  # prep + QKV, attention, o_proj, prep + gate/up, down_proj
    LAUNCHES_TAIL = 3       # prep + lm_head, greedy step

    @property
    def launches_per_step(self):
        return self.shape.n_layers * self.LAUNCHES_PER_LAYER + self.LAUNCHES_TAIL

    def layer(self, li, parts=(0, 1, 2, 3, 4)):
        qa, aa, oa, ga, da = self.layer_args[li]
        c = self.comm_handle
        if 0 in parts:
            _lib.qkv_rope_decode(qa)
        if 1 in parts:
            _lib.paged_attention_decode(aa)
        if 2 in parts:
            _lib.rowparallel_gemm_ar(c, oa)
        if 3 in parts:
            _lib.gate_up_swiglu(ga)
        if 4 in parts:
            _lib.rowparallel_gemm_ar(c, da)

    def tail(self):
        _lib.lm_head_argmax(self.lm_args)
        _lib.greedy_step(self.comm_handle, self.greedy_args)

    def step(self):
        """One decode step of every sequence on the current stream."""
        for li in range(self.shape.n_layers):
            self.layer(li)
        self.tail()

    def capture(self, warm=True):
        """The step as a CUDA graph.  With `warm`, one eager step runs first on a
        side stream (every entry point's first-call set-up happens outside the
        capture) and the state it advanced is put back: the hidden state,
        positions and lengths are restored, and the K/V it wrote at the
        current positions are rewritten identically by the next step."""
        torch = self.torch
        if warm:
            saved = [t.clone() for t in (self.h, self.positions, self.seq_lens, self.tokens, self.next_input)]
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self.step()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            for t, v in zip((self.h, self.positions, self.seq_lens, self.tokens, self.next_input), saved):
                t.copy_(v)
            torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        return g

    # ------------------------------------------------------------ prefill
    def prefill(self, prompts, group=8):
        """Process the prompts of all `batch` sequences (prompts[b]: token ids
        of sequence b, positions 0 .. len - 1), `group` sequences at a time.
        Per layer: the prefill QKV kernel (K/V of every prompt token into the
        pool), causal prefill attention over the pool, o_proj + allreduce +
        residual, gate/up + SwiGLU over the whole group's tokens, down_proj +
        allreduce + residual.  Then the lm_head on each prompt's last token
        and the greedy step: afterwards the next step() processes the chosen
        token at position len(prompts[b]).  The reference's generation loop
        instead re-runs the model over the whole token list for every new
        token (python/kinetic_rt/orchestrator.py:419-448).  Returns the chosen
        tokens (device int32 [batch])."""
        torch, s, w = self.torch, self.shape, self.w
        if len(prompts) != self.B:
            raise ValueError(f"prefill needs one prompt per sequence ({self.B}), got {len(prompts)}")
        dev = self.h.device
        lens = [len(p) for p in prompts]
        if min(lens) < 1 or max(lens) >= self.max_seq_len:
            raise ValueError("prompt lengths must be in 1 .. max_seq_len - 1")
        D, hd, tpb = s.d_model, s.head_dim, s.tokens_per_block
        c = self.comm_handle
        last_h = torch.empty(self.B, D, dtype=torch.bfloat16, device=dev)
        for g0 in range(0, self.B, group):
            seqs = list(range(g0, min(self.B, g0 + group)))
            glens = [lens[b] for b in seqs]
            T = sum(glens)
            ids = torch.cat([torch.as_tensor(prompts[b], dtype=torch.int64).reshape(-1) for b in seqs]).to(dev)
            token_seq = torch.cat([torch.full((n,), b, dtype=torch.int32) for b, n in zip(seqs, glens)]).to(dev)
            positions = torch.cat([torch.arange(n, dtype=torch.int32) for n in glens]).to(dev)
            starts = [0]
            for n in glens:
                starts.append(starts[-1] + n)
            q_start = torch.tensor(starts, dtype=torch.int32, device=dev)
            q_pos0 = torch.zeros(len(seqs), dtype=torch.int32, device=dev)
            table = self.block_table[seqs[0]:seqs[-1] + 1].contiguous()
            hp = w.embed.index_select(0, ids).contiguous()
            qp = torch.empty(T, self.hq * hd, dtype=torch.bfloat16, device=dev)
            attnp = torch.empty_like(qp)
            actp = torch.empty(T, self.ir, dtype=torch.bfloat16, device=dev)
            z = lambda n: torch.zeros(n, dtype=torch.uint8, device=dev)
            ws_q = z(_lib.prefill_workspace_bytes(T, D, self.hq, self.hkv))
            ws_a = z(_lib.prefill_attention_workspace_bytes())
            ws_p = z(_lib.projection_workspace_bytes(T, D))
            ws_g = z(_lib.gemm_ar_workspace_bytes())
            for li in range(s.n_layers):
                _lib.qkv_rope_prefill(_lib.paged_args(hp, w.qkv[li], None, w.g_attn[li], self.cos, self.sin, positions,
                                                      token_seq, self.block_table, self.pools[li], qp, self.hq,
                                                      self.hkv, self.num_blocks, tpb, ws_q, eps=s.eps))
                _lib.paged_attention_prefill(_lib.prefill_attention_args(qp, self.pools[li], table, q_start, q_pos0,
                                                                         attnp, self.hq, self.hkv, self.num_blocks,
                                                                         tpb, max(glens), ws_a))
                _lib.rowparallel_gemm_ar(c, _lib.gemm_ar_args(attnp, w.o[li], hp, ws_g, residual=hp))
                _lib.gate_up_swiglu(_lib.gate_up_args(hp, w.g_mlp[li], w.gate_up[li], actp, ws_p, eps=s.eps))
                _lib.rowparallel_gemm_ar(c, _lib.gemm_ar_args(actp, w.down[li], hp, ws_g, residual=hp))
            last_h[seqs[0]:seqs[-1] + 1] = hp.index_select(0, (q_start[1:] - 1).long())
            for ws in (ws_q, ws_a, ws_p, ws_g):
                rc, bits = _lib.read_status(ws)
                if rc != 0:
                    raise RuntimeError(f"prefill kernel status {bits:#x}")
            del hp, qp, attnp, actp
        # the last prompt token's state, then lm_head + greedy step as in a decode step
        L = torch.tensor(lens, dtype=torch.int32, device=dev)
        self.h.copy_(last_h)
        self.positions.copy_(L - 1)
        self.seq_lens.copy_(L)
        self.next_input.fill_(-1)
        self.tail()
        return self.tokens

    # ------------------------------------------------------------ state
    def start(self, start_tokens, positions):
        """Next step processes token start_tokens[b] at position positions[b]."""
        torch = self.torch
        tok = torch.as_tensor(start_tokens, dtype=torch.int64, device=self.h.device)
        self.h.copy_(self.w.embed.index_select(0, tok))
        pos = torch.as_tensor(positions, dtype=torch.int32, device=self.h.device)
        self.positions.copy_(pos)
        self.seq_lens.copy_(pos + 1)
        self.next_input.fill_(-1)

    def fill_kv_random(self, upto, seed=0, std=1.0):
        """Synthetic K/V for positions 0 .. upto[b]-1 of every sequence (a
        stand-in for the prompt's prefill): random bf16 in every pool."""
        torch = self.torch
        g = torch.Generator(device=self.h.device).manual_seed(seed)
        for pool in self.pools:
            pool.copy_((torch.randn(pool.shape, generator=g, device=pool.device) * std).to(torch.bfloat16))

    def check_status(self):
        for ws in (self.ws_qkv, self.ws_attn, self.ws_proj, self.ws_gemm, self.ws_greedy):
            rc, bits = _lib.read_status(ws)
            if rc != 0:
                raise RuntimeError(f"kernel status {bits:#x}")

    def generate(self, graph, steps, host_tokens=None, prompt=None):
        """Replay `graph` for `steps` decode steps.  With host_tokens (a pinned
        int32 [steps, B] tensor) every step's chosen tokens are copied to the
        host and the host waits for them, as a serving loop does; prompt
        (int32 [n, B], -1 = free) feeds prompt tokens instead of the choices."""
        torch = self.torch
        for i in range(steps):
            if prompt is not None:
                self.next_input.copy_(prompt[i] if i < prompt.shape[0] else torch.full_like(prompt[0], -1),
                                      non_blocking=True)
            graph.replay()
            if host_tokens is not None:
                host_tokens[i].copy_(self.tokens, non_blocking=True)
                torch.cuda.current_stream().synchronize()
