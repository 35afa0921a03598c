/*
 * krt.h -- C ABI of the B200 decoder hot path (libkrt.so).
 *
 * Plain pointers, sizes and POD structs; no exceptions cross this boundary.
 * Every entry point returns KRT_OK (0) or a KRT_ERR_* code and records a
 * message readable with krt_last_error() on the calling thread.  Device
 * pointers are CUDA device addresses on the current device; `stream` is a
 * cudaStream_t (NULL = legacy default stream).
 *
 * Reference interfaces these entry points replace (paths inside the
 * Kinetic-RT project):
 *   krt_fused_rmsnorm_qkv_rope  python/kinetic_rt/fusion_forge.py:21-31 (the
 *                               Triton kernel's 24-argument signature) and
 *                               src/AOTEngine.cpp:489-570 (AOTEngine::launch
 *                               packing the same 24 arguments)
 *   krt_qkv_rope_decode / _prefill
 *                               same computation, plus the K/V scatter into
 *                               BlockManager's pool (include/BlockManager.h:29-95,
 *                               block ids from src/GraphWrapper.cpp:139-145)
 *   krt_comm_* / krt_allreduce  include/Communicator.h:15-26 and
 *                               src/Communicator.cpp:21-27 (all_reduce_async)
 *   krt_rowparallel_gemm_ar     row-parallel o_proj/down_proj
 *                               (scripts/export_hf.py:62-65) followed by
 *                               Communicator::all_reduce_async, as one call
 */
#ifndef KRT_H_
#define KRT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KRT_API __attribute__((visibility("default")))
#else
#define KRT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------- status codes */
#define KRT_OK 0
#define KRT_ERR_INVALID 1     /* bad argument (null pointer, shape, stride)     */
#define KRT_ERR_CUDA 2        /* a CUDA runtime call failed                     */
#define KRT_ERR_UNSUPPORTED 3 /* shape/dtype outside what the kernel handles    */
#define KRT_ERR_WORKSPACE 4   /* workspace missing or too small                 */
#define KRT_ERR_DEVICE 5      /* a kernel reported an error in its status word  */

/* dtype codes: the binding's DataType enum (bindings/python_bindings.cpp:19-28) */
#define KRT_DTYPE_FLOAT32 1
#define KRT_DTYPE_BFLOAT16 3

/* Message of the last failing call on this thread ("" if none). */
KRT_API const char* krt_last_error(void);

/* Library version string. */
KRT_API const char* krt_version(void);

/* -------------------------------------------------------------------------
 * Reference-compatible fused RMSNorm + QKV projection + RoPE.
 *
 * Semantics of fusion_forge.py:21-162 for any d_model (the Triton kernel is
 * limited to d_model <= 128): per token t,
 *   x_hat = cast(x_t * rsqrt(mean(x_t^2) + eps) * rms_weight)
 *   qkv   = qkv_weight @ x_hat (+ qkv_bias)          fp32 accumulation
 *   q, k, v = qkv split [n_heads*hd | n_kv_heads*hd | n_kv_heads*hd]
 *   q, k rotated per head: u*cos + rotate_half(u)*sin
 * cos/sin element for token t, head h, dim d is
 *   freqs[row * stride_f_seq + (h * freqs_head_stride + d) * stride_f_dim]
 * with row = positions ? positions[t] : t.  With n_heads = 1 and
 * head_dim = d_model this is exactly the reference kernel (whose cos/sin use
 * x's strides, fusion_forge.py:92-93).  CUDA cores, fp32 math; any strides.
 * ---------------------------------------------------------------------- */
typedef struct krt_qkv_rope_args {
  const void* x;          /* [seq_len, d_model]                         */
  const void* qkv_weight; /* [(n_heads + 2*n_kv_heads)*head_dim, d_model] */
  const void* qkv_bias;   /* same length as the output rows, or NULL    */
  const void* rms_weight; /* [d_model]                                  */
  const void* freqs_cos;
  const void* freqs_sin;
  void* q_out; /* [seq_len, n_heads*head_dim]    */
  void* k_out; /* [seq_len, n_kv_heads*head_dim] */
  void* v_out; /* [seq_len, n_kv_heads*head_dim] */
  int32_t seq_len, d_model, n_heads, head_dim;
  float eps;
  int64_t stride_x_seq, stride_x_dim;
  int64_t stride_w_out, stride_w_in;
  int64_t stride_q_seq, stride_q_dim;
  int64_t stride_k_seq, stride_k_dim;
  int64_t stride_v_seq, stride_v_dim;
  /* extensions (zero-initialised structs give the reference behaviour) */
  int32_t dtype;             /* KRT_DTYPE_*, 0 = float32                 */
  int32_t n_kv_heads;        /* 0 = n_heads                              */
  int32_t freqs_dtype;       /* 0 = same as dtype                        */
  int32_t freqs_head_stride; /* -1 = head_dim (per-head columns), 0 = shared row */
  int64_t stride_f_seq, stride_f_dim; /* 0,0 = x's strides (reference)   */
  const int32_t* positions;  /* NULL = token index                       */
} krt_qkv_rope_args;

KRT_API int krt_fused_rmsnorm_qkv_rope(const krt_qkv_rope_args* args, void* stream);

/* -------------------------------------------------------------------------
 * Paged fused RMSNorm + QKV + RoPE + K/V scatter (bf16, tcgen05 tensor cores).
 *
 * Same math as above with GQA, bf16 activations/weights, fp32 RoPE tables
 * indexed by position, and K/V written straight into the paged KV pool:
 *   slot(t)  = block_table[token_seq[t] * block_table_stride
 *                          + positions[t] / tokens_per_block]
 *   pool byte offset = (slot * tokens_per_block + positions[t] % tokens_per_block)
 *                      * token_bytes,  token_bytes = 2 * n_kv_heads * head_dim * 2
 *   token layout     = [K | V][kv_head][head_dim] bf16
 * i.e. BlockManager's pool (block i at pool + i * tokens_per_block * token_bytes).
 * Block ids outside [0, num_blocks), positions outside [0, max_position) or
 * block-table columns outside the table skip the write and set KRT_ERR_DEVICE
 * in the status word (krt_read_status).
 *
 * decode : num_tokens <= 256, split-K across the GPU; needs a workspace of
 *          krt_qkv_rope_decode_workspace_size() bytes, zero-filled once when
 *          allocated (the kernel leaves it zeroed after every call).
 * prefill: any num_tokens; needs krt_qkv_rope_prefill_workspace_size() bytes.
 * head_dim must be 128; d_model a multiple of 64.
 * ---------------------------------------------------------------------- */
typedef struct krt_qkv_paged_args {
  const void* x;          /* bf16 [num_tokens, d_model], row stride x_stride */
  const void* qkv_weight; /* bf16 [(n_heads+2*n_kv_heads)*128, d_model], dense rows */
  const void* qkv_bias;   /* bf16 [(n_heads+2*n_kv_heads)*128] or NULL */
  const void* rms_weight; /* bf16 [d_model] */
  const float* rope_cos;  /* fp32 [max_position, 128] */
  const float* rope_sin;  /* fp32 [max_position, 128] */
  const int32_t* positions;   /* [num_tokens] */
  const int32_t* token_seq;   /* [num_tokens] row of block_table for each token */
  const int32_t* block_table; /* [num_seqs, block_table_stride] */
  void* kv_pool;              /* bf16, num_blocks * tokens_per_block * token_bytes bytes */
  void* q_out;                /* bf16 [num_tokens, n_heads, 128] (row stride q_stride) */
  void* k_out;                /* optional dense bf16 [num_tokens, n_kv_heads, 128] */
  void* v_out;                /* optional dense bf16 [num_tokens, n_kv_heads, 128] */
  int32_t num_tokens, d_model, n_heads, n_kv_heads, head_dim;
  int32_t x_stride, q_stride;
  int32_t max_position;
  int32_t num_seqs, block_table_stride, num_blocks, tokens_per_block;
  float eps;
  void* workspace;
  size_t workspace_bytes;
} krt_qkv_paged_args;

KRT_API size_t krt_qkv_rope_decode_workspace_size(int32_t num_tokens, int32_t d_model, int32_t n_heads,
                                          int32_t n_kv_heads, int32_t head_dim);
KRT_API int krt_qkv_rope_decode(const krt_qkv_paged_args* args, void* stream);

KRT_API size_t krt_qkv_rope_prefill_workspace_size(int32_t num_tokens, int32_t d_model, int32_t n_heads,
                                           int32_t n_kv_heads, int32_t head_dim);
KRT_API int krt_qkv_rope_prefill(const krt_qkv_paged_args* args, void* stream);

/* Decode for callers that cannot allocate device memory.  No counterpart in
 * the reference.  Same computation and arguments as krt_qkv_rope_decode, but
 * args->workspace / workspace_bytes are ignored: the workspace is a fixed
 * 4 MiB array in the library's own device memory, reserved on every GPU that
 * loads the library until the process exits.  Meant for callers whose device
 * memory is owned by someone else (a host application's allocator that forbids
 * outside cudaMalloc) or that must not allocate after start-up.
 *  - Calls whose workspace would exceed 4 MiB (krt_qkv_rope_decode_workspace_size)
 *    are rejected with KRT_ERR_UNSUPPORTED.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture on the device.
 *  - Every call on a device shares the one array and clears its header at the
 *    start; calls that can overlap on the GPU (different streams without
 *    ordering) race on it.  The status word of the last call is read with
 *    krt_qkv_rope_decode_noalloc_status.
 *  - Arguments are checked before anything reaches the GPU: a rejected call
 *    leaves the array untouched.
 *  - After cudaDeviceReset the array's address is looked up again (the
 *    context id changed); that first call after a reset, too, must come
 *    before any stream capture.
 *  - Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
KRT_API int krt_qkv_rope_decode_noalloc(const krt_qkv_paged_args* args, void* stream);

/* The status word of the library's fixed decode scratch on the current
 * device, as krt_read_status reports a workspace's (synchronises the stream,
 * clears the word).  Allocates nothing. */
KRT_API int krt_qkv_rope_decode_noalloc_status(void* stream, int32_t* bits);

/* Copy the device status word of a workspace to the host (synchronises the
 * stream), clear it, and return KRT_OK or KRT_ERR_DEVICE with the bits in
 * *bits.  Bits: 1 / 2 / 4 pipeline waits of a kernel ran out (full stage,
 * free stage, accumulator), 8 a token's position or pool block lies outside
 * the table or pool, 16 a wait for another GPU ran out, 32 inconsistent
 * split-K bookkeeping, 64 partials from the other CTAs of a thread-block
 * cluster did not arrive. */
KRT_API int krt_read_status(void* workspace, void* stream, int32_t* bits);

/* -------------------------------------------------------------------------
 * Communicator: symmetric peer buffers over NVLink / NVSwitch.
 *
 * Replaces Communicator(rank, world_size) (include/Communicator.h:15-26),
 * whose RCCL backend the reference left commented out
 * (src/Communicator.cpp:10-27).  One process per GPU:
 *   krt_comm_create      allocates this rank's buffer on the current device
 *                        (sized for outputs of up to max_n_out features)
 *   krt_comm_ipc_handle  writes its CUDA IPC handle (krt_comm_handle_size bytes)
 *   krt_comm_open_peers  maps every rank's buffer; `handles` holds world_size
 *                        handles in rank order (this rank's is skipped)
 * A world_size of 1 needs no peers.  Collectives of one communicator must be
 * issued on one stream per rank, in the same order on every rank.
 * ---------------------------------------------------------------------- */
typedef struct krt_comm krt_comm;

KRT_API int krt_comm_create(int32_t rank, int32_t world_size, int32_t max_n_out, krt_comm** out);
KRT_API size_t krt_comm_handle_size(void);
KRT_API int krt_comm_ipc_handle(krt_comm* comm, void* handle_out);
KRT_API int krt_comm_open_peers(krt_comm* comm, const void* handles);
KRT_API int krt_comm_destroy(krt_comm* comm);

/* NCCL for large messages (the reference's intended backend,
 * src/Communicator.cpp:10-27, whose ncclAllReduce call it left commented
 * out).  libnccl.so.2 is loaded at run time on first use (the copy already in
 * the process, else the system's); nothing else in the library needs it.
 *   krt_nccl_unique_id    one rank creates the id (krt_nccl_id_size bytes) and
 *                         shares it with the others out of band
 *   krt_comm_attach_nccl  collective: ncclCommInitRank for this communicator's
 *                         rank and world; afterwards krt_allreduce of at least
 *                         threshold_bytes, and krt_rowparallel_gemm_ar whose
 *                         bf16 output (num_tokens * n_out * 2 bytes, dense rows)
 *                         is at least that large, run the GEMM without the
 *                         fused exchange followed by one ncclAllReduce in place
 *                         (sum in NCCL's bf16 arithmetic).  SIZE_MAX disables it
 *                         again; calling it twice only changes the threshold.
 * krt_comm_destroy also destroys the NCCL communicator. */
KRT_API size_t krt_nccl_id_size(void);
KRT_API int krt_nccl_unique_id(void* id_out);
KRT_API int krt_comm_attach_nccl(krt_comm* comm, const void* id, size_t threshold_bytes);

/* Recovery after a peer wait ran out (status bit 16), e.g. when one rank
 * skipped or lost a collective call: the exchange epochs of the ranks no
 * longer agree, and every later fused call would wait out its budget.
 * A collective: every rank lets its own stream drain and all ranks meet at a
 * host barrier (so no kernel still writes into a peer's buffer), then each
 * calls krt_comm_reset, which zeroes this rank's flags, flagged words and
 * epoch counters (synchronising `stream`), and all meet at a second host
 * barrier before the next collective (TPComm.reset in python/kinetic_rt/dist.py
 * does exactly this).  The reference's
 * mock has no such state (tests/mock_rccl.h:72-74 only times out). */
KRT_API int krt_comm_reset(krt_comm* comm, void* stream);

/* Allreduce-sum of `count` elements (Communicator::all_reduce_async,
 * src/Communicator.cpp:21-27; every rank's recv receives the elementwise sum
 * of all ranks' send, tests/mock_rccl.h:51-62).  dtype: KRT_DTYPE_FLOAT32
 * (0 is accepted as float32, the mock backend's code, tests/mock_rccl.h:14)
 * or KRT_DTYPE_BFLOAT16; the sum is taken in fp32 in rank order, so every
 * rank gets bit-identical results.  `status` is a device int (a workspace
 * header, krt_read_status) that records peer-wait timeouts. */
KRT_API int krt_allreduce(krt_comm* comm, const void* send, void* recv, size_t count, int32_t dtype, void* status,
                          void* stream);

/* -------------------------------------------------------------------------
 * Row-parallel GEMM fused with the allreduce (o_proj / down_proj under TP).
 *
 * Rank r holds W[:, K_r] and X[:, K_r] (the torch.chunk(dim=1) shards of
 * scripts/export_hf.py:62-65); every rank receives
 *   Y = sum_r X[:, K_r] W[:, K_r]^T          (bf16 out, fp32 accumulation)
 * in one call: a tcgen05 GEMM whose epilogue exchanges the partial products
 * through the ranks' peer buffers (two ranks: each sends its partial to the
 * other and both reduce; more ranks: reduce-scatter to the owner of each
 * 128-feature tile, then all-gather of the bf16 result), with no separate
 * collective.  Partials travel as fp32 rounded to 15-bit mantissas and are
 * summed in fp32 in rank order, so every rank gets bit-identical results.
 * comm may be NULL for a single GPU.  Any num_tokens; k_local % 64 == 0,
 * n_out % 128 == 0.  Up to 256 tokens one launch; more tokens run, without
 * the fused exchange (one GPU, or the NCCL route), as one persistent GEMM
 * over 128- or 256-token blocks that reads each weight tile once per round
 * of CTAs, otherwise in launches of 256 tokens.  Calls that share a
 * communicator must be made in the same order, with the same shapes, on
 * every rank.
 * ---------------------------------------------------------------------- */
typedef struct krt_gemm_ar_args {
  const void* x;      /* bf16 [num_tokens, k_local], row stride x_stride */
  const void* weight; /* bf16 [n_out, k_local], dense rows */
  void* y;            /* bf16 [num_tokens, n_out], row stride y_stride */
  int32_t num_tokens, k_local, n_out, x_stride, y_stride;
  void* workspace;    /* krt_rowparallel_gemm_ar_workspace_size() bytes, zeroed once */
  size_t workspace_bytes;
  /* Optional residual (NULL = none): Y = residual + sum_r X_r W_r^T, summed
   * in fp32 before the one bf16 rounding, as the decoder's residual stream
   * h = h + o_proj(attn) / h + down_proj(act).  bf16, same row stride as y,
   * identical on every rank; it may be y itself (updated in place). */
  const void* residual;
} krt_gemm_ar_args;

KRT_API size_t krt_rowparallel_gemm_ar_workspace_size(void);
KRT_API int krt_rowparallel_gemm_ar(krt_comm* comm, const krt_gemm_ar_args* args, void* stream);

/* -------------------------------------------------------------------------
 * Paged decode attention (one query token per sequence, bf16, GQA).
 *
 * No kernel in the reference: its decoder forward does not exist yet
 * (python/kinetic_rt/orchestrator.py:419-448 re-runs the model per token);
 * this is the attention that reads the pool BlockManager owns
 * (include/BlockManager.h:29-95) after krt_qkv_rope_decode wrote the token's
 * K/V there.  For sequence s and query head h:
 *   out[s, h] = softmax(scale * q[s, h] . K^T) V  over tokens 0 .. seq_lens[s]-1
 * with K/V of KV head h / (n_heads / n_kv_heads), token p at pool slot
 * block_table[s * block_table_stride + p / tokens_per_block] * tokens_per_block
 * + p % tokens_per_block (token layout [K | V][kv_head][128] bf16).  fp32
 * accumulation and softmax; head_dim 128; at most 16 query heads per KV head;
 * tokens_per_block a multiple of 16.  A sequence with seq_lens <= 0 gets
 * zeros; one with seq_lens > max_seq_len attends over its first max_seq_len
 * tokens and sets status bit 8.  Out-of-range block ids are masked and set
 * status bit 8.  The
 * workspace (krt_paged_attention_workspace_size bytes) is zero-filled once
 * when allocated; the kernel leaves its counters at zero after every call.
 * ---------------------------------------------------------------------- */
typedef struct krt_paged_attention_args {
  const void* q;              /* bf16 [num_seqs, q_stride], query head h at h * 128 */
  const void* kv_pool;        /* bf16, num_blocks * tokens_per_block * token_bytes bytes */
  const int32_t* block_table; /* [num_seqs, block_table_stride] */
  const int32_t* seq_lens;    /* [num_seqs] tokens attended, the current one included */
  void* out;                  /* bf16 [num_seqs, out_stride] */
  int32_t num_seqs, n_heads, n_kv_heads, head_dim;
  int32_t q_stride, out_stride;
  int32_t block_table_stride, num_blocks, tokens_per_block;
  int32_t max_seq_len; /* upper bound of seq_lens: sizes the grid and the workspace */
  float scale;         /* softmax scale; 0 = 1 / sqrt(head_dim) */
  void* workspace;
  size_t workspace_bytes;
} krt_paged_attention_args;

KRT_API size_t krt_paged_attention_workspace_size(int32_t num_seqs, int32_t n_heads, int32_t n_kv_heads,
                                                  int32_t max_seq_len);
KRT_API int krt_paged_attention_decode(const krt_paged_attention_args* args, void* stream);

/* Causal paged attention for prompt tokens (prefill), GQA, bf16.  No
 * reference counterpart either (its generate loop recomputes the whole
 * sequence per token, python/kinetic_rt/orchestrator.py:419-448); it reads the
 * pool the prefill QKV kernel (krt_qkv_rope_prefill) scattered K/V into.
 * Sequence s has q_len = q_start[s + 1] - q_start[s] query tokens, rows
 * q_start[s] .. of q and out, at positions q_pos0[s] .. q_pos0[s] + q_len - 1;
 * the query at position p attends to the sequence's pool tokens 0 .. p (with
 * q_pos0 > 0 after a prefix already in the pool).  out[t, h] =
 * softmax(q[t, h] . K^T * scale) V over those tokens, kvh(h) = h / (n_heads /
 * n_kv_heads); n_heads / n_kv_heads must divide 16.  The workspace holds the
 * status word (krt_read_status): bit 8 for a block-table entry out of range
 * (that chunk is masked) or a q_len above max_q_len (rows past it are not
 * written), timeouts as elsewhere. */
typedef struct krt_paged_prefill_attention_args {
  const void* q;       /* bf16 [T, q_stride], query head h at columns h * 128 */
  void* out;           /* bf16 [T, out_stride] */
  const void* kv_pool; /* this layer's pool, [block][token][K|V][kv_head][128] bf16 */
  const int32_t* block_table; /* [num_seqs, block_table_stride] */
  const int32_t* q_start;     /* [num_seqs + 1] first query row of each sequence, then T */
  const int32_t* q_pos0;      /* [num_seqs] position of each sequence's first query token */
  int32_t num_seqs, n_heads, n_kv_heads, head_dim;
  int32_t q_stride, out_stride;
  int32_t block_table_stride, num_blocks, tokens_per_block;
  int32_t max_q_len;   /* upper bound of q_len over the sequences: sizes the grid */
  float scale;         /* softmax scale; 0 = 1 / sqrt(head_dim) */
  void* workspace;
  size_t workspace_bytes;
} krt_paged_prefill_attention_args;

KRT_API size_t krt_paged_attention_prefill_workspace_size(void);
KRT_API int krt_paged_attention_prefill(const krt_paged_prefill_attention_args* args, void* stream);

/* -------------------------------------------------------------------------
 * The rest of a decode step (batch of up to 256 tokens, bf16, fp32
 * accumulation).  The reference has no decoder forward; these are the
 * callers on either side of the hot path that its generation loop
 * (python/kinetic_rt/orchestrator.py:419-448, argmax at 442-444) needs, in
 * Llama's layer order: RMSNorm -> QKV + RoPE (krt_qkv_rope_decode) ->
 * attention -> o_proj + allreduce + residual -> RMSNorm -> gate/up + SwiGLU
 * -> down_proj + allreduce + residual; after the last layer RMSNorm ->
 * lm_head -> greedy argmax -> embedding of the chosen tokens.
 *
 * Both projections below normalise x first (RMSNorm with rms_weight, the
 * same cast-back order as the QKV path) and use a workspace of
 * krt_projection_workspace_size() bytes, zero-filled once before its first
 * use.  That size includes the flags and fp32 partials of the stream-K work
 * split (160 partial slots of 128 x num_tokens floats); a workspace of only
 * the base size (the QKV decode workspace's) still works, without stream-K.
 * After a call that set a timeout bit in the status word, zero the
 * workspace again before reusing it (a stream-K flag may be left raised).
 * ---------------------------------------------------------------------- */
KRT_API size_t krt_projection_workspace_size(int32_t num_tokens, int32_t d_model);

/* act = silu(x_hat W_gate^T) * (x_hat W_up^T), column-parallel over the
 * intermediate features (this rank's inter_local of them).  The weight keeps
 * gate and up rows side by side in 64-row groups: rows 128 i .. 128 i + 63
 * are gate rows of features 64 i .. 64 i + 63 and the next 64 rows are the up
 * rows of the same features (a load-time interleave of the two shards).
 * num_tokens up to 256 for a decode step, or a whole prompt (up to 2^20
 * tokens: the persistent kernel over 256-token blocks). */
typedef struct krt_gate_up_args {
  const void* x;              /* bf16 [num_tokens, d_model], row stride x_stride */
  const void* rms_weight;     /* bf16 [d_model] */
  const void* gate_up_weight; /* bf16 [2 * inter_local, d_model], interleaved as above */
  void* act;                  /* bf16 [num_tokens, act_stride] */
  int32_t num_tokens, d_model, inter_local, x_stride, act_stride;
  float eps;
  void* workspace;
  size_t workspace_bytes;
} krt_gate_up_args;
KRT_API int krt_gate_up_swiglu(const krt_gate_up_args* args, void* stream);

/* Greedy sampling over a vocabulary shard: for every token, the largest
 * logit of x_hat W^T over rows 0 .. vocab_local-1 and its vocabulary index
 * (vocab_offset + row) are folded into argmax_keys[t] (atomic max of an
 * orderable 64-bit key: higher logit first, then the lower index, as
 * torch.argmax picks the first maximum).  argmax_keys must hold 0 (empty)
 * before the first shard; krt_greedy_step reads and clears them. */
typedef struct krt_lm_head_args {
  const void* x;          /* bf16 [num_tokens, d_model], row stride x_stride */
  const void* rms_weight; /* bf16 [d_model] (the final norm) */
  const void* weight;     /* bf16 [vocab_local, d_model] this rank's lm_head rows */
  unsigned long long* argmax_keys; /* [num_tokens] */
  int32_t num_tokens, d_model, vocab_local, vocab_offset, x_stride;
  float eps;
  void* workspace;
  size_t workspace_bytes;
} krt_lm_head_args;
KRT_API int krt_lm_head_argmax(const krt_lm_head_args* args, void* stream);

/* Greedy choice and next-step input (one launch): for every sequence the
 * token with the largest logit over all ranks' vocabulary shards
 * (argmax_keys of this rank, exchanged through the communicator's peer
 * buffers; comm may be NULL for one GPU), written to tokens[] on every rank;
 * argmax_keys are cleared; the chosen token's embedding row is copied into
 * hidden (when embedding is given) and positions / seq_lens, when given, are
 * incremented.  Peer waits are bounded (status bit 16); a token outside the
 * vocabulary sets bit 8 and becomes 0.  Calls sharing a communicator must be
 * made in the same order on every rank. */
typedef struct krt_greedy_step_args {
  unsigned long long* argmax_keys; /* [num_seqs] from krt_lm_head_argmax */
  int32_t* tokens;                 /* [num_seqs] out */
  const void* embedding;           /* bf16 [vocab, d_model] or NULL */
  void* hidden;                    /* bf16 [num_seqs, hidden_stride] out */
  int32_t* positions;              /* [num_seqs] or NULL */
  int32_t* seq_lens;               /* [num_seqs] or NULL */
  int32_t num_seqs, d_model, hidden_stride, vocab;
  void* status;                    /* a workspace header (krt_read_status) */
  const int32_t* next_input;       /* [num_seqs] or NULL: where >= 0, that token's embedding is
                                      fed to the next step instead of the chosen one's (prompt
                                      tokens); tokens[] still receives the choice */
} krt_greedy_step_args;
KRT_API int krt_greedy_step(krt_comm* comm, const krt_greedy_step_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KRT_H_ */
