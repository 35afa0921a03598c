// Shared pieces of the paged fused RMSNorm + QKV + RoPE + K/V-scatter kernels.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda.h>
#include <cstring>

#include "ptx.cuh"

namespace krt {

constexpr int kHeadDim = 128;   // tile rows = one head of Q, K or V
constexpr int kBK = 64;         // k elements per pipeline stage (128-byte rows)
constexpr int kMaxStages = 8;

// Workspace header: [0] status word; the rest of the first 8 KB is reserved.
constexpr int kMaxTiles = 1024;  // head tiles per call
constexpr size_t kWsHeaderBytes = 8192;

struct PagedParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* gamma;
  const float* cos;
  const float* sin;
  const int32_t* positions;
  const int32_t* token_seq;
  const int32_t* block_table;
  __nv_bfloat16* pool;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  int num_tokens, n_pad, d_model, n_heads, n_kv_heads;
  int x_stride, q_stride;
  int max_position, num_seqs, bt_stride, num_blocks, tokens_per_block;
  float eps;
  int splits;         // split-K factor (decode)
  int stages;         // pipeline depth
  int kc;             // 64-column chunks per TMA box / pipeline stage
  int prefetch;       // weight stages requested into L2 ahead of the shared-memory ring
  int tmem_cols;
  int* status;        // workspace status word
  int* tok_pos;       // [num_tokens] position, or -1 when outside the RoPE table
  long long* tok_slot;  // [num_tokens] pool slot, or -1 when the block lookup failed
  __nv_bfloat16* xhat;  // [num_tokens, d_model] bf16(x * rsqrt(mean(x^2)+eps) * gamma)
  // Epilogue of the decode kernel (kEpi*); the fields below serve the
  // non-QKV epilogues.
  int epi;
  __nv_bfloat16* act;   // kEpiSwiglu: [num_tokens, act_stride] silu(gate) * up
  int act_stride;
  unsigned long long* keys;  // kEpiArgmax: [num_tokens] packed (logit, index) maxima
  int vocab_valid;      // kEpiArgmax: weight rows that are real vocabulary entries
  int vocab_offset;     // kEpiArgmax: vocabulary index of weight row 0
  // Persistent projection kernel, stream-K work split (sk != 0): every CTA
  // takes an equal run of (tile, k-box) work; a CTA whose run starts inside
  // a tile leaves its fp32 partial in sk_part[cta] and raises sk_flags[cta],
  // and the CTA holding that tile's first k-box adds it before the epilogue.
  int sk;
  int* sk_flags;        // [kSkMaxCtas] 0 / 1, back to 0 once consumed
  float* sk_part;       // [kSkMaxCtas][n_pad][128] fp32 partials
  // Persistent projection kernel over token blocks of n_pad tokens:
  // tile = block * row_tiles + row tile (row_tiles 0: one token block).
  int row_tiles;
  __nv_bfloat16* y;     // kEpiStore: [num_tokens, y_stride] bf16(acc + residual)
  int y_stride;
  const __nv_bfloat16* residual;  // kEpiStore: optional, same layout as y
  float* y32;           // kEpiStore: fp32 out (row stride y_stride, no residual) instead of y
};

// Epilogues of the decode-shaped (swap-AB, split-K) projection kernel:
//   kEpiQkv     bias, RoPE, Q out, K/V scattered into the paged pool
//   kEpiSwiglu  weight rows in 64-row groups [gate f..f+63 | up f..f+63]:
//               act[t, f + i] = silu(gate) * up
//   kEpiArgmax  logits of a vocabulary shard: per token the largest logit
//               and its index, folded into keys[t] with atomicMax
//   kEpiStore   y[t, row] = bf16(acc + residual[t, row]) (persistent kernel,
//               the row-parallel GEMM at large token counts)
enum : int { kEpiQkv = 0, kEpiSwiglu = 1, kEpiArgmax = 2, kEpiStore = 3 };

// Orderable 64-bit key of (logit, vocabulary index): larger logits give
// larger keys, and for equal logits the smaller index gives the larger key
// (the first maximum, as torch.argmax returns it).
__host__ __device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t u;
#ifdef __CUDA_ARCH__
  u = __float_as_uint(v);
#else
  memcpy(&u, &v, 4);
#endif
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__host__ __device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key) {
  return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

// Workspace layout shared by the decode and prefill paths.
struct WsLayout {
  size_t pos_off, slot_off, xhat_off, total;
};
inline WsLayout ws_layout(int T, int D) {
  auto up = [](size_t v) { return (v + 1023) & ~size_t(1023); };
  WsLayout l;
  l.pos_off = kWsHeaderBytes;
  l.slot_off = up(l.pos_off + 4 * (size_t)T);
  l.xhat_off = up(l.slot_off + 8 * (size_t)T);
  l.total = up(l.xhat_off + 2 * (size_t)T * D);
  return l;
}

// Projection workspace: the layout above, then the stream-K flags and
// partials of the persistent projection kernel (at most kSkMaxCtas CTAs,
// one 128-row partial of n_pad tokens each).
constexpr int kSkMaxCtas = 160;
// Tokens per gate/up call (a prompt runs in 256-token blocks).
constexpr int kMaxPromptTokens = 1 << 20;
struct ProjWsLayout {
  WsLayout base;
  size_t flags_off, part_off, total;
};
inline ProjWsLayout proj_ws_layout(int T, int D) {
  auto up = [](size_t v) { return (v + 1023) & ~size_t(1023); };
  ProjWsLayout l;
  l.base = ws_layout(T, D);
  // partials cover at most one 256-token block (stream-K runs at decode sizes only)
  const size_t n_pad = ((size_t)(T < 256 ? T : 256) + 15) / 16 * 16;
  l.flags_off = l.base.total;
  l.part_off = up(l.flags_off + 4 * (size_t)kSkMaxCtas);
  l.total = up(l.part_off + (size_t)kSkMaxCtas * n_pad * 128 * 4);
  return l;
}

// Pool slot of a token (block_id * tokens_per_block + offset), or -1 when the
// block table, the position or the block id is out of range.
__device__ __forceinline__ long long token_slot(const PagedParams& p, int t) {
  const int pos = p.positions[t];
  const int seq = p.token_seq[t];
  if (pos < 0 || pos >= p.max_position || seq < 0 || seq >= p.num_seqs) return -1;
  const int col = pos / p.tokens_per_block;
  if (col >= p.bt_stride) return -1;
  const int blk = p.block_table[(long long)seq * p.bt_stride + col];
  if (blk < 0 || blk >= p.num_blocks) return -1;
  return (long long)blk * p.tokens_per_block + (pos % p.tokens_per_block);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Row stride (floats) of the token-major staging buffers: 128 rows + 4 pad.
constexpr int kYStride = 132;

// Split-K exchange inside a cluster.  Each CTA parks its fp32 partial tile
// token-major ([n_pad][rows + 4]); the 16-token chunk c is finished by
// cluster rank c % splits, which receives the other ranks' partials of that
// chunk by bulk copy into its receive area:
//   slot(oc, q) = oc * (splits - 1) + (q < owner ? q : q - 1)
// for its oc-th owned chunk and source rank q.
//
// A tile is 128 weight rows (UMMA M = 128) or 64 (M = 64, where the
// accumulator row i sits in TMEM lane 32 * (i / 16) + i % 16).
template <int TM>
struct TileShape {
  static constexpr int kRows = TM;
  static constexpr int kParkStride = TM + 4;                 // floats per parked token row
  static constexpr uint32_t kChunkBytes = 16u * (TM + 4) * 4u;  // one 16-token chunk of a partial
  static constexpr int kRowsPerThread = TM / 8;               // finishing thread: 8 row groups x 16 tokens
  static constexpr uint32_t kSliceBytes = TM * 128u;          // one 64-column slice of the weight tile
};
constexpr uint32_t kChunkBytes = TileShape<128>::kChunkBytes;
__host__ __device__ inline int owned_chunks(int n_chunks, int splits, int rank) {
  return rank < n_chunks ? (n_chunks - 1 - rank) / splits + 1 : 0;
}
__host__ __device__ inline size_t recv_area_bytes(int n_pad, int splits, uint32_t chunk_bytes = kChunkBytes) {
  return splits > 1 ? (size_t)owned_chunks(n_pad / 16, splits, 0) * (splits - 1) * chunk_bytes : 0;
}
__host__ __device__ inline size_t park_area_bytes(int n_pad, int park_stride = kYStride) {
  return (size_t)n_pad * park_stride * sizeof(float);
}
__host__ __device__ inline int recv_slot(int oc, int splits, int owner, int q) {
  return oc * (splits - 1) + (q < owner ? q : q - 1);
}

// N (8 or 16) RoPE table values at `pos`, head rows r0 .. r0 + N - 1.
template <int N>
__device__ __forceinline__ void load_rope_n(const PagedParams& p, int pos, int r0, float4* cs, float4* sn) {
  if (pos < 0) pos = 0;
  const float4* c4 = reinterpret_cast<const float4*>(p.cos + (size_t)pos * kHeadDim + r0);
  const float4* s4 = reinterpret_cast<const float4*>(p.sin + (size_t)pos * kHeadDim + r0);
#pragma unroll
  for (int q = 0; q < N / 4; ++q) {
    cs[q] = __ldg(c4 + q);
    sn[q] = __ldg(s4 + q);
  }
}

// N (8 or 16) consecutive head rows r0 .. r0 + N - 1 of token t in head
// `head` (Q heads, then K, then V): y = the rows, yp = their rotate-half
// partner rows (r0 ^ 64 ..), sign = -1 for the first half of the head.  Q/K
// rows are rotated, V rows are not; Q goes to q[t], K/V to the pool slot and,
// when given, the dense k/v outputs, with 16-byte stores.
template <int N>
__device__ __forceinline__ void store_rows_n(const PagedParams& p, int head, int t, int r0, float sign, int pos,
                                             long long slot, const float* y, const float* yp, const float4* cs,
                                             const float4* sn) {
  const int Hq = p.n_heads, Hkv = p.n_kv_heads;
  const bool is_q = head < Hq;
  const bool is_v = head >= Hq + Hkv;
  const int g = is_q ? head : (is_v ? head - Hq - Hkv : head - Hq);
  float out[N];
  if (!is_v) {
    if (pos < 0) return;
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
      out[4 * q + 0] = y[4 * q + 0] * cs[q].x + sign * yp[4 * q + 0] * sn[q].x;
      out[4 * q + 1] = y[4 * q + 1] * cs[q].y + sign * yp[4 * q + 1] * sn[q].y;
      out[4 * q + 2] = y[4 * q + 2] * cs[q].z + sign * yp[4 * q + 2] * sn[q].z;
      out[4 * q + 3] = y[4 * q + 3] * cs[q].w + sign * yp[4 * q + 3] * sn[q].w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = y[i];
  }
  uint4 v[N / 8];
#pragma unroll
  for (int h = 0; h < N / 8; ++h)
    v[h] = make_uint4(pack_bf16x2(out[8 * h + 0], out[8 * h + 1]), pack_bf16x2(out[8 * h + 2], out[8 * h + 3]),
                      pack_bf16x2(out[8 * h + 4], out[8 * h + 5]), pack_bf16x2(out[8 * h + 6], out[8 * h + 7]));
  if (is_q) {
    uint4* dst = reinterpret_cast<uint4*>(p.q + (size_t)t * p.q_stride + (size_t)head * kHeadDim + r0);
#pragma unroll
    for (int h = 0; h < N / 8; ++h) dst[h] = v[h];
    return;
  }
  const size_t tok_elems = (size_t)2 * Hkv * kHeadDim;
  const size_t head_off = (size_t)(is_v ? Hkv + g : g) * kHeadDim + r0;
  if (slot >= 0) {
    uint4* dst = reinterpret_cast<uint4*>(p.pool + (size_t)slot * tok_elems + head_off);
#pragma unroll
    for (int h = 0; h < N / 8; ++h) dst[h] = v[h];
  }
  __nv_bfloat16* dense = is_v ? p.v : p.k;
  if (dense) {
    uint4* dst = reinterpret_cast<uint4*>(dense + ((size_t)t * Hkv + g) * kHeadDim + r0);
#pragma unroll
    for (int h = 0; h < N / 8; ++h) dst[h] = v[h];
  }
}

__device__ __forceinline__ void ld_smem_16f(const float* src, float* dst) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = reinterpret_cast<const float4*>(src)[q];
    dst[4 * q + 0] = v.x;
    dst[4 * q + 1] = v.y;
    dst[4 * q + 2] = v.z;
    dst[4 * q + 3] = v.w;
  }
}

}  // namespace krt
