// Shared pieces of the paged fused RMSNorm + QKV + RoPE + K/V-scatter kernels.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda.h>

#include "ptx.cuh"

namespace krt {

constexpr int kHeadDim = 128;   // tile rows = one head of Q, K or V
constexpr int kBK = 64;         // k elements per pipeline stage (128-byte rows)
constexpr int kMaxStages = 8;

// Workspace header: [0] status word, [64 .. 64 + 4*kMaxTiles) split-K counters.
constexpr int kMaxTiles = 1024;
constexpr size_t kWsCounterOffset = 64;
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
  int tmem_cols;
  int* status;        // workspace status word
  int* counters;      // split-K arrival counters, one per head tile (decode)
  int* tok_pos;       // [num_tokens] position, or -1 when outside the RoPE table
  long long* tok_slot;  // [num_tokens] pool slot, or -1 when the block lookup failed
  __nv_bfloat16* xhat;  // [num_tokens, d_model] bf16(x * rsqrt(mean(x^2)+eps) * gamma)
  float* partial;     // [tiles][splits][128][n_pad] split-K partial sums (decode)
};

// Workspace layout shared by the decode and prefill paths.
struct WsLayout {
  size_t pos_off, slot_off, xhat_off, partial_off, total;
};
inline WsLayout ws_layout(int T, int D, size_t partial_bytes) {
  auto up = [](size_t v) { return (v + 1023) & ~size_t(1023); };
  WsLayout l;
  l.pos_off = kWsHeaderBytes;
  l.slot_off = up(l.pos_off + 4 * (size_t)T);
  l.xhat_off = up(l.slot_off + 8 * (size_t)T);
  l.partial_off = up(l.xhat_off + 2 * (size_t)T * D);
  l.total = l.partial_off + partial_bytes;
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

// cos/sin values of rows 16*g8 .. +15 at position `pos` (16-byte loads),
// issued ahead of their use so the gather latency overlaps other work.
__device__ __forceinline__ void load_rope16(const PagedParams& p, int pos, int g8, float4* cs, float4* sn) {
  if (pos < 0) pos = 0;
  const float4* c4 = reinterpret_cast<const float4*>(p.cos + (size_t)pos * kHeadDim + 16 * g8);
  const float4* s4 = reinterpret_cast<const float4*>(p.sin + (size_t)pos * kHeadDim + 16 * g8);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    cs[q] = __ldg(c4 + q);
    sn[q] = __ldg(s4 + q);
  }
}

// Epilogue, phase B: thread (token t, row group g8) of a head tile writes
// rows row0 + 16*g8 .. +15 of token t.
//   y[i]  = qkv[t][row0 + 16*g8 + i] (fp32, bias included)
//   yp[i] = the rotate-half partner rows 16*(g8^4) + i (Q/K tiles only)
//   Q/K tiles: out = y*cos + rotate_half(y)*sin with rotate_half = [-y2, y1]
//              per head (fusion_forge.py:92-139); cs/sn from load_rope16;
//   V tiles:   out = y, unrotated (fusion_forge.py:161-162).
// Q goes to q[t][tile*128 + ...]; K/V to pool slot `slot` and, when given, to
// the dense k/v outputs.  Two 16-byte stores per destination.
__device__ __forceinline__ void store_rows16(const PagedParams& p, int tile, int t, int g8, int pos, long long slot,
                                             const float* y, const float* yp, const float4* cs, const float4* sn) {
  const int Hq = p.n_heads, Hkv = p.n_kv_heads;
  const bool is_q = tile < Hq;
  const bool is_v = tile >= Hq + Hkv;
  const int g = is_q ? tile : (is_v ? tile - Hq - Hkv : tile - Hq);
  const int r0 = 16 * g8;
  float out[16];
  if (!is_v) {
    if (pos < 0) return;
    const float sign = g8 < 4 ? -1.f : 1.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      out[4 * q + 0] = y[4 * q + 0] * cs[q].x + sign * yp[4 * q + 0] * sn[q].x;
      out[4 * q + 1] = y[4 * q + 1] * cs[q].y + sign * yp[4 * q + 1] * sn[q].y;
      out[4 * q + 2] = y[4 * q + 2] * cs[q].z + sign * yp[4 * q + 2] * sn[q].z;
      out[4 * q + 3] = y[4 * q + 3] * cs[q].w + sign * yp[4 * q + 3] * sn[q].w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = y[i];
  }
  uint4 v0, v1;
  v0.x = pack_bf16x2(out[0], out[1]);
  v0.y = pack_bf16x2(out[2], out[3]);
  v0.z = pack_bf16x2(out[4], out[5]);
  v0.w = pack_bf16x2(out[6], out[7]);
  v1.x = pack_bf16x2(out[8], out[9]);
  v1.y = pack_bf16x2(out[10], out[11]);
  v1.z = pack_bf16x2(out[12], out[13]);
  v1.w = pack_bf16x2(out[14], out[15]);
  if (is_q) {
    uint4* dst = reinterpret_cast<uint4*>(p.q + (size_t)t * p.q_stride + (size_t)tile * kHeadDim + r0);
    dst[0] = v0;
    dst[1] = v1;
    return;
  }
  const size_t tok_elems = (size_t)2 * Hkv * kHeadDim;
  const size_t head_off = (size_t)(is_v ? Hkv + g : g) * kHeadDim + r0;
  if (slot >= 0) {
    uint4* dst = reinterpret_cast<uint4*>(p.pool + (size_t)slot * tok_elems + head_off);
    dst[0] = v0;
    dst[1] = v1;
  }
  __nv_bfloat16* dense = is_v ? p.v : p.k;
  if (dense) {
    uint4* dst = reinterpret_cast<uint4*>(dense + ((size_t)t * Hkv + g) * kHeadDim + r0);
    dst[0] = v0;
    dst[1] = v1;
  }
}

// Row stride (floats) of the token-major staging buffers: 128 rows + 4 pad.
constexpr int kYStride = 132;

// Split-K exchange inside a cluster.  Each CTA parks its fp32 partial tile
// token-major ([n_pad][kYStride]); the 16-token chunk c is finished by
// cluster rank c % splits, which receives the other ranks' partials of that
// chunk by bulk copy into its receive area:
//   slot(oc, q) = oc * (splits - 1) + (q < owner ? q : q - 1)
// for its oc-th owned chunk and source rank q.
constexpr uint32_t kChunkBytes = 16u * kYStride * 4u;  // one chunk of a partial
__host__ __device__ inline int owned_chunks(int n_chunks, int splits, int rank) {
  return rank < n_chunks ? (n_chunks - 1 - rank) / splits + 1 : 0;
}
__host__ __device__ inline size_t recv_area_bytes(int n_pad, int splits) {
  return splits > 1 ? (size_t)owned_chunks(n_pad / 16, splits, 0) * (splits - 1) * kChunkBytes : 0;
}
__host__ __device__ inline size_t park_area_bytes(int n_pad) { return (size_t)n_pad * kYStride * sizeof(float); }
__host__ __device__ inline int recv_slot(int oc, int splits, int owner, int q) {
  return oc * (splits - 1) + (q < owner ? q : q - 1);
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
