// Paged decode attention over BlockManager's KV pool (bf16, GQA).
//
// One query token per sequence (decode): for sequence b and query head h,
//   o[b, h] = softmax(q[b, h] . K[b, kvh(h)]^T * scale) V[b, kvh(h)]
// over the sequence's first seq_lens[b] tokens, kvh(h) = h / (n_heads /
// n_kv_heads) (Llama's repeated KV heads), scale = 1 / sqrt(128).  K and V
// are read where the fused QKV kernel scattered them: token p of sequence
// b lives at slot block_table[b][p / B] * B + p % B of the pool, whose token
// layout is [K | V][kv_head][128] bf16 (BlockManager geometry,
// include/BlockManager.h:29-95; block ids per sequence as
// src/GraphWrapper.cpp:139-145 allocates them).
//
// The kernel reads every K/V byte once, so it is bound by HBM bandwidth
// (about 4 FLOP per byte for 4 query heads per KV head):
//   * grid (sequence, KV head, split of the context); a CTA's four warps take
//     its 16-token chunks round-robin, each warp with a private ring of three
//     8 KB stages;
//   * one TMA per chunk brings K and V of one KV head for 16 tokens into
//     shared memory: the 5-D tensor map views the pool as
//     {64 dims, token, dim half, K|V, kv head} so the box lands as four
//     [16 tokens x 128 B] tiles with the 128-byte swizzle (conflict-free
//     ldmatrix rows);
//   * Q K^T and P V on the tensor cores with mma.sync m16n8k16 (query heads
//     of the group in rows 0..G-1, the group padded to 16 rows), fp32
//     accumulators, online softmax in base 2 in registers (the work is a few
//     FLOP per byte, so the legacy warp-level MMA is far from limiting);
//   * the four warps' running (max, sum, output) are merged in shared
//     memory; with several splits each CTA leaves its merged partial in the
//     workspace and the last CTA of the (sequence, KV head) to finish merges
//     them all and writes bf16 output (counter in the workspace, reset by
//     that CTA).
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <cuda_runtime.h>

#include "../../include/krt.h"
#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnStages = 3;                 // per warp
constexpr int kAttnChunk = 16;                 // tokens per TMA box
constexpr uint32_t kAttnStageBytes = 8192;     // K and V of 16 tokens, one KV head
constexpr int kAttnMaxGroup = 16;              // query heads per KV head
constexpr int kAttnRowFloats = 2 + kHeadDim;   // max, sum, 128 outputs
constexpr int kAttnMaxCps = 512;               // 16-token chunks per CTA at most

struct AttnParams {
  const __nv_bfloat16* q;    // [num_seqs, q_stride], query head h at h * 128
  __nv_bfloat16* out;        // [num_seqs, out_stride]
  const int32_t* block_table;
  const int32_t* seq_lens;
  float* part;               // [num_seqs][n_kv_heads][max_splits][G][kAttnRowFloats]
  uint32_t* counters;        // [num_seqs][n_kv_heads]
  int* status;
  int num_seqs, bt_stride, num_blocks, tokens_per_block;
  int n_heads, n_kv_heads, group;
  int q_stride, out_stride;
  int chunks_per_split, max_splits;
  int max_len;               // the grid covers this many tokens per sequence
  float scale_log2;          // softmax scale * log2(e)
};

struct AttnSmemTail {
  uint64_t full[kAttnWarps][kAttnStages];
  int tok[kAttnMaxCps];  // first pool token of each of the CTA's chunks, -1 when the lookup failed
  int last;
};

__host__ __device__ inline size_t attn_smem_bytes() {
  return 1024 + (size_t)kAttnWarps * kAttnStages * kAttnStageBytes + sizeof(AttnSmemTail);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D (16x8 fp32) += A (16x16 bf16, row-major) * B (16x8 bf16, column-major).
__device__ __forceinline__ void mma_bf16_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Address of the 16-byte chunk `chunk` (0..7) of token row `tok` in a
// [16 tokens x 128 B] tile written by TMA with the 128-byte swizzle (tile
// base 1024-byte aligned; tokens 0-7 and 8-15 are two swizzle atoms).
__device__ __forceinline__ uint32_t sw128_addr(uint32_t tile, int tok, int chunk) {
  return tile + (uint32_t)tok * 128u + ((uint32_t)(chunk ^ (tok & 7)) << 4);
}

__global__ void __launch_bounds__(kAttnThreads, 2)
    paged_attention_decode_kernel(const __grid_constant__ CUtensorMap tmap_kv, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnSmemTail* tl =
      reinterpret_cast<AttnSmemTail*>(smem + (size_t)kAttnWarps * kAttnStages * kAttnStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int b = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z;
  const int G = p.group;

  if (lane == 0) {
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&tl->full[warp][s], 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 0) tma_prefetch_desc(&tmap_kv);
  __syncwarp();
  pdl_wait();  // q and the pool come from the previous kernel
  pdl_launch_dependents();

  int len = p.seq_lens[b];
  if (len > p.max_len) {
    // beyond the grid (and the workspace): attend over the first max_len tokens and report it
    if (threadIdx.x == 0 && z == 0) atomicOr(p.status, kStatusBadBlock);
    len = p.max_len;
  }
  const int n_chunks = len > 0 ? (len + kAttnChunk - 1) / kAttnChunk : 0;
  const int splits = n_chunks > 0 ? (n_chunks + p.chunks_per_split - 1) / p.chunks_per_split : 1;
  if (z >= splits) return;  // the whole CTA: nothing of this sequence left for it
  const int c_begin = z * p.chunks_per_split;
  const int c_end = min(n_chunks, c_begin + p.chunks_per_split);

  // First pool token of every chunk of this CTA, looked up once by all
  // threads in parallel (-1 when the block table column or block id is out
  // of range: the chunk is then read from token 0 and masked).
  for (int i = threadIdx.x; i < c_end - c_begin; i += kAttnThreads) {
    const int tok = (c_begin + i) * kAttnChunk;
    const int col = tok / p.tokens_per_block;
    int v = -1;
    if (col < p.bt_stride) {
      const int blk = p.block_table[(size_t)b * p.bt_stride + col];
      if (blk >= 0 && blk < p.num_blocks) v = blk * p.tokens_per_block + tok % p.tokens_per_block;
    }
    tl->tok[i] = v;
  }
  __syncthreads();
  uint8_t* wstage = smem + (size_t)warp * kAttnStages * kAttnStageBytes;
  const uint32_t wstage_u32 = smem_u32(wstage);
  // lane 0 issues this warp's loads: the k-th chunk of the warp is
  // c_begin + warp + 4k and uses stage k % 3
  auto issue = [&](int k) {
    const int tok = tl->tok[warp + kAttnWarps * k];
    uint64_t* bar = &tl->full[warp][k % kAttnStages];
    mbar_arrive_expect_tx(bar, kAttnStageBytes);
    const uint64_t pol = make_l2_policy_evict_first();
    tma_load_5d(wstage + (size_t)(k % kAttnStages) * kAttnStageBytes, &tmap_kv, bar, 0, tok < 0 ? 0 : tok, 0, 0,
                kvh, pol);
  };
  const int my_chunks = c_end - c_begin > warp ? (c_end - c_begin - warp + kAttnWarps - 1) / kAttnWarps : 0;
  int issued = my_chunks < kAttnStages ? my_chunks : kAttnStages;  // chunks 0 .. issued-1 requested
  if (lane == 0)
    for (int k = 0; k < issued; ++k) issue(k);

  // Query fragments (A operand, rows = query heads of the group, zero-padded
  // to 16): k-step ks covers dims 16 ks .. 16 ks + 15.
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qrow0 = p.q + (size_t)b * p.q_stride + (size_t)(kvh * G + g) * kHeadDim;
    const __nv_bfloat16* qrow1 = p.q + (size_t)b * p.q_stride + (size_t)(kvh * G + g + 8) * kHeadDim;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int d0 = 16 * ks + 2 * t4;
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t*>(qrow0 + d0) : 0u;
      qa[ks][1] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qrow1 + d0) : 0u;
      qa[ks][2] = g < G ? *reinterpret_cast<const uint32_t*>(qrow0 + d0 + 8) : 0u;
      qa[ks][3] = g + 8 < G ? *reinterpret_cast<const uint32_t*>(qrow1 + d0 + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};  // running max of rows g and g + 8 (base-2 logits)
  float l_r[2] = {0.f, 0.f};              // this lane's share of the running sums
  bool ok = true;

  for (int k = 0; k < my_chunks; ++k) {
    const int s = k % kAttnStages;
    const uint32_t ph = (uint32_t)(k / kAttnStages) & 1u;
    const bool got = mbar_wait_warp(&tl->full[warp][s], ph, nullptr);
    if (!got) {
      ok = false;
      break;
    }
    const uint32_t st = wstage_u32 + (uint32_t)s * kAttnStageBytes;
    const int c = c_begin + warp + kAttnWarps * k;
    // ---- S = Q K^T for the 16 tokens (two n-tiles of 8)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int mat = lane >> 3, r = lane & 7;
      const int tok = r + 8 * (mat >> 1);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int half = ks >> 2, ch = 2 * (ks & 3) + (mat & 1);
        uint32_t bf[4];
        ldsm_x4(sw128_addr(st + (uint32_t)half * 2048u, tok, ch), bf);
        mma_bf16_16816(sc[0], qa[ks], bf[0], bf[1]);
        mma_bf16_16816(sc[1], qa[ks], bf[2], bf[3]);
      }
    }
    // ---- online softmax (base 2); tokens past the sequence end are masked
    const int tok_base = c * kAttnChunk;
    const bool chunk_bad = tl->tok[c - c_begin] < 0;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = tok_base + 8 * j + 2 * t4 + (e & 1);
        float v = sc[j][e] * p.scale_log2;
        if (tk >= len || chunk_bad) v = -INFINITY;
        sc[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float corr[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
      const float m_new = fmaxf(m_r[rr], mx[rr]);
      corr[rr] = m_new == -INFINITY ? 1.f : exp2f(m_r[rr] - m_new);
      m_r[rr] = m_new;
    }
    float pr[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = m_r[e >> 1];
        pr[j][e] = m == -INFINITY ? 0.f : exp2f(sc[j][e] - m);
      }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) l_r[rr] = l_r[rr] * corr[rr] + pr[0][2 * rr] + pr[0][2 * rr + 1] + pr[1][2 * rr] +
                                             pr[1][2 * rr + 1];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // ---- O += P V (P as the A operand: the S accumulators re-packed as bf16)
    uint32_t pa[4];
    pa[0] = pack_bf16x2(pr[0][0], pr[0][1]);
    pa[1] = pack_bf16x2(pr[0][2], pr[0][3]);
    pa[2] = pack_bf16x2(pr[1][0], pr[1][1]);
    pa[3] = pack_bf16x2(pr[1][2], pr[1][3]);
    {
      const int mat = lane >> 3, r = lane & 7;
      const int tok = r + 8 * (mat & 1);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int half = jj >> 2, ch = 2 * (jj & 3) + (mat >> 1);
        uint32_t bf[4];
        ldsm_x4_trans(sw128_addr(st + 4096u + (uint32_t)half * 2048u, tok, ch), bf);
        mma_bf16_16816(o[2 * jj], pa, bf[0], bf[1]);
        mma_bf16_16816(o[2 * jj + 1], pa, bf[2], bf[3]);
      }
    }
    // ---- refill the stage with this warp's chunk k + 3
    __syncwarp();
    if (k + kAttnStages < my_chunks) {
      if (lane == 0) {
        fence_proxy_async_smem();  // the ldmatrix reads above come before the TMA rewrites the stage
        issue(k + kAttnStages);
      }
      issued = k + kAttnStages + 1;
    }
  }
  if (!ok) {
    // A load did not land in time: record it and wait (bounded) for every
    // load this warp still has in flight before the CTA may exit.
    if (lane == 0) {
      atomicOr(p.status, kStatusTimeoutFull);
      for (int k = issued - kAttnStages > 0 ? issued - kAttnStages : 0; k < issued; ++k)
        mbar_wait(&tl->full[warp][k % kAttnStages], (uint32_t)(k / kAttnStages) & 1u, nullptr);
    }
  }
  for (int i = threadIdx.x; i < c_end - c_begin; i += kAttnThreads)
    if (tl->tok[i] < 0) atomicOr(p.status, kStatusBadBlock);
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }

  // ---- merge the four warps: rows [warp][row][max, sum, 128 outputs] in the
  // (now idle) stage buffers
  __syncthreads();
  float* wrow = reinterpret_cast<float*>(smem);
  auto row_at = [&](int w, int row) { return wrow + ((size_t)w * kAttnMaxGroup + row) * kAttnRowFloats; };
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int row = g + 8 * rr;
    if (row >= G) continue;
    float* dst = row_at(warp, row);
    if (t4 == 0) {
      dst[0] = m_r[rr];
      dst[1] = l_r[rr];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      dst[2 + 8 * j + 2 * t4] = o[j][2 * rr];
      dst[2 + 8 * j + 2 * t4 + 1] = o[j][2 * rr + 1];
    }
  }
  __syncthreads();
  // thread -> (row, 8 dims) pairs of the merged result
  const bool single = splits == 1;
  float* part = p.part + (((size_t)b * p.n_kv_heads + kvh) * p.max_splits + z) * (size_t)G * kAttnRowFloats;
  for (int idx = threadIdx.x; idx < G * 16; idx += kAttnThreads) {
    const int row = idx >> 4, d0 = (idx & 15) * 8;
    float mw[kAttnWarps], M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      mw[w] = row_at(w, row)[0];
      M = fmaxf(M, mw[w]);
    }
    float L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = M == -INFINITY ? 0.f : exp2f(mw[w] - M);
      const float* src = row_at(w, row);
      L += f * src[1];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f * src[2 + d0 + i];
    }
    if (single) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      uint4 v = make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                           pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
      *reinterpret_cast<uint4*>(p.out + (size_t)b * p.out_stride + (size_t)(kvh * G + row) * kHeadDim + d0) = v;
    } else {
      float* dst = part + (size_t)row * kAttnRowFloats;
      if (d0 == 0) {
        dst[0] = M;
        dst[1] = L;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[2 + d0 + i] = acc[i];
    }
  }
  if (single) return;

  // ---- several splits: the last CTA of this (sequence, KV head) merges them
  __threadfence();  // this CTA's partial is visible GPU-wide before the count
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* ctr = p.counters + (size_t)b * p.n_kv_heads + kvh;
    const uint32_t prev = atomicAdd(ctr, 1u);
    const bool last = prev + 1 == (uint32_t)splits;
    if (last) *ctr = 0u;  // ready for the next call
    tl->last = last ? 1 : 0;
  }
  __syncthreads();
  if (!tl->last) return;
  __threadfence();
  const float* base = p.part + ((size_t)b * p.n_kv_heads + kvh) * p.max_splits * (size_t)G * kAttnRowFloats;
  for (int idx = threadIdx.x; idx < G * 16; idx += kAttnThreads) {
    const int row = idx >> 4, d0 = (idx & 15) * 8;
    float M = -INFINITY;
    for (int zz = 0; zz < splits; ++zz) M = fmaxf(M, __ldcg(base + ((size_t)zz * G + row) * kAttnRowFloats));
    float L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int zz = 0; zz < splits; ++zz) {
      const float* src = base + ((size_t)zz * G + row) * kAttnRowFloats;
      const float mz = __ldcg(src);
      const float f = M == -INFINITY ? 0.f : exp2f(mz - M);
      L += f * __ldcg(src + 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += f * __ldcg(src + 2 + d0 + i);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    uint4 v = make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                         pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
    *reinterpret_cast<uint4*>(p.out + (size_t)b * p.out_stride + (size_t)(kvh * G + row) * kHeadDim + d0) = v;
  }
}

}  // namespace krt

using namespace krt;

// ------------------------------------------------------------------ C ABI
namespace {

// Tensor map of the pool for one KV head's K and V of 16 tokens per box:
//   d0 = 64 dims (128 contiguous bytes), d1 = token (all blocks' tokens in
//   order; block i's token j is token i * B + j), d2 = dim half (128 B),
//   d3 = K | V, d4 = kv head (256 B); box {64, 16, 2, 2, 1}, so one box is
//   [K lo, K hi, V lo, V hi] x [16 tokens x 128 B], 128-byte swizzled.
int make_tmap_kv_pool(CUtensorMap* map, const void* pool, int num_blocks, int tokens_per_block, int n_kv_heads) {
  const uint64_t token_bytes = (uint64_t)2 * n_kv_heads * kHeadDim * 2;
  return make_tmap_bf16_5d_strided(map, pool, {64, (uint64_t)num_blocks * tokens_per_block, 2, 2, (uint64_t)n_kv_heads},
                                   {token_bytes, 128, (uint64_t)n_kv_heads * 256, 256}, {64, 16, 2, 2, 1});
}

int attn_env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

// 16-token chunks per CTA: at least 16 (256 tokens, before evening out), and
// as many as keep the grid at about one and a half waves of CTAs (B200, batch 128 at context
// 4224: 1 KV head per sequence, 66 chunks per CTA 50.6 us against 59.5 us with
// 29 (four waves) and 93.7 us with 8; 8 KV heads, unsplit 327.8 us against
// 369.4 us with 32 chunks).
int attn_chunks_per_split(int num_seqs, int n_kv_heads, int max_chunks) {
  const int forced = attn_env_int("KRT_ATTN_SPLIT_CHUNKS", 0);
  if (forced > 0) return forced < kAttnMaxCps ? forced : kAttnMaxCps;
  const long long slots = (long long)device_sm_count() * 2;  // two CTAs per SM
  const long long pairs = (long long)num_seqs * n_kv_heads;
  long long cps = (2 * pairs * max_chunks + 3 * slots - 1) / (3 * slots);
  if (cps < 16) cps = 16;
  if (cps > max_chunks) cps = max_chunks;
  if (cps > kAttnMaxCps) cps = kAttnMaxCps;
  if (cps < 1) cps = 1;
  // equal pieces: the same number of splits, the chunks spread evenly over
  // them (264 chunks: 4 x 66 rather than 77, 77, 77, 33; B200, batch 128 at
  // context 4224, one KV head: 51.3 against 53.8 us; within 1 us either way
  // at two KV heads and at the 70B shard's 130 chunks)
  const long long splits = (max_chunks + cps - 1) / cps;
  cps = (max_chunks + splits - 1) / splits;
  return (int)(cps > 0 ? cps : 1);
}

size_t attn_part_floats(int num_seqs, int n_heads, int max_splits) {
  return (size_t)num_seqs * n_heads * max_splits * kAttnRowFloats;
}

}  // namespace

extern "C" size_t krt_paged_attention_workspace_size(int32_t num_seqs, int32_t n_heads, int32_t n_kv_heads,
                                                     int32_t max_seq_len) {
  if (num_seqs <= 0 || n_heads <= 0 || n_kv_heads <= 0 || max_seq_len <= 0 || n_heads % n_kv_heads != 0) return 0;
  const int max_chunks = (max_seq_len + kAttnChunk - 1) / kAttnChunk;
  const int cps = attn_chunks_per_split(num_seqs, n_kv_heads, max_chunks);
  const int max_splits = (max_chunks + cps - 1) / cps;
  const size_t counters = ((size_t)num_seqs * n_kv_heads * 4 + 255) & ~size_t(255);
  return kWsHeaderBytes + counters + attn_part_floats(num_seqs, n_heads, max_splits) * 4;
}

extern "C" int krt_paged_attention_decode(const krt_paged_attention_args* a, void* stream) {
  if (!a) return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: args is NULL");
  if (!a->q || !a->kv_pool || !a->block_table || !a->seq_lens || !a->out || !a->workspace)
    return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: a required pointer is NULL");
  if (a->num_seqs <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->max_seq_len <= 0)
    return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: num_seqs, heads and max_seq_len must be positive");
  if (a->head_dim != kHeadDim) return set_error(KRT_ERR_UNSUPPORTED, "krt_paged_attention_decode: head_dim must be 128");
  if (a->n_heads % a->n_kv_heads != 0 || a->n_heads / a->n_kv_heads > kAttnMaxGroup)
    return set_error(KRT_ERR_UNSUPPORTED,
                     "krt_paged_attention_decode: n_heads must be a multiple of n_kv_heads, at most 16 per KV head");
  if (a->tokens_per_block <= 0 || a->tokens_per_block % kAttnChunk != 0)
    return set_error(KRT_ERR_UNSUPPORTED, "krt_paged_attention_decode: tokens_per_block must be a multiple of 16");
  if (a->num_blocks <= 0 || a->block_table_stride <= 0)
    return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: paged-cache geometry must be positive");
  if ((long long)a->block_table_stride * a->tokens_per_block < a->max_seq_len)
    return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: the block table cannot hold max_seq_len tokens");
  if (a->q_stride < a->n_heads * kHeadDim || a->q_stride % 8 != 0 || a->out_stride < a->n_heads * kHeadDim ||
      a->out_stride % 8 != 0)
    return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: q/out strides must cover the heads, multiples of 8");
  if ((reinterpret_cast<uintptr_t>(a->q) & 15) || (reinterpret_cast<uintptr_t>(a->out) & 15) ||
      (reinterpret_cast<uintptr_t>(a->kv_pool) & 15) || (reinterpret_cast<uintptr_t>(a->workspace) & 15))
    return set_error(KRT_ERR_INVALID, "krt_paged_attention_decode: tensors must be 16-byte aligned");
  const size_t need = krt_paged_attention_workspace_size(a->num_seqs, a->n_heads, a->n_kv_heads, a->max_seq_len);
  if (a->workspace_bytes < need)
    return set_error(KRT_ERR_WORKSPACE, "krt_paged_attention_decode: workspace of %zu bytes, %zu needed",
                     a->workspace_bytes, need);
  const int max_chunks = (a->max_seq_len + kAttnChunk - 1) / kAttnChunk;
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.block_table = a->block_table;
  p.seq_lens = a->seq_lens;
  char* ws = static_cast<char*>(a->workspace);
  p.status = reinterpret_cast<int*>(ws);
  p.counters = reinterpret_cast<uint32_t*>(ws + kWsHeaderBytes);
  const size_t counters = ((size_t)a->num_seqs * a->n_kv_heads * 4 + 255) & ~size_t(255);
  p.part = reinterpret_cast<float*>(ws + kWsHeaderBytes + counters);
  p.num_seqs = a->num_seqs;
  p.bt_stride = a->block_table_stride;
  p.num_blocks = a->num_blocks;
  p.tokens_per_block = a->tokens_per_block;
  p.n_heads = a->n_heads;
  p.n_kv_heads = a->n_kv_heads;
  p.group = a->n_heads / a->n_kv_heads;
  p.q_stride = a->q_stride;
  p.out_stride = a->out_stride;
  p.max_len = a->max_seq_len;
  p.chunks_per_split = attn_chunks_per_split(a->num_seqs, a->n_kv_heads, max_chunks);
  p.max_splits = (max_chunks + p.chunks_per_split - 1) / p.chunks_per_split;
  const float scale = a->scale > 0.f ? a->scale : 0.08838834764831845f;  // 1 / sqrt(128)
  p.scale_log2 = scale * 1.4426950408889634f;
  CUtensorMap tmap;
  int rc = make_tmap_kv_pool(&tmap, a->kv_pool, a->num_blocks, a->tokens_per_block, a->n_kv_heads);
  if (rc) return rc;
  const size_t smem = attn_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(paged_attention_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return cuda_error(e, "krt_paged_attention_decode: shared memory attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a->num_seqs, (unsigned)a->n_kv_heads, (unsigned)p.max_splits);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, paged_attention_decode_kernel, tmap, p);
  if (e != cudaSuccess) return cuda_error(e, "krt_paged_attention_decode launch");
  return clear_error();
}
