// Causal paged attention for prompt tokens (prefill, GQA), bf16.
//
// Sequence s has q_len = q_start[s + 1] - q_start[s] query tokens (rows
// q_start[s] .. of q and out) at positions q_pos0[s] .. q_pos0[s] + q_len - 1;
// the query at position p attends to the sequence's pool tokens 0 .. p, which
// the prefill QKV kernel (or earlier steps) scattered into BlockManager's pool
// (token t of sequence s at slot block_table[s][t / B] * B + t % B, token
// layout [K | V][kv_head][128] bf16, include/BlockManager.h:29-95).  With
// q_pos0 = 0 this is the prompt's own causal attention; q_pos0 > 0 continues
// after a prefix already in the pool (chunked prefill).  kvh(h) = h / G,
// G = n_heads / n_kv_heads (Llama's repeated KV heads).
//
// Unlike decode, the work is about 2 * 128 * G FLOP per K/V byte fetched
// from L2, so the kernel shares each K/V chunk among as many query rows as a
// CTA holds:
//   * grid (query tile, sequence, KV head), tiles with the longest causal
//     range first; a tile is 128 rows = (128 / G) consecutive query tokens x
//     the G query heads of one KV head;
//   * a producer warp streams the tile's causal range of K/V in 16-token
//     chunks through an 8-stage ring (one 5-D TMA box = K and V of one KV head
//     for 16 tokens, 8 KB, the decode kernel's tensor map);
//   * eight compute warps hold 16 rows each (16 / G tokens x G heads) and run
//     Q K^T and P V with mma.sync m16n8k16 over blocks of four chunks (64
//     keys) with one online-softmax update (base 2) per block, so the output
//     rescale and the row reductions are paid once per 64 keys; keys past a
//     row's position are masked, and a warp skips the math of blocks that lie
//     wholly past its last token (it still waits for and releases every
//     stage, so releases stay in step with the fills);
//   * every wait is bounded; a block-table entry out of range reads token 0,
//     masks the chunk and sets status bit 8, as does a sequence with more
//     query tokens than max_q_len (the rows past it are left unwritten).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#include "../../include/krt.h"
#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kPfaWarps = 8;                      // compute warps
constexpr int kPfaThreads = 32 * (kPfaWarps + 1);  // + the producer warp
constexpr int kPfaRows = 16 * kPfaWarps;           // query rows per CTA
constexpr int kPfaStages = 8;                     // two softmax blocks in flight
constexpr int kPfaBlk = 4;                         // 16-token chunks per softmax update (64 keys)
constexpr int kPfaChunk = 16;                      // tokens per TMA box
constexpr uint32_t kPfaStageBytes = 8192;          // K and V of 16 tokens, one KV head

struct PfaParams {
  const __nv_bfloat16* q;  // [T, q_stride], query head h at h * 128
  __nv_bfloat16* out;      // [T, out_stride]
  const int32_t* block_table;
  const int32_t* q_start;  // [num_seqs + 1]
  const int32_t* q_pos0;   // [num_seqs]
  int* status;
  int num_seqs, bt_stride, num_blocks, tokens_per_block;
  int n_heads, n_kv_heads, group;
  int q_stride, out_stride;
  float scale_log2;
};

struct PfaSmemTail {
  uint64_t full[kPfaStages];
  uint64_t empty[kPfaStages];
  int ctok[kPfaStages];  // first pool token of the chunk in each stage, -1 when the lookup failed
};

size_t pfa_smem_bytes() { return 1024 + (size_t)kPfaStages * kPfaStageBytes + sizeof(PfaSmemTail); }

__device__ __forceinline__ void pfa_ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void pfa_ldsm_x4_trans(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D (16x8 fp32) += A (16x16 bf16, row-major) * B (16x8 bf16, column-major).
__device__ __forceinline__ void pfa_mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 16-byte chunk `chunk` of token row `tok` in a 128-byte-swizzled [16 x 128 B] tile.
__device__ __forceinline__ uint32_t pfa_sw128(uint32_t tile, int tok, int chunk) {
  return tile + (uint32_t)tok * 128u + ((uint32_t)(chunk ^ (tok & 7)) << 4);
}

__global__ void __launch_bounds__(kPfaThreads, 1)
    paged_attention_prefill_kernel(const __grid_constant__ CUtensorMap tmap_kv, const PfaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PfaSmemTail* tl = reinterpret_cast<PfaSmemTail*>(smem + (size_t)kPfaStages * kPfaStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group;
  const int qt = kPfaRows / G;  // query tokens per tile
  const int tile = (int)gridDim.x - 1 - (int)blockIdx.x;
  const int seq = blockIdx.y, kvh = blockIdx.z;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfaStages; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], kPfaWarps);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmap_kv);
  }
  __syncthreads();
  pdl_wait();  // q and the pool come from the previous kernel
  pdl_launch_dependents();

  const int qs = p.q_start[seq];
  const int q_len = p.q_start[seq + 1] - qs;
  const int pos0 = p.q_pos0[seq];
  const int t_begin = tile * qt;
  // query rows beyond the grid (q_len > max_q_len) are not computed: report it
  if (tile == 0 && threadIdx.x == 0 && q_len > (int)gridDim.x * qt) atomicOr(p.status, kStatusBadBlock);
  if (t_begin >= q_len || q_len <= 0) return;  // the whole CTA
  const int t_end = min(q_len, t_begin + qt);
  const int n_chunks = (pos0 + t_end - 1) / kPfaChunk + 1;  // causal range of the tile's last token

  if (warp == kPfaWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = make_l2_policy_evict_last();  // the other tiles of the sequence re-read it
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      for (int k = 0; k < n_chunks; ++k) {
        if (k >= kPfaStages && !mbar_wait(&tl->empty[s], ph ^ 1u, nullptr)) {
          atomicOr(p.status, kStatusTimeoutEmpty);
          break;
        }
        const int tok = k * kPfaChunk;
        const int col = tok / p.tokens_per_block;
        int v = -1;
        if (col < p.bt_stride) {
          const int blk = p.block_table[(size_t)seq * p.bt_stride + col];
          if (blk >= 0 && blk < p.num_blocks) v = blk * p.tokens_per_block + tok % p.tokens_per_block;
        }
        if (v < 0) atomicOr(p.status, kStatusBadBlock);
        tl->ctok[s] = v;
        mbar_arrive_expect_tx(&tl->full[s], kPfaStageBytes);
        tma_load_5d(smem + (size_t)s * kPfaStageBytes, &tmap_kv, &tl->full[s], 0, v < 0 ? 0 : v, 0, 0, kvh, pol);
        ++issued;
        if (++s == kPfaStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      // before exiting, every load in flight has landed (bounded)
      for (int k = issued - kPfaStages > 0 ? issued - kPfaStages : 0; k < issued; ++k)
        mbar_wait(&tl->full[k % kPfaStages], (uint32_t)(k / kPfaStages) & 1u, nullptr);
    }
    return;
  }

  // ------------------------------------------------------------ compute warps
  const int g = lane >> 2, t4 = lane & 3;
  const int tpw = 16 / G;                // tokens per warp
  const int wt0 = t_begin + warp * tpw;  // this warp's first token (index within the sequence)
  // rows g and g + 8: token and head
  int row_tok[2], row_pos[2];
  bool row_ok[2];
  const __nv_bfloat16* qrow[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = g + 8 * rr;
    row_tok[rr] = wt0 + r / G;
    row_ok[rr] = row_tok[rr] < t_end;
    row_pos[rr] = pos0 + row_tok[rr];
    qrow[rr] = p.q + (size_t)(qs + (row_ok[rr] ? row_tok[rr] : t_begin)) * p.q_stride +
               (size_t)(kvh * G + r % G) * kHeadDim;
  }
  const int w_last = min(t_end - 1, wt0 + tpw - 1);
  const int w_chunks = wt0 < t_end ? (pos0 + w_last) / kPfaChunk + 1 : 0;  // chunks with any visible key
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d0 = 16 * ks + 2 * t4;
    qa[ks][0] = row_ok[0] ? *reinterpret_cast<const uint32_t*>(qrow[0] + d0) : 0u;
    qa[ks][1] = row_ok[1] ? *reinterpret_cast<const uint32_t*>(qrow[1] + d0) : 0u;
    qa[ks][2] = row_ok[0] ? *reinterpret_cast<const uint32_t*>(qrow[0] + d0 + 8) : 0u;
    qa[ks][3] = row_ok[1] ? *reinterpret_cast<const uint32_t*>(qrow[1] + d0 + 8) : 0u;
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  const uint32_t stages = smem_u32(smem);
  const int n_blocks = (n_chunks + kPfaBlk - 1) / kPfaBlk;
  bool ok = true;
  for (int kb = 0; kb < n_blocks; ++kb) {
    const int k0 = kb * kPfaBlk;
    const int nc = min(kPfaBlk, n_chunks - k0);  // chunks in this block (the last one may be short)
    // Every warp waits for every chunk, also those it has no keys for: its
    // release of a stage must not count toward a later fill of the same stage
    // (the producer refills a stage once all eight warps released it).
    for (int c = 0; c < nc && ok; ++c) {
      const int k = k0 + c;
      if (!mbar_wait_warp(&tl->full[k % kPfaStages], (uint32_t)(k / kPfaStages) & 1u, nullptr)) {
        if (lane == 0) atomicOr(p.status, kStatusTimeoutFull);
        ok = false;
      }
    }
    if (!ok) break;
    if (k0 < w_chunks) {
      // ---- S = Q K^T for the block's (up to) 64 keys: n-tile 2c + j holds keys 16c + 8j ..
      float sc[2 * kPfaBlk][4];
#pragma unroll
      for (int jj = 0; jj < 2 * kPfaBlk; ++jj) sc[jj][0] = sc[jj][1] = sc[jj][2] = sc[jj][3] = 0.f;
      {
        const int mat = lane >> 3, r = lane & 7;
        const int tok = r + 8 * (mat >> 1);
#pragma unroll
        for (int c = 0; c < kPfaBlk; ++c) {
          if (c >= nc) break;
          const uint32_t st = stages + (uint32_t)((k0 + c) % kPfaStages) * kPfaStageBytes;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const int half = ks >> 2, ch = 2 * (ks & 3) + (mat & 1);
            uint32_t bf[4];
            pfa_ldsm_x4(pfa_sw128(st + (uint32_t)half * 2048u, tok, ch), bf);
            pfa_mma(sc[2 * c], qa[ks], bf[0], bf[1]);
            pfa_mma(sc[2 * c + 1], qa[ks], bf[2], bf[3]);
          }
        }
      }
      // ---- causal mask + one online-softmax update (base 2) for the block
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kPfaBlk; ++c) {
        const bool chunk_bad = c >= nc || tl->ctok[(k0 + c) % kPfaStages] < 0;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int kp = (k0 + c) * kPfaChunk + 8 * j + 2 * t4 + (e & 1);
            const int rr = e >> 1;
            float v = sc[2 * c + j][e] * p.scale_log2;
            if (chunk_bad || kp > row_pos[rr] || !row_ok[rr]) v = -INFINITY;
            sc[2 * c + j][e] = v;
            mx[rr] = fmaxf(mx[rr], v);
          }
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
      float lsum[2] = {0.f, 0.f};
#pragma unroll
      for (int jj = 0; jj < 2 * kPfaBlk; ++jj)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float m = m_r[e >> 1];
          const float pv = m == -INFINITY ? 0.f : exp2f(sc[jj][e] - m);
          sc[jj][e] = pv;  // probabilities in place
          lsum[e >> 1] += pv;
        }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) l_r[rr] = l_r[rr] * corr[rr] + lsum[rr];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= corr[0];
        o[j][1] *= corr[0];
        o[j][2] *= corr[1];
        o[j][3] *= corr[1];
      }
      // ---- O += P V, one 16-key k-step per chunk
      {
        const int mat = lane >> 3, r = lane & 7;
        const int tok = r + 8 * (mat & 1);
#pragma unroll
        for (int c = 0; c < kPfaBlk; ++c) {
          if (c >= nc) break;
          const uint32_t st = stages + (uint32_t)((k0 + c) % kPfaStages) * kPfaStageBytes;
          uint32_t pa[4];
          pa[0] = pack_bf16x2(sc[2 * c][0], sc[2 * c][1]);
          pa[1] = pack_bf16x2(sc[2 * c][2], sc[2 * c][3]);
          pa[2] = pack_bf16x2(sc[2 * c + 1][0], sc[2 * c + 1][1]);
          pa[3] = pack_bf16x2(sc[2 * c + 1][2], sc[2 * c + 1][3]);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int half = jj >> 2, ch = 2 * (jj & 3) + (mat >> 1);
            uint32_t bf[4];
            pfa_ldsm_x4_trans(pfa_sw128(st + 4096u + (uint32_t)half * 2048u, tok, ch), bf);
            pfa_mma(o[2 * jj], pa, bf[0], bf[1]);
            pfa_mma(o[2 * jj + 1], pa, bf[2], bf[3]);
          }
        }
      }
      // the ldmatrix reads of the stages come before the TMA that rewrites them
      fence_proxy_async_smem();
    }
    __syncwarp();
    if (lane == 0)
      for (int c = 0; c < nc; ++c) mbar_arrive(&tl->empty[(k0 + c) % kPfaStages]);
  }
  if (!ok) return;
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  // ---- normalised bf16 rows out
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    if (!row_ok[rr]) continue;
    const int r = g + 8 * rr;
    const float inv = l_r[rr] > 0.f ? 1.f / l_r[rr] : 0.f;
    __nv_bfloat16* dst = p.out + (size_t)(qs + row_tok[rr]) * p.out_stride + (size_t)(kvh * G + r % G) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(dst + 8 * j + 2 * t4) = pack_bf16x2(o[j][2 * rr] * inv, o[j][2 * rr + 1] * inv);
  }
}

}  // namespace krt

using namespace krt;

// ------------------------------------------------------------------ C ABI
extern "C" size_t krt_paged_attention_prefill_workspace_size(void) { return kWsHeaderBytes; }

extern "C" int krt_paged_attention_prefill(const krt_paged_prefill_attention_args* a, void* stream) {
  const char* name = "krt_paged_attention_prefill";
  if (!a) return set_error(KRT_ERR_INVALID, "%s: args is NULL", name);
  if (!a->q || !a->out || !a->kv_pool || !a->block_table || !a->q_start || !a->q_pos0 || !a->workspace)
    return set_error(KRT_ERR_INVALID, "%s: a required pointer is NULL", name);
  if (a->head_dim != kHeadDim) return set_error(KRT_ERR_UNSUPPORTED, "%s: head_dim must be 128", name);
  if (a->num_seqs <= 0 || a->num_seqs > 65535 || a->n_heads <= 0 || a->n_kv_heads <= 0 || a->max_q_len <= 0)
    return set_error(KRT_ERR_INVALID, "%s: num_seqs (1..65535), heads and max_q_len must be positive", name);
  if (a->n_heads % a->n_kv_heads != 0) return set_error(KRT_ERR_INVALID, "%s: n_heads %% n_kv_heads != 0", name);
  const int G = a->n_heads / a->n_kv_heads;
  if (G > 16 || 16 % G != 0)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: n_heads / n_kv_heads must be 1, 2, 4, 8 or 16", name);
  if (a->tokens_per_block <= 0 || a->tokens_per_block % kPfaChunk != 0)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: tokens_per_block must be a multiple of 16", name);
  if (a->num_blocks <= 0 || a->block_table_stride <= 0)
    return set_error(KRT_ERR_INVALID, "%s: num_blocks and block_table_stride must be positive", name);
  if (a->q_stride < a->n_heads * kHeadDim || a->q_stride % 8 != 0 || a->out_stride < a->n_heads * kHeadDim ||
      a->out_stride % 8 != 0)
    return set_error(KRT_ERR_INVALID, "%s: strides must cover the heads and be multiples of 8", name);
  if ((reinterpret_cast<uintptr_t>(a->q) & 15) || (reinterpret_cast<uintptr_t>(a->out) & 15) ||
      (reinterpret_cast<uintptr_t>(a->kv_pool) & 15))
    return set_error(KRT_ERR_INVALID, "%s: q, out and kv_pool must be 16-byte aligned", name);
  if (a->workspace_bytes < kWsHeaderBytes)
    return set_error(KRT_ERR_WORKSPACE, "%s: workspace of %zu bytes, %zu needed", name, a->workspace_bytes,
                     (size_t)kWsHeaderBytes);
  PfaParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.out = static_cast<__nv_bfloat16*>(a->out);
  p.block_table = a->block_table;
  p.q_start = a->q_start;
  p.q_pos0 = a->q_pos0;
  p.status = static_cast<int*>(a->workspace);
  p.num_seqs = a->num_seqs;
  p.bt_stride = a->block_table_stride;
  p.num_blocks = a->num_blocks;
  p.tokens_per_block = a->tokens_per_block;
  p.n_heads = a->n_heads;
  p.n_kv_heads = a->n_kv_heads;
  p.group = G;
  p.q_stride = a->q_stride;
  p.out_stride = a->out_stride;
  const float scale = a->scale > 0.f ? a->scale : 1.f / std::sqrt((float)kHeadDim);
  p.scale_log2 = scale * 1.4426950408889634f;
  CUtensorMap tmap;
  const uint64_t token_bytes = (uint64_t)2 * a->n_kv_heads * kHeadDim * 2;
  int rc = make_tmap_bf16_5d_strided(&tmap, a->kv_pool,
                                     {64, (uint64_t)a->num_blocks * a->tokens_per_block, 2, 2, (uint64_t)a->n_kv_heads},
                                     {token_bytes, 128, (uint64_t)a->n_kv_heads * 256, 256}, {64, 16, 2, 2, 1});
  if (rc) return rc;
  const size_t smem = pfa_smem_bytes();
  cudaError_t e =
      cudaFuncSetAttribute(paged_attention_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_error(e, name);
  const int qt = kPfaRows / G;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a->max_q_len + qt - 1) / qt), (unsigned)a->num_seqs, (unsigned)a->n_kv_heads);
  cfg.blockDim = dim3(kPfaThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, paged_attention_prefill_kernel, tmap, p);
  if (e != cudaSuccess) return cuda_error(e, name);
  return clear_error();
}
