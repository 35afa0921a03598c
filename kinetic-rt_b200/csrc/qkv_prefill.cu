// Prefill variant of the fused RMSNorm + QKV projection + RoPE + paged K/V
// scatter (bf16, tcgen05 / TMEM, TMA, persistent).
//
// Shape: thousands of tokens, so the projection is a dense contraction and
// the kernel is tensor-bound:
//
//   1. qkv_prep_kernel (qkv_prep.cu): x_hat = bf16(x * rsqrt(mean(x^2)+eps)
//      * gamma) per token into the workspace (the reference's order of
//      operations, fusion_forge.py:42-47) plus per-token positions and pool
//      slots;
//   2. qkv_rope_prefill_kernel, launched with programmatic dependent launch:
//      persistent, one CTA per SM; tile = (one head of 128 weight rows) x
//      (256 tokens).  Both operands arrive by TMA with the 128-byte swizzle
//      (W and x_hat kept in L2 with an evict-last policy, both are re-read);
//      one thread issues 128 x 256 x 16 UMMAs into one of two TMEM
//      accumulators (2 x 256 columns) so the epilogue of tile i overlaps the
//      main loop of tile i+1.
//
// Epilogue: eight warps in two groups of four (each group covers the 128
// TMEM lanes) take alternate 16-token chunks.  Per chunk, (A) thread r = TMEM
// lane adds the bias and parks row r token-major in its group's buffer;
// (B) thread (token j, rows 16*g8..+15) applies RoPE with the partner rows
// r ^ 64 and writes 16-byte vectors to Q or to the paged pool
// (store_rows_n).  cos/sin gathers are issued before the TMEM load so their
// latency overlaps it; per-token positions and slots are staged in shared
// memory once per tile.
//
// Tiles are ordered token-block-major with heads fastest, so the CTAs working
// on one token block share its x_hat rows in L2 and the weight matrix (50 MB
// for Llama-3-8B shapes) stays L2-resident.
#include <cstdint>
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kPrefillEpiWarps = 8;
constexpr int kPrefillThreads = 64 + 32 * kPrefillEpiWarps;  // 320
constexpr int kPrefillBN = 256;  // tokens per tile (UMMA N)
constexpr int kPrefillStages = 4;
constexpr uint32_t kPfABytes = 128 * 128;         // 128 rows x 64 bf16
constexpr uint32_t kPfBBytes = kPrefillBN * 128;  // 256 rows x 64 bf16
constexpr uint32_t kPfStageBytes = kPfABytes + kPfBBytes;
constexpr int kYBufFloats = 16 * kYStride;        // one 16-token chunk, token-major

struct PrefillSmemTail {
  uint64_t full[kPrefillStages];
  uint64_t empty[kPrefillStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
  int pos[kPrefillBN];
  long long slot[kPrefillBN];
};

size_t prefill_smem_bytes() {
  return 1024 + (size_t)kPrefillStages * kPfStageBytes + 2 * kYBufFloats * sizeof(float) + sizeof(PrefillSmemTail);
}

__device__ __forceinline__ void prefill_fail(const PagedParams& p, PrefillSmemTail* tl, int code) {
  atomicOr(p.status, code);
  tl->abort = 1;
}

__global__ void __launch_bounds__(kPrefillThreads, 1)
    qkv_rope_prefill_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                            const PagedParams p, int num_tiles, int tiles_per_block) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_mem = smem;
  float* ybufs = reinterpret_cast<float*>(smem + (size_t)kPrefillStages * kPfStageBytes);
  PrefillSmemTail* tl = reinterpret_cast<PrefillSmemTail*>(ybufs + 2 * kYBufFloats);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kb = p.d_model / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPrefillStages; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tl->tmem_full[b], 1);
      mbar_init(&tl->tmem_empty[b], kPrefillEpiWarps);
    }
    tl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(&tl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tl->tmem_base;
  volatile int* abort_flag = &tl->abort;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol = make_l2_policy_evict_last();
      pdl_wait();
      uint32_t it = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < num_tiles && alive; tile += gridDim.x) {
        const int head = tile % tiles_per_block;
        const int nb = tile / tiles_per_block;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kPrefillStages;
          const uint32_t ph = (it / kPrefillStages) & 1u;
          if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
            prefill_fail(p, tl, kStatusTimeoutEmpty);
            alive = false;
            break;
          }
          uint8_t* st = stage_mem + (size_t)s * kPfStageBytes;
          mbar_arrive_expect_tx(&tl->full[s], kPfStageBytes);
          tma_load_2d_hint(st, &tmap_w, &tl->full[s], kb * kBK, head * kHeadDim, pol);
          tma_load_2d_hint(st + kPfABytes, &tmap_x, &tl->full[s], kb * kBK, nb * kPrefillBN, pol);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issue
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, kPrefillBN);
      uint32_t it = 0, local = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < num_tiles && alive; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1u;
        const uint32_t use = local >> 1;
        if (!mbar_wait(&tl->tmem_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
          prefill_fail(p, tl, kStatusTimeoutAccum);
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + buf * kPrefillBN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % kPrefillStages;
          const uint32_t ph = (it / kPrefillStages) & 1u;
          if (!mbar_wait(&tl->full[s], ph, abort_flag)) {
            prefill_fail(p, tl, kStatusTimeoutFull);
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stage_mem + (size_t)s * kPfStageBytes);
          const uint64_t ad = umma_desc_sw128(sa);
          const uint64_t bd = umma_desc_sw128(sa + kPfABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(dcol, ad + 2u * kk, bd + 2u * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&tl->empty[s]);
        }
        umma_commit(&tl->tmem_full[buf]);
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int ept = threadIdx.x - 64;   // 0..255
    const int grp = ept >> 7;           // chunk group: 0 takes even chunks, 1 odd
    const int gt = ept & 127;
    const int q4 = warp & 3;            // TMEM lane quadrant of this warp
    const int r = q4 * 32 + lane;       // accumulator row
    const int j = gt & 15, g8 = gt >> 4; // phase-B token / row group (8 lanes: 8 tokens, no bank conflicts)
    const int bar_grp = 1 + grp;        // 128-thread barrier of this group
    float* ybuf = ybufs + grp * kYBufFloats;
    pdl_wait();
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int head = tile % tiles_per_block;
      const int nb = tile / tiles_per_block;
      const uint32_t buf = local & 1u;
      const uint32_t use = local >> 1;
      const int t_base = nb * kPrefillBN;
      // stage this tile's token metadata (the previous tile is finished)
      const int t_ld = t_base + ept;
      tl->pos[ept] = t_ld < p.num_tokens ? p.tok_pos[t_ld] : -1;
      tl->slot[ept] = t_ld < p.num_tokens ? p.tok_slot[t_ld] : -1;
      const bool waited = mbar_wait_warp(&tl->tmem_full[buf], use & 1u, abort_flag);
      if (!waited && lane == 0) prefill_fail(p, tl, kStatusTimeoutAccum);
      tc_fence_after();
      if (named_bar_any(3, 256, !waited || *abort_flag != 0)) break;
      const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16) + buf * kPrefillBN;
      const float bias_r = p.bias ? __bfloat162float(p.bias[head * kHeadDim + r]) : 0.f;
      const bool rot = head < p.n_heads + p.n_kv_heads;
      for (int c0 = grp * 16; c0 < kPrefillBN; c0 += 32) {
        if (t_base + c0 >= p.num_tokens) break;  // uniform within the group
        const int jt = c0 + j;
        const int pos = tl->pos[jt];
        float4 cs[4], sn[4];
        if (rot) load_rope_n<16>(p, pos, 16 * g8, cs, sn);
        float acc[16];
        tmem_ld16(taddr + (uint32_t)c0, acc);
#pragma unroll
        for (int i = 0; i < 16; ++i) ybuf[i * kYStride + r] = acc[i] + bias_r;
        named_bar_sync(bar_grp, 128);
        if (t_base + jt < p.num_tokens) {
          float y[16], yp[16];
          ld_smem_16f(ybuf + j * kYStride + 16 * g8, y);
          ld_smem_16f(ybuf + j * kYStride + 16 * (g8 ^ 4), yp);
          store_rows_n<16>(p, head, t_base + jt, 16 * g8, g8 < 4 ? -1.f : 1.f, pos, tl->slot[jt], y, yp, cs, sn);
        }
        named_bar_sync(bar_grp, 128);
      }
      tc_fence_before();
      named_bar_sync(3, 256);  // both groups are done with this tile's TMEM and metadata
      if (lane == 0) mbar_arrive(&tl->tmem_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

cudaError_t launch_qkv_rope_prefill(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                                    int tiles_per_block, cudaStream_t stream) {
  const size_t smem = prefill_smem_bytes();
  cudaError_t e =
      cudaFuncSetAttribute(qkv_rope_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int n_blocks = (p.num_tokens + kPrefillBN - 1) / kPrefillBN;
  const int num_tiles = n_blocks * tiles_per_block;
  int grid = device_sm_count();
  if (grid > num_tiles) grid = num_tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kPrefillThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qkv_rope_prefill_kernel, tmap_w, tmap_x, p, num_tiles, tiles_per_block);
}

}  // namespace krt
