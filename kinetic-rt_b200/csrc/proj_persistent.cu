// Persistent decode-shaped projection (bf16, tcgen05 / TMEM, TMA): many
// 128-row weight tiles times a batch of up to 256 tokens, full K per tile.
//
// The split-K decode kernel (qkv_decode.cu) gives every CTA one tile (or a
// K slice of one), which suits a few dozen tiles.  With hundreds of tiles
// (gate/up of the MLP: 2 x 14336 / TP rows; the lm_head: 128256 / TP rows)
// its CTAs come in waves, each paying the pipeline fill and the epilogue
// tail, and the last wave leaves SMs idle.  Here one CTA per SM walks the
// tiles blockIdx.x, blockIdx.x + gridDim.x, ...:
//   * warp 0 streams W and x_hat k-blocks through a ring of stages without
//     draining between tiles (the first stages' weight loads are issued
//     before griddepcontrol.wait: weights do not depend on the previous
//     kernel);
//   * warp 1 issues UMMAs (M = 128 weight rows, N = padded tokens) into one
//     of two TMEM accumulators, so the epilogue of tile i overlaps the main
//     loop of tile i + 1;
//   * eight epilogue warps in two groups take alternate 16-token chunks: TMEM
//     lane r parks its 16 values token-major in the group's buffer, then
//     thread (token j, rows 16 g .. 16 g + 15) applies the epilogue with the
//     partner rows 16 (g ^ 4) .. (the same scheme as the prefill kernel).
// Epilogues (PagedParams::epi): kEpiSwiglu (act = silu(gate) * up, gate and
// up rows side by side in 64-row groups) and kEpiArgmax (the CTA keeps each
// token's best (logit, index) over all its tiles in shared memory and folds
// it into the global keys once at the end).  The kEpiQkv branch (bias, RoPE,
// Q out, K/V into the pool) mirrors the prefill kernel's epilogue; the
// launcher does not offer it (QKV runs on the split-K decode kernel).
#include <cstdint>
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kPjEpiWarps = 8;
constexpr int kPjThreads = 64 + 32 * kPjEpiWarps;  // 320
constexpr int kPjMaxStages = 8;
constexpr uint32_t kPjSliceBytes = 128 * 128;      // 128 weight rows x 64 bf16
constexpr int kPjYBufFloats = 16 * kYStride;       // one 16-token chunk, token-major

struct PjSmemTail {
  uint64_t full[kPjMaxStages];
  uint64_t empty[kPjMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
  int pos[256];
  long long slot[256];
  unsigned long long key[256];
};

size_t proj_persistent_smem_bytes(int stages, int kc, int n_pad) {
  return 1024 + (size_t)stages * kc * (kPjSliceBytes + (size_t)n_pad * 128) +
         2 * (size_t)kPjYBufFloats * sizeof(float) + sizeof(PjSmemTail);
}

__device__ __forceinline__ void pj_fail(const PagedParams& p, PjSmemTail* tl, int code) {
  atomicOr(p.status, code);
  tl->abort = 1;
}

template <int EPI>
__global__ void __launch_bounds__(kPjThreads, 1)
    proj_persistent_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                           const PagedParams p, int num_tiles) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages, KC = p.kc, n_pad = p.n_pad;
  const uint32_t a_stage = (uint32_t)KC * kPjSliceBytes;
  const uint32_t b_chunk = (uint32_t)n_pad * 128u;
  const uint32_t b_stage = (uint32_t)KC * b_chunk;
  const uint32_t stage_bytes = a_stage + b_stage;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + (size_t)S * a_stage;
  float* ybufs = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes);
  PjSmemTail* tl = reinterpret_cast<PjSmemTail*>(ybufs + 2 * kPjYBufFloats);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kc = p.d_model / (kBK * KC);
  const int my_tiles = blockIdx.x < num_tiles ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_tiles * num_kc;  // pipeline stages this CTA streams
  const int pre = total < S ? total : S;
  auto tile_of = [&](int it) { return (int)blockIdx.x + (it / num_kc) * (int)gridDim.x; };

  uint64_t pol_w = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tl->tmem_full[b], 1);
      mbar_init(&tl->tmem_empty[b], kPjEpiWarps);
    }
    tl->abort = 0;
    fence_mbar_init();
    // the first stages' weight tiles depend on nothing: request them now
    tma_prefetch_desc(&tmap_w);
    pol_w = make_l2_policy_evict_first();  // weights are streamed once
    for (int it = 0; it < pre; ++it) {
      mbar_arrive_expect_tx(&tl->full[it], stage_bytes);
      tma_load_3d(a_smem + (size_t)it * a_stage, &tmap_w, &tl->full[it], 0, tile_of(it) * 128, (it % num_kc) * KC,
                  pol_w);
    }
    // optionally the next p.prefetch stages' weights into L2 beyond the ring
    for (int it = pre; it < total && it < pre + p.prefetch; ++it)
      tma_prefetch_l2_3d(&tmap_w, 0, tile_of(it) * 128, (it % num_kc) * KC);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(&tl->tmem_base, (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  if (EPI == kEpiArgmax)
    for (int t = threadIdx.x; t < 256; t += kPjThreads) tl->key[t] = 0ull;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const uint32_t tmem_base = tl->tmem_base;
  volatile int* abort_flag = &tl->abort;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_x = make_l2_policy_evict_last();  // x_hat is re-read by every tile
      pdl_wait();  // x_hat comes from the prep kernel
      for (int it = 0; it < pre; ++it)
        tma_load_3d(b_smem + (size_t)it * b_stage, &tmap_x, &tl->full[it], 0, 0, (it % num_kc) * KC, pol_x);
      for (int it = pre; it < total; ++it) {
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
          pj_fail(p, tl, kStatusTimeoutEmpty);
          break;
        }
        mbar_arrive_expect_tx(&tl->full[s], stage_bytes);
        tma_load_3d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, tile_of(it) * 128, (it % num_kc) * KC,
                    pol_w);
        tma_load_3d(b_smem + (size_t)s * b_stage, &tmap_x, &tl->full[s], 0, 0, (it % num_kc) * KC, pol_x);
        const int pf = it + p.prefetch;
        if (p.prefetch > 0 && pf < total) tma_prefetch_l2_3d(&tmap_w, 0, tile_of(pf) * 128, (pf % num_kc) * KC);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issue
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, n_pad);
      int it = 0;
      bool alive = true;
      for (int local = 0; local < my_tiles && alive; ++local) {
        const uint32_t buf = (uint32_t)local & 1u;
        const uint32_t use = (uint32_t)local >> 1;
        if (!mbar_wait(&tl->tmem_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
          pj_fail(p, tl, kStatusTimeoutAccum);
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + buf * (uint32_t)n_pad;
        for (int kb = 0; kb < num_kc; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          if (!mbar_wait(&tl->full[s], ph, abort_flag)) {
            pj_fail(p, tl, kStatusTimeoutFull);
            alive = false;
            break;
          }
          tc_fence_after();
          for (int kc = 0; kc < KC; ++kc) {
            const uint64_t ad = umma_desc_sw128(smem_u32(a_smem + (size_t)s * a_stage + (size_t)kc * kPjSliceBytes));
            const uint64_t bd = umma_desc_sw128(smem_u32(b_smem + (size_t)s * b_stage + (size_t)kc * b_chunk));
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_bf16(dcol, ad + 2u * kk, bd + 2u * kk, idesc, (kb > 0 || kc > 0 || kk > 0) ? 1u : 0u);
          }
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
    const int j = gt & 15, g8 = gt >> 4;
    const int bar_grp = 1 + grp;        // 128-thread barrier of this group
    float* ybuf = ybufs + grp * kPjYBufFloats;
    const int T = p.num_tokens;
    pdl_wait();
    for (int local = 0; local < my_tiles; ++local) {
      const int tile = (int)blockIdx.x + local * (int)gridDim.x;
      const uint32_t buf = (uint32_t)local & 1u;
      const uint32_t use = (uint32_t)local >> 1;
      if (EPI == kEpiQkv && local == 0) {
        // token metadata once (the same batch for every tile)
        for (int t = ept; t < n_pad; t += 256) {
          tl->pos[t] = t < T ? p.tok_pos[t] : -1;
          tl->slot[t] = t < T ? p.tok_slot[t] : -1;
        }
      }
      const bool waited = mbar_wait_warp(&tl->tmem_full[buf], use & 1u, abort_flag);
      if (!waited && lane == 0) pj_fail(p, tl, kStatusTimeoutAccum);
      tc_fence_after();
      if (named_bar_any(3, 256, !waited || *abort_flag != 0)) break;
      const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16) + buf * (uint32_t)n_pad;
      const float bias_r = EPI == kEpiQkv && p.bias ? __bfloat162float(p.bias[tile * kHeadDim + r]) : 0.f;
      const bool rot = EPI == kEpiQkv ? tile < p.n_heads + p.n_kv_heads : (EPI == kEpiSwiglu ? g8 < 4 : false);
      for (int c0 = grp * 16; c0 < n_pad; c0 += 32) {
        if (c0 >= T) break;  // uniform within the group
        const int t = c0 + j;
        const int pos = EPI == kEpiQkv ? tl->pos[t] : 0;
        float4 cs[4], sn[4];
        if (EPI == kEpiQkv && rot) load_rope_n<16>(p, pos, 16 * g8, cs, sn);
        float acc[16];
        tmem_ld16(taddr + (uint32_t)c0, acc);
#pragma unroll
        for (int i = 0; i < 16; ++i) ybuf[i * kYStride + r] = acc[i] + bias_r;
        named_bar_sync(bar_grp, 128);
        if (t < T) {
          float y[16], yp[16];
          ld_smem_16f(ybuf + j * kYStride + 16 * g8, y);
          if (rot) ld_smem_16f(ybuf + j * kYStride + 16 * (g8 ^ 4), yp);
          if (EPI == kEpiQkv) {
            store_rows_n<16>(p, tile, t, 16 * g8, g8 < 4 ? -1.f : 1.f, pos, tl->slot[t], y, yp, cs, sn);
          } else if (EPI == kEpiSwiglu) {
            if (g8 < 4) {
              uint32_t w[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float a0 = y[2 * i] / (1.f + __expf(-y[2 * i])) * yp[2 * i];
                const float a1 = y[2 * i + 1] / (1.f + __expf(-y[2 * i + 1])) * yp[2 * i + 1];
                w[i] = pack_bf16x2(a0, a1);
              }
              uint4* dst = reinterpret_cast<uint4*>(p.act + (size_t)t * p.act_stride + (size_t)tile * 64 + 16 * g8);
              dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
              dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            }
          } else {
            unsigned long long best = 0ull;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int row = tile * 128 + 16 * g8 + i;
              if (row < p.vocab_valid) {
                const unsigned long long k = argmax_key(y[i], (uint32_t)(p.vocab_offset + row));
                best = k > best ? k : best;
              }
            }
            if (best != 0ull) atomicMax(&tl->key[t], best);
          }
        }
        named_bar_sync(bar_grp, 128);
      }
      tc_fence_before();
      named_bar_sync(3, 256);  // both groups are done with this tile's accumulator
      if (lane == 0) mbar_arrive(&tl->tmem_empty[buf]);
    }
    if (EPI == kEpiArgmax) {
      named_bar_sync(3, 256);
      for (int t = ept; t < T; t += 256)
        if (tl->key[t] != 0ull) atomicMax(p.keys + t, tl->key[t]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
  }
}

template <int EPI>
static cudaError_t launch_pj_t(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                               int num_tiles, cudaStream_t stream) {
  const size_t smem = proj_persistent_smem_bytes(p.stages, p.kc, p.n_pad);
  cudaError_t e =
      cudaFuncSetAttribute(proj_persistent_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int grid = device_sm_count();
  if (grid > num_tiles) grid = num_tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kPjThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, proj_persistent_kernel<EPI>, tmap_w, tmap_x, p, num_tiles);
}

cudaError_t launch_proj_persistent(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                                   int num_tiles, cudaStream_t stream) {
  if (p.epi == kEpiSwiglu) return launch_pj_t<kEpiSwiglu>(tmap_w, tmap_x, p, num_tiles, stream);
  if (p.epi == kEpiArgmax) return launch_pj_t<kEpiArgmax>(tmap_w, tmap_x, p, num_tiles, stream);
  return cudaErrorInvalidValue;  // the QKV projection runs on the split-K decode kernel
}

}  // namespace krt
