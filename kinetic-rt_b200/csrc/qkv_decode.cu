// Decode variant of the fused RMSNorm + QKV projection + RoPE + paged K/V
// scatter (bf16, tcgen05 / TMEM, TMA).
//
// Shape: up to 256 tokens (decode batch), W [(Hq+2Hkv)*128, D].  The weight
// stream (50 MB for Llama-3-8B shapes) dominates, so the kernel is HBM-bound
// and is laid out to keep every SM streaming weights:
//
//   * swap-AB: the UMMA M dimension is 128 weight rows (one head of Q, K or
//     V), N is the padded token count, so the accumulator of a head is one
//     128-lane x n_pad-column TMEM tile;
//   * split-K over gridDim.y so that (heads x splits) ~ #SMs, the splits of a
//     head forming one thread-block cluster: after the main loop every CTA
//     parks its fp32 partial tile in its own shared memory, and each CTA
//     finalises a share of the 16-token chunks by summing the partials of
//     all CTAs of the cluster over DSMEM in rank order (deterministic, no
//     global workspace traffic, the finishing work spread over the cluster);
//   * the normalised activations x_hat and the per-token pool slots come from
//     qkv_prep_kernel, launched just before with programmatic dependent
//     launch: the W tiles of the first pipeline stages are requested before
//     griddepcontrol.wait, so the weight stream starts while the prep kernel
//     still runs;
//   * the finishing thread (token, 16-row group) reads its rows and their
//     rotate-half partner rows (r ^ 64) from the parked partials, applies
//     bias and RoPE in fp32 and writes Q densely and K/V into the paged pool
//     with 16-byte stores (store_rows16).
//
// Warp roles (192 threads): warp 0 = TMA producer (W and x_hat tiles),
// warp 1 = TMEM owner + single-thread UMMA issuer, warps 2-5 = epilogue
// (warp w reads TMEM lanes 32*(w%4) .. +31).
#include <cstdint>
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kDecodeThreads = 192;
constexpr uint32_t kTileABytes = 128 * 128;  // 128 rows x 64 bf16

struct DecodeSmemTail {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t accum;
  uint32_t tmem_base;
  int abort;
  int pad[2];
  int pos[256];
  long long slot[256];
};

__device__ __forceinline__ void decode_fail(const PagedParams& p, DecodeSmemTail* tl, int code) {
  atomicOr(p.status, code);
  tl->abort = 1;
}

__global__ void __launch_bounds__(kDecodeThreads, 1)
    qkv_rope_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                           const PagedParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  const int KC = p.kc;
  const int n_pad = p.n_pad;
  const uint32_t b_chunk = (uint32_t)n_pad * 128u;
  const uint32_t a_stage = (uint32_t)KC * kTileABytes;
  const uint32_t b_stage = (uint32_t)KC * b_chunk;
  const uint32_t stage_bytes = a_stage + b_stage;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + (size_t)S * a_stage;
  size_t pipe_bytes = (size_t)S * stage_bytes;
  if (pipe_bytes < (size_t)n_pad * kYStride * sizeof(float)) pipe_bytes = (size_t)n_pad * kYStride * sizeof(float);
  DecodeSmemTail* tl = reinterpret_cast<DecodeSmemTail*>(smem + pipe_bytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int num_kc = p.d_model / (kBK * KC);
  const int kc0 = (int)((long long)split * num_kc / p.splits);
  const int kc1 = (int)((long long)(split + 1) * num_kc / p.splits);
  const int nk = kc1 - kc0;  // pipeline stages (KC chunks each) of this CTA
  const int row0 = tile * kHeadDim;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    mbar_init(&tl->accum, 1);
    tl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(&tl->tmem_base, (uint32_t)p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tl->tmem_base;
  volatile int* abort_flag = &tl->abort;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = make_l2_policy_evict_first();  // weights are streamed once
      const uint64_t pol_x = make_l2_policy_evict_last();   // x_hat is re-read by every head
      // W tiles of the first stages do not depend on the prep kernel.
      const int pre = nk < S ? nk : S;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&tl->full[i], stage_bytes);
        tma_load_3d(a_smem + (size_t)i * a_stage, &tmap_w, &tl->full[i], 0, row0, (kc0 + i) * KC, pol_w);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_3d(b_smem + (size_t)i * b_stage, &tmap_x, &tl->full[i], 0, 0, (kc0 + i) * KC, pol_x);
      for (int i = pre; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
          decode_fail(p, tl, kStatusTimeoutEmpty);
          break;
        }
        mbar_arrive_expect_tx(&tl->full[s], stage_bytes);
        tma_load_3d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, row0, (kc0 + i) * KC, pol_w);
        tma_load_3d(b_smem + (size_t)s * b_stage, &tmap_x, &tl->full[s], 0, 0, (kc0 + i) * KC, pol_x);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ UMMA issue
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, n_pad);
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&tl->full[s], ph, abort_flag)) {
          decode_fail(p, tl, kStatusTimeoutFull);
          break;
        }
        tc_fence_after();
        for (int kc = 0; kc < KC; ++kc) {
          const uint64_t ad = umma_desc_sw128(smem_u32(a_smem + (size_t)s * a_stage + (size_t)kc * kTileABytes));
          const uint64_t bd = umma_desc_sw128(smem_u32(b_smem + (size_t)s * b_stage + (size_t)kc * b_chunk));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(tmem_base, ad + 2u * kk, bd + 2u * kk, idesc, (i > 0 || kc > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&tl->empty[s]);
      }
      umma_commit(&tl->accum);
    }
  } else {
    // ------------------------------------------------ epilogue, phase A (warps 2-5)
    // Park this CTA's partial accumulator, token-major, in its own smem.
    const int ept = threadIdx.x - 64;  // 0..127
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // accumulator row = TMEM lane
    const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16);
    const int T = p.num_tokens;
    pdl_wait();
    for (int t = ept; t < T; t += 128) {
      tl->pos[t] = p.tok_pos[t];
      tl->slot[t] = p.tok_slot[t];
    }
    const bool waited = mbar_wait_warp(&tl->accum, 0u, abort_flag);
    if (!waited && lane == 0) decode_fail(p, tl, kStatusTimeoutAccum);
    tc_fence_after();
    float* part = reinterpret_cast<float*>(smem);  // pipeline buffers are idle now
    if (waited) {
      for (int c0 = 0; c0 < n_pad; c0 += 16) {
        float v[16];
        tmem_ld16(taddr + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) part[(c0 + j) * kYStride + r] = v[j];
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // every partial of the cluster is parked

  if (warp >= 2) {
    // ------------------------------------------------ epilogue, phase B
    // CTA `rank` finalises chunks rank, rank + splits, ...; thread (j, g8)
    // owns token c*16 + j and rows 16*g8 .. +15.
    const int ept = threadIdx.x - 64;
    const int j = ept >> 3, g8 = ept & 7;
    const uint32_t rank = cluster_ctarank();
    const int nranks = p.splits;
    const uint32_t part_base = smem_u32(smem);
    const bool rot = tile < p.n_heads + p.n_kv_heads;
    const int gp = g8 ^ 4;
    float bias_y[16], bias_p[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      bias_y[i] = p.bias ? __bfloat162float(p.bias[row0 + 16 * g8 + i]) : 0.f;
      bias_p[i] = p.bias ? __bfloat162float(p.bias[row0 + 16 * gp + i]) : 0.f;
    }
    if (*abort_flag == 0) {
      for (int c = (int)rank; c * 16 < p.num_tokens; c += nranks) {
        const int t = c * 16 + j;
        if (t >= p.num_tokens) continue;
        const int pos = tl->pos[t];
        float4 cs[4], sn[4];
        if (rot) load_rope16(p, pos, g8, cs, sn);
        float y[16], yp[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          y[i] = bias_y[i];
          yp[i] = bias_p[i];
        }
        for (int q = 0; q < nranks; ++q) {
          const uint32_t base = map_smem_to_rank(part_base, (uint32_t)q) + (uint32_t)(t * kYStride) * 4u;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const float4 a = ld_dsmem_f4(base + (uint32_t)(16 * g8 + 4 * k4) * 4u);
            y[4 * k4 + 0] += a.x;
            y[4 * k4 + 1] += a.y;
            y[4 * k4 + 2] += a.z;
            y[4 * k4 + 3] += a.w;
          }
          if (rot) {
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              const float4 a = ld_dsmem_f4(base + (uint32_t)(16 * gp + 4 * k4) * 4u);
              yp[4 * k4 + 0] += a.x;
              yp[4 * k4 + 1] += a.y;
              yp[4 * k4 + 2] += a.z;
              yp[4 * k4 + 3] += a.w;
            }
          }
        }
        store_rows16(p, tile, t, g8, pos, tl->slot[t], y, yp, cs, sn);
      }
    }
  }

  cluster_sync();  // no CTA leaves while others still read its partial
  if (warp == 1) tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
}

size_t decode_smem_bytes(int stages, int n_pad, int kc) {
  size_t pipe = (size_t)stages * kc * (kTileABytes + (size_t)n_pad * 128);
  const size_t park = (size_t)n_pad * kYStride * sizeof(float);
  if (pipe < park) pipe = park;
  return 1024 + pipe + sizeof(DecodeSmemTail);
}

cudaError_t launch_qkv_rope_decode(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                                   int tiles, cudaStream_t stream) {
  const size_t smem = decode_smem_bytes(p.stages, p.n_pad, p.kc);
  cudaError_t e = cudaFuncSetAttribute(qkv_rope_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, p.splits, 1);
  cfg.blockDim = dim3(kDecodeThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = (unsigned)p.splits;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, qkv_rope_decode_kernel, tmap_w, tmap_x, p);
}

// Largest cluster count that can be resident at once for a given split.
int decode_max_active_clusters(int splits, int n_pad, int stages, int kc) {
  const size_t smem = decode_smem_bytes(stages, n_pad, kc);
  if (cudaFuncSetAttribute(qkv_rope_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, splits, 1);
  cfg.blockDim = dim3(kDecodeThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, qkv_rope_decode_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace krt
