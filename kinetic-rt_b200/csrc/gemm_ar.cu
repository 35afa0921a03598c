// Row-parallel GEMM fused with the allreduce (o_proj / down_proj under tensor
// parallelism), bf16 in and out, fp32 accumulation and reduction.
//
// Rank r holds the column shard W[:, K_r] of the weight and the matching
// activations X[:, K_r] (scripts/export_hf.py:62-65); the layer output is
// Y = sum_r X[:, K_r] W[:, K_r]^T on every rank (Communicator::all_reduce_async,
// src/Communicator.cpp:21-27, with the allreduce semantics of
// tests/mock_rccl.h:51-62).  One launch handles up to 256 tokens.
//
// GEMM part (same structure as the decode QKV kernel): swap-AB, UMMA M = 128
// output features per tile, N = padded tokens, W and X tiles by TMA in
// {64, rows, KC} boxes, split-K across a thread-block cluster with the
// partial tiles reduced over DSMEM.  The finishing thread (token j, features
// 16*g8 .. +15) of chunk `ch` then owns 16 fp32 values of this rank's partial
// product.
//
// Allreduce part, fused into the epilogue (two-shot over NVLink, world > 1;
// every phase covers all the chunks a CTA finishes, one fence per CTA):
//   1. reduce-scatter: the partial chunk (16 tokens x 128 features, fp32) is
//      stored into the owner rank's staging slot [src][tile][chunk]
//      (owner = tile % world) and a flag is released there;
//   2. the owner's CTA for the same chunk waits for all `world` flags, sums
//      the partials in rank order (so every rank ends with bit-identical
//      values), writes bf16 results into every rank's result buffer and its
//      own Y, then releases a flag on each peer;
//   3. every other rank's CTA for that chunk waits for that flag and copies
//      the chunk from its result buffer into Y.
// Flags are reset by their consumer, so the protocol needs no epoch and can
// be replayed from a CUDA graph.  All waits are bounded (status bit 16).
#include <cstdint>
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "comm.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kGemmThreads = 192;
constexpr uint32_t kGemmTileABytes = 128 * 128;

struct GemmSmemTail {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t accum;
  uint64_t recv;  // completes when the other ranks' partials of the owned chunks have arrived
  uint32_t tmem_base;
  int abort;
  int ok;
  int pad;
};

// Pipeline buffers; after the main loop they hold the parked partial.
__host__ __device__ inline size_t gemm_pipe_bytes(int stages, int n_pad, int kc) {
  size_t pipe = (size_t)stages * kc * (kGemmTileABytes + (size_t)n_pad * 128);
  if (pipe < park_area_bytes(n_pad)) pipe = park_area_bytes(n_pad);
  return (pipe + 127) & ~size_t(127);
}

size_t gemm_ar_smem_bytes(int stages, int n_pad, int kc, int splits) {
  return 1024 + gemm_pipe_bytes(stages, n_pad, kc) + recv_area_bytes(n_pad, splits) + sizeof(GemmSmemTail);
}

__device__ __forceinline__ void gemm_fail(const GemmArParams& p, GemmSmemTail* tl, int code) {
  atomicOr(p.status, code);
  tl->abort = 1;
}

__device__ __forceinline__ void st_f4_x4(float* dst, const float* v) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

__device__ __forceinline__ void pack16(const float* v, uint4& a, uint4& b) {
  a = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  b = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                 pack_bf16x2(v[14], v[15]));
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    rowparallel_gemm_ar_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                               const GemmArParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  const int KC = p.kc;
  const int n_pad = p.n_pad;
  const uint32_t b_chunk = (uint32_t)n_pad * 128u;
  const uint32_t a_stage = (uint32_t)KC * kGemmTileABytes;
  const uint32_t b_stage = (uint32_t)KC * b_chunk;
  const uint32_t stage_bytes = a_stage + b_stage;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + (size_t)S * a_stage;
  uint8_t* recv_smem = smem + gemm_pipe_bytes(S, n_pad, KC);
  GemmSmemTail* tl = reinterpret_cast<GemmSmemTail*>(recv_smem + recv_area_bytes(n_pad, p.splits));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int num_kc = p.k_local / (kBK * KC);
  const int kc0 = (int)((long long)split * num_kc / p.splits);
  const int kc1 = (int)((long long)(split + 1) * num_kc / p.splits);
  const int nk = kc1 - kc0;
  const int row0 = tile * 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    mbar_init(&tl->accum, 1);
    mbar_init(&tl->recv, 1);
    tl->abort = 0;
    fence_mbar_init();
    // the partials this CTA will receive: (splits - 1) per owned chunk
    mbar_arrive_expect_tx(&tl->recv, (uint32_t)(owned_chunks(n_pad / 16, p.splits, split) * (p.splits - 1)) *
                                         kChunkBytes);
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
  cluster_arrive_relaxed();  // the receive barriers are initialised; waited on before the first push
  // The next kernel may launch onto free SMs now; it waits for this grid
  // (griddepcontrol.wait) before touching anything this kernel writes.
  if (threadIdx.x == 0) pdl_launch_dependents();
  const uint32_t tmem_base = tl->tmem_base;
  volatile int* abort_flag = &tl->abort;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = make_l2_policy_evict_first();
      const uint64_t pol_x = make_l2_policy_evict_last();
      const int pre = nk < S ? nk : S;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&tl->full[i], stage_bytes);
        tma_load_3d(a_smem + (size_t)i * a_stage, &tmap_w, &tl->full[i], 0, row0, (kc0 + i) * KC, pol_w);
      }
      pdl_wait();  // X may come from the previous kernel
      for (int i = 0; i < pre; ++i)
        tma_load_3d(b_smem + (size_t)i * b_stage, &tmap_x, &tl->full[i], 0, 0, (kc0 + i) * KC, pol_x);
      for (int i = pre; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
          gemm_fail(p, tl, kStatusTimeoutEmpty);
          break;
        }
        mbar_arrive_expect_tx(&tl->full[s], stage_bytes);
        tma_load_3d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, row0, (kc0 + i) * KC, pol_w);
        tma_load_3d(b_smem + (size_t)s * b_stage, &tmap_x, &tl->full[s], 0, 0, (kc0 + i) * KC, pol_x);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, n_pad);
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)(i / S) & 1u;
        if (!mbar_wait(&tl->full[s], ph, abort_flag)) {
          gemm_fail(p, tl, kStatusTimeoutFull);
          break;
        }
        tc_fence_after();
        for (int kc = 0; kc < KC; ++kc) {
          const uint64_t ad = umma_desc_sw128(smem_u32(a_smem + (size_t)s * a_stage + (size_t)kc * kGemmTileABytes));
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
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16);
    const int ept = threadIdx.x - 64;
    const bool waited = mbar_wait_warp(&tl->accum, 0u, abort_flag);
    if (!waited && lane == 0) gemm_fail(p, tl, kStatusTimeoutAccum);
    tc_fence_after();
    cluster_wait();

    // Park the partial token-major in the idle pipeline buffers, one 16-token
    // chunk at a time; a chunk finished by another cluster rank is sent to it
    // by bulk copy as soon as it is parked.
    const int crank = split;  // cluster (1, splits, 1): rank == blockIdx.y
    const int nranks = p.splits;
    float* part = reinterpret_cast<float*>(smem);
    const uint32_t part_u32 = smem_u32(part);
    for (int c = 0; c * 16 < n_pad; ++c) {
      if (waited) {
        float v[16];
        tmem_ld16(taddr + (uint32_t)(c * 16), v);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) part[(c * 16 + jj) * kYStride + r] = v[jj];
      }
      const int cowner = c % nranks;
      if (cowner != crank) {
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (ept == 0) {
          const int slot = recv_slot(c / nranks, nranks, cowner, crank);
          bulk_copy_to_cluster(map_smem_to_rank(smem_u32(recv_smem) + (uint32_t)slot * kChunkBytes, (uint32_t)cowner),
                               part_u32 + (uint32_t)c * kChunkBytes, kChunkBytes,
                               map_smem_to_rank(smem_u32(&tl->recv), (uint32_t)cowner));
        }
      }
    }
    if (ept == 0) bulk_commit_group();
    named_bar_sync(1, 128);  // the owned chunks are parked
    const bool got = mbar_wait_warp_incoming(&tl->recv, 0u);
    if (!got && lane == 0) gemm_fail(p, tl, kStatusTimeoutCluster);

    // Thread (token j, features 16*g8 .. +15) of each chunk this CTA finishes
    // (chunks crank, crank + splits, ...).  Each cross-GPU exchange phase
    // covers all of the CTA's chunks at once, so a launch pays two NVLink
    // round trips.
    const int j = ept >> 3, g8 = ept & 7;
    const int T = p.num_tokens;
    const CommView& cv = p.comm;
    const int world = cv.world;
    const bool alive = *abort_flag == 0;
    const size_t slot_elems = (size_t)16 * 128;
    const int owner = tile % world;
    const float* recv = reinterpret_cast<const float*>(recv_smem);
    pdl_wait();  // Y and the exchange buffers may still be in use by the previous kernel
    // ---- phase 1: this rank's partial of every chunk -> Y (one rank) or the owner's staging slot
    for (int ch = (int)crank; ch * 16 < T; ch += p.splits) {
      const int t = ch * 16 + j;
      float y[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = 0.f;
      // partials of the cluster ranks, summed in rank order
      const int oc = ch / nranks;
      for (int q = 0; q < nranks; ++q) {
        const float* src = q == crank ? part + t * kYStride + 16 * g8
                                      : recv + (size_t)recv_slot(oc, nranks, crank, q) * (kChunkBytes / 4) +
                                            (size_t)j * kYStride + 16 * g8;
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const float4 a = reinterpret_cast<const float4*>(src)[k4];
          y[4 * k4 + 0] += a.x;
          y[4 * k4 + 1] += a.y;
          y[4 * k4 + 2] += a.z;
          y[4 * k4 + 3] += a.w;
        }
      }
      if (world == 1) {
        if (alive && t < T) {
          uint4 a, b;
          pack16(y, a, b);
          __nv_bfloat16* ydst = p.y + (size_t)t * p.y_stride + row0 + 16 * g8;
          reinterpret_cast<uint4*>(ydst)[0] = a;
          reinterpret_cast<uint4*>(ydst)[1] = b;
        }
      } else {
        const size_t chunk_off = (((size_t)cv.rank * cv.L.tiles + tile) * kMaxChunks + ch) * slot_elems;
        st_f4_x4(reinterpret_cast<float*>(cv.base[owner] + cv.L.staging_off) + chunk_off + j * 128 + 16 * g8, y);
      }
    }
    if (world > 1) {
      named_bar_sync(1, 128);
      if (ept == 0) {
        fence_acq_rel_sys();
        uint32_t* pf = reinterpret_cast<uint32_t*>(cv.base[owner] + cv.L.part_flag_off);
        for (int ch = (int)crank; ch * 16 < T; ch += p.splits)
          st_release_sys(pf + ((size_t)tile * kMaxChunks + ch) * kMaxWorld + cv.rank, 1u);
      }
      if (cv.rank == owner) {
        // ---- phase 2 (owner): reduce every chunk in rank order, broadcast bf16 results
        if (ept == 0) {
          uint32_t* pf = reinterpret_cast<uint32_t*>(cv.base[cv.rank] + cv.L.part_flag_off);
          bool ok = true;
          for (int ch = (int)crank; ch * 16 < T && ok; ch += p.splits)
            for (int q = 0; q < world && ok; ++q) ok = wait_flag_sys(pf + ((size_t)tile * kMaxChunks + ch) * kMaxWorld + q, 1u);
          if (ok) {
            for (int ch = (int)crank; ch * 16 < T; ch += p.splits)
              for (int q = 0; q < world; ++q) pf[((size_t)tile * kMaxChunks + ch) * kMaxWorld + q] = 0u;
          } else {
            atomicOr(p.status, kStatusTimeoutPeer);
          }
          tl->ok = ok ? 1 : 0;
        }
        named_bar_sync(1, 128);
        const bool ok = tl->ok != 0;
        if (ok) {
          for (int ch = (int)crank; ch * 16 < T; ch += p.splits) {
            const int t = ch * 16 + j;
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = 0.f;
            for (int q = 0; q < world; ++q) {
              const float4* src = reinterpret_cast<const float4*>(
                  reinterpret_cast<const float*>(cv.base[cv.rank] + cv.L.staging_off) +
                  (((size_t)q * cv.L.tiles + tile) * kMaxChunks + ch) * slot_elems + j * 128 + 16 * g8);
#pragma unroll
              for (int k4 = 0; k4 < 4; ++k4) {
                const float4 a = __ldcg(src + k4);
                acc[4 * k4 + 0] += a.x;
                acc[4 * k4 + 1] += a.y;
                acc[4 * k4 + 2] += a.z;
                acc[4 * k4 + 3] += a.w;
              }
            }
            if (t < T) {
              uint4 a, b;
              pack16(acc, a, b);
              for (int q = 0; q < world; ++q) {
                if (q == cv.rank) continue;
                uint4* rd = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(cv.base[q] + cv.L.result_off) +
                                                     (size_t)t * cv.L.max_n + row0 + 16 * g8);
                rd[0] = a;
                rd[1] = b;
              }
              __nv_bfloat16* ydst = p.y + (size_t)t * p.y_stride + row0 + 16 * g8;
              reinterpret_cast<uint4*>(ydst)[0] = a;
              reinterpret_cast<uint4*>(ydst)[1] = b;
            }
          }
        }
        named_bar_sync(1, 128);
        if (ept == 0 && ok) {
          fence_acq_rel_sys();
          for (int q = 0; q < world; ++q) {
            if (q == cv.rank) continue;
            uint32_t* ff = reinterpret_cast<uint32_t*>(cv.base[q] + cv.L.final_flag_off);
            for (int ch = (int)crank; ch * 16 < T; ch += p.splits)
              st_release_sys(ff + (size_t)tile * kMaxChunks + ch, 1u);
          }
        }
      } else {
        // ---- phase 3 (everyone else): wait for the owner's results, copy them into Y
        if (ept == 0) {
          uint32_t* ff = reinterpret_cast<uint32_t*>(cv.base[cv.rank] + cv.L.final_flag_off);
          bool ok = true;
          for (int ch = (int)crank; ch * 16 < T && ok; ch += p.splits) ok = wait_flag_sys(ff + (size_t)tile * kMaxChunks + ch, 1u);
          if (ok) {
            for (int ch = (int)crank; ch * 16 < T; ch += p.splits) ff[(size_t)tile * kMaxChunks + ch] = 0u;
          } else {
            atomicOr(p.status, kStatusTimeoutPeer);
          }
          tl->ok = ok ? 1 : 0;
        }
        named_bar_sync(1, 128);
        if (tl->ok) {
          for (int ch = (int)crank; ch * 16 < T; ch += p.splits) {
            const int t = ch * 16 + j;
            if (t >= T) continue;
            const uint4* rs = reinterpret_cast<const uint4*>(
                reinterpret_cast<const __nv_bfloat16*>(cv.base[cv.rank] + cv.L.result_off) + (size_t)t * cv.L.max_n +
                row0 + 16 * g8);
            __nv_bfloat16* ydst = p.y + (size_t)t * p.y_stride + row0 + 16 * g8;
            reinterpret_cast<uint4*>(ydst)[0] = __ldcg(rs);
            reinterpret_cast<uint4*>(ydst)[1] = __ldcg(rs + 1);
          }
        }
      }
    }
    if (ept == 0) bulk_wait_group_read0();  // the sent chunks have left this CTA's shared memory
  }

  if (warp < 2) cluster_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
  }
}

cudaError_t launch_rowparallel_gemm_ar(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmArParams& p,
                                       int tiles, cudaStream_t stream) {
  const size_t smem = gemm_ar_smem_bytes(p.stages, p.n_pad, p.kc, p.splits);
  cudaError_t e =
      cudaFuncSetAttribute(rowparallel_gemm_ar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, p.splits, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
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
  return cudaLaunchKernelEx(&cfg, rowparallel_gemm_ar_kernel, tmap_w, tmap_x, p);
}

int gemm_ar_max_active_clusters(int splits, int n_pad, int stages, int kc) {
  const size_t smem = gemm_ar_smem_bytes(stages, n_pad, kc, splits);
  if (cudaFuncSetAttribute(rowparallel_gemm_ar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(splits, splits, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, rowparallel_gemm_ar_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace krt
