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
// or 64 output features per tile (64 up to 128 tokens: twice the tiles, so
// half the K splits fill the SMs and each split exchanges half the data),
// N = padded tokens, W and X tiles by TMA in {64, rows, KC} boxes, split-K
// across a thread-block cluster whose ranks send each other their partial
// chunks by bulk DSMEM copy.  The finishing thread (token j, features
// RG*g .. +RG-1, RG = rows / 8) of chunk `ch` then owns RG fp32 values of
// this rank's partial product.
//
// Allreduce part, fused into the epilogue (world > 1), in flagged 8-byte
// words (epoch and payload in one store each), so that no memory fence and
// no separate flag is on the path.  Two ranks exchange one-shot: each sends
// its partial chunk to both stages (alternating between two copies by epoch
// parity) and both reduce it in rank order (one NVLink hop, the same bytes
// as two-shot).  More ranks run two-shot:
//   1. reduce-scatter: the partial chunk (16 tokens x rows features, fp32
//      rounded to 24-bit floats with a 15-bit mantissa) is stored into the
//      owner rank's stage [src][tile / world][chunk] (owner = tile % world);
//   2. the owner's CTA for the same chunk polls the words of all `world`
//      ranks, sums the partials in rank order (so every rank ends with
//      bit-identical values), writes the bf16 result to its own Y and, as
//      flagged bf16x2 words, into every peer's result area;
//   3. every other rank's CTA for that chunk polls those words and copies
//      them into Y.
// The epoch of a (tile, chunk) is its use counter kept in the communicator's
// own buffer, identical on all ranks because all ranks run the same
// launches; a slot holds at most the previous use's words, which never
// match, so the protocol needs no reset and replays from a CUDA graph.  A
// slot is only rewritten by a launch that the reader's progress already
// allowed.  All polls are bounded (status bit 16).
#include <cstdint>
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "comm.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kGemmThreads = 192;

struct GemmSmemTail {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t accum;
  uint64_t recv;  // completes when the other ranks' partials of the owned chunks have arrived
  uint32_t tmem_base;
  int abort;
  uint32_t epoch[kMaxChunks];  // epoch of each owned chunk (fused allreduce)
  int pad;
};

// Pipeline buffers; after the main loop they hold the parked partial.
template <int TM>
__host__ __device__ inline size_t gemm_pipe_bytes(int stages, int n_pad, int kc) {
  size_t pipe = (size_t)stages * kc * (TileShape<TM>::kSliceBytes + (size_t)n_pad * 128);
  const size_t park = park_area_bytes(n_pad, TileShape<TM>::kParkStride);
  if (pipe < park) pipe = park;
  return (pipe + 127) & ~size_t(127);
}

template <int TM>
size_t gemm_ar_smem_bytes_t(int stages, int n_pad, int kc, int splits) {
  return 1024 + gemm_pipe_bytes<TM>(stages, n_pad, kc) + recv_area_bytes(n_pad, splits, TileShape<TM>::kChunkBytes) +
         sizeof(GemmSmemTail);
}

size_t gemm_ar_smem_bytes(int tile_m, int stages, int n_pad, int kc, int splits) {
  return tile_m == 64 ? gemm_ar_smem_bytes_t<64>(stages, n_pad, kc, splits)
                      : gemm_ar_smem_bytes_t<128>(stages, n_pad, kc, splits);
}

__device__ __forceinline__ void gemm_fail(const GemmArParams& p, GemmSmemTail* tl, int code) {
  atomicOr(p.status, code);
  tl->abort = 1;
}

// Flagged-word areas of the fused exchange (see CommLayout), tile height TM.
// Slot of one chunk; the word pair i of finishing thread `ept` is at
// slot + 2 * (i * 128 + ept).
template <int TM>
__device__ __forceinline__ uint64_t* ll_stage(const CommView& cv, int holder, int src, int tile, int ch,
                                              uint32_t epoch) {
  constexpr int v = TM == 64 ? 1 : 0;
  const int st = cv.world == 2 ? (int)(epoch & 1u) * (cv.L.stage_tiles[v] / 2) + tile : tile / cv.world;
  return reinterpret_cast<uint64_t*>(cv.base[holder] + cv.L.ll_stage_off[v]) +
         (((size_t)src * cv.L.stage_tiles[v] + st) * kMaxChunks + ch) * (TM / 32 * 128 * 2);
}
template <int TM>
__device__ __forceinline__ uint64_t* ll_result(const CommView& cv, int holder, int tile, int ch) {
  constexpr int v = TM == 64 ? 1 : 0;
  return reinterpret_cast<uint64_t*>(cv.base[holder] + cv.L.ll_result_off[v]) +
         ((size_t)tile * kMaxChunks + ch) * (TM / 32 * 128 * 2);
}

// Polls the stage words of up to four source ranks together (NP word pairs
// each, pairs 256 words apart): every load of a round is issued before any
// is checked, so a round costs one memory latency whatever the number of
// sources.  out[s][2i], out[s][2i + 1] receive source s's words.
template <int NP>
__device__ __forceinline__ bool poll_stage_sources(const uint64_t* const* src, int nsrc, uint32_t epoch, uint64_t t0,
                                                   uint64_t (*out)[2 * NP]) {
  while (true) {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (s < nsrc) {
#pragma unroll
        for (int i = 0; i < NP; ++i)
          asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];"
                       : "=l"(out[s][2 * i]), "=l"(out[s][2 * i + 1])
                       : "l"(src[s] + 256 * i)
                       : "memory");
      }
    bool all = true;
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (s < nsrc) {
#pragma unroll
        for (int i = 0; i < 2 * NP; ++i) all = all && (uint32_t)(out[s][i] >> 48) == epoch;
      }
    if (all) return true;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

// RG bf16 values as RG / 8 16-byte vectors.
template <int RG>
__device__ __forceinline__ void store_bf16_rows(__nv_bfloat16* dst, const uint32_t* w) {
#pragma unroll
  for (int h = 0; h < RG / 8; ++h)
    reinterpret_cast<uint4*>(dst)[h] = make_uint4(w[4 * h], w[4 * h + 1], w[4 * h + 2], w[4 * h + 3]);
}

// acc[i] += residual[i] for RG bf16 values (16-byte loads); no-op without a residual.
template <int RG>
__device__ __forceinline__ void add_residual_rows(float* acc, const __nv_bfloat16* res) {
  if (res == nullptr) return;
#pragma unroll
  for (int h = 0; h < RG / 8; ++h) {
    const uint4 v = reinterpret_cast<const uint4*>(res)[h];
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(b2[q]);
      acc[8 * h + 2 * q] += f.x;
      acc[8 * h + 2 * q + 1] += f.y;
    }
  }
}

template <int TM>
__global__ void __launch_bounds__(kGemmThreads, 1)
    rowparallel_gemm_ar_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                               const GemmArParams p) {
  using TS = TileShape<TM>;
  constexpr int RG = TS::kRowsPerThread;  // features per finishing thread
  constexpr int YS = TS::kParkStride;
  constexpr int NP = RG / 4;              // 16-byte word pairs per thread in a flagged slot
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  const int KC = p.kc;
  const int n_pad = p.n_pad;
  const uint32_t b_chunk = (uint32_t)n_pad * 128u;
  const uint32_t a_stage = (uint32_t)KC * TS::kSliceBytes;
  const uint32_t b_stage = (uint32_t)KC * b_chunk;
  const uint32_t stage_bytes = a_stage + b_stage;
  uint8_t* a_smem = smem;
  uint8_t* b_smem = smem + (size_t)S * a_stage;
  uint8_t* recv_smem = smem + gemm_pipe_bytes<TM>(S, n_pad, KC);
  GemmSmemTail* tl = reinterpret_cast<GemmSmemTail*>(recv_smem + recv_area_bytes(n_pad, p.splits, TS::kChunkBytes));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int num_kc = p.k_local / (kBK * KC);
  const int kc0 = (int)((long long)split * num_kc / p.splits);
  const int kc1 = (int)((long long)(split + 1) * num_kc / p.splits);
  const int nk = kc1 - kc0;
  const int row0 = tile * TM;

  const int pre = nk < S ? nk : S;  // stages loaded before the ring turns over
  uint64_t pol_w = 0;                // thread 0 = the TMA producer
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    mbar_init(&tl->accum, 1);
    mbar_init(&tl->recv, 1);
    tl->abort = 0;
    fence_mbar_init();
    // The weight tiles of the first stages depend on nothing: request them
    // before TMEM allocation and the block barrier.
    tma_prefetch_desc(&tmap_w);
    pol_w = make_l2_policy_evict_first();  // weights are streamed once
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&tl->full[i], stage_bytes);
      tma_load_3d(a_smem + (size_t)i * a_stage, &tmap_w, &tl->full[i], 0, row0, (kc0 + i) * KC, pol_w);
    }
    // the next p.prefetch weight stages are requested into L2 beyond the ring
    for (int i = pre; i < nk && i < pre + p.prefetch; ++i) tma_prefetch_l2_3d(&tmap_w, 0, row0, (kc0 + i) * KC);
    // the partials this CTA will receive: (splits - 1) per owned chunk
    mbar_arrive_expect_tx(&tl->recv, (uint32_t)(owned_chunks(n_pad / 16, p.splits, split) * (p.splits - 1)) *
                                         TS::kChunkBytes);
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
      const uint64_t pol_x = make_l2_policy_evict_last();
      pdl_wait();  // X may come from the previous kernel
      for (int i = 0; i < pre; ++i)
        tma_load_3d(b_smem + (size_t)i * b_stage, &tmap_x, &tl->full[i], 0, 0, (kc0 + i) * KC, pol_x);
      // ring slot and phase advance by increment (no divisions on the issue path)
      int s = pre % S;
      uint32_t ph = (uint32_t)(pre / S) & 1u;
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
          gemm_fail(p, tl, kStatusTimeoutEmpty);
          break;
        }
        mbar_arrive_expect_tx(&tl->full[s], stage_bytes);
        tma_load_3d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, row0, (kc0 + i) * KC, pol_w);
        tma_load_3d(b_smem + (size_t)s * b_stage, &tmap_x, &tl->full[s], 0, 0, (kc0 + i) * KC, pol_x);
        if (i + p.prefetch < nk) tma_prefetch_l2_3d(&tmap_w, 0, row0, (kc0 + i + p.prefetch) * KC);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(TM, n_pad);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nk; ++i) {
        if (!mbar_wait(&tl->full[s], ph, abort_flag)) {
          gemm_fail(p, tl, kStatusTimeoutFull);
          break;
        }
        tc_fence_after();
        for (int kc = 0; kc < KC; ++kc) {
          const uint64_t ad =
              umma_desc_sw128(smem_u32(a_smem + (size_t)s * a_stage + (size_t)kc * TS::kSliceBytes));
          const uint64_t bd = umma_desc_sw128(smem_u32(b_smem + (size_t)s * b_stage + (size_t)kc * b_chunk));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(tmem_base, ad + 2u * kk, bd + 2u * kk, idesc, (i > 0 || kc > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&tl->empty[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
      umma_commit(&tl->accum);
    }
  } else {
    const int q4 = warp & 3;
    // accumulator row held by this lane (M = 64: lanes 16-31 of each quarter hold none)
    const int r = TM == 128 ? q4 * 32 + lane : (lane < 16 ? q4 * 16 + lane : -1);
    const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16);
    const int ept = threadIdx.x - 64;
    const bool waited = mbar_wait_warp(&tl->accum, 0u, abort_flag);
    if (!waited && lane == 0) gemm_fail(p, tl, kStatusTimeoutAccum);
    tc_fence_after();
    cluster_wait();

    // Park the partial token-major in the idle pipeline buffers, four 16-token
    // chunks at a time; a chunk finished by another cluster rank is sent to it
    // by bulk copy as soon as its group is parked.
    const int crank = split;  // cluster (1, splits, 1): rank == blockIdx.y
    const int nranks = p.splits;
    float* part = reinterpret_cast<float*>(smem);
    const uint32_t part_u32 = smem_u32(part);
    const int n_chunks = n_pad / 16;
    for (int c0 = 0; c0 < n_chunks; c0 += 4) {
      const int nc = n_chunks - c0 < 4 ? n_chunks - c0 : 4;
      if (waited) {
        uint32_t v[4][16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          if (cc < nc) tmem_ld16_nowait(taddr + (uint32_t)((c0 + cc) * 16), v[cc]);
        tmem_wait_ld();
        if (r >= 0) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc)
            if (cc < nc) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) part[((c0 + cc) * 16 + jj) * YS + r] = __uint_as_float(v[cc][jj]);
            }
        }
      }
      bool remote = false;
      for (int cc = 0; cc < nc; ++cc) remote |= (c0 + cc) % nranks != crank;
      if (remote) {
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        // chunk cc of the group is sent by lane 0 of epilogue warp cc, so the
        // (remote) bulk-copy issues of a group run in parallel
        if ((ept & 31) == 0) {
          for (int cc = ept >> 5; cc < nc; cc += 4) {
            const int c = c0 + cc, cowner = c % nranks;
            if (cowner == crank) continue;
            const int slot = recv_slot(c / nranks, nranks, cowner, crank);
            bulk_copy_to_cluster(
                map_smem_to_rank(smem_u32(recv_smem) + (uint32_t)slot * TS::kChunkBytes, (uint32_t)cowner),
                part_u32 + (uint32_t)c * TS::kChunkBytes, TS::kChunkBytes,
                map_smem_to_rank(smem_u32(&tl->recv), (uint32_t)cowner));
          }
        }
      }
    }
    if ((ept & 31) == 0) bulk_commit_group();
    named_bar_sync(1, 128);  // the owned chunks are parked
    const bool got = mbar_wait_warp_incoming(&tl->recv, 0u);
    if (!got && lane == 0) gemm_fail(p, tl, kStatusTimeoutCluster);

    // Thread (token j, features RG*g .. +RG-1) of each chunk this CTA
    // finishes (chunks crank, crank + splits, ...); 8 consecutive lanes take
    // 8 tokens of one feature group (no bank conflicts).  Each cross-GPU
    // exchange phase covers all of the CTA's chunks at once, so a launch pays
    // two NVLink round trips.
    const int j = ept & 15, g = ept >> 4;
    const int T = p.num_tokens;
    const CommView& cv = p.comm;
    const int world = cv.world;
    const bool alive = *abort_flag == 0;
    const int owner = tile % world;
    const float* recv = reinterpret_cast<const float*>(recv_smem);
    pdl_wait();  // Y and the exchange buffers may still be in use by the previous kernel
    // Epoch of each (tile, chunk) this CTA finishes: its use count, cycling
    // through 1..65534 (so consecutive uses alternate in parity), the same on
    // every rank since every rank runs the same launches.  A slot of the
    // exchange only ever holds this launch's words or an earlier use's,
    // never a matching stale word.
    if (world > 1) {
      if (ept == 0) {
        uint32_t* ctr = reinterpret_cast<uint32_t*>(cv.base[cv.rank] + cv.L.epoch_off[TM == 64 ? 1 : 0]) +
                        (size_t)tile * kMaxChunks;
        for (int ch = crank, oc = 0; ch * 16 < T; ch += p.splits, ++oc) {
          uint32_t e = __ldcg(ctr + ch) + 1u;
          if (e > 65534u) e = 1u;
          ctr[ch] = e;
          tl->epoch[oc] = e;
        }
      }
      named_bar_sync(1, 128);
    }
    // ---- phase 1: this rank's partial of every chunk -> Y (one rank) or the owner's stage
    for (int ch = crank; ch * 16 < T; ch += p.splits) {
      const int t = ch * 16 + j;
      float y[RG];
#pragma unroll
      for (int i = 0; i < RG; ++i) y[i] = 0.f;
      // partials of the cluster ranks, summed in rank order; four ranks per
      // round with all their loads issued before the first add
      const int oc = ch / nranks;
      for (int q0 = 0; q0 < nranks; q0 += 4) {
        float4 a[4][RG / 4];
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int q = q0 + qq < nranks ? q0 + qq : q0;
          const float* src = q == crank ? part + t * YS + RG * g
                                        : recv + (size_t)recv_slot(oc, nranks, crank, q) * (TS::kChunkBytes / 4) +
                                              (size_t)j * YS + RG * g;
#pragma unroll
          for (int k4 = 0; k4 < RG / 4; ++k4) a[qq][k4] = reinterpret_cast<const float4*>(src)[k4];
        }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          if (q0 + qq >= nranks) break;
#pragma unroll
          for (int k4 = 0; k4 < RG / 4; ++k4) {
            y[4 * k4 + 0] += a[qq][k4].x;
            y[4 * k4 + 1] += a[qq][k4].y;
            y[4 * k4 + 2] += a[qq][k4].z;
            y[4 * k4 + 3] += a[qq][k4].w;
          }
        }
      }
      if (world == 1) {
        if (alive && t < T && p.y32) {
          float4* dst = reinterpret_cast<float4*>(p.y32 + (size_t)t * p.n_out + row0 + RG * g);
#pragma unroll
          for (int k4 = 0; k4 < RG / 4; ++k4) dst[k4] = make_float4(y[4 * k4], y[4 * k4 + 1], y[4 * k4 + 2], y[4 * k4 + 3]);
        } else if (alive && t < T) {
          add_residual_rows<RG>(y, p.residual ? p.residual + (size_t)t * p.y_stride + row0 + RG * g : nullptr);
          uint32_t w[RG / 2];
#pragma unroll
          for (int i = 0; i < RG / 2; ++i) w[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
          store_bf16_rows<RG>(p.y + (size_t)t * p.y_stride + row0 + RG * g, w);
        }
      } else {
        // flagged words of two 24-bit floats into the owner's stage (local
        // when this rank owns the tile); with two ranks into both stages
        const uint32_t epoch = tl->epoch[ch / nranks];
        uint64_t w[RG / 2];
#pragma unroll
        for (int i = 0; i < RG / 2; ++i) w[i] = f24_pair_word(y[2 * i], y[2 * i + 1], epoch);
        for (int d = 0; d < (world == 2 ? 2 : 1); ++d) {
          uint64_t* dst = ll_stage<TM>(cv, world == 2 ? d : owner, cv.rank, tile, ch, epoch) + 2 * ept;
#pragma unroll
          for (int i = 0; i < NP; ++i) st_ll2(dst + 256 * i, w[2 * i], w[2 * i + 1]);
        }
      }
    }
    if (world > 1) {
      const uint64_t t0 = globaltimer_ns();
      bool ok = true;
      if (world == 2 || cv.rank == owner) {
        // ---- phase 2 (owner; both ranks when there are two): every rank's
        // words of the chunk, reduced in rank order; the bf16 result goes to
        // Y and, with more than two ranks, as flagged words to every peer
        for (int ch = crank; ch * 16 < T; ch += p.splits) {
          const int t = ch * 16 + j;
          float acc[RG];
#pragma unroll
          for (int i = 0; i < RG; ++i) acc[i] = 0.f;
          const uint32_t epoch = tl->epoch[ch / nranks];
          // up to four ranks' words per polling round, added in rank order
          for (int q0 = 0; q0 < world && ok; q0 += 4) {
            const int nq = world - q0 < 4 ? world - q0 : 4;
            const uint64_t* src[4];
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4)
              src[s4] = ll_stage<TM>(cv, cv.rank, q0 + (s4 < nq ? s4 : 0), tile, ch, epoch) + 2 * ept;
            uint64_t u[4][RG / 2];
            ok = poll_stage_sources<NP>(src, nq, epoch, t0, u);
            if (!ok) break;
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4)
              if (s4 < nq) {
#pragma unroll
                for (int i = 0; i < RG / 2; ++i) {
                  const float2 v = f24_pair_unpack(u[s4][i]);
                  acc[2 * i] += v.x;
                  acc[2 * i + 1] += v.y;
                }
              }
          }
          if (!ok || t >= T) continue;
          add_residual_rows<RG>(acc, p.residual ? p.residual + (size_t)t * p.y_stride + row0 + RG * g : nullptr);
          uint32_t w[RG / 2];
#pragma unroll
          for (int i = 0; i < RG / 2; ++i) w[i] = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
          for (int q = 0; q < world && world > 2; ++q) {
            if (q == cv.rank) continue;
            uint64_t* rd = ll_result<TM>(cv, q, tile, ch) + 2 * ept;
#pragma unroll
            for (int i = 0; i < NP; ++i) st_ll2(rd + 256 * i, ll_word(w[2 * i], epoch), ll_word(w[2 * i + 1], epoch));
          }
          store_bf16_rows<RG>(p.y + (size_t)t * p.y_stride + row0 + RG * g, w);
        }
      } else {
        // ---- phase 3 (everyone else): the owner's flagged bf16 words -> Y
        for (int ch = crank; ch * 16 < T; ch += p.splits) {
          const int t = ch * 16 + j;
          if (t >= T) continue;
          uint32_t w[RG / 2];
#pragma unroll
          for (int i = 0; i < RG / 2; ++i) w[i] = 0u;
          if (ok)
            ok = poll_ll2_batch<NP>(ll_result<TM>(cv, cv.rank, tile, ch) + 2 * ept, 256, tl->epoch[ch / nranks], t0,
                                    w);
          if (!ok) continue;
          store_bf16_rows<RG>(p.y + (size_t)t * p.y_stride + row0 + RG * g, w);
        }
      }
      if (!ok) atomicOr(p.status, kStatusTimeoutPeer);
    }
    if ((ept & 31) == 0) bulk_wait_group_read0();  // the sent chunks have left this CTA's shared memory
  }

  if (warp < 2) cluster_wait();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
  }
}

template <int TM>
static cudaError_t launch_gemm_ar_t(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmArParams& p,
                                    int tiles, cudaStream_t stream) {
  const size_t smem = gemm_ar_smem_bytes_t<TM>(p.stages, p.n_pad, p.kc, p.splits);
  cudaError_t e =
      cudaFuncSetAttribute(rowparallel_gemm_ar_kernel<TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
  return cudaLaunchKernelEx(&cfg, rowparallel_gemm_ar_kernel<TM>, tmap_w, tmap_x, p);
}

cudaError_t launch_rowparallel_gemm_ar(int tile_m, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                                       const GemmArParams& p, int tiles, cudaStream_t stream) {
  return tile_m == 64 ? launch_gemm_ar_t<64>(tmap_w, tmap_x, p, tiles, stream)
                      : launch_gemm_ar_t<128>(tmap_w, tmap_x, p, tiles, stream);
}

template <int TM>
static int gemm_ar_max_active_clusters_t(int splits, int n_pad, int stages, int kc) {
  const size_t smem = gemm_ar_smem_bytes_t<TM>(stages, n_pad, kc, splits);
  if (cudaFuncSetAttribute(rowparallel_gemm_ar_kernel<TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
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
  if (cudaOccupancyMaxActiveClusters(&n, rowparallel_gemm_ar_kernel<TM>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int gemm_ar_max_active_clusters(int tile_m, int splits, int n_pad, int stages, int kc) {
  return tile_m == 64 ? gemm_ar_max_active_clusters_t<64>(splits, n_pad, stages, kc)
                      : gemm_ar_max_active_clusters_t<128>(splits, n_pad, stages, kc);
}

}  // namespace krt
