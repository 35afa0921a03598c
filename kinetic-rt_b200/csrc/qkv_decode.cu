// Decode variant of the fused RMSNorm + QKV projection + RoPE + paged K/V
// scatter (bf16, tcgen05 / TMEM, TMA).
//
// Shape: up to 256 tokens (decode batch), W [(Hq+2Hkv)*128, D].  The weight
// stream (50 MB for Llama-3-8B shapes) dominates, so the kernel is HBM-bound
// and is laid out to keep every SM streaming weights:
//
//   * swap-AB: the UMMA M dimension is a tile of weight rows, N is the padded
//     token count.  A tile is a whole head (M = 128) or, for up to 128
//     tokens, half a head (M = 64: rows 32*h .. +31 and 64 + 32*h .. +31 of
//     the head, h = 0, 1, fetched by one 5-D TMA box), which keeps each
//     row's rotate-half partner (r ^ 64) in the same tile and doubles the
//     tile count, so fewer K splits (less exchange) fill the SMs;
//   * split-K over gridDim.y so that (tiles x splits) ~ #SMs, the splits of a
//     tile forming one thread-block cluster: after the main loop every CTA
//     parks its fp32 partial token-major in its idle pipeline buffers and
//     bulk-copies the 16-token chunks that other ranks finish into their
//     receive areas (cp.async.bulk shared::cta -> shared::cluster, completing
//     the receiver's mbarrier); chunk c is finished by rank c % splits from
//     its own shared memory, partials summed in rank order (deterministic);
//   * the normalised activations x_hat and the per-token pool slots come from
//     qkv_prep_kernel, launched just before with programmatic dependent
//     launch: the W tiles of the first pipeline stages are requested before
//     griddepcontrol.wait, so the weight stream starts while the prep kernel
//     still runs;
//   * the finishing thread (token, row group) applies bias and RoPE in fp32
//     and writes Q densely and K/V into the paged pool with 16-byte stores
//     (store_rows_n); its first token's RoPE values and its bias are fetched
//     while the main loop runs.
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

struct DecodeSmemTail {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t accum;
  uint64_t recv;  // completes when the other ranks' partials of the owned chunks have arrived
  uint32_t tmem_base;
  int abort;
  union {
    struct {
      int pos[256];
      long long slot[256];
    };                            // kEpiQkv: per-token position and pool slot
    unsigned long long key[256];  // kEpiArgmax: the CTA's best (logit, index) per token
  };
};

// Pipeline buffers; after the main loop they hold the parked partial.
template <int TM>
__host__ __device__ inline size_t decode_pipe_bytes(int stages, int n_pad, int kc) {
  size_t pipe = (size_t)stages * kc * (TileShape<TM>::kSliceBytes + (size_t)n_pad * 128);
  const size_t park = park_area_bytes(n_pad, TileShape<TM>::kParkStride);
  if (pipe < park) pipe = park;
  return (pipe + 127) & ~size_t(127);
}

template <int N>
__device__ __forceinline__ void add_f4(float* y, const float4* a) {
#pragma unroll
  for (int k4 = 0; k4 < N / 4; ++k4) {
    y[4 * k4 + 0] += a[k4].x;
    y[4 * k4 + 1] += a[k4].y;
    y[4 * k4 + 2] += a[k4].z;
    y[4 * k4 + 3] += a[k4].w;
  }
}

__device__ __forceinline__ void decode_fail(const PagedParams& p, DecodeSmemTail* tl, int code) {
  atomicOr(p.status, code);
  tl->abort = 1;
}

// Head row of local tile row i.  M = 128: i.  M = 64, half h: rows 0-31 are
// head rows 32h .. 32h+31, rows 32-63 are 64 + 32h .. 64 + 32h + 31.
template <int TM>
__device__ __forceinline__ int head_row(int i, int half) {
  if (TM == 128) return i;
  return i < 32 ? 32 * half + i : 64 + 32 * half + (i - 32);
}

template <int TM, int EPI>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    qkv_rope_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                           const PagedParams p) {
  using TS = TileShape<TM>;
  constexpr int RG = TS::kRowsPerThread;  // rows per finishing thread
  constexpr int YS = TS::kParkStride;
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
  uint8_t* recv_smem = smem + decode_pipe_bytes<TM>(S, n_pad, KC);
  DecodeSmemTail* tl =
      reinterpret_cast<DecodeSmemTail*>(recv_smem + recv_area_bytes(n_pad, p.splits, TS::kChunkBytes));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int head = TM == 128 ? tile : tile >> 1;
  const int half = TM == 128 ? 0 : tile & 1;
  const int num_kc = p.d_model / (kBK * KC);
  const int kc0 = (int)((long long)split * num_kc / p.splits);
  const int kc1 = (int)((long long)(split + 1) * num_kc / p.splits);
  const int nk = kc1 - kc0;  // pipeline stages (KC chunks each) of this CTA

  const int pre = nk < S ? nk : S;  // stages loaded before the ring turns over
  uint64_t pol_w = 0;                // thread 0 = the TMA producer
  auto load_w = [&](int s, int i) {
    if (TM == 128)
      tma_load_3d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, tile * 128, (kc0 + i) * KC, pol_w);
    else
      tma_load_5d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, 0, 0, 4 * head + half, (kc0 + i) * KC,
                  pol_w);
  };
  auto prefetch_w = [&](int i) {
    if (TM == 128)
      tma_prefetch_l2_3d(&tmap_w, 0, tile * 128, (kc0 + i) * KC);
    else
      tma_prefetch_l2_5d(&tmap_w, 0, 0, 0, 4 * head + half, (kc0 + i) * KC);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&tl->full[s], 1);
      mbar_init(&tl->empty[s], 1);
    }
    mbar_init(&tl->accum, 1);
    mbar_init(&tl->recv, 1);
    tl->abort = 0;
    fence_mbar_init();
    // The weight tiles of the first stages depend on nothing (not even the
    // prep kernel): request them before TMEM allocation and the block
    // barrier; the next p.prefetch stages go to L2 beyond the ring.
    tma_prefetch_desc(&tmap_w);
    pol_w = make_l2_policy_evict_first();  // weights are streamed once
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&tl->full[i], stage_bytes);
      load_w(i, i);
    }
    for (int i = pre; i < nk && i < pre + p.prefetch; ++i) prefetch_w(i);
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
  // Epilogue warps: RoPE values of the first finished token and the bias of
  // the thread's row groups, fetched before the main loop ends.
  float4 cs0[RG / 4], sn0[RG / 4];
  float bias_y[RG], bias_p[RG];

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_x = make_l2_policy_evict_last();  // x_hat is re-read by every tile
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_3d(b_smem + (size_t)i * b_stage, &tmap_x, &tl->full[i], 0, 0, (kc0 + i) * KC, pol_x);
      // ring slot and phase advance by increment (no divisions on the issue path)
      int s = pre % S;
      uint32_t ph = (uint32_t)(pre / S) & 1u;
      for (int i = pre; i < nk; ++i) {
        if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
          decode_fail(p, tl, kStatusTimeoutEmpty);
          break;
        }
        mbar_arrive_expect_tx(&tl->full[s], stage_bytes);
        load_w(s, i);
        tma_load_3d(b_smem + (size_t)s * b_stage, &tmap_x, &tl->full[s], 0, 0, (kc0 + i) * KC, pol_x);
        if (i + p.prefetch < nk) prefetch_w(i + p.prefetch);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ UMMA issue
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(TM, n_pad);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nk; ++i) {
        if (!mbar_wait(&tl->full[s], ph, abort_flag)) {
          decode_fail(p, tl, kStatusTimeoutFull);
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
    // ------------------------------------------------ epilogue (warps 2-5)
    const int ept = threadIdx.x - 64;  // 0..127
    const int q4 = warp & 3;
    // accumulator row held by this lane (M = 64: lanes 16-31 of each quarter hold none)
    const int r = TM == 128 ? q4 * 32 + lane : (lane < 16 ? q4 * 16 + lane : -1);
    const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16);
    const int T = p.num_tokens;
    // Finishing thread (j, g): token c*16 + j of chunk c, tile rows RG*g .. +RG-1
    // (8 consecutive lanes: 8 tokens of one row group, no bank conflicts);
    // partner rows RG*(g ^ 4) hold the rotate-half partners.
    const int j = ept & 15, g = ept >> 4, gp = g ^ 4;
    const int hr0 = head_row<TM>(RG * g, half), hrp0 = head_row<TM>(RG * gp, half);
    const float sign = g < 4 ? -1.f : 1.f;
    // rows whose rotate-half / gate-up partner rows are summed as well
    const bool rot = EPI == kEpiQkv ? head < p.n_heads + p.n_kv_heads : (EPI == kEpiSwiglu ? g < 4 : false);
    const int rank = split;  // cluster (1, splits, 1): rank == blockIdx.y
    const int nranks = p.splits;
    pdl_wait();
    if (EPI == kEpiQkv) {
      for (int t = ept; t < T; t += 128) {
        tl->pos[t] = p.tok_pos[t];
        tl->slot[t] = p.tok_slot[t];
      }
    } else if (EPI == kEpiArgmax) {
      for (int t = ept; t < n_pad; t += 128) tl->key[t] = 0ull;
    }
    if (EPI == kEpiQkv) {
      const int t0 = rank * 16 + j;
      if (t0 < T && rot) load_rope_n<RG>(p, p.tok_pos[t0], hr0, cs0, sn0);
#pragma unroll
      for (int i = 0; i < RG; ++i) {
        bias_y[i] = p.bias ? __bfloat162float(p.bias[head * kHeadDim + hr0 + i]) : 0.f;
        bias_p[i] = p.bias ? __bfloat162float(p.bias[head * kHeadDim + hrp0 + i]) : 0.f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < RG; ++i) bias_y[i] = bias_p[i] = 0.f;
    }
    const bool waited = mbar_wait_warp(&tl->accum, 0u, abort_flag);
    if (!waited && lane == 0) decode_fail(p, tl, kStatusTimeoutAccum);
    tc_fence_after();
    cluster_wait();

    // Park the partial token-major in the idle pipeline buffers, four 16-token
    // chunks at a time; a chunk finished by another rank is sent to it by
    // bulk copy as soon as its group is parked.
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
      for (int cc = 0; cc < nc; ++cc) remote |= (c0 + cc) % nranks != rank;
      if (remote) {
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        // chunk cc of the group is sent by lane 0 of epilogue warp cc, so the
        // (remote) bulk-copy issues of a group run in parallel
        if ((ept & 31) == 0) {
          for (int cc = ept >> 5; cc < nc; cc += 4) {
            const int c = c0 + cc, owner = c % nranks;
            if (owner == rank) continue;
            const int slot = recv_slot(c / nranks, nranks, owner, rank);
            bulk_copy_to_cluster(
                map_smem_to_rank(smem_u32(recv_smem) + (uint32_t)slot * TS::kChunkBytes, (uint32_t)owner),
                part_u32 + (uint32_t)c * TS::kChunkBytes, TS::kChunkBytes,
                map_smem_to_rank(smem_u32(&tl->recv), (uint32_t)owner));
          }
        }
      }
    }
    if ((ept & 31) == 0) bulk_commit_group();
    named_bar_sync(1, 128);  // the owned chunks are parked

    // ------------------------------------------------ finish the owned chunks
    const bool got = mbar_wait_warp_incoming(&tl->recv, 0u);
    if (!got && lane == 0) decode_fail(p, tl, kStatusTimeoutCluster);
    if (got && *abort_flag == 0) {
      const float* recv = reinterpret_cast<const float*>(recv_smem);
      for (int c = rank; c * 16 < T; c += nranks) {
        const int t = c * 16 + j;
        if (t >= T) continue;
        if (EPI == kEpiSwiglu && g >= 4) continue;  // up rows: read as partners of the gate rows
        const int pos = EPI == kEpiQkv ? tl->pos[t] : 0;
        float4 cs[RG / 4], sn[RG / 4];
        if (EPI == kEpiQkv && rot) {
          if (c == rank) {
#pragma unroll
            for (int k4 = 0; k4 < RG / 4; ++k4) {
              cs[k4] = cs0[k4];
              sn[k4] = sn0[k4];
            }
          } else {
            load_rope_n<RG>(p, pos, hr0, cs, sn);
          }
        }
        float y[RG], yp[RG];
#pragma unroll
        for (int i = 0; i < RG; ++i) {
          y[i] = bias_y[i];
          yp[i] = bias_p[i];
        }
        // partials summed in rank order; two ranks per round with all their
        // loads issued before the first add
        const int oc = c / nranks;
        for (int q0 = 0; q0 < nranks; q0 += 2) {
          float4 a[2][RG / 4], b[2][RG / 4];
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int q = q0 + qq < nranks ? q0 + qq : q0;
            const float* src = q == rank ? part + t * YS
                                         : recv + (size_t)recv_slot(oc, nranks, rank, q) * (TS::kChunkBytes / 4) +
                                               (size_t)j * YS;
#pragma unroll
            for (int k4 = 0; k4 < RG / 4; ++k4) a[qq][k4] = reinterpret_cast<const float4*>(src + RG * g)[k4];
            if (rot) {
#pragma unroll
              for (int k4 = 0; k4 < RG / 4; ++k4) b[qq][k4] = reinterpret_cast<const float4*>(src + RG * gp)[k4];
            }
          }
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            if (q0 + qq >= nranks) break;
            add_f4<RG>(y, a[qq]);
            if (rot) add_f4<RG>(yp, b[qq]);
          }
        }
        if (EPI == kEpiQkv) {
          store_rows_n<RG>(p, head, t, hr0, sign, pos, tl->slot[t], y, yp, cs, sn);
        } else if (EPI == kEpiSwiglu) {
          // features tile * 64 + RG * g .. +RG-1: silu(gate) * up
          uint32_t w[RG / 2];
#pragma unroll
          for (int i = 0; i < RG / 2; ++i) {
            const float a0 = y[2 * i] / (1.f + __expf(-y[2 * i])) * yp[2 * i];
            const float a1 = y[2 * i + 1] / (1.f + __expf(-y[2 * i + 1])) * yp[2 * i + 1];
            w[i] = pack_bf16x2(a0, a1);
          }
          uint4* dst = reinterpret_cast<uint4*>(p.act + (size_t)t * p.act_stride + (size_t)tile * 64 + RG * g);
#pragma unroll
          for (int h = 0; h < RG / 8; ++h) dst[h] = make_uint4(w[4 * h], w[4 * h + 1], w[4 * h + 2], w[4 * h + 3]);
        } else {
          // vocabulary rows tile * 128 + RG * g + i
          unsigned long long best = 0ull;
#pragma unroll
          for (int i = 0; i < RG; ++i) {
            const int row = tile * 128 + RG * g + i;
            if (row < p.vocab_valid) {
              const unsigned long long k = argmax_key(y[i], (uint32_t)(p.vocab_offset + row));
              best = k > best ? k : best;
            }
          }
          atomicMax(&tl->key[t], best);
        }
      }
    }
    if (EPI == kEpiArgmax) {
      named_bar_sync(1, 128);
      for (int t = ept; t < T; t += 128)
        if (tl->key[t] != 0ull) atomicMax(p.keys + t, tl->key[t]);
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
size_t decode_smem_bytes_t(int stages, int n_pad, int kc, int splits) {
  return 1024 + decode_pipe_bytes<TM>(stages, n_pad, kc) +
         recv_area_bytes(n_pad, splits, TileShape<TM>::kChunkBytes) + sizeof(DecodeSmemTail);
}

size_t decode_smem_bytes(int tile_m, int stages, int n_pad, int kc, int splits) {
  return tile_m == 64 ? decode_smem_bytes_t<64>(stages, n_pad, kc, splits)
                      : decode_smem_bytes_t<128>(stages, n_pad, kc, splits);
}

template <int TM, int EPI>
static cudaError_t launch_decode_t(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                                   int tiles, cudaStream_t stream) {
  const size_t smem = decode_smem_bytes_t<TM>(p.stages, p.n_pad, p.kc, p.splits);
  cudaError_t e =
      cudaFuncSetAttribute(qkv_rope_decode_kernel<TM, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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
  return cudaLaunchKernelEx(&cfg, qkv_rope_decode_kernel<TM, EPI>, tmap_w, tmap_x, p);
}

cudaError_t launch_qkv_rope_decode(int tile_m, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                                   const PagedParams& p, int tiles, cudaStream_t stream) {
  if (p.epi == kEpiSwiglu) return launch_decode_t<128, kEpiSwiglu>(tmap_w, tmap_x, p, tiles, stream);
  if (p.epi == kEpiArgmax) return launch_decode_t<128, kEpiArgmax>(tmap_w, tmap_x, p, tiles, stream);
  return tile_m == 64 ? launch_decode_t<64, kEpiQkv>(tmap_w, tmap_x, p, tiles, stream)
                      : launch_decode_t<128, kEpiQkv>(tmap_w, tmap_x, p, tiles, stream);
}

// Largest cluster count that can be resident at once for a given split.
template <int TM>
static int decode_max_active_clusters_t(int splits, int n_pad, int stages, int kc) {
  const size_t smem = decode_smem_bytes_t<TM>(stages, n_pad, kc, splits);
  if (cudaFuncSetAttribute(qkv_rope_decode_kernel<TM, kEpiQkv>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
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
  if (cudaOccupancyMaxActiveClusters(&n, qkv_rope_decode_kernel<TM, kEpiQkv>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int decode_max_active_clusters(int tile_m, int splits, int n_pad, int stages, int kc) {
  return tile_m == 64 ? decode_max_active_clusters_t<64>(splits, n_pad, stages, kc)
                      : decode_max_active_clusters_t<128>(splits, n_pad, stages, kc);
}

}  // namespace krt
