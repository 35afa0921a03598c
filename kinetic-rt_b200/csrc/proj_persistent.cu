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
// Work split.  Tile-granular (p.sk == 0): CTA c takes tiles c, c + G, ...
// (G = gridDim.x), full K each.  With T tiles not a multiple of G the last
// round leaves SMs idle (B200, gate/up at TP=1: 224 tiles on 148 SMs, the
// SMs busy 72 % of the kernel).  Stream-K (p.sk != 0): the T x KB k-boxes
// are cut into G equal runs, run c = boxes [c T KB / G, (c+1) T KB / G) in
// (tile, k) order, so every SM streams the same number of weight bytes.  A
// run is a list of segments (tile, k0, k1):
//   * k0 == 0 and k1 == KB: a whole tile, epilogue as usual;
//   * k0 > 0 (only a run's first segment): the tail of a tile another CTA
//     started.  The epilogue stores the raw fp32 accumulator to
//     sk_part[c] and releases sk_flags[c];
//   * k0 == 0 and k1 < KB (only a run's last segment): the head of a tile
//     that continues in runs c + 1, c + 2, ...  The epilogue acquires their
//     flags (bounded wait, status bit 64 when it runs out), adds their
//     partials in run order and applies the epilogue; then it clears the
//     flags for the next launch.
// A head waits only for runs that start with their tile, i.e. at the
// beginning of those CTAs' work, while the head comes at the end of its own:
// all G CTAs are resident together (one per SM, G <= #SMs), and the
// dependent kernel cannot take an SM before every CTA here has started.
// Token blocks (p.row_tiles > 0, more than 256 tokens): tile = tb * row_tiles
// + rt covers weight rows 128 rt .. and tokens n_pad tb .. (n_pad = 256); row
// tiles run fastest, so the CTAs of one round share a few token blocks of X
// and walk W in step (both kept in L2 with an evict-last policy).
// Epilogues (PagedParams::epi): kEpiSwiglu (act = silu(gate) * up, gate and
// up rows side by side in 64-row groups), kEpiArgmax (the CTA keeps each
// token's best (logit, index) over all its tiles in shared memory and folds
// it into the global keys once at the end; one token block) and kEpiStore
// (y = bf16(acc + residual): the row-parallel GEMM at large token counts).
// kEpiQkv (bias, RoPE, Q out, K/V into the paged pool; tile = one head x
// one token block) serves the QKV prefill: every tile stages its block's
// positions and pool slots in shared memory once the previous tile's
// epilogue is done with them.  (Decode-sized QKV runs on the split-K kernel.)
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
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  // this CTA's k-boxes: [box0, box0 + total) of the (tile, k) order (stream-K),
  // or its tiles' boxes one after another (tile-granular)
  const long long all_boxes = (long long)num_tiles * num_kc;
  const long long box0 = p.sk ? all_boxes * c / G : 0;
  const int my_tiles = c < num_tiles ? (num_tiles - 1 - c) / G + 1 : 0;
  const int total = p.sk ? (int)(all_boxes * (c + 1) / G - box0) : my_tiles * num_kc;
  const int pre = total < S ? total : S;
  auto tile_of = [&](int it) {
    return p.sk ? (int)((box0 + it) / num_kc) : c + (it / num_kc) * G;
  };
  auto kb_of = [&](int it) { return p.sk ? (int)((box0 + it) % num_kc) : it % num_kc; };
  // segments: (tile, k0, k1); tile-granular runs have my_tiles whole tiles
  const int first_tile = p.sk ? (int)(box0 / num_kc) : c;
  const int num_segs = p.sk ? (total > 0 ? tile_of(total - 1) - first_tile + 1 : 0) : my_tiles;
  auto seg_tile = [&](int i) { return p.sk ? first_tile + i : c + i * G; };
  auto seg_k0 = [&](int i) { return (p.sk && i == 0) ? (int)(box0 - (long long)first_tile * num_kc) : 0; };
  auto seg_k1 = [&](int i) {
    if (!p.sk) return num_kc;
    const long long end = box0 + total - (long long)seg_tile(i) * num_kc;
    return end < num_kc ? (int)end : num_kc;
  };
  // tile -> (weight row tile, token block)
  const int RT = p.row_tiles > 0 ? p.row_tiles : num_tiles;
  auto w_row = [&](int tile) { return (tile % RT) * 128; };
  auto x_row = [&](int tile) { return (tile / RT) * n_pad; };

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
    // weights are streamed once, unless several token blocks re-read them
    pol_w = RT < num_tiles ? make_l2_policy_evict_last() : make_l2_policy_evict_first();
    for (int it = 0; it < pre; ++it) {
      mbar_arrive_expect_tx(&tl->full[it], stage_bytes);
      tma_load_3d(a_smem + (size_t)it * a_stage, &tmap_w, &tl->full[it], 0, w_row(tile_of(it)), kb_of(it) * KC, pol_w);
    }
    // optionally the next p.prefetch stages' weights into L2 beyond the ring
    for (int it = pre; it < total && it < pre + p.prefetch; ++it)
      tma_prefetch_l2_3d(&tmap_w, 0, w_row(tile_of(it)), kb_of(it) * KC);
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
      // The segments' k-boxes in order; the ring slot and its phase advance
      // by increment (no divisions between a slot turning free and its loads).
      int it = 0, s = 0;
      uint32_t ph = 0;
      bool alive = true;
      for (int seg = 0; seg < num_segs && alive; ++seg) {
        const int tile = seg_tile(seg);
        const int wr = w_row(tile), xr = x_row(tile);
        const int k1 = seg_k1(seg);
        for (int kb = seg_k0(seg); kb < k1; ++kb, ++it) {
          if (it >= pre) {
            if (!mbar_wait(&tl->empty[s], ph ^ 1u, abort_flag)) {
              pj_fail(p, tl, kStatusTimeoutEmpty);
              alive = false;
              break;
            }
            mbar_arrive_expect_tx(&tl->full[s], stage_bytes);
            tma_load_3d(a_smem + (size_t)s * a_stage, &tmap_w, &tl->full[s], 0, wr, kb * KC, pol_w);
            const int pf = it + p.prefetch;
            if (p.prefetch > 0 && pf < total) tma_prefetch_l2_3d(&tmap_w, 0, w_row(tile_of(pf)), kb_of(pf) * KC);
          }
          // (the first `pre` slots' weight boxes were requested before the wait)
          tma_load_3d(b_smem + (size_t)s * b_stage, &tmap_x, &tl->full[s], 0, xr, kb * KC, pol_x);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issue
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(128, n_pad);
      int s = 0;  // ring slot and phase, advanced by increment
      uint32_t ph = 0;
      bool alive = true;
      for (int local = 0; local < num_segs && alive; ++local) {
        const uint32_t buf = (uint32_t)local & 1u;
        const uint32_t use = (uint32_t)local >> 1;
        if (!mbar_wait(&tl->tmem_empty[buf], (use & 1u) ^ 1u, abort_flag)) {
          pj_fail(p, tl, kStatusTimeoutAccum);
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem_base + buf * (uint32_t)n_pad;
        const int k0 = seg_k0(local), k1 = seg_k1(local);
        for (int kb = k0; kb < k1; ++kb) {
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
              umma_bf16(dcol, ad + 2u * kk, bd + 2u * kk, idesc, (kb > k0 || kc > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&tl->empty[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
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
    pdl_wait();
    for (int local = 0; local < num_segs; ++local) {
      const int tile = seg_tile(local);
      const int t_base = x_row(tile);  // first token of the tile's block
      const int T = p.num_tokens - t_base < n_pad ? p.num_tokens - t_base : n_pad;
      const int k0 = seg_k0(local), k1 = seg_k1(local);
      const bool tail = k0 > 0;                  // partial for the CTA that holds k-box 0
      const bool head = k0 == 0 && k1 < num_kc;  // add the partials of runs c + 1, ...
      int partners = 0;                          // runs that continue this tile
      if (head) {
        const long long tile_end = (long long)(tile + 1) * num_kc;
        while (c + 1 + partners < G && all_boxes * (c + 1 + partners) / G < tile_end) ++partners;
      }
      const uint32_t buf = (uint32_t)local & 1u;
      const uint32_t use = (uint32_t)local >> 1;
      const int qh = tile % RT;  // kEpiQkv: the head (weight row tile)
      if (EPI == kEpiQkv) {
        // this tile's token metadata (the previous tile's epilogue is done with it)
        for (int t = ept; t < n_pad; t += 256) {
          tl->pos[t] = t < T ? p.tok_pos[t_base + t] : -1;
          tl->slot[t] = t < T ? p.tok_slot[t_base + t] : -1;
        }
      }
      const bool waited = mbar_wait_warp(&tl->tmem_full[buf], use & 1u, abort_flag);
      if (!waited && lane == 0) pj_fail(p, tl, kStatusTimeoutAccum);
      tc_fence_after();
      bool got = true;
      if (head && ept == 0) {
        for (int q = 1; q <= partners && got; ++q) got = wait_flag_gpu(reinterpret_cast<const uint32_t*>(p.sk_flags + c + q), 1u);
        if (!got) pj_fail(p, tl, kStatusTimeoutCluster);
      }
      if (named_bar_any(3, 256, !waited || !got || *abort_flag != 0)) break;
      const uint32_t taddr = tmem_base + ((uint32_t)(q4 * 32) << 16) + buf * (uint32_t)n_pad;
      if (tail) {
        // the raw accumulator to this run's partial slot, token-major
        float* part = p.sk_part + (size_t)c * n_pad * 128 + r;
        for (int c0 = grp * 16; c0 < n_pad && c0 < T; c0 += 32) {
          float acc[16];
          tmem_ld16(taddr + (uint32_t)c0, acc);
#pragma unroll
          for (int i = 0; i < 16; ++i) __stcg(part + (size_t)(c0 + i) * 128, acc[i]);
        }
        tc_fence_before();
        named_bar_sync(3, 256);
        if (ept == 0) {
          __threadfence();
          st_release_gpu(reinterpret_cast<uint32_t*>(p.sk_flags + c), 1u);
        }
        if (lane == 0) mbar_arrive(&tl->tmem_empty[buf]);
        continue;
      }
      const float bias_r = EPI == kEpiQkv && p.bias ? __bfloat162float(p.bias[qh * kHeadDim + r]) : 0.f;
      const bool rot = EPI == kEpiQkv ? qh < p.n_heads + p.n_kv_heads : (EPI == kEpiSwiglu ? g8 < 4 : false);
      for (int c0 = grp * 16; c0 < n_pad; c0 += 32) {
        if (c0 >= T) break;  // uniform within the group
        const int t = c0 + j;
        const int pos = EPI == kEpiQkv ? tl->pos[t] : 0;
        float4 cs[4], sn[4];
        if (EPI == kEpiQkv && rot) load_rope_n<16>(p, pos, 16 * g8, cs, sn);
        float acc[16];
        tmem_ld16(taddr + (uint32_t)c0, acc);
        for (int q = 1; q <= partners; ++q) {
          const float* part = p.sk_part + (size_t)(c + q) * n_pad * 128 + r;
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[i] += __ldcg(part + (size_t)(c0 + i) * 128);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) ybuf[i * kYStride + r] = acc[i] + bias_r;
        named_bar_sync(bar_grp, 128);
        if (t < T) {
          float y[16], yp[16];
          ld_smem_16f(ybuf + j * kYStride + 16 * g8, y);
          if (rot) ld_smem_16f(ybuf + j * kYStride + 16 * (g8 ^ 4), yp);
          if (EPI == kEpiQkv) {
            store_rows_n<16>(p, qh, t_base + t, 16 * g8, g8 < 4 ? -1.f : 1.f, pos, tl->slot[t], y, yp, cs, sn);
          } else if (EPI == kEpiStore && p.y32) {
            float4* dst = reinterpret_cast<float4*>(p.y32 + (size_t)(t_base + t) * p.y_stride + w_row(tile) + 16 * g8);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
          } else if (EPI == kEpiStore) {
            const size_t off = (size_t)(t_base + t) * p.y_stride + w_row(tile) + 16 * g8;
            if (p.residual) {
              const uint4* res = reinterpret_cast<const uint4*>(p.residual + off);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint4 v = res[h];
                const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float2 f = __bfloat1622float2(b2[q]);
                  y[8 * h + 2 * q] += f.x;
                  y[8 * h + 2 * q + 1] += f.y;
                }
              }
            }
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = pack_bf16x2(y[2 * i], y[2 * i + 1]);
            uint4* dst = reinterpret_cast<uint4*>(p.y + off);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          } else if (EPI == kEpiSwiglu) {
            if (g8 < 4) {
              uint32_t w[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float a0 = y[2 * i] / (1.f + __expf(-y[2 * i])) * yp[2 * i];
                const float a1 = y[2 * i + 1] / (1.f + __expf(-y[2 * i + 1])) * yp[2 * i + 1];
                w[i] = pack_bf16x2(a0, a1);
              }
              uint4* dst = reinterpret_cast<uint4*>(p.act + (size_t)(t_base + t) * p.act_stride +
                                                    (size_t)(tile % RT) * 64 + 16 * g8);
              dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
              dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
            }
          } else {
            unsigned long long best = 0ull;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int row = w_row(tile) + 16 * g8 + i;
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
      // the partials are consumed: clear their flags for the next launch
      if (ept < partners) p.sk_flags[c + 1 + ept] = 0;
    }
    if (EPI == kEpiArgmax) {
      named_bar_sync(3, 256);
      for (int t = ept; t < p.num_tokens; t += 256)
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
  if (p.sk) {
    const long long boxes = (long long)num_tiles * (p.d_model / (kBK * p.kc));
    if (grid > kSkMaxCtas) grid = kSkMaxCtas;
    if (grid > boxes) grid = (int)boxes;
  } else if (grid > num_tiles) {
    grid = num_tiles;
  }
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
  if (p.epi == kEpiStore) return launch_pj_t<kEpiStore>(tmap_w, tmap_x, p, num_tiles, stream);
  if (p.epi == kEpiQkv) return launch_pj_t<kEpiQkv>(tmap_w, tmap_x, p, num_tiles, stream);
  return cudaErrorInvalidValue;
}

}  // namespace krt
