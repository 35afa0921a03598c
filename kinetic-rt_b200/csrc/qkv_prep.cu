// Per-token preparation shared by the decode and prefill paths.
//
// One CTA per token (warps 0-3 normalise, warp 4 looks the slot up):
//   * x_hat[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * gamma), the
//     reference's RMSNorm with the cast back to the activation dtype before
//     the projection (python/kinetic_rt/fusion_forge.py:42-47);
//   * tok_pos[t]  = positions[t], or -1 outside the RoPE table;
//   * tok_slot[t] = block_table[seq][pos / B] * B + pos % B, or -1 when the
//     table column or the block id is out of range (BlockManager geometry,
//     include/BlockManager.h:46-49); failures set a bit in the status word.
// Programmatic dependent launch on both sides: the kernel starts while the
// previous kernel drains (and waits for it before reading anything), and
// triggers the dependent projection kernel at once, so that kernel streams
// weights while this one runs.
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

constexpr int kPrepThreads = 160;  // warps 0-3: RMSNorm of the token; warp 4: its pool slot
constexpr int kPrepCache = 8;      // 16-byte vectors per thread held in registers (d_model <= 8192)

// ss + sum of the squares of 8 bf16 values, in element order.
__device__ __forceinline__ float sum_squares8(const uint4 raw, float ss) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    ss += f.x * f.x + f.y * f.y;
  }
  return ss;
}

// bf16(x * r * gamma) of 8 values.
__device__ __forceinline__ uint4 scale8(const uint4 raw, const uint4 graw, float r) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&graw);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    const float2 gg = __bfloat1622float2(g[j]);
    o[j] = pack_bf16x2(f.x * r * gg.x, f.y * r * gg.y);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(kPrepThreads) qkv_prep_kernel(const PagedParams p) {
  pdl_launch_dependents();
  pdl_wait();  // every input may come from the previous kernel
  __shared__ float red[4];
  const int t = blockIdx.x;
  if (t >= p.num_tokens) return;
  if (threadIdx.x >= 128) {
    // Warp 4: the slot lookup, whose dependent loads overlap the RMS pass
    // (only the QKV projection has positions and pool slots).
    if (threadIdx.x == 128 && p.positions != nullptr) {
      const int pos = p.positions[t];
      const bool pos_ok = pos >= 0 && pos < p.max_position;
      const long long sl = token_slot(p, t);
      p.tok_pos[t] = pos_ok ? pos : -1;
      p.tok_slot[t] = sl;
      if (!pos_ok || sl < 0) atomicOr(p.status, kStatusBadBlock);
    }
    return;
  }
  const __nv_bfloat16* row = p.x + (size_t)t * p.x_stride;
  const int nvec = p.d_model >> 3;
  __nv_bfloat16* orow = p.xhat + (size_t)t * p.d_model;
  // x and gamma of vectors threadIdx.x + 128*i, i < kPrepCache, stay in
  // registers between the two passes; gamma is requested before the reduction.
  uint4 xc[kPrepCache], gc[kPrepCache];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kPrepCache; ++i) {
    const int v = threadIdx.x + 128 * i;
    if (v < nvec) {
      xc[i] = *reinterpret_cast<const uint4*>(row + v * 8);
      gc[i] = *reinterpret_cast<const uint4*>(p.gamma + v * 8);
    }
  }
#pragma unroll
  for (int i = 0; i < kPrepCache; ++i)
    if ((int)threadIdx.x + 128 * i < nvec) ss = sum_squares8(xc[i], ss);
  for (int v = threadIdx.x + 128 * kPrepCache; v < nvec; v += 128)
    ss = sum_squares8(*reinterpret_cast<const uint4*>(row + v * 8), ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  named_bar_sync(1, 128);
  const float r = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)p.d_model + p.eps);
#pragma unroll
  for (int i = 0; i < kPrepCache; ++i) {
    const int v = threadIdx.x + 128 * i;
    if (v < nvec) *reinterpret_cast<uint4*>(orow + v * 8) = scale8(xc[i], gc[i], r);
  }
  for (int v = threadIdx.x + 128 * kPrepCache; v < nvec; v += 128)
    *reinterpret_cast<uint4*>(orow + v * 8) = scale8(*reinterpret_cast<const uint4*>(row + v * 8),
                                                     *reinterpret_cast<const uint4*>(p.gamma + v * 8), r);
}

cudaError_t launch_qkv_prep(const PagedParams& p, cudaStream_t stream) {
  // Programmatic dependent launch: the CTAs start while the previous kernel
  // drains and wait (griddepcontrol.wait) before reading their inputs.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.num_tokens, 1, 1);
  cfg.blockDim = dim3(kPrepThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qkv_prep_kernel, p);
}

}  // namespace krt
