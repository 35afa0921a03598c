// Per-token preparation shared by the decode and prefill paths.
//
// One 128-thread CTA per token:
//   * x_hat[t] = bf16(x[t] * rsqrt(mean(x[t]^2) + eps) * gamma), the
//     reference's RMSNorm with the cast back to the activation dtype before
//     the projection (python/kinetic_rt/fusion_forge.py:42-47);
//   * tok_pos[t]  = positions[t], or -1 outside the RoPE table;
//   * tok_slot[t] = block_table[seq][pos / B] * B + pos % B, or -1 when the
//     table column or the block id is out of range (BlockManager geometry,
//     include/BlockManager.h:46-49); failures set a bit in the status word.
// It triggers the dependent GEMM launch at once, so the GEMM kernel streams
// weights while this kernel runs (programmatic dependent launch).
#include <cuda_runtime.h>

#include "capi_internal.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

namespace krt {

__global__ void __launch_bounds__(128) qkv_prep_kernel(const PagedParams p) {
  pdl_launch_dependents();
  __shared__ float red[4];
  const int t = blockIdx.x;
  if (t >= p.num_tokens) return;
  const __nv_bfloat16* row = p.x + (size_t)t * p.x_stride;
  const int nvec = p.d_model >> 3;
  float ss = 0.f;
  for (int v = threadIdx.x; v < nvec; v += 128) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + v * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float r = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)p.d_model + p.eps);
  __nv_bfloat16* orow = p.xhat + (size_t)t * p.d_model;
  for (int v = threadIdx.x; v < nvec; v += 128) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + v * 8);
    const uint4 graw = *reinterpret_cast<const uint4*>(p.gamma + v * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&graw);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      const float2 gg = __bfloat1622float2(g[j]);
      o[j] = pack_bf16x2(f.x * r * gg.x, f.y * r * gg.y);
    }
    *reinterpret_cast<uint4*>(orow + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (threadIdx.x == 0) {
    const int pos = p.positions[t];
    const bool pos_ok = pos >= 0 && pos < p.max_position;
    const long long sl = token_slot(p, t);
    p.tok_pos[t] = pos_ok ? pos : -1;
    p.tok_slot[t] = sl;
    if (!pos_ok || sl < 0) atomicOr(p.status, kStatusBadBlock);
  }
}

cudaError_t launch_qkv_prep(const PagedParams& p, cudaStream_t stream) {
  qkv_prep_kernel<<<p.num_tokens, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace krt
