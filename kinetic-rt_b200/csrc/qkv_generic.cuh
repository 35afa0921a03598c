// Reference-compatible fused RMSNorm + QKV projection + RoPE on CUDA cores.
//
// Follows python/kinetic_rt/fusion_forge.py:21-162 step by step, without its
// d_model <= 128 limit:
//   (1) RMSNorm in fp32, result cast back to the activation dtype (lines 42-47)
//   (2) qkv = W x_hat (+ b), fp32 accumulation (lines 57-75)
//   (3) split Q | K | V (lines 79-87; GQA widths when n_kv_heads != n_heads)
//   (4) rotate-half RoPE on Q and K per head, fp32 (lines 92-139)
//   (5) strided stores (lines 155-162)
// One CTA per token (grid-stride, so any launch grid is correct); warps own
// output rows and reduce along d_model with shuffles.  This path carries the
// fp32 known-answer and small-shape cases; the bf16 production shapes run on
// the tcgen05 kernels.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

namespace krt {

struct GenericArgs {
  const void* x;
  const void* w;
  const void* bias;
  const void* gamma;
  const void* cos;
  const void* sin;
  void* q;
  void* k;
  void* v;
  int seq_len, d_model, n_heads, n_kv_heads, head_dim;
  float eps;
  int64_t sx_seq, sx_dim, sw_out, sw_in, sq_seq, sq_dim, sk_seq, sk_dim, sv_seq, sv_dim;
  int64_t sf_seq, sf_dim;
  int f_head_stride;
  const int32_t* positions;
};

template <typename T>
__device__ __forceinline__ float ld_as_f32(const void* p, int64_t i) {
  return static_cast<float>(static_cast<const T*>(p)[i]);
}
template <>
__device__ __forceinline__ float ld_as_f32<__nv_bfloat16>(const void* p, int64_t i) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
template <typename T>
__device__ __forceinline__ void st_from_f32(void* p, int64_t i, float v) {
  static_cast<T*>(p)[i] = static_cast<T>(v);
}
template <>
__device__ __forceinline__ void st_from_f32<__nv_bfloat16>(void* p, int64_t i, float v) {
  static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return v;
}
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Dynamic shared memory: d_model floats (x_hat) + n_out floats (qkv) + 32.
template <typename T, typename TF>
__device__ __forceinline__ void qkv_rope_generic_body(const GenericArgs& a) {
  extern __shared__ float smem[];
  float* xh = smem;
  const int n_q = a.n_heads * a.head_dim;
  const int n_kv = a.n_kv_heads * a.head_dim;
  const int n_out = n_q + 2 * n_kv;
  float* y = xh + a.d_model;
  float* red = y + n_out;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
  const int half = a.head_dim >> 1;

  for (int t = blockIdx.x; t < a.seq_len; t += gridDim.x) {
    // (1) RMSNorm
    float ss = 0.f;
    for (int i = tid; i < a.d_model; i += nthr) {
      const float xv = ld_as_f32<T>(a.x, (int64_t)t * a.sx_seq + (int64_t)i * a.sx_dim);
      xh[i] = xv;
      ss += xv * xv;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float s = lane < nwarps ? red[lane] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) red[0] = s;
    }
    __syncthreads();
    const float r = rsqrtf(red[0] / (float)a.d_model + a.eps);
    for (int i = tid; i < a.d_model; i += nthr) xh[i] = round_to<T>(xh[i] * r * ld_as_f32<T>(a.gamma, i));
    __syncthreads();

    // (2) projection: one warp per output row
    for (int o = warp; o < n_out; o += nwarps) {
      float acc = 0.f;
      const int64_t wrow = (int64_t)o * a.sw_out;
      for (int i = lane; i < a.d_model; i += 32) acc += ld_as_f32<T>(a.w, wrow + (int64_t)i * a.sw_in) * xh[i];
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
      if (lane == 0) {
        if (a.bias != nullptr) acc += ld_as_f32<T>(a.bias, o);
        y[o] = acc;
      }
    }
    __syncthreads();

    // (3)-(5) split, RoPE, store
    const int64_t frow = (int64_t)(a.positions ? a.positions[t] : t) * a.sf_seq;
    for (int o = tid; o < n_out; o += nthr) {
      if (o < n_q + n_kv) {
        const bool is_q = o < n_q;
        const int base = is_q ? 0 : n_q;
        const int h = (o - base) / a.head_dim;
        const int d = (o - base) - h * a.head_dim;
        const int head0 = base + h * a.head_dim;
        const float u = y[o];
        const float rot = d < half ? -y[head0 + d + half] : y[head0 + d - half];
        const int64_t fi = frow + (int64_t)(h * a.f_head_stride + d) * a.sf_dim;
        const float out = u * ld_as_f32<TF>(a.cos, fi) + rot * ld_as_f32<TF>(a.sin, fi);
        if (is_q)
          st_from_f32<T>(a.q, (int64_t)t * a.sq_seq + (int64_t)(o - base) * a.sq_dim, out);
        else
          st_from_f32<T>(a.k, (int64_t)t * a.sk_seq + (int64_t)(o - base) * a.sk_dim, out);
      } else {
        st_from_f32<T>(a.v, (int64_t)t * a.sv_seq + (int64_t)(o - n_q - n_kv) * a.sv_dim, y[o]);
      }
    }
    __syncthreads();
  }
}

}  // namespace krt
