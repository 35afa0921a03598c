// Kernel image carried inside .kin artifacts (compiled to an sm_100a cubin).
//
// The exported symbol and its 24 parameters match what AOTEngine::launch
// packs for "fused_rmsnorm_qkv_rope" (src/AOTEngine.cpp:541-567 of the
// reference): x, W, b, gamma, cos, sin, q, k, v, seq_len, d_model, n_heads,
// head_dim, eps and ten int strides, with cos/sin indexed by x's strides
// (python/kinetic_rt/fusion_forge.py:92-93).  The body is the CUDA-core
// fused kernel of qkv_generic.cuh; tokens are grid-strided, so any grid is
// correct.  Needs (d_model + 3*d_model + 32) * 4 bytes of dynamic shared
// memory and a block size that is a multiple of 32.
#include "qkv_generic.cuh"

namespace {
__device__ __forceinline__ krt::GenericArgs pack(const void* x, const void* w, const void* b, const void* g,
                                                 const void* cs, const void* sn, void* q, void* k, void* v,
                                                 int seq_len, int d_model, int n_heads, int head_dim, float eps,
                                                 int sxs, int sxd, int swo, int swi, int sqs, int sqd, int sks,
                                                 int skd, int svs, int svd) {
  krt::GenericArgs a;
  a.x = x;
  a.w = w;
  a.bias = b;
  a.gamma = g;
  a.cos = cs;
  a.sin = sn;
  a.q = q;
  a.k = k;
  a.v = v;
  a.seq_len = seq_len;
  a.d_model = d_model;
  a.n_heads = n_heads;
  a.n_kv_heads = n_heads;
  a.head_dim = head_dim;
  a.eps = eps;
  a.sx_seq = sxs;
  a.sx_dim = sxd;
  a.sw_out = swo;
  a.sw_in = swi;
  a.sq_seq = sqs;
  a.sq_dim = sqd;
  a.sk_seq = sks;
  a.sk_dim = skd;
  a.sv_seq = svs;
  a.sv_dim = svd;
  a.sf_seq = sxs;
  a.sf_dim = sxd;
  a.f_head_stride = head_dim;
  a.positions = nullptr;
  return a;
}
}  // namespace

extern "C" __global__ void __launch_bounds__(1024)
    fused_rmsnorm_qkv_rope(const float* x, const float* w, const float* b, const float* g, const float* cs,
                           const float* sn, float* q, float* k, float* v, int seq_len, int d_model, int n_heads,
                           int head_dim, float eps, int sxs, int sxd, int swo, int swi, int sqs, int sqd, int sks,
                           int skd, int svs, int svd) {
  if ((blockDim.x & 31) != 0) return;
  const krt::GenericArgs a =
      pack(x, w, b, g, cs, sn, q, k, v, seq_len, d_model, n_heads, head_dim, eps, sxs, sxd, swo, swi, sqs, sqd,
           sks, skd, svs, svd);
  krt::qkv_rope_generic_body<float, float>(a);
}

extern "C" __global__ void __launch_bounds__(1024)
    fused_rmsnorm_qkv_rope_bf16(const __nv_bfloat16* x, const __nv_bfloat16* w, const __nv_bfloat16* b,
                                const __nv_bfloat16* g, const __nv_bfloat16* cs, const __nv_bfloat16* sn,
                                __nv_bfloat16* q, __nv_bfloat16* k, __nv_bfloat16* v, int seq_len, int d_model,
                                int n_heads, int head_dim, float eps, int sxs, int sxd, int swo, int swi, int sqs,
                                int sqd, int sks, int skd, int svs, int svd) {
  if ((blockDim.x & 31) != 0) return;
  const krt::GenericArgs a =
      pack(x, w, b, g, cs, sn, q, k, v, seq_len, d_model, n_heads, head_dim, eps, sxs, sxd, swo, swi, sqs, sqd,
           sks, skd, svs, svd);
  krt::qkv_rope_generic_body<__nv_bfloat16, __nv_bfloat16>(a);
}
