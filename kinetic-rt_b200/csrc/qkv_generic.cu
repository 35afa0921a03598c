// Launchers of the reference-compatible CUDA-core kernel (qkv_generic.cuh)
// and the extern "C" kernel with the reference's 24-argument signature that
// the .kin artifact carries (compiled separately to a cubin by the build).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/krt.h"
#include "capi_internal.h"
#include "qkv_generic.cuh"

namespace krt {

template <typename T, typename TF>
__global__ void __launch_bounds__(1024) qkv_rope_generic_kernel(const GenericArgs a) {
  qkv_rope_generic_body<T, TF>(a);
}

size_t generic_smem_bytes(int d_model, int n_out) { return ((size_t)d_model + n_out + 32) * sizeof(float); }

cudaError_t launch_qkv_rope_generic(const GenericArgs& a, int dtype, int freqs_dtype, int grid, int block,
                                    cudaStream_t stream) {
  const int n_out = (a.n_heads + 2 * a.n_kv_heads) * a.head_dim;
  const size_t smem = generic_smem_bytes(a.d_model, n_out);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (grid <= 0) grid = a.seq_len < 4096 ? a.seq_len : 4096;
  if (block <= 0) block = 256;
  void (*kern)(GenericArgs) = nullptr;
  if (dtype == KRT_DTYPE_FLOAT32)
    kern = freqs_dtype == KRT_DTYPE_FLOAT32 ? qkv_rope_generic_kernel<float, float>
                                            : qkv_rope_generic_kernel<float, __nv_bfloat16>;
  else
    kern = freqs_dtype == KRT_DTYPE_FLOAT32 ? qkv_rope_generic_kernel<__nv_bfloat16, float>
                                            : qkv_rope_generic_kernel<__nv_bfloat16, __nv_bfloat16>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<grid, block, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace krt
