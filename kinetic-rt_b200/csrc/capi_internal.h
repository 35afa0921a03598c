// Internal declarations shared by the C-ABI layer and the kernel files.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstddef>
#include <cstdint>
#include <initializer_list>

struct krt_qkv_paged_args;

namespace krt {

struct GenericArgs;
struct PagedParams;

int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
int clear_error();
int device_sm_count();
int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint32_t box_rows, uint32_t kc);
int make_tmap_bf16_5d_strided(CUtensorMap* map, const void* base, std::initializer_list<uint64_t> dims,
                              std::initializer_list<uint64_t> strides, std::initializer_list<uint32_t> box);
int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint32_t box_rows);

// capi.cu: argument checks of krt_qkv_rope_decode, workspace excluded
int decode_args_check(const krt_qkv_paged_args* a, const char* name);

// qkv_generic.cu
cudaError_t launch_qkv_rope_generic(const GenericArgs& a, int dtype, int freqs_dtype, int grid, int block,
                                    cudaStream_t stream);
size_t generic_smem_bytes(int d_model, int n_out);

// qkv_decode.cu
// tile_m = 128 (one head per tile) or 64 (half a head per tile)
size_t decode_smem_bytes(int tile_m, int stages, int n_pad, int kc, int splits);
cudaError_t launch_qkv_rope_decode(int tile_m, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                                   const PagedParams& p, int tiles, cudaStream_t stream);

int decode_max_active_clusters(int tile_m, int splits, int n_pad, int stages, int kc);

// qkv_prep.cu
cudaError_t launch_qkv_prep(const PagedParams& p, cudaStream_t stream);

// qkv_prefill.cu
size_t prefill_smem_bytes();
cudaError_t launch_qkv_rope_prefill(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                                    int tiles_per_block, cudaStream_t stream);

// proj_persistent.cu
size_t proj_persistent_smem_bytes(int stages, int kc, int n_pad);
cudaError_t launch_proj_persistent(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const PagedParams& p,
                                   int num_tiles, cudaStream_t stream);

// gemm_ar.cu
struct GemmArParams;
size_t gemm_ar_smem_bytes(int tile_m, int stages, int n_pad, int kc, int splits);
int gemm_ar_max_active_clusters(int tile_m, int splits, int n_pad, int stages, int kc);
cudaError_t launch_rowparallel_gemm_ar(int tile_m, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                                       const GemmArParams& p, int tiles, cudaStream_t stream);

}  // namespace krt
