// C-ABI entry points of libkrt.so (declared in include/krt.h).
//
// Argument validation, launch-shape selection, TMA descriptor encoding and
// error reporting live here; the kernels are in qkv_generic.cu,
// qkv_decode.cu and qkv_prefill.cu.  Nothing here allocates device memory:
// callers pass every buffer, including workspaces.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <map>
#include <mutex>
#include <tuple>
#include <string>

#include "../../include/krt.h"
#include "capi_internal.h"
#include "qkv_generic.cuh"
#include "qkv_paged.cuh"

namespace krt {

namespace {
thread_local std::string g_last_error;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(KRT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int clear_error() {
  g_last_error.clear();
  return KRT_OK;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with a row pitch
// of `pitch_elems`, box = [box_rows, 64 cols], 128-byte swizzle.
int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(KRT_ERR_INVALID, "TMA base address must be 16-byte aligned");
  if ((pitch_elems * 2) % 16 != 0) return set_error(KRT_ERR_INVALID, "row pitch must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
  return KRT_OK;
}

// 3-D view of a row-major bf16 [rows, cols] matrix as [cols/64][rows][64]:
// one box = `kc` consecutive 64-column chunks of `box_rows` rows, landing in
// shared memory as kc back-to-back [box_rows x 64] 128-byte-swizzled tiles,
// so each row contributes kc * 128 contiguous bytes per request.
int make_tmap_bf16_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint32_t box_rows, uint32_t kc) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(KRT_ERR_INVALID, "TMA base address must be 16-byte aligned");
  if ((pitch_elems * 2) % 16 != 0) return set_error(KRT_ERR_INVALID, "row pitch must be a multiple of 16 bytes");
  if (cols % 64 != 0) return set_error(KRT_ERR_INVALID, "columns must be a multiple of 64");
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {pitch_elems * 2, 128};
  cuuint32_t box[3] = {64, box_rows, kc};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (CUresult %d)", (int)r);
  return KRT_OK;
}

// Weight tiles of half a head: the 64 rows {32h .. 32h+31} and {64+32h ..
// 64+32h+31} of head `head` (h = 0, 1) as one box.  View of W [heads*128, K]:
//   d0 = 64 columns (128 bytes), d1 = 32 rows, d2 = 2 (the 64-row hop),
//   d3 = 32-row block index 4*head + h, d4 = 64-column chunk;
// box {64, 32, 2, 1, kc} lands as kc back-to-back [64 rows x 64] 128-byte-
// swizzled slices (rows 0-31 then 32-63), the K-major UMMA A operand of M = 64.
int make_tmap_bf16_half_heads(CUtensorMap* map, const void* base, int heads, uint64_t cols, uint32_t kc) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(KRT_ERR_INVALID, "TMA base address must be 16-byte aligned");
  if (cols % 64 != 0) return set_error(KRT_ERR_INVALID, "columns must be a multiple of 64");
  const uint64_t row = cols * 2;  // bytes
  cuuint64_t dims[5] = {64, 32, 2, (cuuint64_t)(4 * heads - 2), cols / 64};
  cuuint64_t strides[4] = {row, 64 * row, 32 * row, 128};
  cuuint32_t box[5] = {64, 32, 2, 1, kc};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled (5-D) failed (CUresult %d)", (int)r);
  return KRT_OK;
}

// bf16 tensor map of any rank <= 5 with explicit byte strides (dims[0] is
// contiguous, the other strides in any order, multiples of 16), 128-byte
// swizzle (box[0] * 2 must be 128 bytes).
int make_tmap_bf16_5d_strided(CUtensorMap* map, const void* base, std::initializer_list<uint64_t> dims,
                              std::initializer_list<uint64_t> strides, std::initializer_list<uint32_t> box) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(KRT_ERR_INVALID, "TMA base address must be 16-byte aligned");
  const int rank = (int)dims.size();
  if (rank < 2 || rank > 5 || (int)strides.size() != rank - 1 || (int)box.size() != rank)
    return set_error(KRT_ERR_INVALID, "tensor map: inconsistent rank");
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  int i = 0;
  for (uint64_t v : dims) d[i++] = v;
  i = 0;
  for (uint64_t v : strides) {
    if (v % 16 != 0) return set_error(KRT_ERR_INVALID, "tensor map: strides must be multiples of 16 bytes");
    st[i++] = v;
  }
  i = 0;
  for (uint32_t v : box) bx[i++] = v;
  for (i = 0; i < rank; ++i) es[i] = 1;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KRT_ERR_CUDA, "cuTensorMapEncodeTiled (%d-D) failed (CUresult %d)", rank, (int)r);
  return KRT_OK;
}

}  // namespace krt

using namespace krt;

extern "C" const char* krt_last_error(void) { return g_last_error.c_str(); }

extern "C" const char* krt_version(void) { return "kinetic-rt-b200 0.1 (sm_100a)"; }

// ------------------------------------------------------------------ generic
extern "C" int krt_fused_rmsnorm_qkv_rope(const krt_qkv_rope_args* a, void* stream) {
  if (!a) return set_error(KRT_ERR_INVALID, "krt_fused_rmsnorm_qkv_rope: args is NULL");
  if (!a->x || !a->qkv_weight || !a->rms_weight || !a->freqs_cos || !a->freqs_sin || !a->q_out || !a->k_out ||
      !a->v_out)
    return set_error(KRT_ERR_INVALID,
                     "Cannot launch fused_rmsnorm_qkv_rope: descriptor is missing required weight, frequency, or "
                     "Q/K/V buffers.");
  if (a->seq_len <= 0 || a->d_model <= 0 || a->n_heads <= 0 || a->head_dim <= 0)
    return set_error(KRT_ERR_INVALID,
                     "Cannot launch fused_rmsnorm_qkv_rope: seq_len, d_model, n_heads, and head_dim must be positive.");
  if (a->head_dim % 2 != 0) return set_error(KRT_ERR_INVALID, "head_dim must be even for rotate-half RoPE");
  const int dtype = a->dtype == 0 ? KRT_DTYPE_FLOAT32 : a->dtype;
  const int fdtype = a->freqs_dtype == 0 ? dtype : a->freqs_dtype;
  if ((dtype != KRT_DTYPE_FLOAT32 && dtype != KRT_DTYPE_BFLOAT16) ||
      (fdtype != KRT_DTYPE_FLOAT32 && fdtype != KRT_DTYPE_BFLOAT16))
    return set_error(KRT_ERR_UNSUPPORTED, "fused_rmsnorm_qkv_rope supports float32 and bfloat16 only");
  GenericArgs g;
  g.x = a->x;
  g.w = a->qkv_weight;
  g.bias = a->qkv_bias;
  g.gamma = a->rms_weight;
  g.cos = a->freqs_cos;
  g.sin = a->freqs_sin;
  g.q = a->q_out;
  g.k = a->k_out;
  g.v = a->v_out;
  g.seq_len = a->seq_len;
  g.d_model = a->d_model;
  g.n_heads = a->n_heads;
  g.n_kv_heads = a->n_kv_heads > 0 ? a->n_kv_heads : a->n_heads;
  g.head_dim = a->head_dim;
  g.eps = a->eps;
  g.sx_seq = a->stride_x_seq;
  g.sx_dim = a->stride_x_dim;
  g.sw_out = a->stride_w_out;
  g.sw_in = a->stride_w_in;
  g.sq_seq = a->stride_q_seq;
  g.sq_dim = a->stride_q_dim;
  g.sk_seq = a->stride_k_seq;
  g.sk_dim = a->stride_k_dim;
  g.sv_seq = a->stride_v_seq;
  g.sv_dim = a->stride_v_dim;
  const bool f_default = a->stride_f_seq == 0 && a->stride_f_dim == 0;
  g.sf_seq = f_default ? a->stride_x_seq : a->stride_f_seq;
  g.sf_dim = f_default ? a->stride_x_dim : a->stride_f_dim;
  g.f_head_stride = a->freqs_head_stride < 0 ? a->head_dim : a->freqs_head_stride;
  g.positions = a->positions;
  cudaError_t e = launch_qkv_rope_generic(g, dtype, fdtype, 0, 0, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_error(e, "fused_rmsnorm_qkv_rope launch");
  return clear_error();
}

// ------------------------------------------------------------------- paged
namespace {

int paged_common_checks(const krt_qkv_paged_args* a, const char* name, bool need_workspace = true) {
  if (!a) return set_error(KRT_ERR_INVALID, "%s: args is NULL", name);
  if (!a->x || !a->qkv_weight || !a->rms_weight || !a->rope_cos || !a->rope_sin || !a->positions ||
      !a->token_seq || !a->block_table || !a->kv_pool || !a->q_out)
    return set_error(KRT_ERR_INVALID, "%s: a required pointer is NULL", name);
  if (a->num_tokens <= 0 || a->d_model <= 0 || a->n_heads <= 0 || a->n_kv_heads <= 0)
    return set_error(KRT_ERR_INVALID, "%s: num_tokens, d_model, n_heads and n_kv_heads must be positive", name);
  if (a->head_dim != kHeadDim) return set_error(KRT_ERR_UNSUPPORTED, "%s: head_dim must be 128", name);
  if (a->d_model % kBK != 0) return set_error(KRT_ERR_UNSUPPORTED, "%s: d_model must be a multiple of 64", name);
  if (a->n_heads + 2 * a->n_kv_heads > kMaxTiles)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: too many heads", name);
  if (a->x_stride < a->d_model || a->x_stride % 8 != 0)
    return set_error(KRT_ERR_INVALID, "%s: x_stride must be >= d_model and a multiple of 8", name);
  if (a->q_stride < a->n_heads * kHeadDim)
    return set_error(KRT_ERR_INVALID, "%s: q_stride must be >= n_heads * 128", name);
  if ((reinterpret_cast<uintptr_t>(a->x) & 15) || (reinterpret_cast<uintptr_t>(a->rms_weight) & 15) ||
      (reinterpret_cast<uintptr_t>(a->qkv_weight) & 15) || (reinterpret_cast<uintptr_t>(a->q_out) & 15) ||
      (reinterpret_cast<uintptr_t>(a->kv_pool) & 15) || (reinterpret_cast<uintptr_t>(a->k_out) & 15) ||
      (reinterpret_cast<uintptr_t>(a->v_out) & 15) || (reinterpret_cast<uintptr_t>(a->rope_cos) & 15) ||
      (reinterpret_cast<uintptr_t>(a->rope_sin) & 15))
    return set_error(KRT_ERR_INVALID, "%s: tensors must be 16-byte aligned", name);
  if (a->q_stride % 8 != 0) return set_error(KRT_ERR_INVALID, "%s: q_stride must be a multiple of 8", name);
  if (a->max_position <= 0 || a->num_seqs <= 0 || a->block_table_stride <= 0 || a->num_blocks <= 0 ||
      a->tokens_per_block <= 0)
    return set_error(KRT_ERR_INVALID, "%s: paged-cache geometry must be positive", name);
  if (need_workspace && !a->workspace) return set_error(KRT_ERR_WORKSPACE, "%s: workspace is NULL", name);
  return KRT_OK;
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

// Shared memory per CTA the stage count may use: 227 KB (one CTA per SM) by
// default; KRT_SMEM_CAP_KB lowers it for tuning (at 113 KB two kernels' CTAs
// can share an SM, but the shallower weight pipeline measured slower on
// B200: a Llama-3-8B decode layer step of 66.6 us against 51.3 us).
size_t smem_cap_bytes() { return (size_t)env_int("KRT_SMEM_CAP_KB", 227) * 1024; }

int decode_stages(int tile_m, int n_pad, int kc, int splits) {
  for (int st = kMaxStages; st >= 1; --st)
    if (decode_smem_bytes(tile_m, st, n_pad, kc, splits) <= smem_cap_bytes()) return st;
  return 0;
}

// 64-column chunks per decode pipeline stage (TMA box depth): the deepest of
// 4, 2, 1 that divides the k-blocks and still leaves two pipeline stages.
// KRT_DECODE_KC overrides the starting value for tuning.
int decode_kc(int tile_m, int num_kb, int n_pad, int splits) {
  int kc = env_int("KRT_DECODE_KC", 4);
  if (kc < 1) kc = 1;
  while (kc > 1 && ((num_kb % kc) != 0 || num_kb / kc < splits || decode_stages(tile_m, n_pad, kc, splits) < 2))
    kc >>= 1;
  return kc;
}

struct DecodeCfg {
  int tile_m, tiles, kc, stages, splits;
};

// Tile height: a whole head (M = 128), or half a head (M = 64) when there are
// at most 12 heads and at most 128 tokens: few head tiles would need up to 8
// K splits, whose partial exchange then costs more than the X tiles that
// half-height tiles re-read (measured on B200: 6 heads 8.8 us vs 10.2 us,
// 12 heads 10.6 vs 10.8, 24 heads 13.8 vs 11.6, 48 heads 21.0 vs 16.1 at
// 64 tokens).  KRT_DECODE_TILE_M overrides.  Split-K factor = cluster size along
// gridDim.y: as many splits as fit (tiles * splits <= #SMs, at most 8 =
// portable cluster size) while every cluster of the grid can be resident at
// once; box depth and stage count follow from the shared memory left beside
// the split's receive area.  KRT_DECODE_SPLITS overrides the split factor.
DecodeCfg decode_config(int heads, int num_kb, int n_pad, bool whole_tiles = false) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, DecodeCfg> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, heads, num_kb, n_pad, whole_tiles ? 1 : 0);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  // Above 128 tokens whole-head tiles park 135 KB of partial and leave room
  // for 2 splits only (B200, 256 tokens, 10 heads: 20 CTAs, 41.6 us); half
  // heads need half of it: 24.7 us at 4 splits, 21.6 us at 6 (but 48 heads:
  // 40.4 us against 29.0 on whole heads).
  const bool wide = n_pad > 128;
  int tile_m = env_int("KRT_DECODE_TILE_M", (heads <= 12 && !wide) || (heads <= 24 && wide) ? 64 : 128);
  if (tile_m != 64 || whole_tiles) tile_m = 128;
  const int tiles = heads * (128 / tile_m);
  DecodeCfg cfg{tile_m, tiles, 1, 1, 1};
  const int forced = env_int("KRT_DECODE_SPLITS", 0);
  // splits fill about two thirds of the SMs: more CTAs exchange more partials
  // than their extra streaming gains (B200, 64 tokens: 24 half-head tiles
  // x 4 splits 10.1 us, x 6 splits 10.6 us); above 128 tokens five sixths
  // (the 256-token case above)
  // (projections on whole tiles, gate/up at TP=8: 28 tiles x 4 splits 16.7 us,
  // x 3 splits 19.4 us, x 5 splits 26.4 us: about four fifths of the SMs)
  const int num = whole_tiles ? 4 : (wide ? 5 : 2), den = whole_tiles ? 5 : (wide ? 6 : 3);
  int s = forced > 0 ? forced : device_sm_count() * num / den / tiles;
  if (s > 8) s = 8;
  if (s < 1) s = 1;
  for (; s >= 1; --s) {
    const int kc = decode_kc(tile_m, num_kb, n_pad, s);
    const int st = decode_stages(tile_m, n_pad, kc, s);
    if (st < 1 || s > num_kb / kc) continue;
    cfg = DecodeCfg{tile_m, tiles, kc, st, s};
    if (forced > 0 || s == 1 || decode_max_active_clusters(tile_m, s, n_pad, st, kc) >= tiles) break;
  }
  cache[key] = cfg;
  return cfg;
}

}  // namespace

namespace krt {
// Argument checks of the decode path without the workspace (for callers
// that supply the workspace themselves); KRT_OK or an error with `name`.
int decode_args_check(const krt_qkv_paged_args* a, const char* name) {
  int rc = paged_common_checks(a, name, false);
  if (rc) return rc;
  if (a->num_tokens > 256)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: num_tokens must be <= 256 (use the prefill path)", name);
  return KRT_OK;
}
}  // namespace krt

extern "C" size_t krt_qkv_rope_decode_workspace_size(int32_t num_tokens, int32_t d_model, int32_t n_heads,
                                                     int32_t n_kv_heads, int32_t head_dim) {
  if (num_tokens <= 0 || num_tokens > 256 || d_model <= 0 || head_dim != kHeadDim || n_heads <= 0 ||
      n_kv_heads <= 0)
    return 0;
  return ws_layout(num_tokens, d_model).total;
}

extern "C" int krt_qkv_rope_decode(const krt_qkv_paged_args* a, void* stream) {
  int rc = paged_common_checks(a, "krt_qkv_rope_decode");
  if (rc) return rc;
  if (a->num_tokens > 256)
    return set_error(KRT_ERR_UNSUPPORTED, "krt_qkv_rope_decode: num_tokens must be <= 256 (use the prefill path)");
  const int tiles = a->n_heads + 2 * a->n_kv_heads;
  const int num_kb = a->d_model / kBK;
  const size_t need =
      krt_qkv_rope_decode_workspace_size(a->num_tokens, a->d_model, a->n_heads, a->n_kv_heads, a->head_dim);
  if (a->workspace_bytes < need)
    return set_error(KRT_ERR_WORKSPACE, "krt_qkv_rope_decode: workspace of %zu bytes, %zu needed",
                     a->workspace_bytes, need);
  PagedParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.bias = static_cast<const __nv_bfloat16*>(a->qkv_bias);
  p.gamma = static_cast<const __nv_bfloat16*>(a->rms_weight);
  p.cos = a->rope_cos;
  p.sin = a->rope_sin;
  p.positions = a->positions;
  p.token_seq = a->token_seq;
  p.block_table = a->block_table;
  p.pool = static_cast<__nv_bfloat16*>(a->kv_pool);
  p.q = static_cast<__nv_bfloat16*>(a->q_out);
  p.k = static_cast<__nv_bfloat16*>(a->k_out);
  p.v = static_cast<__nv_bfloat16*>(a->v_out);
  p.num_tokens = a->num_tokens;
  p.n_pad = (a->num_tokens + 15) / 16 * 16;
  p.d_model = a->d_model;
  p.n_heads = a->n_heads;
  p.n_kv_heads = a->n_kv_heads;
  p.x_stride = a->x_stride;
  p.q_stride = a->q_stride;
  p.max_position = a->max_position;
  p.num_seqs = a->num_seqs;
  p.bt_stride = a->block_table_stride;
  p.num_blocks = a->num_blocks;
  p.tokens_per_block = a->tokens_per_block;
  p.eps = a->eps;
  const DecodeCfg cfg = decode_config(tiles, num_kb, p.n_pad);
  p.kc = cfg.kc;
  p.stages = cfg.stages;
  p.splits = cfg.splits;
  // L2 prefetch of weight stages ahead of the ring: off by default.  It
  // shortens the kernel alone (48 heads, 64 tokens: 16.4 -> 15.7 us) but
  // lengthens a PDL-chained decoder-layer step on B200 (53.7 -> 54.9 us);
  // KRT_L2_PREFETCH_STAGES turns it on.
  p.prefetch = env_int("KRT_L2_PREFETCH_STAGES", 0);
  int cols = 32;
  while (cols < p.n_pad) cols <<= 1;
  p.tmem_cols = cols;
  char* ws = static_cast<char*>(a->workspace);
  const WsLayout L = ws_layout(p.num_tokens, p.d_model);
  p.status = reinterpret_cast<int*>(ws);
  p.tok_pos = reinterpret_cast<int*>(ws + L.pos_off);
  p.tok_slot = reinterpret_cast<long long*>(ws + L.slot_off);
  p.xhat = reinterpret_cast<__nv_bfloat16*>(ws + L.xhat_off);

  cudaStream_t s = (cudaStream_t)stream;
  CUtensorMap tmap_w, tmap_x;
  if (cfg.tile_m == 64)
    rc = make_tmap_bf16_half_heads(&tmap_w, a->qkv_weight, tiles, (uint64_t)a->d_model, (uint32_t)p.kc);
  else
    rc = make_tmap_bf16_3d(&tmap_w, a->qkv_weight, (uint64_t)tiles * kHeadDim, (uint64_t)a->d_model,
                           (uint64_t)a->d_model, 128, (uint32_t)p.kc);
  if (rc) return rc;
  rc = make_tmap_bf16_3d(&tmap_x, p.xhat, (uint64_t)p.num_tokens, (uint64_t)a->d_model, (uint64_t)a->d_model,
                         (uint32_t)p.n_pad, (uint32_t)p.kc);
  if (rc) return rc;
  cudaError_t e = launch_qkv_prep(p, s);
  if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_decode prep launch");
  e = launch_qkv_rope_decode(cfg.tile_m, tmap_w, tmap_x, p, cfg.tiles, s);
  if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_decode launch");
  return clear_error();
}

extern "C" int krt_read_status(void* workspace, void* stream, int32_t* bits) {
  if (!workspace || !bits) return set_error(KRT_ERR_INVALID, "krt_read_status: NULL argument");
  int v = 0;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_error(e, "krt_read_status");
  *bits = v;
  if (v != 0) {
    // Clear the status word (and the rest of the reserved header) for the next call.
    e = cudaMemsetAsync(workspace, 0, kWsHeaderBytes, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_error(e, "krt_read_status clear");
    return set_error(KRT_ERR_DEVICE, "kernel status bits 0x%x", v);
  }
  return clear_error();
}

// --------------------------------------------- decode-shaped projections
namespace {

// RMSNorm prep + the swap-AB split-K projection kernel with a non-QKV
// epilogue (p.epi), weight rows in 128-row tiles.
int run_projection(PagedParams& p, const void* weight, int weight_rows, const char* name, cudaStream_t s) {
  const int tiles = (weight_rows + 127) / 128;
  const int num_kb = p.d_model / kBK;
  const int sms = device_sm_count();
  // Kernel and work split by tiles per SM, as measured on B200 (148 SMs) at
  // 128 tokens, gate/up + SwiGLU and lm_head + argmax at the Llama-3-8B TP
  // shards (us per call):
  //   gate/up TP=1 (224 tiles): stream-K 54.4, whole tiles 56.0, split-K 72.0
  //   gate/up TP=2 (112):       stream-K 35.6, whole tiles 32.9, split-K 37.3
  //   gate/up TP=4 (56):        stream-K 28.3, split-K 33.9
  //   gate/up TP=8 (28):        stream-K 27.3, split-K 19.3
  //   lm_head TP=1 (1002):      stream-K 188.6, whole tiles 183.7
  //   lm_head TP=8 (126):       stream-K 36.7, whole tiles 32.4
  // (and stream-K over whole tiles by 10-12 % for gate/up at TP=1 with 1..64
  // tokens).  So: the persistent kernel above a quarter tile per SM, one CTA
  // per SM walking the tiles with the weight stream never drained; stream-K
  // below 0.6 tiles per SM and between one and three, whole tiles otherwise.
  // KRT_PROJ_PERSISTENT=0 / 1 and KRT_PROJ_STREAMK=0 / 1 force either choice.
  // More than 256 tokens (a prompt): the persistent kernel over 256-token
  // blocks, whole tiles.
  const bool blocks = p.num_tokens > 256;
  if (blocks) {
    p.n_pad = 256;
    p.row_tiles = tiles;
    p.sk_part = nullptr;
    p.sk_flags = nullptr;
  }
  const int n_blocks = (p.num_tokens + 255) / 256;
  const int forced = blocks ? 1 : env_int("KRT_PROJ_PERSISTENT", -1);
  const int sk_forced = env_int("KRT_PROJ_STREAMK", -1);
  const bool sk_possible = p.sk_part != nullptr && sk_forced != 0;  // the workspace holds the partials
  const bool sk_auto = 10 * tiles < 6 * sms || (tiles >= sms && tiles < 3 * sms);
  if (forced == 1 || (forced != 0 && (2 * tiles > sms || (4 * tiles > sms && sk_possible)))) {
    const size_t budget = smem_cap_bytes() - proj_persistent_smem_bytes(0, 1, p.n_pad);
    int kc = env_int("KRT_PROJ_KC", 2) == 1 ? 1 : 2;
    if (num_kb % 2 != 0 || budget / (2 * (16384 + (size_t)p.n_pad * 128)) < 3) kc = 1;
    int stages = (int)(budget / ((size_t)kc * (16384 + (size_t)p.n_pad * 128)));
    if (stages > 8) stages = 8;
    if (stages >= 2) {
      p.kc = kc;
      p.stages = stages;
      p.splits = 1;
      p.prefetch = env_int("KRT_L2_PREFETCH_STAGES", 0);
      p.sk = sk_possible && (sk_forced == 1 || sk_auto) ? 1 : 0;
      int cols = 32;
      while (cols < 2 * p.n_pad) cols <<= 1;
      p.tmem_cols = cols;
      CUtensorMap tmap_w, tmap_x;
      int rc = make_tmap_bf16_3d(&tmap_w, weight, (uint64_t)weight_rows, (uint64_t)p.d_model, (uint64_t)p.d_model,
                                 128, (uint32_t)kc);
      if (rc) return rc;
      rc = make_tmap_bf16_3d(&tmap_x, p.xhat, (uint64_t)p.num_tokens, (uint64_t)p.d_model, (uint64_t)p.d_model,
                             (uint32_t)p.n_pad, (uint32_t)kc);
      if (rc) return rc;
      cudaError_t e = launch_qkv_prep(p, s);
      if (e != cudaSuccess) return cuda_error(e, name);
      e = launch_proj_persistent(tmap_w, tmap_x, p, tiles * n_blocks, s);
      if (e != cudaSuccess) return cuda_error(e, name);
      return clear_error();
    }
    if (blocks) return set_error(KRT_ERR_UNSUPPORTED, "%s: shared memory too small for 256-token blocks", name);
  }
  const DecodeCfg cfg = decode_config(tiles, num_kb, p.n_pad, true);
  p.kc = cfg.kc;
  p.stages = cfg.stages;
  p.splits = cfg.splits;
  p.prefetch = env_int("KRT_L2_PREFETCH_STAGES", 0);
  int cols = 32;
  while (cols < p.n_pad) cols <<= 1;
  p.tmem_cols = cols;
  CUtensorMap tmap_w, tmap_x;
  int rc = make_tmap_bf16_3d(&tmap_w, weight, (uint64_t)weight_rows, (uint64_t)p.d_model, (uint64_t)p.d_model, 128,
                             (uint32_t)p.kc);
  if (rc) return rc;
  rc = make_tmap_bf16_3d(&tmap_x, p.xhat, (uint64_t)p.num_tokens, (uint64_t)p.d_model, (uint64_t)p.d_model,
                         (uint32_t)p.n_pad, (uint32_t)p.kc);
  if (rc) return rc;
  cudaError_t e = launch_qkv_prep(p, s);
  if (e != cudaSuccess) return cuda_error(e, name);
  e = launch_qkv_rope_decode(128, tmap_w, tmap_x, p, tiles, s);
  if (e != cudaSuccess) return cuda_error(e, name);
  return clear_error();
}

// Shared checks and parameters of the RMSNorm + projection calls.
int projection_params(PagedParams& p, const char* name, const void* x, const void* gamma, const void* weight,
                      int num_tokens, int d_model, int x_stride, float eps, void* workspace, size_t ws_bytes,
                      int max_tokens = 256) {
  if (!x || !gamma || !weight || !workspace) return set_error(KRT_ERR_INVALID, "%s: a required pointer is NULL", name);
  if (num_tokens <= 0 || num_tokens > max_tokens)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: num_tokens must be in 1..%d", name, max_tokens);
  if (d_model <= 0 || d_model % kBK != 0)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: d_model must be a positive multiple of 64", name);
  if (x_stride < d_model || x_stride % 8 != 0)
    return set_error(KRT_ERR_INVALID, "%s: x_stride must be >= d_model and a multiple of 8", name);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(gamma) & 15) ||
      (reinterpret_cast<uintptr_t>(weight) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return set_error(KRT_ERR_INVALID, "%s: tensors must be 16-byte aligned", name);
  const size_t need = ws_layout(num_tokens, d_model).total;
  if (ws_bytes < need) return set_error(KRT_ERR_WORKSPACE, "%s: workspace of %zu bytes, %zu needed", name, ws_bytes, need);
  const ProjWsLayout PL = proj_ws_layout(num_tokens, d_model);
  std::memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.gamma = static_cast<const __nv_bfloat16*>(gamma);
  p.num_tokens = num_tokens;
  p.n_pad = (num_tokens + 15) / 16 * 16;
  p.d_model = d_model;
  p.x_stride = x_stride;
  p.eps = eps;
  char* ws = static_cast<char*>(workspace);
  const WsLayout L = ws_layout(num_tokens, d_model);
  p.status = reinterpret_cast<int*>(ws);
  p.tok_pos = reinterpret_cast<int*>(ws + L.pos_off);
  p.tok_slot = reinterpret_cast<long long*>(ws + L.slot_off);
  p.xhat = reinterpret_cast<__nv_bfloat16*>(ws + L.xhat_off);
  // a workspace of krt_projection_workspace_size() bytes also holds the
  // stream-K flags and partials; a smaller one (the base layout) keeps the
  // persistent kernel on whole tiles
  if (ws_bytes >= PL.total) {
    p.sk_flags = reinterpret_cast<int*>(ws + PL.flags_off);
    p.sk_part = reinterpret_cast<float*>(ws + PL.part_off);
  }
  return KRT_OK;
}

}  // namespace

extern "C" size_t krt_projection_workspace_size(int32_t num_tokens, int32_t d_model) {
  if (num_tokens <= 0 || num_tokens > kMaxPromptTokens || d_model <= 0) return 0;
  return proj_ws_layout(num_tokens, d_model).total;
}

extern "C" int krt_gate_up_swiglu(const krt_gate_up_args* a, void* stream) {
  const char* name = "krt_gate_up_swiglu";
  if (!a) return set_error(KRT_ERR_INVALID, "%s: args is NULL", name);
  PagedParams p;
  int rc = projection_params(p, name, a->x, a->rms_weight, a->gate_up_weight, a->num_tokens, a->d_model, a->x_stride,
                             a->eps, a->workspace, a->workspace_bytes, kMaxPromptTokens);
  if (rc) return rc;
  if (!a->act) return set_error(KRT_ERR_INVALID, "%s: act is NULL", name);
  if (a->inter_local <= 0 || a->inter_local % 64 != 0)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: inter_local must be a positive multiple of 64", name);
  if (a->act_stride < a->inter_local || a->act_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(a->act) & 15))
    return set_error(KRT_ERR_INVALID, "%s: act must be 16-byte aligned with a stride >= inter_local, multiple of 8",
                     name);
  p.epi = kEpiSwiglu;
  p.act = static_cast<__nv_bfloat16*>(a->act);
  p.act_stride = a->act_stride;
  return run_projection(p, a->gate_up_weight, 2 * a->inter_local, name, (cudaStream_t)stream);
}

extern "C" int krt_lm_head_argmax(const krt_lm_head_args* a, void* stream) {
  const char* name = "krt_lm_head_argmax";
  if (!a) return set_error(KRT_ERR_INVALID, "%s: args is NULL", name);
  PagedParams p;
  int rc = projection_params(p, name, a->x, a->rms_weight, a->weight, a->num_tokens, a->d_model, a->x_stride, a->eps,
                             a->workspace, a->workspace_bytes);
  if (rc) return rc;
  if (!a->argmax_keys || (reinterpret_cast<uintptr_t>(a->argmax_keys) & 7))
    return set_error(KRT_ERR_INVALID, "%s: argmax_keys must be an 8-byte aligned buffer", name);
  if (a->vocab_local <= 0 || a->vocab_offset < 0)
    return set_error(KRT_ERR_INVALID, "%s: vocab_local must be positive and vocab_offset >= 0", name);
  p.epi = kEpiArgmax;
  p.keys = a->argmax_keys;
  p.vocab_valid = a->vocab_local;
  p.vocab_offset = a->vocab_offset;
  return run_projection(p, a->weight, a->vocab_local, name, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ prefill
extern "C" size_t krt_qkv_rope_prefill_workspace_size(int32_t num_tokens, int32_t d_model, int32_t n_heads,
                                                      int32_t n_kv_heads, int32_t head_dim) {
  (void)n_heads;
  (void)n_kv_heads;
  if (num_tokens <= 0 || d_model <= 0 || head_dim != kHeadDim) return 0;
  return ws_layout(num_tokens, d_model).total;
}

extern "C" int krt_qkv_rope_prefill(const krt_qkv_paged_args* a, void* stream) {
  int rc = paged_common_checks(a, "krt_qkv_rope_prefill");
  if (rc) return rc;
  const int tiles = a->n_heads + 2 * a->n_kv_heads;
  const size_t need =
      krt_qkv_rope_prefill_workspace_size(a->num_tokens, a->d_model, a->n_heads, a->n_kv_heads, a->head_dim);
  if (a->workspace_bytes < need)
    return set_error(KRT_ERR_WORKSPACE, "krt_qkv_rope_prefill: workspace of %zu bytes, %zu needed",
                     a->workspace_bytes, need);
  PagedParams p;
  std::memset(&p, 0, sizeof(p));
  p.x = static_cast<const __nv_bfloat16*>(a->x);
  p.bias = static_cast<const __nv_bfloat16*>(a->qkv_bias);
  p.gamma = static_cast<const __nv_bfloat16*>(a->rms_weight);
  p.cos = a->rope_cos;
  p.sin = a->rope_sin;
  p.positions = a->positions;
  p.token_seq = a->token_seq;
  p.block_table = a->block_table;
  p.pool = static_cast<__nv_bfloat16*>(a->kv_pool);
  p.q = static_cast<__nv_bfloat16*>(a->q_out);
  p.k = static_cast<__nv_bfloat16*>(a->k_out);
  p.v = static_cast<__nv_bfloat16*>(a->v_out);
  p.num_tokens = a->num_tokens;
  p.n_pad = a->num_tokens;
  p.d_model = a->d_model;
  p.n_heads = a->n_heads;
  p.n_kv_heads = a->n_kv_heads;
  p.x_stride = a->x_stride;
  p.q_stride = a->q_stride;
  p.max_position = a->max_position;
  p.num_seqs = a->num_seqs;
  p.bt_stride = a->block_table_stride;
  p.num_blocks = a->num_blocks;
  p.tokens_per_block = a->tokens_per_block;
  p.eps = a->eps;
  char* ws = static_cast<char*>(a->workspace);
  const WsLayout L = ws_layout(p.num_tokens, p.d_model);
  p.status = reinterpret_cast<int*>(ws);
  p.tok_pos = reinterpret_cast<int*>(ws + L.pos_off);
  p.tok_slot = reinterpret_cast<long long*>(ws + L.slot_off);
  p.xhat = reinterpret_cast<__nv_bfloat16*>(ws + L.xhat_off);

  cudaStream_t s = (cudaStream_t)stream;
  // KRT_PREFILL_KERNEL=1: the persistent projection kernel's QKV epilogue
  // over head x 256-token tiles instead of the dedicated prefill kernel (the
  // same speed on B200 at 8 x 2048 tokens: 1112 vs 1115 TFLOP/s).
  if (env_int("KRT_PREFILL_KERNEL", 0) == 1) {
    PagedParams q = p;
    q.epi = kEpiQkv;
    q.n_pad = 256;
    q.row_tiles = tiles;
    const size_t budget = smem_cap_bytes() - proj_persistent_smem_bytes(0, 1, q.n_pad);
    const size_t stage1 = 16384 + (size_t)q.n_pad * 128;
    q.kc = (a->d_model / kBK) % 2 == 0 && budget / (2 * stage1) >= 3 ? 2 : 1;
    q.stages = (int)(budget / (q.kc * stage1));
    if (q.stages > 8) q.stages = 8;
    q.tmem_cols = 512;
    if (q.stages >= 2) {
      CUtensorMap tmap_w, tmap_x;
      rc = make_tmap_bf16_3d(&tmap_w, a->qkv_weight, (uint64_t)tiles * kHeadDim, (uint64_t)a->d_model,
                             (uint64_t)a->d_model, 128, (uint32_t)q.kc);
      if (rc) return rc;
      rc = make_tmap_bf16_3d(&tmap_x, p.xhat, (uint64_t)a->num_tokens, (uint64_t)a->d_model, (uint64_t)a->d_model,
                             256, (uint32_t)q.kc);
      if (rc) return rc;
      cudaError_t e = launch_qkv_prep(p, s);
      if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_prefill prep launch");
      e = launch_proj_persistent(tmap_w, tmap_x, q, tiles * ((a->num_tokens + 255) / 256), s);
      if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_prefill launch");
      return clear_error();
    }
  }
  CUtensorMap tmap_w, tmap_x;
  rc = make_tmap_bf16_2d(&tmap_w, a->qkv_weight, (uint64_t)tiles * kHeadDim, (uint64_t)a->d_model,
                         (uint64_t)a->d_model, 128);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tmap_x, p.xhat, (uint64_t)a->num_tokens, (uint64_t)a->d_model, (uint64_t)a->d_model, 256);
  if (rc) return rc;
  cudaError_t e = launch_qkv_prep(p, s);
  if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_prefill prep launch");
  e = launch_qkv_rope_prefill(tmap_w, tmap_x, p, tiles, s);
  if (e != cudaSuccess) return cuda_error(e, "krt_qkv_rope_prefill launch");
  return clear_error();
}
