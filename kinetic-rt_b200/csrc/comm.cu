// Communicator plumbing of the C ABI (krt_comm_*), the standalone allreduce
// and the entry point of the fused row-parallel GEMM + allreduce.
//
// Setup (not on the hot path): krt_comm_create allocates this rank's
// symmetric buffer (layout in comm.h), zero-fills it and exports a CUDA IPC
// handle; the caller exchanges the handles (e.g. torch.distributed
// all_gather_object) and passes all of them to krt_comm_open_peers, which
// maps every peer's buffer.  Ranks are processes, one GPU each.
//
// krt_allreduce is the reference's Communicator::all_reduce_async
// (src/Communicator.cpp:21-27; semantics tests/mock_rccl.h:51-62: every
// rank receives the elementwise sum of all ranks' send buffers), done as a
// two-shot exchange over the mapped peer buffers: rank o owns the o-th slice,
// every rank pushes its slice o to o, o sums in rank order and pushes the
// result to everyone.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <climits>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <new>
#include <vector>

#include "../../include/krt.h"
#include "capi_internal.h"
#include "comm.h"
#include "ptx.cuh"
#include "qkv_paged.cuh"

struct krt_comm {
  int rank = 0, world = 1, device = 0, max_n = 0;
  krt::CommLayout L;
  char* local = nullptr;
  char* peer[krt::kMaxWorld] = {};
  bool peers_open = false;
  ncclComm_t nccl = nullptr;      // krt_comm_attach_nccl
  size_t nccl_threshold = SIZE_MAX;  // messages of at least this many bytes go through NCCL
  float* nccl_f32 = nullptr;         // fp32 partials of the GEMM's NCCL route: [kNcclSliceTokens, max_n]
};

namespace {
// NCCL, resolved at run time from libnccl.so.2 (the copy the process already
// loaded, e.g. torch's, or the system's): only its header is used at build
// time, so the library links no NCCL and runs without one until a caller
// attaches an NCCL communicator.
struct NcclApi {
  bool ok = false;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};
const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
  });
  return api;
}
int nccl_error(ncclResult_t r, const char* what) {
  return krt::set_error(KRT_ERR_CUDA, "%s: NCCL error %d (%s)", what, (int)r,
                        nccl_api().error_string ? nccl_api().error_string(r) : "?");
}
}  // namespace

namespace krt {

// ------------------------------------------------------ standalone allreduce
constexpr int kArThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f32(float v) {
  return static_cast<T>(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// One launch reduces `count` elements: staging row q (count floats) holds
// rank q's copy of the owner's slice, the result area holds count elements.  CTA b handles
// the b-th sub-range of every rank's slice.
template <typename T>
__global__ void __launch_bounds__(kArThreads) allreduce_kernel(const T* __restrict__ send, T* __restrict__ recv,
                                                               long long count, CommView cv, int* status) {
  __shared__ int ok_s;
  const int world = cv.world, me = cv.rank, b = blockIdx.x, nb = gridDim.x;
  auto slice_lo = [&](int o) { return count * o / world; };
  // sub-range of slice o handled by this CTA
  auto sub = [&](int o, long long& lo, long long& hi) {
    const long long s0 = slice_lo(o), s1 = slice_lo(o + 1);
    lo = s0 + (s1 - s0) * b / nb;
    hi = s0 + (s1 - s0) * (b + 1) / nb;
  };
  // 1. push my slice o to owner o's staging row [me]
  for (int o = 0; o < world; ++o) {
    long long lo, hi;
    sub(o, lo, hi);
    float* stg = reinterpret_cast<float*>(cv.base[o] + cv.L.staging_off) + (size_t)me * count;
    for (long long i = lo + threadIdx.x; i < hi; i += kArThreads) stg[i - slice_lo(o)] = to_f32(send[i]);
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int o = 0; o < world; ++o)
      st_release_sys(reinterpret_cast<uint32_t*>(cv.base[o] + cv.L.ar_part_off) + (size_t)b * kMaxWorld + me, 1u);
  // 2. as owner of slice `me`: reduce in rank order, push to everyone
  if (threadIdx.x == 0) {
    uint32_t* pf = reinterpret_cast<uint32_t*>(cv.base[me] + cv.L.ar_part_off) + (size_t)b * kMaxWorld;
    bool ok = true;
    for (int q = 0; q < world && ok; ++q) ok = wait_flag_sys(pf + q, 1u);
    if (ok)
      for (int q = 0; q < world; ++q) pf[q] = 0u;
    else
      atomicOr(status, kStatusTimeoutPeer);
    ok_s = ok;
  }
  __syncthreads();
  {
    long long lo, hi;
    sub(me, lo, hi);
    const size_t row = (size_t)count;
    const float* stg = reinterpret_cast<const float*>(cv.base[me] + cv.L.staging_off);
    if (ok_s) {
      for (long long i = lo + threadIdx.x; i < hi; i += kArThreads) {
        float acc = 0.f;
        for (int q = 0; q < world; ++q) acc += __ldcg(stg + (size_t)q * row + (i - slice_lo(me)));
        const T v = from_f32<T>(acc);
        for (int q = 0; q < world; ++q) reinterpret_cast<T*>(cv.base[q] + cv.L.result_off)[i] = v;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && ok_s)
    for (int q = 0; q < world; ++q)
      st_release_sys(reinterpret_cast<uint32_t*>(cv.base[q] + cv.L.ar_final_off) + (size_t)me * kArMaxCtas + b, 1u);
  // 3. collect every owner's result slice into recv
  for (int o = 0; o < world; ++o) {
    if (threadIdx.x == 0) {
      uint32_t* ff = reinterpret_cast<uint32_t*>(cv.base[me] + cv.L.ar_final_off) + (size_t)o * kArMaxCtas + b;
      const bool ok = wait_flag_sys(ff, 1u);
      if (ok)
        *ff = 0u;
      else
        atomicOr(status, kStatusTimeoutPeer);
      ok_s = ok;
    }
    __syncthreads();
    long long lo, hi;
    sub(o, lo, hi);
    const T* res = reinterpret_cast<const T*>(cv.base[me] + cv.L.result_off);
    if (ok_s)
      for (long long i = lo + threadIdx.x; i < hi; i += kArThreads) {
        T v;
        if (sizeof(T) == 4) {
          const float f = __ldcg(reinterpret_cast<const float*>(res) + i);
          v = from_f32<T>(f);
        } else {
          const unsigned short h = __ldcg(reinterpret_cast<const unsigned short*>(res) + i);
          v = *reinterpret_cast<const T*>(&h);
        }
        recv[i] = v;
      }
    __syncthreads();
  }
}

// ------------------------------------------------------ greedy sampling
struct GreedyParams {
  unsigned long long* keys;
  int32_t* tokens;
  const __nv_bfloat16* embedding;
  __nv_bfloat16* hidden;
  int32_t* positions;
  int32_t* seq_lens;
  const int32_t* next_input;
  int* status;
  int num_seqs, d_model, hidden_stride, vocab;
};

// 49-bit form of a (logit, index) key for the flagged exchange: the
// orderable logit bits above a 17-bit inverted index (vocabularies below
// 2^17 entries); 0 stays 0 (no entry).
__device__ __forceinline__ uint64_t key49(unsigned long long key) {
  if (key == 0ull) return 0ull;
  const uint32_t idx = argmax_key_index(key);
  return ((uint64_t)(key >> 32) << 17) | (uint64_t)(0x1FFFFu - (idx & 0x1FFFFu));
}

// One CTA per sequence: the chosen token (max over ranks' keys), then its
// embedding row into the hidden state of the next step.
__global__ void __launch_bounds__(128) greedy_step_kernel(const GreedyParams g, const CommView cv) {
  pdl_wait();  // the keys come from the lm_head kernel
  pdl_launch_dependents();
  __shared__ int tok_s;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    const unsigned long long key = g.keys[b];
    g.keys[b] = 0ull;  // empty for the next lm_head call
    int tok = 0;
    bool have = key != 0ull;
    if (cv.world == 1) {
      if (have) tok = (int)argmax_key_index(key);
    } else {
      uint32_t* ep = reinterpret_cast<uint32_t*>(cv.base[cv.rank] + cv.L.greedy_epoch_off) + b;
      uint32_t e = *ep + 1u;
      if (e > 32767u) e = 1u;
      *ep = e;
      const uint64_t word = ((uint64_t)e << 49) | key49(key);
      const size_t slot = ((size_t)(e & 1u) * kMaxWorld + cv.rank) * kMaxGreedySeqs + b;
      for (int q = 0; q < cv.world; ++q) {
        uint64_t* dst = reinterpret_cast<uint64_t*>(cv.base[q] + cv.L.greedy_off) + slot;
        asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(word) : "memory");
      }
      uint64_t best = 0ull;
      const uint64_t t0 = globaltimer_ns();
      bool ok = true;
      for (int q = 0; q < cv.world && ok; ++q) {
        const uint64_t* src = reinterpret_cast<const uint64_t*>(cv.base[cv.rank] + cv.L.greedy_off) +
                              ((size_t)(e & 1u) * kMaxWorld + q) * kMaxGreedySeqs + b;
        while (true) {
          uint64_t w;
          asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(src) : "memory");
          if ((uint32_t)(w >> 49) == e) {
            const uint64_t k = w & ((1ull << 49) - 1ull);
            best = k > best ? k : best;
            break;
          }
          if (globaltimer_ns() - t0 > kWaitBudgetNs) {
            ok = false;
            break;
          }
        }
      }
      if (!ok) atomicOr(g.status, kStatusTimeoutPeer);
      have = ok && best != 0ull;
      if (have) tok = (int)(0x1FFFFu - (uint32_t)(best & 0x1FFFFu));
    }
    if (tok < 0 || tok >= g.vocab) {
      atomicOr(g.status, kStatusBadBlock);
      tok = 0;
    }
    g.tokens[b] = tok;
    if (g.next_input) {
      const int forced = g.next_input[b];
      if (forced >= 0 && forced < g.vocab) tok = forced;
    }
    tok_s = tok;
    if (g.positions) g.positions[b] += 1;
    if (g.seq_lens) g.seq_lens[b] += 1;
  }
  __syncthreads();
  if (g.embedding) {
    const uint4* src = reinterpret_cast<const uint4*>(g.embedding + (size_t)tok_s * g.d_model);
    uint4* dst = reinterpret_cast<uint4*>(g.hidden + (size_t)b * g.hidden_stride);
    for (int v = threadIdx.x; v < g.d_model / 8; v += blockDim.x) dst[v] = src[v];
  }
}

}  // namespace krt

using namespace krt;

// ------------------------------------------------------------------ C ABI
extern "C" int krt_comm_create(int32_t rank, int32_t world_size, int32_t max_n_out, krt_comm** out) {
  if (!out) return set_error(KRT_ERR_INVALID, "krt_comm_create: out is NULL");
  *out = nullptr;
  if (world_size < 1 || world_size > kMaxWorld || rank < 0 || rank >= world_size)
    return set_error(KRT_ERR_INVALID, "krt_comm_create: rank %d / world_size %d outside 1..%d", rank, world_size,
                     kMaxWorld);
  if (max_n_out <= 0 || max_n_out % 128 != 0)
    return set_error(KRT_ERR_INVALID, "krt_comm_create: max_n_out must be a positive multiple of 128");
  krt_comm* c = new (std::nothrow) krt_comm();
  if (!c) return set_error(KRT_ERR_INVALID, "krt_comm_create: out of host memory");
  c->rank = rank;
  c->world = world_size;
  c->max_n = max_n_out;
  c->L = comm_layout(world_size, max_n_out);
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->local), c->L.total);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->L.total);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return cuda_error(e, "krt_comm_create");
  }
  c->peer[rank] = c->local;
  if (world_size == 1) c->peers_open = true;
  *out = c;
  return clear_error();
}

extern "C" size_t krt_comm_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int krt_comm_ipc_handle(krt_comm* c, void* handle_out) {
  if (!c || !handle_out) return set_error(KRT_ERR_INVALID, "krt_comm_ipc_handle: NULL argument");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) return cuda_error(e, "krt_comm_ipc_handle");
  std::memcpy(handle_out, &h, sizeof(h));
  return clear_error();
}

extern "C" int krt_comm_open_peers(krt_comm* c, const void* handles) {
  if (!c || !handles) return set_error(KRT_ERR_INVALID, "krt_comm_open_peers: NULL argument");
  if (c->peers_open) return clear_error();
  const char* hp = static_cast<const char*>(handles);
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hp + (size_t)q * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int r = 0; r < q; ++r)
        if (r != c->rank && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]), c->peer[r] = nullptr;
      return cuda_error(e, "krt_comm_open_peers: cudaIpcOpenMemHandle");
    }
    c->peer[q] = static_cast<char*>(ptr);
  }
  c->peers_open = true;
  return clear_error();
}

extern "C" int krt_comm_reset(krt_comm* c, void* stream) {
  if (!c) return set_error(KRT_ERR_INVALID, "krt_comm_reset: communicator is NULL");
  // Every exchange area of this rank's buffer (flags, flagged words, epoch
  // counters) back to the state krt_comm_create left it in.
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(c->local, 0, c->L.total, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_error(e, "krt_comm_reset");
  return clear_error();
}

extern "C" size_t krt_nccl_id_size(void) { return sizeof(ncclUniqueId); }

extern "C" int krt_nccl_unique_id(void* id_out) {
  if (!id_out) return set_error(KRT_ERR_INVALID, "krt_nccl_unique_id: NULL argument");
  const NcclApi& api = nccl_api();
  if (!api.ok) return set_error(KRT_ERR_UNSUPPORTED, "krt_nccl_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_error(r, "krt_nccl_unique_id");
  std::memcpy(id_out, &id, sizeof(id));
  return clear_error();
}

extern "C" int krt_comm_attach_nccl(krt_comm* c, const void* id, size_t threshold_bytes) {
  if (!c || !id) return set_error(KRT_ERR_INVALID, "krt_comm_attach_nccl: NULL argument");
  const NcclApi& api = nccl_api();
  if (!api.ok) return set_error(KRT_ERR_UNSUPPORTED, "krt_comm_attach_nccl: libnccl.so.2 could not be loaded");
  if (!c->nccl) {
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t nc = nullptr;
    ncclResult_t r = api.comm_init_rank(&nc, c->world, uid, c->rank);
    if (r != ncclSuccess) return nccl_error(r, "krt_comm_attach_nccl: ncclCommInitRank");
    c->nccl = nc;
  }
  if (!c->nccl_f32) {
    cudaError_t e = cudaMalloc(&c->nccl_f32, (size_t)krt::kNcclSliceTokens * c->max_n * sizeof(float));
    if (e != cudaSuccess) {
      c->nccl_f32 = nullptr;
      return krt::cuda_error(e, "krt_comm_attach_nccl: fp32 partial buffer");
    }
  }
  c->nccl_threshold = threshold_bytes;
  return clear_error();
}

extern "C" int krt_comm_destroy(krt_comm* c) {
  if (!c) return clear_error();
  if (c->nccl && nccl_api().ok) nccl_api().comm_destroy(c->nccl);
  if (c->nccl_f32) cudaFree(c->nccl_f32);
  for (int q = 0; q < c->world; ++q)
    if (q != c->rank && c->peer[q]) cudaIpcCloseMemHandle(c->peer[q]);
  if (c->local) cudaFree(c->local);
  delete c;
  return clear_error();
}

namespace {
int comm_view(krt_comm* c, CommView* v) {
  if (!c) return set_error(KRT_ERR_INVALID, "communicator is NULL");
  if (!c->peers_open) return set_error(KRT_ERR_INVALID, "communicator peers are not open (krt_comm_open_peers)");
  std::memset(v, 0, sizeof(*v));
  v->rank = c->rank;
  v->world = c->world;
  v->L = c->L;
  for (int q = 0; q < c->world; ++q) v->base[q] = c->peer[q];
  return KRT_OK;
}
}  // namespace

extern "C" int krt_allreduce(krt_comm* c, const void* send, void* recv, size_t count, int32_t dtype, void* status,
                             void* stream) {
  CommView v;
  int rc = comm_view(c, &v);
  if (rc) return rc;
  if (!send || !recv || !status) return set_error(KRT_ERR_INVALID, "krt_allreduce: NULL buffer");
  if (dtype == 0) dtype = KRT_DTYPE_FLOAT32;  // the mock backend's fp32 code (tests/mock_rccl.h:14)
  if (dtype != KRT_DTYPE_FLOAT32 && dtype != KRT_DTYPE_BFLOAT16)
    return set_error(KRT_ERR_UNSUPPORTED, "krt_allreduce: float32 and bfloat16 only");
  const size_t esize = dtype == KRT_DTYPE_FLOAT32 ? 4 : 2;
  if (c->nccl && count * esize >= c->nccl_threshold) {
    ncclResult_t r = nccl_api().all_reduce(send, recv, count, dtype == KRT_DTYPE_FLOAT32 ? ncclFloat32 : ncclBfloat16,
                                           ncclSum, c->nccl, (cudaStream_t)stream);
    if (r != ncclSuccess) return nccl_error(r, "krt_allreduce: ncclAllReduce");
    return clear_error();
  }
  // Elements per launch: staging holds world rows of (slice + count) floats,
  // the result area holds count elements.
  const size_t stg_bytes = v.L.result_off - v.L.staging_off;
  const size_t res_bytes = v.L.part_flag_off - v.L.result_off;
  size_t seg = res_bytes / esize;
  const size_t by_stage = stg_bytes / (sizeof(float) * (size_t)v.world);
  if (seg > by_stage) seg = by_stage;
  cudaStream_t s = (cudaStream_t)stream;
  for (size_t off = 0; off < count; off += seg) {
    const long long n = (long long)((count - off) < seg ? (count - off) : seg);
    int ctas = (int)((n + 4095) / 4096);
    if (ctas < 1) ctas = 1;
    if (ctas > kArMaxCtas) ctas = kArMaxCtas;
    if (dtype == KRT_DTYPE_FLOAT32)
      allreduce_kernel<float><<<ctas, kArThreads, 0, s>>>(static_cast<const float*>(send) + off,
                                                          static_cast<float*>(recv) + off, n, v,
                                                          static_cast<int*>(status));
    else
      allreduce_kernel<__nv_bfloat16><<<ctas, kArThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(send) + off, static_cast<__nv_bfloat16*>(recv) + off, n, v,
          static_cast<int*>(status));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "krt_allreduce launch");
  }
  (void)esize;
  return clear_error();
}

// ------------------------------------------------------ fused GEMM + allreduce
namespace {

int env_int_value(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v && *v) ? std::atoi(v) : dflt;
}

int gemm_stages(int tile_m, int n_pad, int kc, int splits) {
  const size_t cap = (size_t)env_int_value("KRT_SMEM_CAP_KB", 227) * 1024;
  for (int st = kMaxStages; st >= 1; --st)
    if (gemm_ar_smem_bytes(tile_m, st, n_pad, kc, splits) <= cap) return st;
  return 0;
}

// Box depth with the most weight bytes in flight, leaving every split at
// least one box of the K range; a 64-column box gives way to a 128-column
// one that still double-buffers and keeps two thirds of its bytes in
// flight, because one box costs an mbarrier round trip and an MMA issue
// either way (B200, 128 tokens, 4 splits: K = 14336 -> 4096 down projection
// 33.2 us with 64-column boxes in 5 stages, 31.3 us with 128-column boxes
// in 2; K = 4096 o projection 15.1 -> 13.8 us).
int gemm_kc(int tile_m, int num_kb, int n_pad, int splits) {
  const int forced = env_int_value("KRT_GEMM_KC", 0);  // box depth for tuning
  if ((forced == 1 || forced == 2 || forced == 4) && num_kb % forced == 0 && num_kb / forced >= splits &&
      gemm_stages(tile_m, n_pad, forced, splits) >= 1)
    return forced;
  int best = 1;
  size_t best_bytes = 0;
  for (int kc = 4; kc >= 1; kc >>= 1) {
    if (num_kb % kc != 0 || num_kb / kc < splits) continue;
    const size_t bytes = (size_t)gemm_stages(tile_m, n_pad, kc, splits) * kc * tile_m * 128;
    if (bytes > best_bytes) {
      best_bytes = bytes;
      best = kc;
    }
  }
  if (best == 1 && num_kb % 2 == 0 && num_kb / 2 >= splits) {
    const int st2 = gemm_stages(tile_m, n_pad, 2, splits);
    if (st2 >= 2 && (size_t)st2 * 2 * tile_m * 128 * 3 >= best_bytes * 2) best = 2;
  }
  return best;
}

struct GemmCfg {
  int tile_m, tiles, kc, stages, splits;
};

// Tile height 128; 64 (twice the tiles, half the K splits and half the
// exchange per split, but every tile re-reads X) is slower at every decode
// shape measured on B200 (K = 512 .. 14336, N = 4096, 64 tokens) and only
// runs when KRT_GEMM_TILE_M=64 asks for it.  Split-K factor = cluster size:
// as many splits as fit (tiles * splits <= #SMs, at most 8, on one GPU at
// least four 64-column blocks each) while every cluster can be resident at
// once.
// KRT_GEMM_SPLITS overrides the split factor.
GemmCfg gemm_config(int n_out, int num_kb, int n_pad, int world) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, GemmCfg> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, n_out, num_kb, n_pad, world);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int tile_m = env_int_value("KRT_GEMM_TILE_M", 128);
  if (tile_m != 64) tile_m = 128;
  const int tiles = n_out / tile_m;
  GemmCfg cfg{tile_m, tiles, 1, 1, 1};
  const int forced = env_int_value("KRT_GEMM_SPLITS", 0);
  int s = forced > 0 ? forced : device_sm_count() / tiles;
  if (s > 8) s = 8;
  // On one GPU, at least four 64-column blocks per split: shorter K ranges
  // gain less streaming time than their partial exchange costs (B200,
  // K = 512, N = 4096, 64 tokens: 2 splits 5.2 us, 4 splits 5.9 us).  With
  // a fused allreduce, fewer splits leave each CTA more chunks to exchange
  // across GPUs one after another (8 GPUs, K = 512: 2 splits 19.6 us,
  // 4 splits 14.1 us), so all splits stay.
  if (forced <= 0 && world == 1 && s > num_kb / 4) s = num_kb / 4 > 0 ? num_kb / 4 : 1;
  if (s < 1) s = 1;
  for (; s >= 1; --s) {
    const int kc = gemm_kc(tile_m, num_kb, n_pad, s);
    const int st = gemm_stages(tile_m, n_pad, kc, s);
    if (st < 1 || s > num_kb / kc) continue;
    cfg = GemmCfg{tile_m, tiles, kc, st, s};
    if (forced > 0 || s == 1 || gemm_ar_max_active_clusters(tile_m, s, n_pad, st, kc) >= tiles) break;
  }
  cache[key] = cfg;
  return cfg;
}

// Large token counts without the fused exchange (one GPU, or the NCCL route):
// the persistent projection kernel over token blocks (tile = 128 output
// features x 256 tokens, or 128 when 256-token blocks would leave SMs idle;
// row tiles fastest, two TMEM accumulators), y = bf16(x W^T + residual).  The
// 256-token slices of the decode-shaped kernel re-stream the whole weight
// shard per slice; here the CTAs of one round walk W together and share it
// through L2.  Taken when the tiles cover at least half the SMs
// (KRT_GEMM_LARGE_T=0 keeps the slices).
int gemm_large_t_block(const krt_gemm_ar_args* a) {
  const long long row_tiles = a->n_out / 128, sms = device_sm_count();
  if (row_tiles * ((a->num_tokens + 255) / 256) >= sms) return 256;
  return 128;
}

bool gemm_large_t_eligible(const krt_gemm_ar_args* a) {
  if (a->num_tokens <= 256 || env_int_value("KRT_GEMM_LARGE_T", 1) == 0) return false;
  const int bs = gemm_large_t_block(a);
  const long long tiles = (long long)(a->n_out / 128) * ((a->num_tokens + bs - 1) / bs);
  return 2 * tiles >= device_sm_count();
}

// y32 != nullptr: fp32 [T, n_out] out instead of bf16 y (no residual).
int gemm_large_t(const krt_gemm_ar_args* a, const void* residual, float* y32, int* status, cudaStream_t s) {
  PagedParams q;
  std::memset(&q, 0, sizeof(q));
  q.num_tokens = a->num_tokens;
  q.n_pad = gemm_large_t_block(a);
  q.d_model = a->k_local;
  q.status = status;
  q.epi = kEpiStore;
  q.y = static_cast<__nv_bfloat16*>(a->y);
  q.y_stride = y32 ? a->n_out : a->y_stride;
  q.y32 = y32;
  q.residual = y32 ? nullptr : static_cast<const __nv_bfloat16*>(residual);
  q.row_tiles = a->n_out / 128;
  const size_t cap = (size_t)env_int_value("KRT_SMEM_CAP_KB", 227) * 1024;
  const size_t budget = cap - proj_persistent_smem_bytes(0, 1, q.n_pad);
  const size_t stage1 = 16384 + (size_t)q.n_pad * 128;
  q.kc = (a->k_local / 64) % 2 == 0 && budget / (2 * stage1) >= 3 ? 2 : 1;
  q.stages = (int)(budget / (q.kc * stage1));
  if (q.stages > 8) q.stages = 8;
  if (q.stages < 2) return set_error(KRT_ERR_UNSUPPORTED, "krt_rowparallel_gemm_ar: shared memory too small");
  q.tmem_cols = 2 * q.n_pad;
  CUtensorMap tmap_w, tmap_x;
  int rc = make_tmap_bf16_3d(&tmap_w, a->weight, (uint64_t)a->n_out, (uint64_t)a->k_local, (uint64_t)a->k_local, 128,
                             (uint32_t)q.kc);
  if (rc) return rc;
  rc = make_tmap_bf16_3d(&tmap_x, a->x, (uint64_t)a->num_tokens, (uint64_t)a->k_local, (uint64_t)a->x_stride,
                         (uint32_t)q.n_pad, (uint32_t)q.kc);
  if (rc) return rc;
  const int tiles = q.row_tiles * ((a->num_tokens + q.n_pad - 1) / q.n_pad);
  cudaError_t e = launch_proj_persistent(tmap_w, tmap_x, q, tiles, s);
  if (e != cudaSuccess) return cuda_error(e, "krt_rowparallel_gemm_ar launch");
  return KRT_OK;
}

// One launch per 256 tokens of the decode-shaped GEMM (+ exchange when
// p.comm.world > 1).  Every slice's parameters and tensor maps are built
// before the first launch: with a communicator, every rank must make the same
// launches (the exchange epochs count them), so a call that fails on the host
// fails before any of its kernels run.  y32 != nullptr: fp32 [T, n_out] out
// (world 1, no residual).
struct GemmSlice {
  GemmArParams p;
  GemmCfg cfg;
  CUtensorMap tmap_w, tmap_x;
};
int build_gemm_slices(const krt_gemm_ar_args* a, const void* residual, float* y32, const GemmArParams& base,
                      std::vector<GemmSlice>& slices) {
  const int num_kb = a->k_local / 64;
  slices.reserve((size_t)(a->num_tokens + 255) / 256);
  for (int t0 = 0; t0 < a->num_tokens; t0 += 256) {
    const int T = (a->num_tokens - t0) < 256 ? (a->num_tokens - t0) : 256;
    GemmSlice sl;
    sl.p = base;
    sl.p.num_tokens = T;
    sl.p.n_pad = (T + 15) / 16 * 16;
    sl.cfg = gemm_config(a->n_out, num_kb, sl.p.n_pad, base.comm.world);
    sl.p.kc = sl.cfg.kc;
    sl.p.stages = sl.cfg.stages;
    sl.p.splits = sl.cfg.splits;
    // L2 prefetch of weight stages ahead of the ring: off by default (it
    // shortens o_proj alone, 10.7 -> 10.3 us, but lengthens the chained
    // decoder-layer step); KRT_L2_PREFETCH_STAGES turns it on.
    sl.p.prefetch = env_int_value("KRT_L2_PREFETCH_STAGES", 0);
    int cols = 32;
    while (cols < sl.p.n_pad) cols <<= 1;
    sl.p.tmem_cols = cols;
    sl.p.y = static_cast<__nv_bfloat16*>(a->y) + (size_t)t0 * a->y_stride;
    sl.p.y32 = y32 ? y32 + (size_t)t0 * a->n_out : nullptr;
    sl.p.residual = residual && !y32 ? static_cast<const __nv_bfloat16*>(residual) + (size_t)t0 * a->y_stride
                                     : nullptr;
    const void* xp = static_cast<const __nv_bfloat16*>(a->x) + (size_t)t0 * a->x_stride;
    int rc = make_tmap_bf16_3d(&sl.tmap_w, a->weight, (uint64_t)a->n_out, (uint64_t)a->k_local,
                               (uint64_t)a->k_local, (uint32_t)sl.cfg.tile_m, (uint32_t)sl.p.kc);
    if (rc) return rc;
    rc = make_tmap_bf16_3d(&sl.tmap_x, xp, (uint64_t)T, (uint64_t)a->k_local, (uint64_t)a->x_stride,
                           (uint32_t)sl.p.n_pad, (uint32_t)sl.p.kc);
    if (rc) return rc;
    slices.push_back(sl);
  }
  return KRT_OK;
}

// This GPU's product alone, any token count: bf16 y (+ residual), or fp32
// y32 [T, n_out] (no residual).
int gemm_local(const krt_gemm_ar_args* a, const void* residual, float* y32, int* status, cudaStream_t s) {
  if (gemm_large_t_eligible(a)) return gemm_large_t(a, residual, y32, status, s);
  GemmArParams p;
  std::memset(&p, 0, sizeof(p));
  p.comm.world = 1;
  p.comm.rank = 0;
  p.n_out = a->n_out;
  p.k_local = a->k_local;
  p.y_stride = a->y_stride;
  p.status = status;
  std::vector<GemmSlice> slices;
  int rc = build_gemm_slices(a, residual, y32, p, slices);
  if (rc) return rc;
  for (const GemmSlice& sl : slices) {
    cudaError_t e = launch_rowparallel_gemm_ar(sl.cfg.tile_m, sl.tmap_w, sl.tmap_x, sl.p, sl.cfg.tiles, s);
    if (e != cudaSuccess) return cuda_error(e, "krt_rowparallel_gemm_ar launch");
  }
  return KRT_OK;
}

// y[t, n] = bf16(y32[t, n] + residual[t, n]): the NCCL route's single
// rounding, eight features per thread (16-byte loads and stores).
__global__ void __launch_bounds__(256) nccl_finish_kernel(const float* __restrict__ y32,
                                                          const __nv_bfloat16* __restrict__ residual,
                                                          __nv_bfloat16* __restrict__ y, int T, int n_out,
                                                          int y_stride) {
  const long long groups = (long long)T * (n_out / 8);
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(g / (n_out / 8));
    const int n = (int)(g % (n_out / 8)) * 8;
    const float4* src = reinterpret_cast<const float4*>(y32 + (size_t)t * n_out + n);
    float v[8];
    const float4 a0 = src[0], a1 = src[1];
    v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
    v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    if (residual) {
      const uint4 r = *reinterpret_cast<const uint4*>(residual + (size_t)t * y_stride + n);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(b2[q]);
        v[2 * q] += f.x;
        v[2 * q + 1] += f.y;
      }
    }
    *reinterpret_cast<uint4*>(y + (size_t)t * y_stride + n) =
        make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

cudaError_t launch_nccl_finish(const float* y32, const __nv_bfloat16* residual, __nv_bfloat16* y, int T, int n_out,
                               int y_stride, cudaStream_t s) {
  const long long groups = (long long)T * (n_out / 8);
  long long blocks = (groups + 255) / 256;
  const long long cap = 4LL * device_sm_count();
  if (blocks > cap) blocks = cap;
  nccl_finish_kernel<<<(unsigned)blocks, 256, 0, s>>>(y32, residual, y, T, n_out, y_stride);
  return cudaGetLastError();
}

}  // namespace

extern "C" size_t krt_rowparallel_gemm_ar_workspace_size(void) { return kWsHeaderBytes; }

extern "C" int krt_rowparallel_gemm_ar(krt_comm* c, const krt_gemm_ar_args* a, void* stream) {
  if (!a) return set_error(KRT_ERR_INVALID, "krt_rowparallel_gemm_ar: args is NULL");
  if (!a->x || !a->weight || !a->y) return set_error(KRT_ERR_INVALID, "krt_rowparallel_gemm_ar: NULL tensor");
  if (a->num_tokens <= 0 || a->k_local <= 0 || a->n_out <= 0)
    return set_error(KRT_ERR_INVALID, "krt_rowparallel_gemm_ar: num_tokens, k_local and n_out must be positive");
  if (a->k_local % 64 != 0) return set_error(KRT_ERR_UNSUPPORTED, "krt_rowparallel_gemm_ar: k_local % 64 != 0");
  if (a->n_out % 128 != 0) return set_error(KRT_ERR_UNSUPPORTED, "krt_rowparallel_gemm_ar: n_out % 128 != 0");
  if (a->x_stride < a->k_local || a->x_stride % 8 != 0 || a->y_stride < a->n_out || a->y_stride % 8 != 0)
    return set_error(KRT_ERR_INVALID, "krt_rowparallel_gemm_ar: strides must cover the rows and be multiples of 8");
  if ((reinterpret_cast<uintptr_t>(a->x) & 15) || (reinterpret_cast<uintptr_t>(a->weight) & 15) ||
      (reinterpret_cast<uintptr_t>(a->y) & 15))
    return set_error(KRT_ERR_INVALID, "krt_rowparallel_gemm_ar: tensors must be 16-byte aligned");
  if (!a->workspace || a->workspace_bytes < kWsHeaderBytes)
    return set_error(KRT_ERR_WORKSPACE, "krt_rowparallel_gemm_ar: workspace of %zu bytes, %zu needed",
                     a->workspace_bytes, (size_t)kWsHeaderBytes);
  if (a->residual && (reinterpret_cast<uintptr_t>(a->residual) & 15))
    return set_error(KRT_ERR_INVALID, "krt_rowparallel_gemm_ar: residual must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  int* status = static_cast<int*>(a->workspace);
  // Large outputs with an NCCL communicator attached: per slice of up to
  // kNcclSliceTokens tokens the GEMM writes this rank's fp32 partial into the
  // communicator's buffer, one ncclAllReduce sums the partials in fp32, and
  // nccl_finish_kernel adds the residual and rounds to bf16 once (bf16
  // partials can miss the bf16 tolerance where partials cancel).  Every rank
  // takes the same route (same sizes, same threshold).
  const bool via_nccl = c && c->world > 1 && c->nccl && c->nccl_f32 &&
                        (size_t)a->num_tokens * a->n_out * 2 >= c->nccl_threshold;
  if (via_nccl) {
    if (a->n_out > c->max_n)
      return set_error(KRT_ERR_UNSUPPORTED, "krt_rowparallel_gemm_ar: n_out %d exceeds the communicator's %d",
                       a->n_out, c->max_n);
    for (int t0 = 0; t0 < a->num_tokens; t0 += kNcclSliceTokens) {
      krt_gemm_ar_args sub = *a;
      sub.num_tokens = a->num_tokens - t0 < kNcclSliceTokens ? a->num_tokens - t0 : kNcclSliceTokens;
      sub.x = static_cast<const __nv_bfloat16*>(a->x) + (size_t)t0 * a->x_stride;
      sub.y = static_cast<__nv_bfloat16*>(a->y) + (size_t)t0 * a->y_stride;
      sub.residual = a->residual ? static_cast<const __nv_bfloat16*>(a->residual) + (size_t)t0 * a->y_stride
                                 : nullptr;
      int rc = gemm_local(&sub, nullptr, c->nccl_f32, status, s);
      if (rc) return rc;
      const size_t count = (size_t)sub.num_tokens * a->n_out;
      ncclResult_t r = nccl_api().all_reduce(c->nccl_f32, c->nccl_f32, count, ncclFloat32, ncclSum, c->nccl, s);
      if (r != ncclSuccess) return nccl_error(r, "krt_rowparallel_gemm_ar: ncclAllReduce");
      cudaError_t e = launch_nccl_finish(c->nccl_f32, static_cast<const __nv_bfloat16*>(sub.residual),
                                         static_cast<__nv_bfloat16*>(sub.y), sub.num_tokens, a->n_out, a->y_stride, s);
      if (e != cudaSuccess) return cuda_error(e, "krt_rowparallel_gemm_ar: finish launch");
    }
    return clear_error();
  }
  if (!c || c->world == 1) {
    int rc = gemm_local(a, a->residual, nullptr, status, s);
    return rc ? rc : clear_error();
  }
  // The fused exchange, in launches of up to 256 tokens.
  GemmArParams p;
  std::memset(&p, 0, sizeof(p));
  int rc = comm_view(c, &p.comm);
  if (rc) return rc;
  if (a->n_out > c->max_n)
    return set_error(KRT_ERR_UNSUPPORTED, "krt_rowparallel_gemm_ar: n_out %d exceeds the communicator's %d",
                     a->n_out, c->max_n);
  p.n_out = a->n_out;
  p.k_local = a->k_local;
  p.y_stride = a->y_stride;
  p.status = status;
  std::vector<GemmSlice> slices;
  rc = build_gemm_slices(a, a->residual, nullptr, p, slices);
  if (rc) return rc;
  for (const GemmSlice& sl : slices) {
    cudaError_t e = launch_rowparallel_gemm_ar(sl.cfg.tile_m, sl.tmap_w, sl.tmap_x, sl.p, sl.cfg.tiles, s);
    if (e != cudaSuccess) return cuda_error(e, "krt_rowparallel_gemm_ar launch");
  }
  return clear_error();
}

// ------------------------------------------------------ greedy sampling
extern "C" int krt_greedy_step(krt_comm* c, const krt_greedy_step_args* a, void* stream) {
  const char* name = "krt_greedy_step";
  if (!a) return set_error(KRT_ERR_INVALID, "%s: args is NULL", name);
  if (!a->argmax_keys || !a->tokens || !a->status) return set_error(KRT_ERR_INVALID, "%s: NULL buffer", name);
  if (a->num_seqs <= 0 || a->num_seqs > kMaxGreedySeqs)
    return set_error(KRT_ERR_UNSUPPORTED, "%s: num_seqs must be in 1..%d", name, kMaxGreedySeqs);
  if (a->vocab <= 0 || a->vocab > (1 << 17))
    return set_error(KRT_ERR_UNSUPPORTED, "%s: vocab must be in 1..131072", name);
  if (a->embedding) {
    if (!a->hidden) return set_error(KRT_ERR_INVALID, "%s: hidden is NULL", name);
    if (a->d_model <= 0 || a->d_model % 8 != 0 || a->hidden_stride < a->d_model || a->hidden_stride % 8 != 0 ||
        (reinterpret_cast<uintptr_t>(a->embedding) & 15) || (reinterpret_cast<uintptr_t>(a->hidden) & 15))
      return set_error(KRT_ERR_INVALID, "%s: embedding rows and hidden must be 16-byte aligned, d_model % 8 == 0",
                       name);
  }
  GreedyParams g;
  g.keys = a->argmax_keys;
  g.tokens = a->tokens;
  g.embedding = static_cast<const __nv_bfloat16*>(a->embedding);
  g.hidden = static_cast<__nv_bfloat16*>(a->hidden);
  g.positions = a->positions;
  g.seq_lens = a->seq_lens;
  g.next_input = a->next_input;
  g.status = static_cast<int*>(a->status);
  g.num_seqs = a->num_seqs;
  g.d_model = a->d_model;
  g.hidden_stride = a->hidden_stride;
  g.vocab = a->vocab;
  CommView v;
  if (c) {
    int rc = comm_view(c, &v);
    if (rc) return rc;
  } else {
    std::memset(&v, 0, sizeof(v));
    v.world = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a->num_seqs, 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, greedy_step_kernel, g, v);
  if (e != cudaSuccess) return cuda_error(e, name);
  return clear_error();
}
