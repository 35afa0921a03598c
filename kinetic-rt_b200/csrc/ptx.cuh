// Inline-PTX building blocks for sm_100a: mbarriers, TMA tile loads,
// tcgen05 (TMEM allocation, UMMA issue, commit, TMEM loads) and bounded waits.
//
// Every wait in this file is bounded by wall-clock time (%globaltimer).  A
// wait that runs out returns false; callers record an error code and leave
// their loop, so a broken producer/consumer protocol ends the kernel with an
// error status instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace krt {

// Error codes written to the device status word.
enum : int {
  kStatusOk = 0,
  kStatusTimeoutFull = 1,     // consumer gave up waiting for a full stage
  kStatusTimeoutEmpty = 2,    // producer gave up waiting for a free stage
  kStatusTimeoutAccum = 4,    // epilogue gave up waiting for the accumulator
  kStatusBadBlock = 8,        // paged scatter: block id / position outside the pool
  kStatusTimeoutPeer = 16,    // cross-GPU flag wait ran out
  kStatusBadSplit = 32,       // split-K bookkeeping inconsistent
  kStatusTimeoutCluster = 64, // split-K partials of the other CTAs (cluster or stream-K runs) did not arrive
};

// Wall-clock budget for any single wait: 2 s.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait until the phase with the given parity has completed, or give up after
// kWaitBudgetNs or as soon as *abort becomes non-zero.  Returns true on success.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && *abort) return false;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

// Make generic-proxy writes to shared memory visible to the async proxy
// (tensor cores and TMA read shared memory through it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// 2-D tile load with an L2 cache policy (from make_l2_policy_*).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                                 int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// 3-D tile load with an L2 cache policy (from make_l2_policy_*).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_5d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "l"(policy)
      : "memory");
}
// Bulk tensor prefetch of one box into L2 (no shared memory, no completion
// tracking): it only raises the bytes in flight ahead of the loads.
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(map), "r"(c0), "r"(c1),
               "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_l2_5d(const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4) {
  asm volatile("cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(c2), "r"(c3), "r"(c4)
               : "memory");
}
__device__ __forceinline__ uint64_t make_l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t make_l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ----------------------------------------------------------------- tcgen05
// TMEM allocation is warp-collective; the base address is written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
// Issued by a single thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(m0), "r"(m1), "r"(m2), "r"(m3)
      : "memory");
}

// Arrive once on an mbarrier when all previously issued tcgen05 ops of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
// 16 columns without waiting: issue several, then one tmem_wait_ld().
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for a K-major bf16 tile whose rows are 128
// bytes (64 elements) and were written with the 128-byte swizzle: 8-row
// groups 1024 bytes apart (SBO), LBO unused, descriptor version 1,
// layout type 2 (SWIZZLE_128B).  The tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // LBO (ignored for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // SBO
  d |= (uint64_t)1 << 46;                 // version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A bf16
         | (1u << 10)                    // B bf16
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also returns the OR of `pred` over the participating
// threads, so a decision taken after it is uniform across them.
__device__ __forceinline__ bool named_bar_any(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// Warp-uniform bounded wait: lane 0 polls, the result is broadcast.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Wait for data that other CTAs of the cluster send into this CTA's shared
// memory.  The senders always send, also after their own failures, so this
// wait ignores the CTA's abort flag (the CTA must not exit while copies may
// still land) and allows two wait budgets, covering a sender that reaches
// its send only after one of its own bounded waits ran out.
__device__ __forceinline__ bool mbar_wait_warp_incoming(uint64_t* bar, uint32_t parity) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, nullptr) || mbar_wait(bar, parity, nullptr);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// ------------------------------------------------------- flagged words
// 8-byte words carrying (epoch << 32) | payload; aligned 8-byte accesses are
// single-copy atomic, so payload and flag arrive together.
__device__ __forceinline__ uint64_t ll_word(uint32_t payload, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | payload;
}
__device__ __forceinline__ void st_ll2(uint64_t* dst, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a), "l"(b) : "memory");
}

// 24-bit float: fp32 rounded to nearest-even at mantissa bit 8 (sign,
// 8-bit exponent, 15-bit mantissa); two of them and a 16-bit epoch fill one
// flagged word: (epoch << 48) | (b << 24) | a.
__device__ __forceinline__ uint64_t f24_pair_word(float a, float b, uint32_t epoch16) {
  auto f24 = [](float v) -> uint64_t {
    const uint32_t u = __float_as_uint(v);
    return (uint64_t)((u + 0x7Fu + ((u >> 8) & 1u)) >> 8) & 0xFFFFFFull;
  };
  return ((uint64_t)epoch16 << 48) | (f24(b) << 24) | f24(a);
}
__device__ __forceinline__ float2 f24_pair_unpack(uint64_t w) {
  return make_float2(__uint_as_float((uint32_t)(w & 0xFFFFFFull) << 8),
                     __uint_as_float((uint32_t)((w >> 24) & 0xFFFFFFull) << 8));
}

// Poll N word pairs at src + stride * i (i < N) until every word carries
// `epoch` in its bits [SHIFT, 64), all N loads issued together per round so a
// round costs one memory latency; out[2i], out[2i+1] receive the words.
// False once the wait budget, counted from t0, is spent.
template <int N, int SHIFT>
__device__ __forceinline__ bool poll_words_batch(const uint64_t* src, int stride, uint32_t epoch, uint64_t t0,
                                                 uint64_t* out) {
  while (true) {
    uint64_t x[N], y[N];
#pragma unroll
    for (int i = 0; i < N; ++i)
      asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];"
                   : "=l"(x[i]), "=l"(y[i])
                   : "l"(src + (size_t)stride * i)
                   : "memory");
    bool all = true;
#pragma unroll
    for (int i = 0; i < N; ++i) all = all && (uint32_t)(x[i] >> SHIFT) == epoch && (uint32_t)(y[i] >> SHIFT) == epoch;
    if (all) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        out[2 * i] = x[i];
        out[2 * i + 1] = y[i];
      }
      return true;
    }
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

// Poll N word pairs at src + stride * i (i < N) until every word carries
// `epoch`, all N loads issued together per round so a round costs one memory
// latency; out[2i], out[2i+1] receive the payloads.  False once the wait
// budget, counted from t0, is spent.
template <int N>
__device__ __forceinline__ bool poll_ll2_batch(const uint64_t* src, int stride, uint32_t epoch, uint64_t t0,
                                               uint32_t* out) {
  while (true) {
    uint64_t x[N], y[N];
#pragma unroll
    for (int i = 0; i < N; ++i)
      asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];"
                   : "=l"(x[i]), "=l"(y[i])
                   : "l"(src + (size_t)stride * i)
                   : "memory");
    bool all = true;
#pragma unroll
    for (int i = 0; i < N; ++i) all = all && (uint32_t)(x[i] >> 32) == epoch && (uint32_t)(y[i] >> 32) == epoch;
    if (all) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        out[2 * i] = (uint32_t)x[i];
        out[2 * i + 1] = (uint32_t)y[i];
      }
      return true;
    }
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

// ----------------------------------------------------------------- cluster
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Split cluster barrier: arrive early (after the mbarrier inits), wait
// later, right before the first access to another CTA's shared memory.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Bulk copy of `bytes` (multiple of 16, 16-byte aligned ends) from this
// CTA's shared memory to shared memory of another CTA of the cluster; the
// transfer completes `bytes` of transaction count on the mbarrier at
// `mbar_cluster` (an address in the destination CTA).
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, uint32_t src_smem, uint32_t bytes,
                                                     uint32_t mbar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(src_smem), "r"(bytes), "r"(mbar_cluster)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the source buffers of all committed bulk copies have been read.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_smem_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// ------------------------------------------------------- cross-GPU flags
// Flags live in symmetric buffers that peers write over NVLink.  A producer
// fences its data stores system-wide, then releases the flag; the consumer
// acquires it.  Waits are bounded by kWaitBudgetNs.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Wait until *flag == expect; false after kWaitBudgetNs.
__device__ __forceinline__ bool wait_flag_sys(const uint32_t* flag, uint32_t expect) {
  if (ld_acquire_sys(flag) == expect) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_sys(flag) == expect) return true;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
    __nanosleep(64);
  }
}

// The same between CTAs of one GPU (device scope).
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool wait_flag_gpu(const uint32_t* flag, uint32_t expect) {
  if (ld_acquire_gpu(flag) == expect) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_gpu(flag) == expect) return true;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
    __nanosleep(32);
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace krt
