// Symmetric peer buffers shared by the fused row-parallel GEMM + allreduce
// and the standalone allreduce.
//
// Every rank allocates one device buffer with the same layout, exports it as
// a CUDA IPC handle, and maps every peer's buffer into its own address space
// (krt_comm_open_peers).  Kernels then write partial sums and flags straight
// into peers' buffers over NVLink / NVSwitch with ordinary stores; no TMA or
// multicast load ever reads peer memory.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_bf16.h>

namespace krt {

constexpr int kMaxWorld = 8;
constexpr int kArMaxCtas = 64;     // CTAs of the standalone allreduce
constexpr int kMaxChunks = 16;     // 256 tokens per launch
constexpr int kMaxGreedySeqs = 1024;  // sequences per krt_greedy_step call

struct CommLayout {
  int world, max_n, tiles;
  size_t staging_off;      // fp32 [world][tiles][kMaxChunks][16 * 128]
  size_t result_off;       // [256][max_n] bf16 (fused) / raw bytes (standalone)
  size_t part_flag_off;    // u32 [tiles][kMaxChunks][kMaxWorld]
  size_t final_flag_off;   // u32 [tiles][kMaxChunks]
  size_t ar_part_off;      // u32 [kArMaxCtas][kMaxWorld]
  size_t ar_final_off;     // u32 [kMaxWorld][kArMaxCtas]
  // Fused GEMM + allreduce exchange in flagged 8-byte words, each written
  // with one 8-byte store and carrying the epoch of its (tile, chunk), so a
  // reader that sees the current epoch in a word also sees its payload and
  // no fence or separate flag is needed:
  //   stage words  (epoch << 48) | two 24-bit floats (fp32 rounded at bit 8)
  //   result words (epoch << 32) | bf16x2
  // Slots are laid out [word pair][finishing thread] (16 bytes per thread
  // and pair), so a warp's store covers 512 contiguous bytes.  One set of
  // areas per tile height (index 0: 128 rows, 1: 64 rows), so the slots and
  // epochs of the two tilings never alias.
  // Two ranks exchange one-shot (each rank sends its whole partial to the
  // other and both reduce), so their stage holds every tile, twice: uses of
  // a (tile, chunk) alternate between the two copies by epoch parity, since
  // nothing tells a sender that its peer has finished reading the previous
  // use (a rank runs at most one launch ahead of the other).  More ranks
  // reduce-scatter, and a rank's stage holds only the tiles it owns.
  size_t ll_stage_off[2];   // [world (source)][stage tiles][kMaxChunks][rows/32 pairs][128 threads]
  size_t ll_result_off[2];  // [tiles][kMaxChunks][rows/32 pairs][128 threads]
  size_t epoch_off[2];      // u32 [tiles][kMaxChunks] uses of each (tile, chunk), cycling 1..65534
  // Greedy sampling across vocabulary shards: per sequence one flagged word
  // (15-bit epoch << 49 | 49-bit (logit, index) key) from every rank, in
  // two copies alternating by epoch parity; per-sequence epoch counters.
  size_t greedy_off;        // u64 [2][kMaxWorld (source)][kMaxGreedySeqs]
  size_t greedy_epoch_off;  // u32 [kMaxGreedySeqs]
  int owned_tiles[2];       // ceil(tiles / world): tile t is reduced by rank t % world
  int stage_tiles[2];       // tile slots per source: 2 x all tiles (world 2) or the owned ones
  size_t total;
};

inline CommLayout comm_layout(int world, int max_n) {
  auto up = [](size_t v) { return (v + 4095) & ~size_t(4095); };
  CommLayout L;
  L.world = world;
  L.max_n = max_n;
  L.tiles = max_n / 128;
  L.staging_off = 0;
  L.result_off = up(L.staging_off + (size_t)world * L.tiles * kMaxChunks * 16 * 128 * sizeof(float));
  L.part_flag_off = up(L.result_off + (size_t)kMaxChunks * 16 * max_n * 2);
  L.final_flag_off = up(L.part_flag_off + (size_t)L.tiles * kMaxChunks * kMaxWorld * 4);
  L.ar_part_off = up(L.final_flag_off + (size_t)L.tiles * kMaxChunks * 4);
  L.ar_final_off = up(L.ar_part_off + (size_t)kArMaxCtas * kMaxWorld * 4);
  size_t off = up(L.ar_final_off + (size_t)kMaxWorld * kArMaxCtas * 4);
  for (int v = 0; v < 2; ++v) {
    const int rows = v == 0 ? 128 : 64;
    const int tiles = max_n / rows;
    const size_t slot = (size_t)rows * 64;  // bytes: rows/32 pairs x 128 threads x 16
    L.owned_tiles[v] = (tiles + world - 1) / world;
    L.stage_tiles[v] = world == 2 ? 2 * tiles : L.owned_tiles[v];
    L.ll_stage_off[v] = off;
    L.ll_result_off[v] = up(off + (size_t)world * L.stage_tiles[v] * kMaxChunks * slot);
    L.epoch_off[v] = up(L.ll_result_off[v] + (size_t)tiles * kMaxChunks * slot);
    off = up(L.epoch_off[v] + (size_t)tiles * kMaxChunks * 4);
  }
  L.greedy_off = off;
  L.greedy_epoch_off = up(off + (size_t)2 * kMaxWorld * kMaxGreedySeqs * 8);
  off = up(L.greedy_epoch_off + (size_t)kMaxGreedySeqs * 4);
  L.total = off;
  return L;
}

// Device-side view of a communicator: each rank's buffer as mapped here.
struct CommView {
  int rank, world;
  char* base[kMaxWorld];
  CommLayout L;
};

// Launch parameters of the fused row-parallel GEMM + allreduce (gemm_ar.cu).
// Tokens per NCCL-route slice: the communicator's fp32 partial buffer holds
// kNcclSliceTokens x max_n floats.
constexpr int kNcclSliceTokens = 4096;

struct GemmArParams {
  __nv_bfloat16* y;
  float* y32;  // world 1 only: fp32 out [num_tokens, n_out] instead of y (no residual)
  const __nv_bfloat16* residual;  // optional: y = residual + sum (same strides as y; may be y itself)
  int y_stride;
  int num_tokens, n_pad, n_out, k_local;
  int splits, stages, kc, tmem_cols;
  int prefetch;  // weight stages requested into L2 ahead of the shared-memory ring
  int* status;
  CommView comm;
};

}  // namespace krt
