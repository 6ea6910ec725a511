// Block sum in the exact fp32 order of the reference's block reduction.
//
// The reference test kernel `blockReduceSum`
// (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:229-312,
// generated text core/src/test/scala/flight4s/core/codegen/CudaCodegenSuite.scala:133-216)
// sums one 256-element tile with a shared-memory tree:
//     for stride in 128, 64, 32, 16, 8, 4, 2, 1:  s[t] += s[t + stride]  (t < stride)
// This kernel extends it to n elements as a 256-ary tree: level 1 sums each
// 256-element tile (zero padded) in that order and writes one partial per
// tile; level 2 sums each run of 256 tile partials the same way; and so on
// until one value remains.  Every level reproduces the reference's pairing,
// so the result is bit-identical to running the reference kernel level by
// level.
//
// B200 mapping (no shared-memory barriers inside a tile; for arrays above
// 2^23 elements one clustered launch):
//   * one warp owns one tile: lane l holds x[l + 32k], k = 0..7, which are
//     eight coalesced 128-byte rows.  Strides 128/64/32 of the reference are
//     register adds between those eight values, strides 16..1 are
//     __shfl_down_sync steps, so the pairing is unchanged;
//   * a CTA of 1024 threads owns 32 tiles, a cluster of 8 CTAs owns 256
//     tiles = one level-2 node.  Tile partials are written straight into the
//     cluster leader's shared memory through DSMEM; after one cluster barrier
//     the leader's warp 0 computes the level-2 partial;
//   * the last cluster to finish (atomic ticket, no waiting) computes the
//     remaining levels from the level-2 partials in global workspace.
//
// Arrays of up to kBlockSumSmallMaxTiles tiles (2^23 elements) take two
// launches instead and no workspace: a tiles kernel (level 1 only) and a
// one-CTA upper pass (levels 2+) launched as its programmatic dependent, so
// it is already resident when the last tile partial lands.  Same tree, same
// bits.  Measured at n = 2^20 by CUDA-graph replay on B200: empty launch of
// the level-1 shape 0.59 us, level 1 alone 1.72 us, level 1 + the ticket of
// the former one-launch form 2.48 us, that form complete 3.31-3.34 us
// (L2-flushed 4.74-4.84), this pair 3.08-3.21 us (flushed 4.40-4.44).
// Slots polled by the last or a designated CTA instead of a ticket, and a
// one-warp upper pass, measured slower (3.46-4.48 us).
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace f4s {

constexpr int kTile = 256;
constexpr int kBlockSumThreads = 1024;
constexpr int kBlockSumWarps = kBlockSumThreads / kWarp;    // 32 tiles per CTA
constexpr int kBlockSumCluster = 8;                         // 256 tiles per cluster
// Workspace layout: [0,4) ticket; level-2 partials from byte 256.
constexpr int kBlockSumLevel2Offset = 256;
// Largest tile count of the two-launch form: its upper pass holds the
// level-2 nodes (one per 256 tiles) in a 256-entry shared array.
constexpr unsigned kBlockSumSmallMaxTiles = 128u * kTile;
constexpr int kBlockSumUpperThreads = 512;

// One 256-ary tree node in the reference order; `v[k]` = element
// (lane + 32k) of the node's 256 inputs.  Returns the node value in lane 0.
__device__ __forceinline__ float tree256(const float (&v)[8]) {
  // strides 128 and 64 and 32 (element t pairs with t + stride)
  const float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
  const float b0 = a0 + a2, b1 = a1 + a3;
  float c = b0 + b1;
  // strides 16..1 inside the warp
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) c += __shfl_down_sync(0xffffffffu, c, s);
  return c;
}

// Warp-cooperative: reduce `count` values at `src` (global or shared) into
// ceil(count/256) node values at dst[], one node per warp, warps striding.
__device__ __forceinline__ void tree_level(const float* src, unsigned count, float* dst,
                                           int warp, int lane, int nwarps, bool from_global) {
  const unsigned nodes = (count + kTile - 1) / kTile;
  for (unsigned node = warp; node < nodes; node += nwarps) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const unsigned i = node * kTile + lane + 32 * k;
      v[k] = (i < count) ? (from_global ? __ldcg(src + i) : src[i]) : 0.0f;
    }
    const float r = tree256(v);
    if (lane == 0) dst[node] = r;
  }
}

__device__ __forceinline__ unsigned ticket_acq_rel(unsigned* ticket) {
  unsigned prior;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prior) : "l"(ticket) : "memory");
  return prior;
}

}  // namespace f4s

// (in, n, partials[ceil(n/256)], out[1], workspace).  Launch with
// blockDim 1024, cluster (8,1,1), grid = 8 * max(1, ceil(n / 65536)).
extern "C" __global__ void __launch_bounds__(f4s::kBlockSumThreads)
f4s_block_reduce_sum_f32(const float* __restrict__ in, int n, float* __restrict__ partials,
                         float* __restrict__ out, unsigned char* __restrict__ workspace) {
  namespace cg = cooperative_groups;
  using namespace f4s;
  const cg::cluster_group cluster = cg::this_cluster();
  __shared__ float tile_sums[kBlockSumWarps * kBlockSumCluster];  // leader only
  __shared__ float level_a[kTile];
  __shared__ float level_b[kTile];
  __shared__ int is_last;

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const unsigned rank = cluster.block_rank();
  const unsigned tiles = (static_cast<unsigned>(n) + kTile - 1) / kTile;
  const unsigned tile = blockIdx.x * kBlockSumWarps + warp;

  // level 1: one tile per warp (zero padded past n)
  float v[8];
  const size_t tile_base = static_cast<size_t>(tile) * kTile;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const size_t i = tile_base + lane + 32 * k;
    v[k] = (tile < tiles && i < static_cast<size_t>(n)) ? __ldcs(in + i) : 0.0f;
  }
  const float tile_sum = tree256(v);
  if (lane == 0) {
    if (tile < tiles) partials[tile] = tile_sum;
    *cluster.map_shared_rank(&tile_sums[rank * kBlockSumWarps + warp], 0) = tile_sum;
  }
  cluster.sync();
  if (rank != 0) return;

  // level 2 on the cluster leader: tiles [256c, 256c + 256)
  const unsigned cluster_id = blockIdx.x / kBlockSumCluster;
  const unsigned num_clusters = gridDim.x / kBlockSumCluster;
  unsigned int* ticket = reinterpret_cast<unsigned int*>(workspace);
  float* level2 = reinterpret_cast<float*>(workspace + kBlockSumLevel2Offset);
  if (warp == 0) {
    // Padding tiles past `tiles` already hold +0.0 from zero-filled loads.
    float w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = tile_sums[lane + 32 * k];
    // A single tile is already the final value: the tree stops at one value.
    const float node = (tiles <= 1) ? w[0] : tree256(w);
    if (lane == 0) {
      level2[cluster_id] = node;
      // One acquire-release RMW orders this cluster's level-2 store before
      // its ticket and, for the last arriver, every other cluster's store
      // before its reads (cheaper than a full fence plus a relaxed atomic).
      is_last = (ticket_acq_rel(ticket) == num_clusters - 1) ? 1 : 0;
    }
  }
  __syncthreads();
  if (!is_last) return;

  // remaining levels on the last cluster's leader CTA (the barrier above
  // carries the acquire of thread 0 to the CTA's other threads)
  unsigned count = num_clusters;
  if (count == 1) {
    if (threadIdx.x == 0) {
      out[0] = __ldcg(level2);
      *ticket = 0u;
    }
    return;
  }
  tree_level(level2, count, level_a, warp, lane, kBlockSumWarps, true);
  count = (count + kTile - 1) / kTile;
  float* cur = level_a;
  float* nxt = level_b;
  __syncthreads();
  while (count > 1) {
    tree_level(cur, count, nxt, warp, lane, kBlockSumWarps, false);
    count = (count + kTile - 1) / kTile;
    float* tmp = cur;
    cur = nxt;
    nxt = tmp;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[0] = cur[0];
    *ticket = 0u;
  }
}

// Arrays of up to 2^23 elements: two launches, no workspace.
//
// f4s_block_sum_tiles_f32 (in, n, partials[ceil(n/256)]): level 1, one tile
// per warp.  Launch with blockDim 1024, grid = max(1, ceil(n / 8192)).
// Every CTA first lets the dependent launch start, so the one-CTA upper pass
// below is resident and waiting before the last tile is summed.
extern "C" __global__ void __launch_bounds__(f4s::kBlockSumThreads)
f4s_block_sum_tiles_f32(const float* __restrict__ in, int n, float* __restrict__ partials) {
  using namespace f4s;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const unsigned tiles = (static_cast<unsigned>(n) + kTile - 1) / kTile;
  const unsigned tile = blockIdx.x * kBlockSumWarps + warp;
  float v[8];
  const size_t tile_base = static_cast<size_t>(tile) * kTile;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const size_t i = tile_base + lane + 32 * k;
    v[k] = (tile < tiles && i < static_cast<size_t>(n)) ? __ldcs(in + i) : 0.0f;
  }
  const float tile_sum = tree256(v);
  if (lane == 0 && tile < tiles) partials[tile] = tile_sum;
}

// f4s_block_sum_upper_f32 (partials, n, out): levels 2+ from the tile
// partials, one CTA of kBlockSumUpperThreads.  Launched right after the tiles
// kernel on the same stream as its programmatic dependent: griddepcontrol.wait
// returns once that grid has completed and its partial stores are visible
// (for an ordinary launch it returns at once, the stream having already
// ordered the two).  Nothing is read before the wait.
extern "C" __global__ void __launch_bounds__(f4s::kBlockSumUpperThreads)
f4s_block_sum_upper_f32(const float* __restrict__ partials, int n, float* __restrict__ out) {
  using namespace f4s;
  __shared__ float level_a[kTile];
  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  constexpr int kWarps = kBlockSumUpperThreads / kWarp;
  const unsigned count = (static_cast<unsigned>(n) + kTile - 1) / kTile;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (count <= 1) {  // one tile (or none) is already the final value
    if (threadIdx.x == 0) out[0] = (count == 1) ? __ldcg(partials) : 0.0f;
    return;
  }
  // level 2: one node per warp, from the tile partials in L2
  const unsigned nodes = (count + kTile - 1) / kTile;  // <= 128 for n <= 2^23
  if (nodes == 1) {  // warp 0 holds the final value: no barrier needed
    if (warp == 0) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const unsigned i = lane + 32 * k;
        v[k] = (i < count) ? __ldcg(partials + i) : 0.0f;
      }
      const float r = tree256(v);
      if (lane == 0) out[0] = r;
    }
    return;
  }
  tree_level(partials, count, level_a, warp, lane, kWarps, true);
  __syncthreads();
  // level 3 (the last one: at most 128 nodes) on warp 0
  if (warp == 0) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const unsigned i = lane + 32 * k;
      v[k] = (i < nodes) ? level_a[i] : 0.0f;
    }
    const float r = tree256(v);
    if (lane == 0) out[0] = r;
  }
}
