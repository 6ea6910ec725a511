// Order-fixed ("Deterministic") floating-point sums.
//
// The reference's ReduceSum carries a ReductionPolicy {Strict,
// Deterministic, Fast} (core/src/main/scala/flight4s/core/ir/IR.scala:79-82)
// that its serial codegen never needed to read.  The fast kernels in
// reduce.cuh associate partial sums by launch geometry (grid, cluster size,
// SM count), so the rounding of a floating-point sum can change with the
// device or the number of GPUs.  These kernels fix the association by the
// element index alone:
//
//   tile  = 256 consecutive 16-byte vectors (4 KiB), one warp: lane l sums
//           vectors l + 32u (u = 0..7) with the op's vector arithmetic, then
//           a fixed warp tree (lane 0);
//   group = 64 consecutive tiles (256 KiB): a fixed tree over the 64 tile
//           partials, written to workspace[group];
//   total = F(group partials): thread t (of 512) adds groups t, t + 512, ...
//           in order, then a fixed block tree; plus the unaligned head
//           elements, added in order.
//
// Every partial is a function of its elements only, so the result is the
// same on any grid, cluster size or B200, and -- when each GPU holds whole
// groups of one 16-byte-aligned array -- for any number of GPUs: their
// group partials, concatenated, go through the same F
// (f4s_reduce_ordered_final).  Costs one 8-byte store per 256 KiB of input.
#pragma once

#include "reduce.cuh"

namespace f4s {

constexpr int kOrderedBlock = 512;
constexpr int kOrderedWarps = kOrderedBlock / kWarp;              // 16
constexpr int kTileVectors = kWarp * kReduceUnroll;              // 256 vectors = 4 KiB
constexpr int kGroupTiles = 64;                                  // 256 KiB per group
constexpr int kTilesPerWarp = kGroupTiles / kOrderedWarps;       // 4
constexpr int kOrderedGroupOffset = 256;                         // workspace: [0,4) ticket

// The partial last vector of the body: its `tail` elements followed by
// zeros (built once per thread, kept in registers).
template <class Op>
__device__ __forceinline__ uint4 load_tail_vector(const unsigned char* p, int tail) {
  constexpr int kElem = Op::kElemBytes;
  constexpr int kPerVec = 16 / kElem;
  uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < kPerVec; ++j) {
    if (j < tail) {
      const uint64_t bits = load_element_bits<kElem>(p + j * kElem);
      if constexpr (kElem == 8) {
        w[2 * j] = static_cast<uint32_t>(bits);
        w[2 * j + 1] = static_cast<uint32_t>(bits >> 32);
      } else {
        w[(j * kElem) / 4] |= static_cast<uint32_t>(bits) << (8 * ((j * kElem) % 4));
      }
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// How many of the vectors first + 32u (u < kReduceUnroll) lie below `end`.
__device__ __forceinline__ int lane_vectors(uint64_t first, uint64_t end) {
  if (first >= end) return 0;
  const uint64_t k = (end - first + kWarp - 1) / kWarp;
  return k < kReduceUnroll ? static_cast<int>(k) : kReduceUnroll;
}

// Fixed warp tree: lane 0 receives the sum.
__device__ __forceinline__ double warp_tree_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;
}

// F over `count` group partials, run by one whole CTA of kOrderedBlock
// threads; thread 0 returns the value.
__device__ __forceinline__ double ordered_total(const double* groups, uint64_t count, double* scratch) {
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  double acc = 0.0;
  uint64_t g = tid;
  for (; g + 3 * kOrderedBlock < count; g += 4 * kOrderedBlock) {
    const double a = __ldcg(groups + g), b = __ldcg(groups + g + kOrderedBlock);
    const double c = __ldcg(groups + g + 2 * kOrderedBlock), d = __ldcg(groups + g + 3 * kOrderedBlock);
    acc += a;
    acc += b;
    acc += c;
    acc += d;
  }
  for (; g < count; g += kOrderedBlock) acc += __ldcg(groups + g);
  acc = warp_tree_f64(acc);
  if (lane == 0) scratch[warp] = acc;
  __syncthreads();
  double total = 0.0;
  if (warp == 0) {
    total = warp_tree_f64(lane < kOrderedWarps ? scratch[lane] : 0.0);
  }
  return total;
}

template <class Op>
__device__ __forceinline__ void reduce_ordered(const void* __restrict__ in_ptr, uint64_t n, double* __restrict__ out,
                                               unsigned char* __restrict__ workspace, double* __restrict__ groups,
                                               int accumulate) {
  constexpr int kElem = Op::kElemBytes;
  constexpr int kPerVec = 16 / kElem;
  static_assert(Op::kUnroll == kReduceUnroll, "order-fixed tiles are 8 vectors per lane");
  __shared__ double tile_partials[2][kGroupTiles];
  __shared__ double scratch[kOrderedWarps];
  __shared__ int is_last;

  const unsigned char* in = static_cast<const unsigned char*>(in_ptr);
  const uint64_t addr = reinterpret_cast<uint64_t>(in);
  uint64_t head = ((16u - (addr & 15u)) & 15u) / kElem;
  if (head > n) head = n;
  const unsigned char* body = in + head * kElem;
  const uint64_t nvec_full = (n - head) / kPerVec;
  const int tail = static_cast<int>((n - head) % kPerVec);
  const uint64_t nvec = nvec_full + (tail > 0 ? 1 : 0);
  const uint64_t ntiles = (nvec + kTileVectors - 1) / kTileVectors;
  const uint64_t whole_tiles = nvec_full / kTileVectors;
  const uint64_t ngroups = (ntiles + kGroupTiles - 1) / kGroupTiles;
  unsigned int* ticket = reinterpret_cast<unsigned int*>(workspace);

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const uint4 tail_vec = tail > 0 ? load_tail_vector<Op>(body + nvec_full * 16, tail) : make_uint4(0, 0, 0, 0);
  int buf = 0;
  for (uint64_t g = blockIdx.x; g < ngroups; g += gridDim.x) {
    const uint64_t tile0 = g * kGroupTiles + warp * kTilesPerWarp;
    if (tile0 + kTilesPerWarp <= whole_tiles) {
      // This warp's tiles are all whole: two at a time, 16 unconditional
      // loads in flight per lane (measured +7-30 % over one tile at a time
      // at 8 GiB; the association, hence every bit, is unchanged).
#pragma unroll 1
      for (int j = 0; j < kTilesPerWarp; j += 2) {
        const uint4* vp = reinterpret_cast<const uint4*>(body) + (tile0 + j) * kTileVectors + lane;
        uint4 a[kReduceUnroll], b[kReduceUnroll];
#pragma unroll
        for (int u = 0; u < kReduceUnroll; ++u) a[u] = ld_stream_u4(vp + u * kWarp);
#pragma unroll
        for (int u = 0; u < kReduceUnroll; ++u) b[u] = ld_stream_u4(vp + kTileVectors + u * kWarp);
        typename Op::Thread ta, tb;
        Op::body(ta, a, 0, kWarp, kReduceUnroll);
        Op::body(tb, b, 0, kWarp, kReduceUnroll);
        const double pa = warp_tree_f64(Op::finish(ta, 0));
        const double pb = warp_tree_f64(Op::finish(tb, 0));
        if (lane == 0) {
          tile_partials[buf][warp * kTilesPerWarp + j] = pa;
          tile_partials[buf][warp * kTilesPerWarp + j + 1] = pb;
        }
      }
    } else {
#pragma unroll 1
      for (int j = 0; j < kTilesPerWarp; ++j) {
        const int local = warp * kTilesPerWarp + j;
        const uint64_t tile = g * kGroupTiles + local;
        double p = 0.0;
        if (tile < ntiles) {
          // this lane's vectors: first + 32u, u < 8; `full` of them are whole
          // vectors, and the zero-padded tail vector (if any) comes right after
          const uint64_t first = tile * kTileVectors + lane;
          const int full = lane_vectors(first, nvec_full);
          const int count = lane_vectors(first, nvec);
          const uint4* vp = reinterpret_cast<const uint4*>(body) + first;
          uint4 v[kReduceUnroll];
#pragma unroll
          for (int u = 0; u < kReduceUnroll; ++u) {
            v[u] = u < full ? ld_stream_u4(vp + u * kWarp) : (u < count ? tail_vec : make_uint4(0, 0, 0, 0));
          }
          typename Op::Thread t;
          Op::body(t, v, first, kWarp, count);
          p = Op::finish(t, 0);
        }
        p = warp_tree_f64(p);
        if (lane == 0) tile_partials[buf][local] = p;
      }
    }
    __syncthreads();
    if (warp == 0) {
      const double gp = warp_tree_f64(tile_partials[buf][lane] + tile_partials[buf][lane + kWarp]);
      if (lane == 0) groups[g] = gp;
    }
    buf ^= 1;  // the next group writes the other buffer; the barrier above orders reuse
  }

  // last CTA to finish computes the total (nothing waits)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    is_last = (atomicAdd(ticket, 1u) == gridDim.x - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  double total = ordered_total(groups, ngroups, scratch);
  if (threadIdx.x == 0) {
    typename Op::Thread h;
    for (uint64_t i = 0; i < head; ++i) Op::scalar(h, load_element_bits<kElem>(in + i * kElem), i);
    total += Op::finish(h, 0);
    *out = accumulate ? *out + total : total;
    *ticket = 0u;
  }
}

}  // namespace f4s

// (in, n_lo, n_hi, out f64, workspace, groups f64[], accumulate).  Launch
// with blockDim 512, any grid; workspace holds the ticket (4 bytes, zeroed
// once; each launch leaves it zeroed), `groups` receives one f64 partial
// per 256 KiB group (the single-array layout puts it at workspace + 256).
#define F4S_REDUCE_ORDERED_KERNEL(NAME, OP, MIN_CTAS)                                                    \
  extern "C" __global__ void __launch_bounds__(f4s::kOrderedBlock, MIN_CTAS)                              \
      NAME(const void* in, uint32_t n_lo, uint32_t n_hi, double* out, unsigned char* workspace,           \
           double* groups, int accumulate) {                                                              \
    f4s::reduce_ordered<OP>(in, f4s::join_u64(n_lo, n_hi), out, workspace, groups, accumulate);           \
  }
// Co-resident CTAs per SM (the launch uses one persistent wave of them):
// one for the 4-byte and 16-bit types (measured best with the registers
// free), two for FP8, whose per-vector decode needs more warps to hide.
F4S_REDUCE_ORDERED_KERNEL(f4s_reduce_ordered_f32, f4s::SumF32TileOp, 1)
F4S_REDUCE_ORDERED_KERNEL(f4s_reduce_ordered_bf16, f4s::SumHalfOp<true>, 1)
F4S_REDUCE_ORDERED_KERNEL(f4s_reduce_ordered_f16, f4s::SumHalfOp<false>, 1)
F4S_REDUCE_ORDERED_KERNEL(f4s_reduce_ordered_f64, f4s::SumF64TileOp, 1)
F4S_REDUCE_ORDERED_KERNEL(f4s_reduce_ordered_e4m3, f4s::SumFp8TileOp<true>, 2)
F4S_REDUCE_ORDERED_KERNEL(f4s_reduce_ordered_e5m2, f4s::SumFp8TileOp<false>, 2)
#undef F4S_REDUCE_ORDERED_KERNEL

// F alone over `count` group partials (e.g. several GPUs' partials
// concatenated in array order): one CTA of 512 threads.
extern "C" __global__ void __launch_bounds__(f4s::kOrderedBlock)
    f4s_reduce_ordered_final(const double* groups, uint32_t count_lo, uint32_t count_hi, double* out,
                             int accumulate) {
  __shared__ double scratch[f4s::kOrderedWarps];
  const double total = f4s::ordered_total(groups, f4s::join_u64(count_lo, count_hi), scratch);
  if (threadIdx.x == 0) *out = accumulate ? *out + total : total;
}
