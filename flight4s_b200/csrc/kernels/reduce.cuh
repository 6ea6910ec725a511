// Full-array reductions over one device buffer: f32 sum (f64 accumulation),
// i32 sum (two's-complement wrap, bit-exact in any order), and f32 max with
// lowest-index argmax under IEEE totalOrder.
//
// The reference IR has a single reduction node, `ReduceSum`
// (core/src/main/scala/flight4s/core/ir/IR.scala:96-107), which its code
// generator lowers to a per-thread serial loop
// (core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:383-403).
// These kernels are the parallel lowering of that node (and of the max/argmax
// the reference lacks) for sm_100a:
//
//   1. a grid-stride streaming pass with 128-bit loads, kReduceUnroll vectors
//      per thread in flight;
//   2. warp combine (shuffles, or redux.sync for i32) then a CTA combine in
//      shared memory;
//   3. a thread-block-cluster combine: every CTA deposits its partial in the
//      cluster leader's shared memory through DSMEM, so only one partial per
//      cluster reaches global memory;
//   4. the last cluster to finish (atomic ticket, nothing waits) folds all
//      cluster partials in index order and writes the result.  The result is
//      deterministic for a given grid, and no second kernel is launched.
//
// Accumulation follows the reference's `AccumulatorType` rules
// (core/src/main/scala/flight4s/core/types/CudaType.scala:199-230): I32
// accumulates in I32 (wrapping); F32 sums are carried in f64 above 32-element
// fp32 runs, which costs no bandwidth and keeps a 2^32-element sum accurate
// to ~1e-12 of sum|x|.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace f4s {
namespace cg = cooperative_groups;

constexpr int kReduceBlock = 512;
constexpr int kReduceUnroll = 8;
constexpr int kReduceMaxCluster = 8;
// Workspace layout: [0,4) ticket counter; cluster partials from byte 256,
// 16 bytes each.
constexpr int kReducePartialOffset = 256;
constexpr int kReducePartialBytes = 16;

struct ArgmaxPartial {
  int64_t key;    // order key of the value (32-bit keys sign-extended)
  int64_t index;  // INT64_MAX: no candidate
};

// (key desc, index asc): keep the lexicographic winner.
__device__ __forceinline__ void argmax_merge(ArgmaxPartial& a, const ArgmaxPartial& b) {
  if (b.key > a.key || (b.key == a.key && b.index < a.index)) a = b;
}

// --------------------------------------------------------------- op policies
// Each policy supplies: the per-thread state, the vector-body step, the
// scalar head/tail step, the partial type with its identity / merge / warp
// merge, and how the final partial is written to `out`.

__device__ __forceinline__ float u2f(uint32_t b) { return __uint_as_float(b); }

// Pairwise tree over the U per-vector fp32 sums, then one f64 add: the
// accumulation rule of the f32 sums below.
template <int U>
__device__ __forceinline__ double fold_unrolled(float (&s)[U]) {
#pragma unroll
  for (int w = 1; w < U; w <<= 1) {
#pragma unroll
    for (int u = 0; u + w < U; u += 2 * w) s[u] += s[u + w];
  }
  return static_cast<double>(s[0]);
}

// The same tree in f64 over the per-vector f32 sums of the narrow types:
// an E4M3 vector sum is exact in f32, so E4M3 totals stay exact while they
// fit f64's 53 bits at the 2^-9 grid (below 2^44, i.e. any n < 2^35).
template <int U>
__device__ __forceinline__ double fold_unrolled_f64(const float (&s)[U]) {
  double d[U];
#pragma unroll
  for (int u = 0; u < U; ++u) d[u] = static_cast<double>(s[u]);
#pragma unroll
  for (int w = 1; w < U; w <<= 1) {
#pragma unroll
    for (int u = 0; u + w < U; u += 2 * w) d[u] += d[u + w];
  }
  return d[0];
}

struct SumF64PartialBase {
  static constexpr int kUnroll = kReduceUnroll;
  using Partial = double;
  struct Thread {
    double acc = 0.0;
  };
  static __device__ __forceinline__ Partial finish(Thread& t, uint64_t) { return t.acc; }
  static __device__ __forceinline__ void before_body(Thread&, uint64_t) {}
  static __device__ __forceinline__ Partial identity() { return 0.0; }
  static __device__ __forceinline__ Partial merge(Partial a, Partial b) { return a + b; }
  static __device__ __forceinline__ Partial warp_merge(Partial v) { return warp_sum_f64(v); }
  static __device__ __forceinline__ Partial load_cg(const Partial* p) { return __ldcg(p); }
  static __device__ __forceinline__ void write(void* out, Partial r, uint64_t, int accumulate) {
    double* o = static_cast<double*>(out);
    *o = accumulate ? *o + r : r;
  }
};

// f32 in, f64 out: fp32 pairs inside a 16-byte vector, a pairwise fp32
// tree over the U vectors of a step, f64 above.  Both the fast kernel and
// the order-fixed kernel's tiles step 8 vectors per lane (the fast kernel
// at 2 CTAs per SM in 16 waves: +1.2 % at 2^32 and +0.4 % at 2^29 elements
// over 4 vectors at 4 CTAs per SM in 8 waves, A/B on B200).
template <int U>
struct SumF32OpT : SumF64PartialBase {
  static constexpr int kElemBytes = 4;
  static constexpr int kUnroll = U;
  static __device__ __forceinline__ void body(Thread& t, const uint4* v, uint64_t, uint64_t, int count) {
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      s[u] = (u < count) ? (u2f(v[u].x) + u2f(v[u].y)) + (u2f(v[u].z) + u2f(v[u].w)) : 0.0f;
    }
    t.acc += fold_unrolled<U>(s);
  }
  static __device__ __forceinline__ void scalar(Thread& t, uint64_t bits, uint64_t) {
    t.acc += static_cast<double>(u2f(static_cast<uint32_t>(bits)));
  }
};
using SumF32Op = SumF32OpT<kReduceUnroll>;  // fast kernel
using SumF32TileOp = SumF32OpT<kReduceUnroll>;  // order-fixed tiles

// 16-bit floats (bf16 or f16) in, f64 out.  Each vector is summed in f32
// by sm_100's mixed-precision add (add.rn.f32.{f16,bf16}: widen exactly,
// add, one rounding) in two chains of four elements, then chain + chain;
// vector sums are combined in f64.
template <bool kBf16>
struct SumHalfOp : SumF64PartialBase {
  static constexpr int kElemBytes = 2;
  static __device__ __forceinline__ float word(float acc, uint32_t w) {
    if constexpr (kBf16) return add_bf16x2_to_f32(acc, w); else return add_f16x2_to_f32(acc, w);
  }
  static __device__ __forceinline__ void body(Thread& t, const uint4* v, uint64_t, uint64_t, int count) {
    float s[kReduceUnroll];
#pragma unroll
    for (int u = 0; u < kReduceUnroll; ++u) {
      s[u] = (u < count) ? word(word(0.0f, v[u].x), v[u].y) + word(word(0.0f, v[u].z), v[u].w) : 0.0f;
    }
    t.acc += fold_unrolled_f64<kReduceUnroll>(s);
  }
  static __device__ __forceinline__ void scalar(Thread& t, uint64_t bits, uint64_t) {
    const uint32_t w = static_cast<uint32_t>(bits);
    t.acc += static_cast<double>(kBf16 ? bf16_lo(w) : f16_to_f32(static_cast<uint16_t>(w)));
  }
};

// FP8 (E4M3 or E5M2) in, f64 out: pairs of codes become f16x2 exactly
// (cvt.rn.f16x2.{e4m3,e5m2}x2), which the mixed-precision add accumulates in
// f32 in two chains of eight; every partial sum of E4M3 values is exact in
// f32 (at most 21 significant bits).  Vector sums are combined in f64, U per
// step (8 for both kernels: with two CTAs per SM the fast kernel gains 6 %
// at 2 GiB and 2.4 % at 8 GiB over 4 vectors at four CTAs per SM).
template <bool kE4m3, int U>
struct SumFp8OpT : SumF64PartialBase {
  static constexpr int kElemBytes = 1;
  static constexpr int kUnroll = U;
  static __device__ __forceinline__ uint32_t to_f16x2(uint32_t two_codes) {
    if constexpr (kE4m3) return e4m3x2_to_f16x2(two_codes); else return e5m2x2_to_f16x2(two_codes);
  }
  static __device__ __forceinline__ float word(float acc, uint32_t w) {
    return add_f16x2_to_f32(add_f16x2_to_f32(acc, to_f16x2(w & 0xFFFFu)), to_f16x2(w >> 16));
  }
  static __device__ __forceinline__ void body(Thread& t, const uint4* v, uint64_t, uint64_t, int count) {
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      s[u] = (u < count) ? word(word(0.0f, v[u].x), v[u].y) + word(word(0.0f, v[u].z), v[u].w) : 0.0f;
    }
    t.acc += fold_unrolled_f64<U>(s);
  }
  static __device__ __forceinline__ void scalar(Thread& t, uint64_t bits, uint64_t) {
    const uint32_t c = static_cast<uint32_t>(bits) & 0xFFu;
    t.acc += static_cast<double>(kE4m3 ? unpack_e4m3x2(c).x : unpack_e5m2x2(c).x);
  }
};
template <bool kE4m3>
using SumFp8Op = SumFp8OpT<kE4m3, kReduceUnroll>;
template <bool kE4m3>
using SumFp8TileOp = SumFp8OpT<kE4m3, kReduceUnroll>;

// f64 in, f64 out, U vectors per step (8 for both kernels; the fast one at
// two CTAs per SM, +4 % over 4 vectors at four CTAs per SM).
template <int U>
struct SumF64OpT : SumF64PartialBase {
  static constexpr int kElemBytes = 8;
  static constexpr int kUnroll = U;
  static __device__ __forceinline__ double d(uint32_t lo, uint32_t hi) {
    return __hiloint2double(static_cast<int>(hi), static_cast<int>(lo));
  }
  static __device__ __forceinline__ void body(Thread& t, const uint4* v, uint64_t, uint64_t, int count) {
    double s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) s[u] = (u < count) ? d(v[u].x, v[u].y) + d(v[u].z, v[u].w) : 0.0;
#pragma unroll
    for (int w = 1; w < U; w <<= 1) {
#pragma unroll
      for (int u = 0; u + w < U; u += 2 * w) s[u] += s[u + w];
    }
    t.acc += s[0];
  }
  static __device__ __forceinline__ void scalar(Thread& t, uint64_t bits, uint64_t) {
    t.acc += __longlong_as_double(static_cast<long long>(bits));
  }
};
using SumF64Op = SumF64OpT<kReduceUnroll>;
using SumF64TileOp = SumF64OpT<kReduceUnroll>;

// i32 or u32 in, 32-bit two's-complement wrap out (bit-identical for both).
struct SumWrap32Op {
  static constexpr int kElemBytes = 4;
  // 8 vectors per lane per step at 2 CTAs per SM in 16 waves: +0.6 % at
  // 2^32 elements over 4 vectors at 3 CTAs per SM in 8 waves (A/B on B200)
  static constexpr int kUnroll = kReduceUnroll;
  using Partial = int32_t;
  struct Thread {
    uint32_t acc = 0;
  };
  static __device__ __forceinline__ void body(Thread& t, const uint4* v, uint64_t, uint64_t, int count) {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (u < count) t.acc += (v[u].x + v[u].y) + (v[u].z + v[u].w);
    }
  }
  static __device__ __forceinline__ void scalar(Thread& t, uint64_t bits, uint64_t) {
    t.acc += static_cast<uint32_t>(bits);
  }
  static __device__ __forceinline__ Partial finish(Thread& t, uint64_t) { return static_cast<int32_t>(t.acc); }
  static __device__ __forceinline__ void before_body(Thread&, uint64_t) {}
  static __device__ __forceinline__ Partial identity() { return 0; }
  static __device__ __forceinline__ Partial merge(Partial a, Partial b) {
    return static_cast<int32_t>(static_cast<uint32_t>(a) + static_cast<uint32_t>(b));
  }
  static __device__ __forceinline__ Partial warp_merge(Partial v) {
    return static_cast<int32_t>(__reduce_add_sync(0xffffffffu, static_cast<uint32_t>(v)));
  }
  static __device__ __forceinline__ Partial load_cg(const Partial* p) { return __ldcg(p); }
  static __device__ __forceinline__ void write(void* out, Partial r, uint64_t, int accumulate) {
    int32_t* o = static_cast<int32_t*>(out);
    *o = accumulate ? merge(*o, r) : r;
  }
};

// Order keys: a signed integer whose order is the element type's order
// (IEEE totalOrder for the floating-point types: -NaN < -inf < ... < -0 <
// +0 < ... < +inf < +NaN), per OrderedType of the reference
// (core/src/main/scala/flight4s/core/types/CudaType.scala:182-188).
struct ArgmaxKeyF32 {
  static constexpr int kBytes = 4;
  using Key = int32_t;
  static __device__ __forceinline__ Key key(uint64_t b) {
    return total_order_key(__uint_as_float(static_cast<uint32_t>(b)));
  }
};
struct ArgmaxKeyI32 {
  static constexpr int kBytes = 4;
  using Key = int32_t;
  static __device__ __forceinline__ Key key(uint64_t b) { return static_cast<int32_t>(static_cast<uint32_t>(b)); }
};
struct ArgmaxKeyU32 {
  static constexpr int kBytes = 4;
  using Key = int32_t;
  static __device__ __forceinline__ Key key(uint64_t b) {
    return static_cast<int32_t>(static_cast<uint32_t>(b) ^ 0x80000000u);
  }
};
// f16 and bf16 share the sign-magnitude layout, so one key serves both.
struct ArgmaxKeyHalf {
  static constexpr int kBytes = 2;
  using Key = int32_t;
  static __device__ __forceinline__ Key key(uint64_t b) {
    const int32_t v = static_cast<int16_t>(static_cast<uint16_t>(b));
    return v ^ (static_cast<int32_t>(static_cast<uint32_t>(v >> 31) >> 17));
  }
  // The same keys two at a time: each 16-bit lane of `w` XOR 0x7FFF where
  // its sign bit is set ((sign bits >> 15) * 0x7FFF stays inside each lane).
  static __device__ __forceinline__ uint32_t keys2(uint32_t w) { return w ^ (((w >> 15) & 0x00010001u) * 0x7FFFu); }
  static __device__ __forceinline__ uint32_t max_s16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.s16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  // max key of a 16-byte vector (8 elements), as key() would give it.
  static __device__ __forceinline__ Key vector_max(const uint4& v) {
    const uint32_t m = max_s16x2(max_s16x2(keys2(v.x), keys2(v.y)), max_s16x2(keys2(v.z), keys2(v.w)));
    return max(static_cast<int32_t>(static_cast<int16_t>(m & 0xFFFFu)), static_cast<int32_t>(m) >> 16);
  }
};
struct ArgmaxKeyF64 {
  static constexpr int kBytes = 8;
  using Key = int64_t;
  static __device__ __forceinline__ Key key(uint64_t b) {
    const int64_t v = static_cast<int64_t>(b);
    return v ^ static_cast<int64_t>(static_cast<uint64_t>(v >> 63) >> 1);
  }
};

// Element j of a 16-byte vector as raw bits.
template <int kBytes>
__device__ __forceinline__ uint64_t vector_element(const uint4& v, int j) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (kBytes == 8) return static_cast<uint64_t>(w[2 * j]) | (static_cast<uint64_t>(w[2 * j + 1]) << 32);
  else if constexpr (kBytes == 4) return w[j];
  else return (w[j / 2] >> (16 * (j % 2))) & 0xFFFFu;
}

// Output record of the argmax kernels (two 64-bit words):
//   out[0] = for 32-bit keys (every type but f64): (i64)key << 32 |
//            (0xFFFFFFFF - index), the packed form whose signed 64-bit max
//            across devices (NCCL int64 MAX) is again the (max value, lowest
//            index) pair, valid while index < 2^32; for f64: the 64-bit key
//            itself; INT64_MIN for an empty input;
//   out[1] = the index as a signed 64-bit integer, -1 for an empty input.
template <class K, int U = 4>
struct ArgmaxOp {
  static constexpr int kElemBytes = K::kBytes;
  static constexpr int kPerVec = 16 / K::kBytes;
  // U vectors in flight per lane at 2 CTAs per SM, launched in 16 waves:
  // 8 (6 for f64's 64-bit keys).  A/B on B200 against 4 vectors at 3 CTAs
  // per SM in 8 waves: f32 +1.2 % at 16 GiB, +0.5 % at 2 GiB; f16 +3 %,
  // i32 / u32 +4 %, f64 +2.4 % at 8 GiB.
  static constexpr int kUnroll = U;
  using Key = typename K::Key;
  using Partial = ArgmaxPartial;
  static constexpr Key kKeyMin = sizeof(Key) == 8 ? static_cast<Key>(INT64_MIN) : static_cast<Key>(INT32_MIN);
  struct Thread {
    Key vkey = kKeyMin;  // best key seen in the vector body
    uint64_t best_vec = UINT64_MAX;
    uint4 best = make_uint4(0, 0, 0, 0);  // that vector's values
    ArgmaxPartial s{INT64_MIN, INT64_MAX};  // scalar head/tail candidate
  };
  static __device__ __forceinline__ Key vector_max(const uint4& v) {
    if constexpr (kElemBytes == 2) {
      return K::vector_max(v);  // packed 16-bit keys
    } else {
      Key k = K::key(vector_element<kElemBytes>(v, 0));
#pragma unroll
      for (int j = 1; j < kPerVec; ++j) k = max(k, K::key(vector_element<kElemBytes>(v, j)));
      return k;
    }
  }
  static __device__ __forceinline__ void body(Thread& t, const uint4* v, uint64_t base,
                                              uint64_t stride, int count) {
    // The hot loop tracks only the best vector (kept in registers; the
    // update branch is rarely taken); the lane inside it is resolved once
    // at the end.  Vectors arrive in increasing index order, so a strict
    // '>' keeps the lowest index.
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (u < count) {
        const Key k = vector_max(v[u]);
        if (k > t.vkey) {
          t.vkey = k;
          t.best_vec = base + u * stride;
          t.best = v[u];
        }
      }
    }
  }
  static __device__ __forceinline__ void scalar(Thread& t, uint64_t bits, uint64_t index) {
    argmax_merge(t.s, ArgmaxPartial{static_cast<int64_t>(K::key(bits)), static_cast<int64_t>(index)});
  }
  // Before the body: the lane's lowest-index vector, if it reads any, is
  // the candidate until a vector with a larger key than the smallest one
  // turns up (the strict '>' against the initial key never fires for a
  // lane that sees only the smallest key, e.g. an i32 array of INT32_MIN;
  // its answer is then the first element of its first vector).
  static __device__ __forceinline__ void before_body(Thread& t, uint64_t first) { t.best_vec = first; }
  static __device__ __forceinline__ Partial finish(Thread& t, uint64_t head) {
    ArgmaxPartial p = t.s;
    if (t.best_vec != UINT64_MAX) {
      int lane = kPerVec - 1;
#pragma unroll
      for (int j = kPerVec - 2; j >= 0; --j)
        if (K::key(vector_element<kElemBytes>(t.best, j)) == t.vkey) lane = j;
      if (t.vkey == kKeyMin) lane = 0;  // never updated: every key seen was the smallest
      argmax_merge(p, ArgmaxPartial{static_cast<int64_t>(t.vkey),
                                    static_cast<int64_t>(head + kPerVec * t.best_vec + lane)});
    }
    return p;
  }
  static __device__ __forceinline__ Partial identity() { return ArgmaxPartial{INT64_MIN, INT64_MAX}; }
  static __device__ __forceinline__ Partial merge(Partial a, Partial b) {
    argmax_merge(a, b);
    return a;
  }
  static __device__ __forceinline__ Partial warp_merge(Partial v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgmaxPartial other{__shfl_xor_sync(0xffffffffu, v.key, o), __shfl_xor_sync(0xffffffffu, v.index, o)};
      argmax_merge(v, other);
    }
    return v;
  }
  static __device__ __forceinline__ Partial load_cg(const Partial* p) {
    const longlong2 raw = __ldcg(reinterpret_cast<const longlong2*>(p));
    return ArgmaxPartial{static_cast<int64_t>(raw.x), static_cast<int64_t>(raw.y)};
  }
  static __device__ __forceinline__ void write(void* out, Partial r, uint64_t index_base, int accumulate) {
    int64_t* o = static_cast<int64_t*>(out);
    constexpr bool kPacked = sizeof(Key) == 4;
    if (r.index != INT64_MAX) r.index += static_cast<int64_t>(index_base);
    if (accumulate && o[1] >= 0) argmax_merge(r, ArgmaxPartial{kPacked ? (o[0] >> 32) : o[0], o[1]});
    if (r.index == INT64_MAX) {
      o[0] = INT64_MIN;
      o[1] = -1;
      return;
    }
    if constexpr (kPacked) {
      const uint32_t low = (r.index <= 0xFFFFFFFFll) ? 0xFFFFFFFFu - static_cast<uint32_t>(r.index) : 0u;
      o[0] = static_cast<int64_t>((static_cast<uint64_t>(static_cast<uint32_t>(r.key)) << 32) | low);
    } else {
      o[0] = r.key;
    }
    o[1] = r.index;
  }
};
using ArgmaxF32Op = ArgmaxOp<ArgmaxKeyF32>;

// Partials are stored as 16-byte records so one workspace layout serves
// every op.
template <class Partial>
__device__ __forceinline__ void store_partial(unsigned char* slot, const Partial& p) {
  *reinterpret_cast<Partial*>(slot) = p;
}
template <>
__device__ __forceinline__ void store_partial<ArgmaxPartial>(unsigned char* slot, const ArgmaxPartial& p) {
  *reinterpret_cast<longlong2*>(slot) = make_longlong2(p.key, p.index);
}

// --------------------------------------------------------------- the kernel
template <int kBytes>
__device__ __forceinline__ uint64_t load_element_bits(const unsigned char* p) {
  if constexpr (kBytes == 1) return *p;
  else if constexpr (kBytes == 2) return *reinterpret_cast<const uint16_t*>(p);
  else if constexpr (kBytes == 4) return *reinterpret_cast<const uint32_t*>(p);
  else return *reinterpret_cast<const unsigned long long*>(p);
}

// in: n elements of Op::kElemBytes bytes, aligned to the element size.
template <class Op>
__device__ __forceinline__ void reduce_full(const void* __restrict__ in_ptr, uint64_t n,
                                            void* __restrict__ out,
                                            unsigned char* __restrict__ workspace,
                                            uint64_t index_base, int accumulate) {
  using Partial = typename Op::Partial;
  constexpr int kElem = Op::kElemBytes;
  constexpr int kPerVec = 16 / kElem;
  const unsigned char* in = static_cast<const unsigned char*>(in_ptr);
  const cg::cluster_group cluster = cg::this_cluster();

  __shared__ Partial warp_partials[kReduceBlock / kWarp];
  __shared__ Partial cluster_partials[kReduceMaxCluster];
  __shared__ int is_last;

  // A kernel launched after this one as a programmatic dependent (launch
  // overlap, off unless the host asks) may start once every CTA here has
  // started; without such a launch this has no effect.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t nthreads = static_cast<uint64_t>(gridDim.x) * blockDim.x;

  // [0,n) = scalar head up to the first 16-byte boundary, vector body,
  // scalar tail (fewer than one vector each).
  const uint64_t addr = reinterpret_cast<uint64_t>(in);
  uint64_t head = ((16u - (addr & 15u)) & 15u) / kElem;
  if (head > n) head = n;
  const uint64_t nvec = (n - head) / kPerVec;
  const uint64_t tail_begin = head + static_cast<uint64_t>(kPerVec) * nvec;

  typename Op::Thread t;
  for (uint64_t i = tid; i < head; i += nthreads) Op::scalar(t, load_element_bits<kElem>(in + i * kElem), i);
  for (uint64_t i = tail_begin + tid; i < n; i += nthreads)
    Op::scalar(t, load_element_bits<kElem>(in + i * kElem), i);

  // Body in warp tiles of 32 * Op::kUnroll vectors (4 KiB at 8): lane l of
  // a warp loads vectors l + 32u (u < Op::kUnroll) of its tile, so each
  // warp streams contiguous memory per step; warps stride over the tiles.
  // (Measured against a thread-strided layout: equal for f32/i32/argmax,
  // +10% for the bf16 and FP8 sums.)  Each lane still sees its vectors in
  // increasing index order.
  constexpr int kUnroll = Op::kUnroll;
  const uint4* vin = reinterpret_cast<const uint4*>(in + head * kElem);
  const uint64_t tile_lane = threadIdx.x % kWarp;
  const uint64_t nwarps = nthreads / kWarp;
  const uint64_t full_tiles = nvec / (kWarp * kUnroll);
  uint64_t tile = tid / kWarp;
  {
    // the lowest-index vector this lane reads, if any
    const uint64_t first = tile * (kWarp * kUnroll) + tile_lane;
    Op::before_body(t, (tile <= full_tiles && first < nvec) ? first : UINT64_MAX);
  }
  for (; tile < full_tiles; tile += nwarps) {
    const uint64_t base = tile * (kWarp * kUnroll) + tile_lane;
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream_u4(vin + base + u * kWarp);
    Op::body(t, v, base, kWarp, kUnroll);
  }
  if (tile == full_tiles) {  // exactly one warp owns the partial last tile
    const uint64_t base = tile * (kWarp * kUnroll) + tile_lane;
    uint4 v[kUnroll];
    int count = 0;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (base + u * kWarp < nvec) {
        v[u] = ld_stream_u4(vin + base + u * kWarp);
        count = u + 1;
      } else {
        v[u] = make_uint4(0, 0, 0, 0);
      }
    }
    if (count > 0) Op::body(t, v, base, kWarp, count);
  }

  // Launched as a programmatic dependent, this kernel may have streamed its
  // input while the previous kernel on the stream was finishing: wait for
  // that kernel (complete, its writes visible) before touching the workspace
  // and the output, which it may share.  A no-op for an ordinary launch.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // thread -> warp -> CTA
  Partial p = Op::warp_merge(Op::finish(t, head));
  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  if (lane == 0) warp_partials[warp] = p;
  __syncthreads();

  // CTA -> cluster leader through distributed shared memory
  const unsigned rank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  if (threadIdx.x == 0) {
    Partial c = warp_partials[0];
#pragma unroll
    for (int w = 1; w < kReduceBlock / kWarp; ++w) c = Op::merge(c, warp_partials[w]);
    *cluster.map_shared_rank(&cluster_partials[rank], 0) = c;
  }
  cluster.sync();
  if (rank != 0) return;

  // cluster leader: publish one partial and take a ticket
  const unsigned cluster_id = blockIdx.x / csize;
  const unsigned num_clusters = gridDim.x / csize;
  unsigned int* ticket = reinterpret_cast<unsigned int*>(workspace);
  unsigned char* partials = workspace + kReducePartialOffset;
  if (threadIdx.x == 0) {
    Partial c = cluster_partials[0];
    for (unsigned r = 1; r < csize; ++r) c = Op::merge(c, cluster_partials[r]);
    store_partial(partials + static_cast<size_t>(cluster_id) * kReducePartialBytes, c);
    __threadfence();
    is_last = (atomicAdd(ticket, 1u) == num_clusters - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!is_last) return;

  // last cluster: fold every cluster partial in a fixed order
  __threadfence();
  Partial acc = Op::identity();
  for (unsigned i = threadIdx.x; i < num_clusters; i += blockDim.x) {
    acc = Op::merge(acc, Op::load_cg(reinterpret_cast<const Partial*>(
                             partials + static_cast<size_t>(i) * kReducePartialBytes)));
  }
  acc = Op::warp_merge(acc);
  if (lane == 0) warp_partials[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    Partial r = warp_partials[0];
#pragma unroll
    for (int w = 1; w < kReduceBlock / kWarp; ++w) r = Op::merge(r, warp_partials[w]);
    *ticket = 0u;  // leave the workspace ready for the next launch
    Op::write(out, r, index_base, accumulate);
  }
}

}  // namespace f4s

// Kernel entry points.  Parameters use only launch-ABI descriptor codes
// 10 (device pointer), 3 (u32) and 2 (i32): (in, n_lo, n_hi, out, workspace,
// index_base_lo, index_base_hi, accumulate).
// max / argmax over every OrderedType, 2 CTAs per SM (MIN_CTAS) with
// UNROLL vectors per lane per step.
#define F4S_ARGMAX_KERNEL(NAME, KEY, MIN_CTAS, UNROLL)                                                 \
  extern "C" __global__ void __launch_bounds__(f4s::kReduceBlock, MIN_CTAS)                             \
      NAME(const void* in, uint32_t n_lo, uint32_t n_hi, void* out, unsigned char* workspace,           \
           uint32_t base_lo, uint32_t base_hi, int accumulate) {                                        \
    f4s::reduce_full<f4s::ArgmaxOp<f4s::KEY, UNROLL>>(in, f4s::join_u64(n_lo, n_hi), out, workspace,    \
                                                      f4s::join_u64(base_lo, base_hi), accumulate);     \
  }
F4S_ARGMAX_KERNEL(f4s_reduce_argmax_f32, ArgmaxKeyF32, 2, 8)
F4S_ARGMAX_KERNEL(f4s_reduce_argmax_i32, ArgmaxKeyI32, 2, 8)
F4S_ARGMAX_KERNEL(f4s_reduce_argmax_u32, ArgmaxKeyU32, 2, 8)
F4S_ARGMAX_KERNEL(f4s_reduce_argmax_half, ArgmaxKeyHalf, 2, 8)  // f16 and bf16
F4S_ARGMAX_KERNEL(f4s_reduce_argmax_f64, ArgmaxKeyF64, 2, 6)    // 8 would spill more
#undef F4S_ARGMAX_KERNEL
// Sums: f32 -> f64, i32 / u32 -> 32-bit wrap, and the other AccumulatorType
// inputs (core/src/main/scala/flight4s/core/types/CudaType.scala:199-230),
// accumulated in f64: bf16, f16, f64, FP8 E4M3, FP8 E5M2.  Two CTAs per SM
// (the register room lets each lane keep 8-vector steps in flight),
// launched in twice the waves; for bf16 / f16 +1.0 % at 8 GiB and +1.2 % at
// 2 GiB over 3 CTAs per SM in 8 waves (A/B on B200).
#define F4S_REDUCE_KERNEL_2(NAME, OP)                                                        \
  extern "C" __global__ void __launch_bounds__(f4s::kReduceBlock, 2)                          \
      NAME(const void* in, uint32_t n_lo, uint32_t n_hi, void* out, unsigned char* workspace, \
           uint32_t base_lo, uint32_t base_hi, int accumulate) {                              \
    f4s::reduce_full<OP>(in, f4s::join_u64(n_lo, n_hi), out, workspace,                      \
                         f4s::join_u64(base_lo, base_hi), accumulate);                       \
  }
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_f32, f4s::SumF32Op)
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_i32, f4s::SumWrap32Op)
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_f64, f4s::SumF64Op)
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_bf16, f4s::SumHalfOp<true>)
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_f16, f4s::SumHalfOp<false>)
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_e4m3, f4s::SumFp8Op<true>)
F4S_REDUCE_KERNEL_2(f4s_reduce_sum_e5m2, f4s::SumFp8Op<false>)
#undef F4S_REDUCE_KERNEL_2
