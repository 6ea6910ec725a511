// Elementwise Convert: the reference's conversion node over whole arrays.
//
// Convert (core/src/main/scala/flight4s/core/ir/IR.scala:54-70) carries a
// RoundingMode and a SaturationMode; its codegen
// (core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:405-449,506-538)
// lowers f32 -> f16 / bf16 to __float2half_{rn,rz,ru,rd} /
// __float2bfloat16_{rn,rz,ru,rd}, f32 -> FP8 to
// __nv_cvt_float_to_fp8(v, __NV_NOSAT | __NV_SATFINITE, __NV_E4M3 | __NV_E5M2)
// (always nearest-even), and the widening back to __half2float,
// __bfloat162float and static_cast<float>.  These kernels call the same
// CUDA conversion functions on each element (FP8 pairs through the x2 form),
// so every code equals the reference's; the decodes use the exact
// f16x2 <- fp8x2 conversion instruction.
//
// B200 mapping: one thread per 16 elements, moved with 128/256-bit
// streaming loads and stores (L1 bypassed, L2 evict-first); a scalar path
// for the ragged tail and for buffers not 32-byte aligned.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace f4s {

constexpr int kConvertBlock = 256;
constexpr int kConvertChunk = 16;  // elements per thread step

enum RoundingOrdinal : int { kRoundNearestEven = 0, kRoundTowardZero = 1, kRoundUp = 2, kRoundDown = 3 };

template <int kRounding>
__device__ __forceinline__ uint32_t f32_to_f16_bits(float x) {
  __half h;
  if constexpr (kRounding == kRoundNearestEven) h = __float2half_rn(x);
  else if constexpr (kRounding == kRoundTowardZero) h = __float2half_rz(x);
  else if constexpr (kRounding == kRoundUp) h = __float2half_ru(x);
  else h = __float2half_rd(x);
  return __half_as_ushort(h);
}

template <int kRounding>
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float x) {
  __nv_bfloat16 b;
  if constexpr (kRounding == kRoundNearestEven) b = __float2bfloat16_rn(x);
  else if constexpr (kRounding == kRoundTowardZero) b = __float2bfloat16_rz(x);
  else if constexpr (kRounding == kRoundUp) b = __float2bfloat16_ru(x);
  else b = __float2bfloat16_rd(x);
  return __bfloat16_as_ushort(b);
}

// f32 -> 16-bit float with a rounding mode: 16 f32 words -> 8 packed words.
template <bool kBf16, int kRounding>
struct ToHalfConvert {
  static constexpr int kIn = 4, kOut = 2;
  static __device__ __forceinline__ uint32_t one(uint64_t bits) {
    const float x = __uint_as_float(static_cast<uint32_t>(bits));
    return kBf16 ? f32_to_bf16_bits<kRounding>(x) : f32_to_f16_bits<kRounding>(x);
  }
  static __device__ __forceinline__ void chunk(const uint32_t (&in)[16], uint32_t (&out)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = one(in[2 * i]) | (one(in[2 * i + 1]) << 16);
  }
};

// f32 -> FP8, nearest-even, saturating to the largest finite value or not.
template <bool kE4m3, bool kSaturate>
struct ToFp8Convert {
  static constexpr int kIn = 4, kOut = 1;
  static __device__ __forceinline__ uint32_t pair(uint32_t a, uint32_t b) {
    const float2 v = make_float2(__uint_as_float(a), __uint_as_float(b));
    return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(v, kSaturate ? __NV_SATFINITE : __NV_NOSAT,
                                                          kE4m3 ? __NV_E4M3 : __NV_E5M2));
  }
  static __device__ __forceinline__ uint32_t one(uint64_t bits) {
    return pair(static_cast<uint32_t>(bits), 0u) & 0xFFu;
  }
  static __device__ __forceinline__ void chunk(const uint32_t (&in)[16], uint32_t (&out)[4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = pair(in[4 * i], in[4 * i + 1]) | (pair(in[4 * i + 2], in[4 * i + 3]) << 16);
  }
};

// 16-bit float -> f32 (exact).
template <bool kBf16>
struct FromHalfConvert {
  static constexpr int kIn = 2, kOut = 4;
  static __device__ __forceinline__ uint32_t one(uint64_t bits) {
    const uint32_t b = static_cast<uint32_t>(bits) & 0xFFFFu;
    return kBf16 ? (b << 16) : __float_as_uint(f16_to_f32(static_cast<uint16_t>(b)));
  }
  static __device__ __forceinline__ void chunk(const uint32_t (&in)[8], uint32_t (&out)[16]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      out[2 * i] = one(in[i] & 0xFFFFu);
      out[2 * i + 1] = one(in[i] >> 16);
    }
  }
};

// FP8 -> f32 (exact, through f16x2).
template <bool kE4m3>
struct FromFp8Convert {
  static constexpr int kIn = 1, kOut = 4;
  static __device__ __forceinline__ float2 two(uint32_t codes) {
    return kE4m3 ? unpack_e4m3x2(codes) : unpack_e5m2x2(codes);
  }
  static __device__ __forceinline__ uint32_t one(uint64_t bits) {
    return __float_as_uint(two(static_cast<uint32_t>(bits) & 0xFFu).x);
  }
  static __device__ __forceinline__ void chunk(const uint32_t (&in)[4], uint32_t (&out)[16]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = two(in[i] & 0xFFFFu), b = two(in[i] >> 16);
      out[4 * i] = __float_as_uint(a.x);
      out[4 * i + 1] = __float_as_uint(a.y);
      out[4 * i + 2] = __float_as_uint(b.x);
      out[4 * i + 3] = __float_as_uint(b.y);
    }
  }
};

// Same type on both sides (the reference emits the value unchanged): a
// copy, 16 elements of kBytes each.
template <int kBytes>
struct CopyConvert {
  static constexpr int kIn = kBytes, kOut = kBytes;
  static __device__ __forceinline__ uint64_t one(uint64_t bits) { return bits; }
  template <int W>
  static __device__ __forceinline__ void chunk(const uint32_t (&in)[W], uint32_t (&out)[W]) {
#pragma unroll
    for (int i = 0; i < W; ++i) out[i] = in[i];
  }
};

// 16 * B bytes <-> words with 128/256-bit streaming accesses.
template <int W>
__device__ __forceinline__ void load_words(const unsigned char* p, uint32_t (&w)[W]) {
  static_assert(W == 4 || W % 8 == 0, "chunk of 16 bytes or a multiple of 32");
  if constexpr (W == 4) {
    const uint4 v = ld_stream_u4(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
#pragma unroll
    for (int h = 0; h < W / 8; ++h) {
      const u32x8 v = ld_stream_v8(p + 32 * h);
      w[8 * h + 0] = v.lo.x; w[8 * h + 1] = v.lo.y; w[8 * h + 2] = v.lo.z; w[8 * h + 3] = v.lo.w;
      w[8 * h + 4] = v.hi.x; w[8 * h + 5] = v.hi.y; w[8 * h + 6] = v.hi.z; w[8 * h + 7] = v.hi.w;
    }
  }
}

template <int W>
__device__ __forceinline__ void store_words(unsigned char* p, const uint32_t (&w)[W]) {
  if constexpr (W == 4) {
    st_stream_u4(p, make_uint4(w[0], w[1], w[2], w[3]));
  } else {
#pragma unroll
    for (int h = 0; h < W / 8; ++h) {
      u32x8 v;
      v.lo = make_uint4(w[8 * h + 0], w[8 * h + 1], w[8 * h + 2], w[8 * h + 3]);
      v.hi = make_uint4(w[8 * h + 4], w[8 * h + 5], w[8 * h + 6], w[8 * h + 7]);
      st_stream_v8(p + 32 * h, v);
    }
  }
}

template <int kBytes>
__device__ __forceinline__ void store_element_bits(unsigned char* p, uint64_t bits) {
  if constexpr (kBytes == 1) *p = static_cast<unsigned char>(bits);
  else if constexpr (kBytes == 2) *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(bits);
  else if constexpr (kBytes == 4) *reinterpret_cast<uint32_t*>(p) = static_cast<uint32_t>(bits);
  else *reinterpret_cast<unsigned long long*>(p) = bits;
}

template <int kBytes>
__device__ __forceinline__ uint64_t read_element_bits(const unsigned char* p) {
  if constexpr (kBytes == 1) return *p;
  else if constexpr (kBytes == 2) return *reinterpret_cast<const uint16_t*>(p);
  else if constexpr (kBytes == 4) return *reinterpret_cast<const uint32_t*>(p);
  else return *reinterpret_cast<const unsigned long long*>(p);
}

// out[i] = C(in[i]), i < n.  Threads take 16-element chunks (vector path
// when both buffers are 32-byte aligned); the rest goes element by element.
template <class C>
__device__ __forceinline__ void convert_body(const unsigned char* __restrict__ in, unsigned char* __restrict__ out,
                                             uint64_t n) {
  constexpr int kInWords = kConvertChunk * C::kIn / 4, kOutWords = kConvertChunk * C::kOut / 4;
  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t nthreads = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  uint64_t done = 0;
  if (((reinterpret_cast<uint64_t>(in) | reinterpret_cast<uint64_t>(out)) & 31u) == 0) {
    const uint64_t chunks = n / kConvertChunk;
    for (uint64_t c = tid; c < chunks; c += nthreads) {
      uint32_t w[kInWords], o[kOutWords];
      load_words<kInWords>(in + c * (kConvertChunk * C::kIn), w);
      C::chunk(w, o);
      store_words<kOutWords>(out + c * (kConvertChunk * C::kOut), o);
    }
    done = chunks * kConvertChunk;
  }
  for (uint64_t i = done + tid; i < n; i += nthreads)
    store_element_bits<C::kOut>(out + i * C::kOut, C::one(read_element_bits<C::kIn>(in + i * C::kIn)));
}

}  // namespace f4s

namespace f4s {
// one alias per kernel (template arguments cannot pass through the macro)
using Convert_f32_f16_rn = ToHalfConvert<false, kRoundNearestEven>;
using Convert_f32_f16_rz = ToHalfConvert<false, kRoundTowardZero>;
using Convert_f32_f16_ru = ToHalfConvert<false, kRoundUp>;
using Convert_f32_f16_rd = ToHalfConvert<false, kRoundDown>;
using Convert_f32_bf16_rn = ToHalfConvert<true, kRoundNearestEven>;
using Convert_f32_bf16_rz = ToHalfConvert<true, kRoundTowardZero>;
using Convert_f32_bf16_ru = ToHalfConvert<true, kRoundUp>;
using Convert_f32_bf16_rd = ToHalfConvert<true, kRoundDown>;
using Convert_f32_e4m3_sat = ToFp8Convert<true, true>;
using Convert_f32_e4m3_nosat = ToFp8Convert<true, false>;
using Convert_f32_e5m2_sat = ToFp8Convert<false, true>;
using Convert_f32_e5m2_nosat = ToFp8Convert<false, false>;
using Convert_f16_f32 = FromHalfConvert<false>;
using Convert_bf16_f32 = FromHalfConvert<true>;
using Convert_e4m3_f32 = FromFp8Convert<true>;
using Convert_e5m2_f32 = FromFp8Convert<false>;
using Convert_copy_1 = CopyConvert<1>;
using Convert_copy_2 = CopyConvert<2>;
using Convert_copy_4 = CopyConvert<4>;
using Convert_copy_8 = CopyConvert<8>;
}  // namespace f4s

// (in, out, n_lo, n_hi).  Grid: one 256-thread block per 4096 elements
// (capped by the host), block 256.
#define F4S_CONVERT_KERNEL(NAME, C)                                                             \
  extern "C" __global__ void __launch_bounds__(f4s::kConvertBlock)                               \
      NAME(const void* in, void* out, uint32_t n_lo, uint32_t n_hi) {                           \
    f4s::convert_body<C>(static_cast<const unsigned char*>(in), static_cast<unsigned char*>(out), \
                         f4s::join_u64(n_lo, n_hi));                                             \
  }
F4S_CONVERT_KERNEL(f4s_convert_f32_f16_rn, f4s::Convert_f32_f16_rn)
F4S_CONVERT_KERNEL(f4s_convert_f32_f16_rz, f4s::Convert_f32_f16_rz)
F4S_CONVERT_KERNEL(f4s_convert_f32_f16_ru, f4s::Convert_f32_f16_ru)
F4S_CONVERT_KERNEL(f4s_convert_f32_f16_rd, f4s::Convert_f32_f16_rd)
F4S_CONVERT_KERNEL(f4s_convert_f32_bf16_rn, f4s::Convert_f32_bf16_rn)
F4S_CONVERT_KERNEL(f4s_convert_f32_bf16_rz, f4s::Convert_f32_bf16_rz)
F4S_CONVERT_KERNEL(f4s_convert_f32_bf16_ru, f4s::Convert_f32_bf16_ru)
F4S_CONVERT_KERNEL(f4s_convert_f32_bf16_rd, f4s::Convert_f32_bf16_rd)
F4S_CONVERT_KERNEL(f4s_convert_f32_e4m3_sat, f4s::Convert_f32_e4m3_sat)
F4S_CONVERT_KERNEL(f4s_convert_f32_e4m3_nosat, f4s::Convert_f32_e4m3_nosat)
F4S_CONVERT_KERNEL(f4s_convert_f32_e5m2_sat, f4s::Convert_f32_e5m2_sat)
F4S_CONVERT_KERNEL(f4s_convert_f32_e5m2_nosat, f4s::Convert_f32_e5m2_nosat)
F4S_CONVERT_KERNEL(f4s_convert_f16_f32, f4s::Convert_f16_f32)
F4S_CONVERT_KERNEL(f4s_convert_bf16_f32, f4s::Convert_bf16_f32)
F4S_CONVERT_KERNEL(f4s_convert_e4m3_f32, f4s::Convert_e4m3_f32)
F4S_CONVERT_KERNEL(f4s_convert_e5m2_f32, f4s::Convert_e5m2_f32)
F4S_CONVERT_KERNEL(f4s_convert_copy_1, f4s::Convert_copy_1)
F4S_CONVERT_KERNEL(f4s_convert_copy_2, f4s::Convert_copy_2)
F4S_CONVERT_KERNEL(f4s_convert_copy_4, f4s::Convert_copy_4)
F4S_CONVERT_KERNEL(f4s_convert_copy_8, f4s::Convert_copy_8)
#undef F4S_CONVERT_KERNEL
