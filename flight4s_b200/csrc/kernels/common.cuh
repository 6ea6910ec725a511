// Shared device helpers for the sm_100a hot-path kernels.
//
// Everything here is plain integer / IEEE arithmetic or a documented PTX
// instruction; no CUDA math-library routine is restated.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace f4s {

constexpr int kWarp = 32;

// ---------------------------------------------------------------- loads/stores
// Streaming 128-bit global loads: the hot paths touch every byte exactly
// once, so they bypass L1.  (sm_100 accepts an L2 eviction hint only on the
// 256-bit forms below.)
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 256-bit global load / store (sm_100), evict-first in L2.
struct u32x8 {
  uint4 lo, hi;
};
__device__ __forceinline__ u32x8 ld_stream_v8(const void* p) {
  u32x8 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(v.lo.x), "=r"(v.lo.y), "=r"(v.lo.z), "=r"(v.lo.w), "=r"(v.hi.x), "=r"(v.hi.y),
        "=r"(v.hi.z), "=r"(v.hi.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream_v8(void* p, const u32x8& v) {
  asm volatile(
      "st.global.L1::no_allocate.L2::evict_first.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
      :
      : "l"(p), "r"(v.lo.x), "r"(v.lo.y), "r"(v.lo.z), "r"(v.lo.w), "r"(v.hi.x), "r"(v.hi.y),
        "r"(v.hi.z), "r"(v.hi.w)
      : "memory");
}

__device__ __forceinline__ float4 ld_stream_f4(const void* p) {
  uint4 v = ld_stream_u4(p);
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y),
                     __uint_as_float(v.z), __uint_as_float(v.w));
}

__device__ __forceinline__ void st_stream_u4(void* p, uint4 v) {
  asm volatile(
      "st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};"
      :
      : "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
      : "memory");
}

__device__ __forceinline__ void st_stream_u2(void* p, uint2 v) {
  asm volatile(
      "st.global.L1::no_allocate.v2.u32 [%0], {%1,%2};"
      :
      : "l"(p), "r"(v.x), "r"(v.y)
      : "memory");
}

// ------------------------------------------------------------------ bf16 bits
// bf16 -> f32 is exact: the bf16 pattern is the top half of the f32 pattern.
__device__ __forceinline__ float bf16_lo(uint32_t pair) {
  return __uint_as_float(pair << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t pair) {
  return __uint_as_float(pair & 0xFFFF0000u);
}

// Two f32 -> packed bf16x2 with IEEE round-to-nearest-even (subnormals kept).
// `lo` lands in bits [15:0], `hi` in bits [31:16].
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// ------------------------------------------------------------------ e4m3 bits
// Two f32 -> packed e4m3x2, round-to-nearest-even, saturating finite values
// to +-448 (OCP FP8 E4M3).  `lo` lands in bits [7:0], `hi` in bits [15:8].
__device__ __forceinline__ uint32_t pack_e4m3x2_satfinite(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Packed e4m3x2 (low 16 bits of `codes`) -> two f32, exact (every E4M3 value
// is representable in f16, and every f16 in f32).
__device__ __forceinline__ float2 unpack_e4m3x2(uint32_t codes) {
  uint32_t h2;
  uint16_t c = static_cast<uint16_t>(codes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c));
  float lo, hi;
  asm("{.reg .f16 l, h;\n"
      " mov.b32 {l, h}, %2;\n"
      " cvt.f32.f16 %0, l;\n"
      " cvt.f32.f16 %1, h;}"
      : "=f"(lo), "=f"(hi)
      : "r"(h2));
  return make_float2(lo, hi);
}

// Packed e5m2x2 (low 16 bits) -> two f32, exact (E5M2 is a subset of f16).
__device__ __forceinline__ float2 unpack_e5m2x2(uint32_t codes) {
  uint32_t h2;
  uint16_t c = static_cast<uint16_t>(codes);
  asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(c));
  float lo, hi;
  asm("{.reg .f16 l, h;\n"
      " mov.b32 {l, h}, %2;\n"
      " cvt.f32.f16 %0, l;\n"
      " cvt.f32.f16 %1, h;}"
      : "=f"(lo), "=f"(hi)
      : "r"(h2));
  return make_float2(lo, hi);
}

// Packed e4m3x2 / e5m2x2 (low 16 bits) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t codes) {
  uint32_t h2;
  const uint16_t c = static_cast<uint16_t>(codes);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c));
  return h2;
}
__device__ __forceinline__ uint32_t e5m2x2_to_f16x2(uint32_t codes) {
  uint32_t h2;
  const uint16_t c = static_cast<uint16_t>(codes);
  asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(c));
  return h2;
}

// acc + lo + hi for a packed f16x2 / bf16x2 word, with sm_100's
// mixed-precision add (the 16-bit operand widened exactly; each add rounds
// once to f32), low half first.
__device__ __forceinline__ float add_f16x2_to_f32(float acc, uint32_t w) {
  asm("{.reg .f16 l, h;\n"
      " mov.b32 {l, h}, %1;\n"
      " add.rn.f32.f16 %0, l, %0;\n"
      " add.rn.f32.f16 %0, h, %0;}"
      : "+f"(acc)
      : "r"(w));
  return acc;
}
__device__ __forceinline__ float add_bf16x2_to_f32(float acc, uint32_t w) {
  asm("{.reg .b16 l, h;\n"
      " mov.b32 {l, h}, %1;\n"
      " add.rn.f32.bf16 %0, l, %0;\n"
      " add.rn.f32.bf16 %0, h, %0;}"
      : "+f"(acc)
      : "r"(w));
  return acc;
}

// IEEE binary16 bits -> f32, exact.
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
  float f;
  asm("{.reg .f16 t;\n mov.b16 t, %1;\n cvt.f32.f16 %0, t;}" : "=f"(f) : "h"(h));
  return f;
}

// ---------------------------------------------------------------- total order
// Signed-int image of an f32 under IEEE-754 totalOrder:
// -NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN.
__device__ __forceinline__ int32_t total_order_key(float v) {
  int32_t b = __float_as_int(v);
  return b ^ static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
}
__device__ __forceinline__ float from_total_order_key(int32_t k) {
  int32_t b = k ^ static_cast<int32_t>(static_cast<uint32_t>(k >> 31) >> 1);
  return __int_as_float(b);
}

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ex2.approx: hardware base-2 exponential (documented PTX instruction).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 64-bit element counts travel as two u32 launch arguments so that every
// kernel parameter has a descriptor code the existing launch ABI knows.
__device__ __forceinline__ uint64_t join_u64(uint32_t lo, uint32_t hi) {
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

}  // namespace f4s
