// Elementwise vectorAdd, c[i] = a[i] + b[i], in fp32 and bf16.
//
// Reference: the DSL-generated `vectorAdd` test kernel
// (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:108-227,
// generated text core/src/test/scala/flight4s/core/codegen/CudaCodegenSuite.scala:15-61):
// one guarded scalar add per thread, parameters (left, right, output,
// elementCount:int).  These kernels keep that parameter list and meaning.
//
// B200 mapping: one thread per 32-byte vector of each operand, loaded and
// stored with the sm_100 256-bit global instructions (L1 bypassed, L2
// evict-first: every byte is touched once).  The bf16 variant widens to
// f32, adds, and rounds to nearest-even, which equals the correctly rounded
// bf16 sum (the exact sum of two bf16 values is representable in f32
// whenever rounding could matter).  Misaligned or ragged inputs take a
// scalar path with the same arithmetic.
#pragma once

#include "common.cuh"

namespace f4s {

constexpr int kAddBlock = 256;

__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  return pack_bf16x2_rn(bf16_lo(a) + bf16_lo(b), bf16_hi(a) + bf16_hi(b));
}

__device__ __forceinline__ uint16_t add_bf16(uint16_t a, uint16_t b) {
  const float s = __uint_as_float(static_cast<uint32_t>(a) << 16) +
                  __uint_as_float(static_cast<uint32_t>(b) << 16);
  return static_cast<uint16_t>(pack_bf16x2_rn(s, 0.0f) & 0xFFFFu);
}

__device__ __forceinline__ uint32_t add_f32_bits(uint32_t a, uint32_t b) {
  return __float_as_uint(__uint_as_float(a) + __uint_as_float(b));
}

// IEEE binary16 add, round to nearest-even: two lanes at once (add.f16x2)
// and one (add.f16).  These are the operation the reference's `+` on
// __half operands performs.
__device__ __forceinline__ uint32_t add_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint16_t add_f16(uint16_t a, uint16_t b) {
  uint16_t d;
  asm("{.reg .f16 x, y, z;\n mov.b16 x, %1;\n mov.b16 y, %2;\n add.rn.f16 z, x, y;\n mov.b16 %0, z;}"
      : "=h"(d)
      : "h"(a), "h"(b));
  return d;
}

__device__ __forceinline__ uint2 add_f64_bits(uint32_t alo, uint32_t ahi, uint32_t blo, uint32_t bhi) {
  const double r = __hiloint2double(static_cast<int>(ahi), static_cast<int>(alo)) +
                   __hiloint2double(static_cast<int>(bhi), static_cast<int>(blo));
  return make_uint2(static_cast<uint32_t>(__double2loint(r)), static_cast<uint32_t>(__double2hiint(r)));
}

// Element kinds of c = a + b, one per AdditiveType of the reference
// (core/src/main/scala/flight4s/core/types/CudaType.scala:154-160).
enum class AddKind { kF32, kBf16, kF16, kF64, kWrap32 };

// Four 32-bit words of c = a + b.
template <AddKind K>
__device__ __forceinline__ uint4 add4(uint4 a, uint4 b) {
  if constexpr (K == AddKind::kBf16) {
    return make_uint4(add_bf16x2(a.x, b.x), add_bf16x2(a.y, b.y), add_bf16x2(a.z, b.z), add_bf16x2(a.w, b.w));
  } else if constexpr (K == AddKind::kF16) {
    return make_uint4(add_f16x2(a.x, b.x), add_f16x2(a.y, b.y), add_f16x2(a.z, b.z), add_f16x2(a.w, b.w));
  } else if constexpr (K == AddKind::kF64) {
    const uint2 lo = add_f64_bits(a.x, a.y, b.x, b.y), hi = add_f64_bits(a.z, a.w, b.z, b.w);
    return make_uint4(lo.x, lo.y, hi.x, hi.y);
  } else if constexpr (K == AddKind::kWrap32) {
    return make_uint4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  } else {
    return make_uint4(add_f32_bits(a.x, b.x), add_f32_bits(a.y, b.y), add_f32_bits(a.z, b.z),
                      add_f32_bits(a.w, b.w));
  }
}

// One element of c = a + b.
template <AddKind K, class T>
__device__ __forceinline__ T add1(T a, T b) {
  if constexpr (K == AddKind::kBf16) return add_bf16(a, b);
  else if constexpr (K == AddKind::kF16) return add_f16(a, b);
  else if constexpr (K == AddKind::kWrap32) return static_cast<T>(static_cast<uint32_t>(a) + static_cast<uint32_t>(b));
  else return a + b;
}

// One 32-byte vector per operand per thread: the host sizes the grid to
// cover the array, so the loop below normally runs once (measured faster
// on B200 than persistent grid-stride forms, which leave SMs idle at the
// tail); any other grid, e.g. the reference's one-element-per-thread
// LaunchConfig, is still correct.  The < 32-byte tail, or the whole array
// when the pointers are not 32-byte aligned, takes scalar loads.
template <AddKind K, class T>
__device__ __forceinline__ void vector_add_body(const T* __restrict__ left, const T* __restrict__ right,
                                                T* __restrict__ output, int element_count) {
  constexpr int kPerVec = 32 / sizeof(T);
  const size_t n = element_count > 0 ? static_cast<size_t>(element_count) : 0;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nthreads = static_cast<size_t>(gridDim.x) * blockDim.x;
  const bool aligned = ((reinterpret_cast<uintptr_t>(left) | reinterpret_cast<uintptr_t>(right) |
                         reinterpret_cast<uintptr_t>(output)) & 31u) == 0;
  const size_t nvec = aligned ? n / kPerVec : 0;
  for (size_t v = tid; v < nvec; v += nthreads) {
    const u32x8 a = ld_stream_v8(left + v * kPerVec);
    const u32x8 b = ld_stream_v8(right + v * kPerVec);
    u32x8 c;
    c.lo = add4<K>(a.lo, b.lo);
    c.hi = add4<K>(a.hi, b.hi);
    st_stream_v8(output + v * kPerVec, c);
  }
  for (size_t i = nvec * kPerVec + tid; i < n; i += nthreads) output[i] = add1<K>(left[i], right[i]);
}

}  // namespace f4s

// Parameters (left, right, output, elementCount) as in the reference's
// generated vectorAdd.  Fastest with blockDim 256 and a grid of
// ceil(n / elements-per-32-bytes) threads.
#define F4S_VECTOR_ADD(NAME, KIND, T)                                                              \
  extern "C" __global__ void __launch_bounds__(f4s::kAddBlock)                                     \
      NAME(const T* __restrict__ left, const T* __restrict__ right, T* __restrict__ output,         \
           int element_count) {                                                                    \
    f4s::vector_add_body<f4s::AddKind::KIND>(left, right, output, element_count);                  \
  }
F4S_VECTOR_ADD(f4s_vector_add_f32, kF32, float)
F4S_VECTOR_ADD(f4s_vector_add_bf16, kBf16, uint16_t)
// the other AdditiveTypes: f16 (IEEE add, nearest-even), f64, and i32 / u32
// (32-bit wrap: one kernel, the bits are the same)
F4S_VECTOR_ADD(f4s_vector_add_f16, kF16, uint16_t)
F4S_VECTOR_ADD(f4s_vector_add_f64, kF64, double)
F4S_VECTOR_ADD(f4s_vector_add_i32, kWrap32, uint32_t)
#undef F4S_VECTOR_ADD
