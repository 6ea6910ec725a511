// Elementwise vectorAdd, c[i] = a[i] + b[i], in fp32 and bf16.
//
// Reference: the DSL-generated `vectorAdd` test kernel
// (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:108-227,
// generated text core/src/test/scala/flight4s/core/codegen/CudaCodegenSuite.scala:15-61):
// one guarded scalar add per thread, parameters (left, right, output,
// elementCount:int).  These kernels keep that parameter list and meaning.
//
// B200 mapping: a persistent grid (a multiple of the SM count) strides over
// 16-byte vectors with kAddUnroll vectors of each operand in flight per
// thread; loads bypass L1 and stores are marked evict-first, since every
// byte is touched once.  The bf16 variant widens to f32, adds, and rounds
// to nearest-even, which equals the correctly rounded bf16 sum (the exact
// sum of two bf16 values is representable in f32 whenever rounding could
// matter).  Misaligned or ragged inputs take a scalar path with the same
// arithmetic.
#pragma once

#include "common.cuh"

namespace f4s {

constexpr int kAddBlock = 256;
constexpr int kAddUnroll = 4;

__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  return pack_bf16x2_rn(bf16_lo(a) + bf16_lo(b), bf16_hi(a) + bf16_hi(b));
}

__device__ __forceinline__ uint16_t add_bf16(uint16_t a, uint16_t b) {
  const float s = __uint_as_float(static_cast<uint32_t>(a) << 16) +
                  __uint_as_float(static_cast<uint32_t>(b) << 16);
  return static_cast<uint16_t>(pack_bf16x2_rn(s, 0.0f) & 0xFFFFu);
}

}  // namespace f4s

extern "C" __global__ void __launch_bounds__(f4s::kAddBlock)
f4s_vector_add_f32(const float* __restrict__ left, const float* __restrict__ right,
                   float* __restrict__ output, int element_count) {
  using namespace f4s;
  const size_t n = element_count > 0 ? static_cast<size_t>(element_count) : 0;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nthreads = static_cast<size_t>(gridDim.x) * blockDim.x;
  const bool aligned = ((reinterpret_cast<uintptr_t>(left) | reinterpret_cast<uintptr_t>(right) |
                         reinterpret_cast<uintptr_t>(output)) & 15u) == 0;
  size_t done = 0;
  if (aligned) {
    const size_t nvec = n / 4;
    const uint4* a = reinterpret_cast<const uint4*>(left);
    const uint4* b = reinterpret_cast<const uint4*>(right);
    uint4* c = reinterpret_cast<uint4*>(output);
    size_t base = tid;
    for (; base + (kAddUnroll - 1) * nthreads < nvec; base += kAddUnroll * nthreads) {
      uint4 va[kAddUnroll], vb[kAddUnroll];
#pragma unroll
      for (int u = 0; u < kAddUnroll; ++u) {
        va[u] = ld_stream_u4(a + base + u * nthreads);
        vb[u] = ld_stream_u4(b + base + u * nthreads);
      }
#pragma unroll
      for (int u = 0; u < kAddUnroll; ++u) {
        uint4 r;
        r.x = __float_as_uint(__uint_as_float(va[u].x) + __uint_as_float(vb[u].x));
        r.y = __float_as_uint(__uint_as_float(va[u].y) + __uint_as_float(vb[u].y));
        r.z = __float_as_uint(__uint_as_float(va[u].z) + __uint_as_float(vb[u].z));
        r.w = __float_as_uint(__uint_as_float(va[u].w) + __uint_as_float(vb[u].w));
        st_stream_u4(c + base + u * nthreads, r);
      }
    }
    for (; base < nvec; base += nthreads) {
      const uint4 va = ld_stream_u4(a + base), vb = ld_stream_u4(b + base);
      uint4 r;
      r.x = __float_as_uint(__uint_as_float(va.x) + __uint_as_float(vb.x));
      r.y = __float_as_uint(__uint_as_float(va.y) + __uint_as_float(vb.y));
      r.z = __float_as_uint(__uint_as_float(va.z) + __uint_as_float(vb.z));
      r.w = __float_as_uint(__uint_as_float(va.w) + __uint_as_float(vb.w));
      st_stream_u4(c + base, r);
    }
    done = nvec * 4;
  }
  for (size_t i = done + tid; i < n; i += nthreads) output[i] = left[i] + right[i];
}

extern "C" __global__ void __launch_bounds__(f4s::kAddBlock)
f4s_vector_add_bf16(const uint16_t* __restrict__ left, const uint16_t* __restrict__ right,
                    uint16_t* __restrict__ output, int element_count) {
  using namespace f4s;
  const size_t n = element_count > 0 ? static_cast<size_t>(element_count) : 0;
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nthreads = static_cast<size_t>(gridDim.x) * blockDim.x;
  const bool aligned = ((reinterpret_cast<uintptr_t>(left) | reinterpret_cast<uintptr_t>(right) |
                         reinterpret_cast<uintptr_t>(output)) & 15u) == 0;
  size_t done = 0;
  if (aligned) {
    const size_t nvec = n / 8;
    const uint4* a = reinterpret_cast<const uint4*>(left);
    const uint4* b = reinterpret_cast<const uint4*>(right);
    uint4* c = reinterpret_cast<uint4*>(output);
    size_t base = tid;
    for (; base + (kAddUnroll - 1) * nthreads < nvec; base += kAddUnroll * nthreads) {
      uint4 va[kAddUnroll], vb[kAddUnroll];
#pragma unroll
      for (int u = 0; u < kAddUnroll; ++u) {
        va[u] = ld_stream_u4(a + base + u * nthreads);
        vb[u] = ld_stream_u4(b + base + u * nthreads);
      }
#pragma unroll
      for (int u = 0; u < kAddUnroll; ++u) {
        uint4 r;
        r.x = add_bf16x2(va[u].x, vb[u].x);
        r.y = add_bf16x2(va[u].y, vb[u].y);
        r.z = add_bf16x2(va[u].z, vb[u].z);
        r.w = add_bf16x2(va[u].w, vb[u].w);
        st_stream_u4(c + base + u * nthreads, r);
      }
    }
    for (; base < nvec; base += nthreads) {
      const uint4 va = ld_stream_u4(a + base), vb = ld_stream_u4(b + base);
      uint4 r;
      r.x = add_bf16x2(va.x, vb.x);
      r.y = add_bf16x2(va.y, vb.y);
      r.z = add_bf16x2(va.z, vb.z);
      r.w = add_bf16x2(va.w, vb.w);
      st_stream_u4(c + base, r);
    }
    done = nvec * 8;
  }
  for (size_t i = done + tid; i < n; i += nthreads) output[i] = add_bf16(left[i], right[i]);
}
