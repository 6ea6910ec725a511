// FP8 E4M3 block quantize (with fused amax) and dequantize, 1x128 blocks.
//
// Element conversion is the reference's: f32 -> E4M3 with round-to-nearest-
// even and finite saturation, i.e. the `__nv_cvt_float_to_fp8(v,
// __NV_SATFINITE, __NV_E4M3)` call its code generator emits
// (core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:418-428,525-538)
// for `convert.f32ToFP8E4M3` (core/src/main/scala/flight4s/core/dsl/CudaDsl.scala:526-535);
// here it is the `cvt.rn.satfinite.e4m3x2.f32` instruction.  The block
// scaling around it is new (the reference has no amax or block quantizer):
//
//   amax  = max |x| over the block (NaN ignored; max(NaN, v) = v)
//   scale = amax / 448                      (f32, IEEE division)
//   inv   = amax > 0 ? min(448 / amax, FLT_MAX) : 0
//   q     = e4m3_rn_satfinite(x * inv)     (f32 multiply, one rounding)
//   deq   = bf16_rn(f32(q) * scale)
//
// Every step is an IEEE-754 operation with one rounding, so a CPU
// restatement reproduces the codes and the dequantized values bit for bit.
//
// Layout: x bf16 [rows x cols] row-major; codes u8 [rows x cols]; scales f32
// [rows x ceil(cols/128)].  When cols % 128 == 0 the blocks tile memory
// contiguously and the vector kernels treat the tensor as a flat run of
// 128-element blocks; other widths use the per-row kernels.
#pragma once

#include "common.cuh"

namespace f4s {

constexpr int kFp8Block = 128;
constexpr int kFp8Threads = 256;
constexpr int kQuantUnroll = 4;    // 4-block steps in flight per warp
constexpr int kDequantUnroll = 2;
constexpr float kE4m3Max = 448.0f;
constexpr float kFltMax = 3.402823466e38f;

__device__ __forceinline__ float abs_max_bf16x2(float m, uint32_t pair) {
  return fmaxf(m, fmaxf(fabsf(bf16_lo(pair)), fabsf(bf16_hi(pair))));
}

__device__ __forceinline__ void block_scale(float amax, float& scale, float& inv) {
  scale = __fdiv_rn(amax, kE4m3Max);
  inv = amax > 0.0f ? fminf(__fdiv_rn(kE4m3Max, amax), kFltMax) : 0.0f;
}

__device__ __forceinline__ uint32_t quant_bf16x2(uint32_t pair, float inv) {
  return pack_e4m3x2_satfinite(__fmul_rn(bf16_lo(pair), inv), __fmul_rn(bf16_hi(pair), inv));
}

// four e4m3 codes -> four bf16 (two packed words)
__device__ __forceinline__ uint2 dequant_x4(uint32_t codes, float scale) {
  const float2 a = unpack_e4m3x2(codes & 0xFFFFu);
  const float2 b = unpack_e4m3x2(codes >> 16);
  return make_uint2(pack_bf16x2_rn(__fmul_rn(a.x, scale), __fmul_rn(a.y, scale)),
                    pack_bf16x2_rn(__fmul_rn(b.x, scale), __fmul_rn(b.y, scale)));
}

}  // namespace f4s

// Flat vector kernels: every block is 128 contiguous elements (cols % 128
// == 0), so the tensor is a flat run of blocks.  A quarter-warp (8 lanes)
// owns one block and each lane 16 elements: the quantizer reads them with
// one 256-bit load (32 bytes of bf16), takes the amax with 3 xor shuffles
// inside the quarter-warp and stores 16 codes (16 bytes); the dequantizer
// reads 16 codes and writes 32 bytes of bf16 with one 256-bit store.  A warp
// covers 4 blocks per step and keeps kQuantUnroll / kDequantUnroll steps in
// flight; the host launches enough warps that each runs its loop about once.
// (minBlocksPerSM = 2 lets ptxas keep all four 32-byte loads in registers:
// without it, it stops at 64 registers and spills.)
extern "C" __global__ void __launch_bounds__(f4s::kFp8Threads, 2)
f4s_fp8_quant_flat(const uint16_t* __restrict__ x, uint8_t* __restrict__ codes,
                   float* __restrict__ scales, int num_blocks) {
  using namespace f4s;
  const int lane = threadIdx.x % kWarp;
  const int quarter = lane >> 3;  // which block of the warp's four
  const int sub = lane & 7;       // 16-element slice within the block
  const size_t warp_id = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const size_t nwarps = static_cast<size_t>(gridDim.x) * blockDim.x / kWarp;
  const size_t quads = (static_cast<size_t>(num_blocks) + 3) / 4;
  for (size_t q0 = warp_id; q0 < quads; q0 += nwarps * kQuantUnroll) {
    u32x8 raw[kQuantUnroll];
    bool live[kQuantUnroll];
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const size_t blk = 4 * (q0 + u * nwarps) + quarter;
      live[u] = (q0 + u * nwarps) < quads && blk < static_cast<size_t>(num_blocks);
      if (live[u]) {
        raw[u] = ld_stream_v8(x + blk * kFp8Block + sub * 16);
      } else {
        raw[u].lo = make_uint4(0, 0, 0, 0);
        raw[u].hi = raw[u].lo;
      }
    }
#pragma unroll
    for (int u = 0; u < kQuantUnroll; ++u) {
      const uint32_t w[8] = {raw[u].lo.x, raw[u].lo.y, raw[u].lo.z, raw[u].lo.w,
                             raw[u].hi.x, raw[u].hi.y, raw[u].hi.z, raw[u].hi.w};
      float amax = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = abs_max_bf16x2(amax, w[j]);
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      float scale, inv;
      block_scale(amax, scale, inv);
      if (live[u]) {
        const size_t blk = 4 * (q0 + u * nwarps) + quarter;
        uint4 q;
        q.x = quant_bf16x2(w[0], inv) | (quant_bf16x2(w[1], inv) << 16);
        q.y = quant_bf16x2(w[2], inv) | (quant_bf16x2(w[3], inv) << 16);
        q.z = quant_bf16x2(w[4], inv) | (quant_bf16x2(w[5], inv) << 16);
        q.w = quant_bf16x2(w[6], inv) | (quant_bf16x2(w[7], inv) << 16);
        st_stream_u4(codes + blk * kFp8Block + sub * 16, q);
        if (sub == 0) scales[blk] = scale;
      }
    }
  }
}

extern "C" __global__ void __launch_bounds__(f4s::kFp8Threads)
f4s_fp8_dequant_flat(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                     uint16_t* __restrict__ y, int num_blocks) {
  using namespace f4s;
  const int lane = threadIdx.x % kWarp;
  const int quarter = lane >> 3;
  const int sub = lane & 7;
  const size_t warp_id = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const size_t nwarps = static_cast<size_t>(gridDim.x) * blockDim.x / kWarp;
  const size_t quads = (static_cast<size_t>(num_blocks) + 3) / 4;
  for (size_t q0 = warp_id; q0 < quads; q0 += nwarps * kDequantUnroll) {
    uint4 raw[kDequantUnroll];
    float sc[kDequantUnroll];
    bool live[kDequantUnroll];
#pragma unroll
    for (int u = 0; u < kDequantUnroll; ++u) {
      const size_t blk = 4 * (q0 + u * nwarps) + quarter;
      live[u] = (q0 + u * nwarps) < quads && blk < static_cast<size_t>(num_blocks);
      raw[u] = live[u] ? ld_stream_u4(codes + blk * kFp8Block + sub * 16) : make_uint4(0, 0, 0, 0);
      sc[u] = live[u] ? __ldg(scales + blk) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kDequantUnroll; ++u) {
      if (live[u]) {
        const size_t blk = 4 * (q0 + u * nwarps) + quarter;
        const uint2 a = dequant_x4(raw[u].x, sc[u]);
        const uint2 b = dequant_x4(raw[u].y, sc[u]);
        const uint2 c = dequant_x4(raw[u].z, sc[u]);
        const uint2 d = dequant_x4(raw[u].w, sc[u]);
        u32x8 o;
        o.lo = make_uint4(a.x, a.y, b.x, b.y);
        o.hi = make_uint4(c.x, c.y, d.x, d.y);
        st_stream_v8(y + blk * kFp8Block + sub * 16, o);
      }
    }
  }
}

// Per-row kernels for any width: (x, codes, scales, rows, cols) and
// (codes, scales, y, rows, cols).  One warp per 128-element block (the last
// block of a row may be short), scalar loads, same arithmetic.
extern "C" __global__ void __launch_bounds__(f4s::kFp8Threads)
f4s_fp8_quant_rows(const uint16_t* __restrict__ x, uint8_t* __restrict__ codes,
                   float* __restrict__ scales, int rows, int cols) {
  using namespace f4s;
  const int lane = threadIdx.x % kWarp;
  const size_t warp_id = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const size_t nwarps = static_cast<size_t>(gridDim.x) * blockDim.x / kWarp;
  const int bpr = (cols + kFp8Block - 1) / kFp8Block;
  const size_t total = static_cast<size_t>(rows) * bpr;
  for (size_t b = warp_id; b < total; b += nwarps) {
    const size_t r = b / bpr;
    const int c0 = static_cast<int>(b % bpr) * kFp8Block;
    float v[4];
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      v[k] = (c < cols) ? __uint_as_float(static_cast<uint32_t>(x[r * cols + c]) << 16) : 0.0f;
      amax = fmaxf(amax, fabsf(v[k]));
    }
    amax = warp_max_f32(amax);
    float scale, inv;
    block_scale(amax, scale, inv);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      if (c < cols)
        codes[r * cols + c] = static_cast<uint8_t>(pack_e4m3x2_satfinite(__fmul_rn(v[k], inv), 0.0f));
    }
    if (lane == 0) scales[b] = scale;
  }
}

extern "C" __global__ void __launch_bounds__(f4s::kFp8Threads)
f4s_fp8_dequant_rows(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                     uint16_t* __restrict__ y, int rows, int cols) {
  using namespace f4s;
  const int lane = threadIdx.x % kWarp;
  const size_t warp_id = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarp;
  const size_t nwarps = static_cast<size_t>(gridDim.x) * blockDim.x / kWarp;
  const int bpr = (cols + kFp8Block - 1) / kFp8Block;
  const size_t total = static_cast<size_t>(rows) * bpr;
  for (size_t b = warp_id; b < total; b += nwarps) {
    const size_t r = b / bpr;
    const int c0 = static_cast<int>(b % bpr) * kFp8Block;
    const float scale = scales[b];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      if (c < cols) {
        const float q = unpack_e4m3x2(codes[r * cols + c]).x;
        y[r * cols + c] = static_cast<uint16_t>(pack_bf16x2_rn(__fmul_rn(q, scale), 0.0f) & 0xFFFFu);
      }
    }
  }
}
