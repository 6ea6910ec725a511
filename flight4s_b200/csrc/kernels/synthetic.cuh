// Seeded synthetic inputs generated on the device.
//
// Counter-based Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC'11).  Element i of stream s under key
// `seed` takes word (i % 4) of philox(counter = {i/4 lo, i/4 hi, s, 0},
// key = {seed lo, seed hi}), so any shard of an array can be generated
// independently and the host can regenerate uniform and integer streams
// bit for bit.
//
// Distributions (all exact integer / IEEE steps except the normal):
//   uniform f32 [-1,1):   (w >> 8) * 2^-23 - 1
//   uniform i32 [lo,hi]:  lo + w % (hi - lo + 1)
//   normal f32 (mean, sd): Box-Muller on words (2j, 2j+1) of one draw,
//                          u1 = ((w0 >> 8) + 1) * 2^-24 in (0,1],
//                          u2 = (w1 >> 8) * 2^-24 in [0,1);
//                          outlier option: with probability p (word of
//                          stream s+1 below p * 2^32) the value is scaled.
// The normal uses the device's logf / sincospif, so host code downloads
// normal-distributed data instead of regenerating it.
#pragma once

#include "common.cuh"

namespace f4s {

__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint2 key) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, ctr.x), lo0 = kM0 * ctr.x;
    const uint32_t hi1 = __umulhi(kM1, ctr.z), lo1 = kM1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += kW0;
    key.y += kW1;
  }
  return ctr;
}

__device__ __forceinline__ uint4 philox_draw(uint64_t group, uint32_t stream, uint64_t seed) {
  return philox4x32_10(make_uint4(static_cast<uint32_t>(group), static_cast<uint32_t>(group >> 32),
                                  stream, 0u),
                       make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32)));
}

__device__ __forceinline__ float uniform_pm1(uint32_t w) {
  return static_cast<float>(w >> 8) * 0x1p-23f - 1.0f;
}

__device__ __forceinline__ float2 box_muller(uint32_t w0, uint32_t w1) {
  const float u1 = static_cast<float>((w0 >> 8) + 1u) * 0x1p-24f;
  const float u2 = static_cast<float>(w1 >> 8) * 0x1p-24f;
  const float rad = sqrtf(-2.0f * logf(u1));
  float s, c;
  sincospif(2.0f * u2, &s, &c);
  return make_float2(rad * c, rad * s);
}

}  // namespace f4s

// Element ranges are [offset, offset + n) of the global stream, written to
// out[0, n).  kind selects the distribution:
//   0 uniform f32 [-1,1)            -> f32
//   1 uniform f32 [-1,1) -> bf16 rn -> bf16
//   2 normal f32 (p0 = mean, p1 = sd)
//   3 normal -> bf16 rn
//   4 uniform i32 [ilo, ihi]
//   5 normal -> bf16 rn with outliers: probability p2, factor p3
extern "C" __global__ void f4s_fill_synthetic(void* __restrict__ out, uint32_t n_lo, uint32_t n_hi,
                                              uint32_t off_lo, uint32_t off_hi, uint32_t seed_lo,
                                              uint32_t seed_hi, uint32_t stream, int kind, float p0,
                                              float p1, float p2, float p3, int ilo, int ihi) {
  using namespace f4s;
  const uint64_t n = join_u64(n_lo, n_hi);
  const uint64_t offset = join_u64(off_lo, off_hi);
  const uint64_t seed = join_u64(seed_lo, seed_hi);
  const uint64_t nthreads = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  // One thread per group of 4 global elements.
  const uint64_t g_first = offset / 4;
  const uint64_t g_last = (offset + n + 3) / 4;
  for (uint64_t g = g_first + static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       g < g_last; g += nthreads) {
    const uint4 w = philox_draw(g, stream, seed);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    float vals[4];
    if (kind == 2 || kind == 3 || kind == 5) {
      const float2 z0 = box_muller(w.x, w.y);
      const float2 z1 = box_muller(w.z, w.w);
      vals[0] = p0 + p1 * z0.x;
      vals[1] = p0 + p1 * z0.y;
      vals[2] = p0 + p1 * z1.x;
      vals[3] = p0 + p1 * z1.y;
      if (kind == 5) {
        const uint4 o = philox_draw(g, stream + 1u, seed);
        const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
        const uint32_t threshold = static_cast<uint32_t>(p2 * 4294967296.0f);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (ow[j] < threshold) vals[j] *= p3;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) vals[j] = uniform_pm1(words[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint64_t gi = 4 * g + j;
      if (gi < offset || gi >= offset + n) continue;
      const uint64_t i = gi - offset;
      switch (kind) {
        case 0:
        case 2:
          static_cast<float*>(out)[i] = vals[j];
          break;
        case 1:
        case 3:
        case 5:
          static_cast<uint16_t*>(out)[i] = static_cast<uint16_t>(pack_bf16x2_rn(vals[j], 0.0f) & 0xFFFFu);
          break;
        case 4: {
          const uint32_t span = static_cast<uint32_t>(ihi - ilo) + 1u;
          static_cast<int32_t*>(out)[i] = ilo + static_cast<int32_t>(words[j] % span);
          break;
        }
        default:
          break;
      }
    }
  }
}
