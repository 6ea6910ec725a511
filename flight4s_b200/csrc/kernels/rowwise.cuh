// Row-wise softmax and RMSNorm over bf16 [rows x cols] with fp32 math.
//
// The reference has neither op (no exp, rsqrt or row max in its DSL or
// codegen); its data model fixes the types: bf16 storage accumulates in f32
// (core/src/main/scala/flight4s/core/types/CudaType.scala:222-224) and f32 ->
// bf16 stores round to nearest-even (`__float2bfloat16_rn`,
// core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:518-523).
//
//   softmax: y = bf16_rn( exp(x - max) * (1 / sum exp(x - max)) )
//   rmsnorm: y = bf16_rn( (x * rsqrt(mean(x^2) + eps)) * w )
//
// B200 mapping: a 256-thread CTA per row; a row of up to 256*8*VPT bf16
// lives in registers (VPT 16-byte vectors per thread), so HBM sees exactly
// one read and one write per element.  Softmax gives each CTA two rows and
// loads the second while reducing the first (one row per CTA at the widest
// register width).
// RMSNorm on rows of 2049..8192 elements stages whole rows in shared memory
// with bulk copies (TMA) in persistent CTAs; other widths use persistent
// CTAs that keep the weight slice in registers and prefetch their next row.  Row reductions are warp shuffles plus
// one shared-memory exchange.  Rows that are not a multiple of 8 elements
// wide, or too wide for registers, use a looped kernel that re-reads the row
// (from L2 for realistic widths) with the same arithmetic.
#pragma once

#include "common.cuh"
#include "staging.cuh"

namespace f4s {

constexpr int kRowBlock = 256;
constexpr int kRowWarps = kRowBlock / kWarp;
constexpr float kLog2e = 1.4426950408889634f;

// Block-wide reductions; every thread receives the result.  `scratch` holds
// kRowWarps floats and must not be reused until after the next barrier.
__device__ __forceinline__ float block_max(float v, float* scratch) {
  v = warp_max_f32(v);
  if ((threadIdx.x % kWarp) == 0) scratch[threadIdx.x / kWarp] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll
  for (int w = 1; w < kRowWarps; ++w) r = fmaxf(r, scratch[w]);
  return r;
}

__device__ __forceinline__ float block_sum(float v, float* scratch) {
  v = warp_sum_f32(v);
  if ((threadIdx.x % kWarp) == 0) scratch[threadIdx.x / kWarp] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll
  for (int w = 1; w < kRowWarps; ++w) r += scratch[w];
  return r;
}

template <int VPT>
__device__ __forceinline__ void store_row(uint16_t* row, const float (&y)[VPT * 8],
                                          const bool (&valid)[VPT]) {
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    if (valid[k]) {
      uint4 r;
      r.x = pack_bf16x2_rn(y[k * 8 + 0], y[k * 8 + 1]);
      r.y = pack_bf16x2_rn(y[k * 8 + 2], y[k * 8 + 3]);
      r.z = pack_bf16x2_rn(y[k * 8 + 4], y[k * 8 + 5]);
      r.w = pack_bf16x2_rn(y[k * 8 + 6], y[k * 8 + 7]);
      st_stream_u4(reinterpret_cast<uint4*>(row) + threadIdx.x + k * kRowBlock, r);
    }
  }
}

// Softmax of one row held as raw bf16 vectors (`raw[k]` = the row's 16-byte
// vector threadIdx.x + k * kRowBlock, zero past nvec): max, exp and sum in
// f32, one block reduction each, then the row scaled and stored.
template <int VPT>
__device__ __forceinline__ void softmax_row_math(const uint4 (&raw)[VPT], int nvec, uint16_t* out,
                                                 float* red_a, float* red_b) {
  float x[VPT * 8];
  bool valid[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    valid[k] = static_cast<int>(threadIdx.x) + k * kRowBlock < nvec;
    const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[k * 8 + 2 * j] = bf16_lo(w[j]);
      x[k * 8 + 2 * j + 1] = bf16_hi(w[j]);
    }
  }
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < VPT; ++k)
    if (valid[k])
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, x[k * 8 + j]);
  m = block_max(m, red_a);
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // (x - m) first: folding m into an FMA (x*log2e - m*log2e) cancels
      // catastrophically when |m| is large.
      const float e = valid[k] ? fast_exp2((x[k * 8 + j] - m) * kLog2e) : 0.0f;
      x[k * 8 + j] = e;
      s += e;
    }
  s = block_sum(s, red_b);
  const float inv = 1.0f / s;
#pragma unroll
  for (int k = 0; k < VPT * 8; ++k) x[k] *= inv;
  store_row<VPT>(out, x, valid);
}

template <int VPT>
__device__ __forceinline__ void load_row_raw(const uint16_t* row, int nvec, uint4 (&raw)[VPT]) {
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * kRowBlock;
    raw[k] = v < nvec ? ld_stream_u4(reinterpret_cast<const uint4*>(row) + v) : make_uint4(0, 0, 0, 0);
  }
}

template <int VPT>
__device__ __forceinline__ void softmax_row_regs(const uint16_t* in, uint16_t* out, int cols,
                                                 float* red_a, float* red_b) {
  uint4 raw[VPT];
  load_row_raw<VPT>(in, cols / 8, raw);
  softmax_row_math<VPT>(raw, cols / 8, out, red_a, red_b);
}

// Rows 2 * blockIdx.x and 2 * blockIdx.x + 1: the second row's loads are
// issued before the first row's reductions, so the CTA keeps a row of
// loads in flight across its barriers.  Same arithmetic and order as
// softmax_row_regs (bit-identical output); at 8192 columns, 4 CTAs per SM,
// 6.23 -> 6.61 TB/s against one row per CTA.
template <int VPT>
__device__ __forceinline__ void softmax_row_pair(const uint16_t* __restrict__ in, uint16_t* __restrict__ out,
                                                 int rows, int cols) {
  __shared__ float red[2][2][kRowWarps];  // per row: a fresh pair, no barrier needed between rows
  const int nvec = cols / 8;
  const int first = 2 * static_cast<int>(blockIdx.x);
  const int end = min(rows, first + 2);
  uint4 cur[VPT], nxt[VPT];
  load_row_raw<VPT>(in + static_cast<size_t>(first) * cols, nvec, cur);
  for (int r = first; r < end; ++r) {
    const int p = r - first;
    if (r + 1 < end) load_row_raw<VPT>(in + static_cast<size_t>(r + 1) * cols, nvec, nxt);
    softmax_row_math<VPT>(cur, nvec, out + static_cast<size_t>(r) * cols, red[p][0], red[p][1]);
#pragma unroll
    for (int k = 0; k < VPT; ++k) cur[k] = nxt[k];
  }
}

// RMSNorm over the rows blockIdx.x, blockIdx.x + gridDim.x, ...: the weight
// slice and the current row stay packed (bf16 pairs) in registers, and the
// next row's loads are issued before the current row's reduction, so a CTA
// keeps a row of loads in flight across its barrier.
template <int VPT>
__device__ __forceinline__ void rmsnorm_rows_packed(const uint16_t* __restrict__ in,
                                                    const uint16_t* __restrict__ weight,
                                                    uint16_t* __restrict__ out, int rows, int cols, float eps) {
  __shared__ float red[2][kRowWarps];
  const int nvec = cols / 8;
  uint4 w[VPT], cur[VPT], nxt[VPT];
  load_row_raw<VPT>(weight, nvec, w);
  int r = blockIdx.x;
  if (r < rows) load_row_raw<VPT>(in + static_cast<size_t>(r) * cols, nvec, cur);
  int parity = 0;
  for (; r < rows; r += gridDim.x) {
    const int next = r + gridDim.x;
    if (next < rows) load_row_raw<VPT>(in + static_cast<size_t>(next) * cols, nvec, nxt);
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const uint32_t q[4] = {cur[k].x, cur[k].y, cur[k].z, cur[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf16_lo(q[j]), b = bf16_hi(q[j]);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
    }
    ss = block_sum(ss, red[parity]);
    parity ^= 1;
    const float rs = rsqrtf(ss / static_cast<float>(cols) + eps);
    uint4* o = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * cols);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = threadIdx.x + k * kRowBlock;
      if (v < nvec) {
        const uint32_t q[4] = {cur[k].x, cur[k].y, cur[k].z, cur[k].w};
        const uint32_t ww[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
        uint32_t y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          y[j] = pack_bf16x2_rn((bf16_lo(q[j]) * rs) * bf16_lo(ww[j]), (bf16_hi(q[j]) * rs) * bf16_hi(ww[j]));
        st_stream_u4(o + v, make_uint4(y[0], y[1], y[2], y[3]));
      }
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) cur[k] = nxt[k];
  }
}

// RMSNorm with TMA row staging: every CTA keeps kStages whole rows in
// flight in shared memory (one 1-D bulk copy per row, completion on an
// mbarrier), reads the current row from shared memory, and writes the
// output straight to global memory.  The copy for the CTA's row j + kStages
// is issued as soon as row j's stage is free, independent of the threads'
// progress through the reduction.  Same arithmetic and summation order as
// rmsnorm_rows_packed, so the outputs are bit-identical.
template <int VPT, int kStages>
__device__ __forceinline__ void rmsnorm_rows_staged(const uint16_t* __restrict__ in,
                                                    const uint16_t* __restrict__ weight,
                                                    uint16_t* __restrict__ out, int rows, int cols, float eps) {
  constexpr int kStageBytes = kRowBlock * 8 * VPT * 2;
  __shared__ __align__(128) unsigned char stage[kStages][kStageBytes];
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ float red[kRowWarps];
  const int nvec = cols / 8;
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 2u;
  const int count = rows > static_cast<int>(blockIdx.x)
                        ? (rows - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                        : 0;
  auto row_ptr = [&](int j) {
    return in + (static_cast<size_t>(blockIdx.x) + static_cast<size_t>(j) * gridDim.x) * cols;
  };
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int j = 0; j < kStages && j < count; ++j) {
      mbar_expect_tx(&full[j], row_bytes);
      bulk_copy_g2s(stage[j], row_ptr(j), row_bytes, &full[j]);
    }
  }
  uint4 w[VPT];
  load_row_raw<VPT>(weight, nvec, w);
  for (int j = 0; j < count; ++j) {
    const int s = j % kStages;
    const bool ready = mbar_wait_bounded(&full[s], static_cast<uint32_t>(j / kStages) & 1u);
    if (__syncthreads_or(!ready)) {
      // A row never arrived: count it, wait (bounded) for this CTA's copies
      // still in flight so none lands after the CTA is gone, and leave.
      if (threadIdx.x == 0) {
        atomicAdd(&f4s_wait_timeouts, 1u);
        for (int p = j; p < count && p < j + kStages; ++p)
          mbar_wait_bounded(&full[p % kStages], static_cast<uint32_t>(p / kStages) & 1u);
      }
      return;
    }
    const uint4* row = reinterpret_cast<const uint4*>(stage[s]);
    uint4 cur[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = threadIdx.x + k * kRowBlock;
      cur[k] = v < nvec ? row[v] : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const uint32_t q[4] = {cur[k].x, cur[k].y, cur[k].z, cur[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf16_lo(q[i]), b = bf16_hi(q[i]);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
    }
    ss = block_sum(ss, red);
    const float rs = rsqrtf(ss / static_cast<float>(cols) + eps);
    uint4* o = reinterpret_cast<uint4*>(out + (static_cast<size_t>(blockIdx.x) + static_cast<size_t>(j) * gridDim.x) * cols);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = threadIdx.x + k * kRowBlock;
      if (v < nvec) {
        const uint32_t q[4] = {cur[k].x, cur[k].y, cur[k].z, cur[k].w};
        const uint32_t ww[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
        uint32_t y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          y[i] = pack_bf16x2_rn((bf16_lo(q[i]) * rs) * bf16_lo(ww[i]), (bf16_hi(q[i]) * rs) * bf16_hi(ww[i]));
        st_stream_u4(o + v, make_uint4(y[0], y[1], y[2], y[3]));
      }
    }
    __syncthreads();  // stage s and red are free again
    if (threadIdx.x == 0 && j + kStages < count) {
      fence_proxy_async_smem();
      mbar_expect_tx(&full[s], row_bytes);
      bulk_copy_g2s(stage[s], row_ptr(j + kStages), row_bytes, &full[s]);
    }
  }
}

}  // namespace f4s

// (in, weight, out, rows, cols, eps) with 2048 < cols <= 8192, cols % 8 == 0,
// in / weight 16-byte aligned: TMA-staged rows, 2 stages of 16 KiB per CTA.
// Measured fastest at exactly 2 CTAs per SM (persistent).
extern "C" __global__ void __launch_bounds__(f4s::kRowBlock)
f4s_rmsnorm_rows_bf16_tma(const uint16_t* __restrict__ in, const uint16_t* __restrict__ weight,
                          uint16_t* __restrict__ out, int rows, int cols, float eps) {
  f4s::rmsnorm_rows_staged<4, 2>(in, weight, out, rows, cols, eps);
}

// (in, out, rows, cols); cols % 8 == 0 and cols <= 2048 * VPT.  VPT 1, 2, 4:
// two rows per CTA, grid = ceil(rows / 2), at least 4 CTAs per SM; VPT 8:
// one row per CTA, grid = rows.
#define F4S_SOFTMAX_PAIR(VPT)                                                               \
  extern "C" __global__ void __launch_bounds__(f4s::kRowBlock, 4)                            \
      f4s_softmax_rows_bf16_v##VPT(const uint16_t* __restrict__ in,                          \
                                   uint16_t* __restrict__ out, int rows, int cols) {         \
    f4s::softmax_row_pair<VPT>(in, out, rows, cols);                                         \
  }
F4S_SOFTMAX_PAIR(1)
F4S_SOFTMAX_PAIR(2)
F4S_SOFTMAX_PAIR(4)
#undef F4S_SOFTMAX_PAIR
extern "C" __global__ void __launch_bounds__(f4s::kRowBlock)
f4s_softmax_rows_bf16_v8(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, int rows, int cols) {
  __shared__ float red_a[f4s::kRowWarps];
  __shared__ float red_b[f4s::kRowWarps];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    f4s::softmax_row_regs<8>(in + static_cast<size_t>(r) * cols, out + static_cast<size_t>(r) * cols, cols,
                             red_a, red_b);
    __syncthreads();
  }
}

// (in, weight, out, rows, cols, eps); cols % 8 == 0 and cols <= 2048 * VPT.
#define F4S_RMSNORM_REGS(VPT)                                                                 \
  extern "C" __global__ void __launch_bounds__(f4s::kRowBlock)                                 \
      f4s_rmsnorm_rows_bf16_v##VPT(const uint16_t* __restrict__ in,                             \
                                   const uint16_t* __restrict__ weight,                         \
                                   uint16_t* __restrict__ out, int rows, int cols, float eps) {  \
    f4s::rmsnorm_rows_packed<VPT>(in, weight, out, rows, cols, eps);                            \
  }
F4S_RMSNORM_REGS(1)
F4S_RMSNORM_REGS(2)
F4S_RMSNORM_REGS(4)
F4S_RMSNORM_REGS(8)
#undef F4S_RMSNORM_REGS

// Looped fallbacks for any width: (in, out, rows, cols) and
// (in, weight, out, rows, cols, eps).  Same arithmetic as above.
extern "C" __global__ void __launch_bounds__(f4s::kRowBlock)
f4s_softmax_rows_bf16_any(const uint16_t* __restrict__ in, uint16_t* __restrict__ out,
                          int rows, int cols) {
  using namespace f4s;
  __shared__ float red_a[kRowWarps];
  __shared__ float red_b[kRowWarps];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t* x = in + static_cast<size_t>(r) * cols;
    uint16_t* y = out + static_cast<size_t>(r) * cols;
    float m = -INFINITY;
    for (int c = threadIdx.x; c < cols; c += kRowBlock)
      m = fmaxf(m, __uint_as_float(static_cast<uint32_t>(x[c]) << 16));
    m = block_max(m, red_a);
    float s = 0.0f;
    for (int c = threadIdx.x; c < cols; c += kRowBlock)
      s += fast_exp2((__uint_as_float(static_cast<uint32_t>(x[c]) << 16) - m) * kLog2e);
    s = block_sum(s, red_b);
    const float inv = 1.0f / s;
    for (int c = threadIdx.x; c < cols; c += kRowBlock) {
      const float e = fast_exp2((__uint_as_float(static_cast<uint32_t>(x[c]) << 16) - m) * kLog2e);
      y[c] = static_cast<uint16_t>(pack_bf16x2_rn(e * inv, 0.0f) & 0xFFFFu);
    }
    __syncthreads();
  }
}

extern "C" __global__ void __launch_bounds__(f4s::kRowBlock)
f4s_rmsnorm_rows_bf16_any(const uint16_t* __restrict__ in, const uint16_t* __restrict__ weight,
                          uint16_t* __restrict__ out, int rows, int cols, float eps) {
  using namespace f4s;
  __shared__ float red[2][kRowWarps];
  int parity = 0;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const uint16_t* x = in + static_cast<size_t>(r) * cols;
    uint16_t* y = out + static_cast<size_t>(r) * cols;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < cols; c += kRowBlock) {
      const float v = __uint_as_float(static_cast<uint32_t>(x[c]) << 16);
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red[parity]);
    parity ^= 1;
    const float rs = rsqrtf(ss / static_cast<float>(cols) + eps);
    for (int c = threadIdx.x; c < cols; c += kRowBlock) {
      const float v = __uint_as_float(static_cast<uint32_t>(x[c]) << 16);
      const float wv = __uint_as_float(static_cast<uint32_t>(weight[c]) << 16);
      y[c] = static_cast<uint16_t>(pack_bf16x2_rn((v * rs) * wv, 0.0f) & 0xFFFFu);
    }
  }
}
