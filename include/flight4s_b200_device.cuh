/* Device-side reduction and math intrinsics for generated kernels.
 *
 * The reference's code generator emits CUDA C++ text and compiles it with
 * NVRTC (core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala,
 * native/src/nvrtc_compiler.cpp).  Its IR has no warp, block or cluster
 * reduction and no exp / rsqrt (core/src/main/scala/flight4s/core/ir/Validation.scala:96-106
 * lists the intrinsics it accepts); a kernel that needs them can include
 * this header (NVRTC option -I<this directory>) and call:
 *
 *   f4s_warp_sum_{f32,f64,i32}   every lane of a full warp gets the sum
 *   f4s_warp_max_f32             every lane gets the max (NaN ignored)
 *   f4s_warp_argmax_f32          (max value, lowest index) by IEEE totalOrder
 *   f4s_block_sum_f32            every thread of the CTA gets the CTA's sum
 *   f4s_block_argmax_f32         every thread gets the CTA's (value, index)
 *   f4s_cluster_sum_f32          every thread of every CTA of the thread-block
 *                                cluster gets the cluster's sum (DSMEM)
 *   f4s_exp_f32, f4s_rsqrt_f32   CUDA's expf / rsqrtf
 *
 * Every combine has a fixed order that depends only on lane, warp and
 * cluster rank, so a result is reproducible for a given launch shape:
 *   warp    xor butterfly over offsets 16, 8, 4, 2, 1 (v += shfl_xor(v, o));
 *           IEEE addition is commutative, so all 32 lanes hold the same bits;
 *   block   each warp's butterfly sum into slot[warp], then warp 0 runs the
 *           butterfly over slot[0..31] (missing warps contribute +0);
 *   cluster each CTA's block sum into the leader CTA's slot[rank] through
 *           distributed shared memory, then every CTA adds slot[0..n-1] in
 *           rank order, left to right.
 * i32 sums wrap (two's complement), like the reference's I32 accumulator
 * (core/src/main/scala/flight4s/core/types/CudaType.scala:204-206).
 *
 * Requirements: whole warps (all 32 lanes active at the call); block
 * functions called by every thread of the CTA with blockDim.x a multiple of
 * 32, no more than 1024; the cluster function called by every thread of
 * every CTA of the cluster (at most 16 CTAs).  Self-contained: no includes,
 * so NVRTC needs no extra header path.  sm_90 or later (redux.sync, DSMEM);
 * built and tested here for sm_100a.
 */
#ifndef FLIGHT4S_B200_DEVICE_CUH
#define FLIGHT4S_B200_DEVICE_CUH

#define F4S_DEVICE static __device__ __forceinline__

/* ------------------------------------------------------------------ warp */

F4S_DEVICE float f4s_warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

F4S_DEVICE double f4s_warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

/* 32-bit wrapping sum in one redux.sync. */
F4S_DEVICE int f4s_warp_sum_i32(int v) {
  return static_cast<int>(__reduce_add_sync(0xffffffffu, static_cast<unsigned>(v)));
}

/* fmaxf semantics: a NaN operand is ignored unless both are NaN. */
F4S_DEVICE float f4s_warp_max_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

/* IEEE totalOrder as a signed integer: -NaN < -inf < ... < -0 < +0 < ...
 * < +inf < +NaN. */
F4S_DEVICE int f4s_total_order_key_f32(float v) {
  const int b = __float_as_int(v);
  return b ^ static_cast<int>(static_cast<unsigned>(b >> 31) >> 1);
}

/* Larger key wins; on equal keys the lower index. */
F4S_DEVICE void f4s_argmax_merge(int& key, long long& index, int other_key, long long other_index) {
  if (other_key > key || (other_key == key && other_index < index)) {
    key = other_key;
    index = other_index;
  }
}

/* (max value, lowest index) over the warp's 32 (value, index) pairs by
 * totalOrder; every lane receives the result.  Pass index -1 for a lane
 * with no element: such lanes never win unless all are empty, and then the
 * result index is -1. */
F4S_DEVICE void f4s_warp_argmax_f32(float v, long long index, float* out_value, long long* out_index) {
  int key = index < 0 ? static_cast<int>(0x80000000u) : f4s_total_order_key_f32(v);
  long long idx = index < 0 ? 0x7fffffffffffffffll : index;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int k2 = __shfl_xor_sync(0xffffffffu, key, o);
    const long long i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    f4s_argmax_merge(key, idx, k2, i2);
  }
  *out_value = __int_as_float(key ^ static_cast<int>(static_cast<unsigned>(key >> 31) >> 1));
  *out_index = idx == 0x7fffffffffffffffll ? -1 : idx;
}

/* ----------------------------------------------------------------- block */

/* `scratch`: 32 floats of shared memory, free on entry, reused on return. */
F4S_DEVICE float f4s_block_sum_f32(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
  v = f4s_warp_sum_f32(v);
  __syncthreads();  /* scratch may still be read by an earlier call */
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < warps ? scratch[lane] : 0.0f;
    s = f4s_warp_sum_f32(s);
    if (lane == 0) scratch[0] = s;
  }
  __syncthreads();
  return scratch[0];
}

/* `scratch_v`: 32 floats, `scratch_i`: 32 long longs of shared memory. */
F4S_DEVICE void f4s_block_argmax_f32(float v, long long index, float* scratch_v, long long* scratch_i,
                                     float* out_value, long long* out_index) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
  float wv;
  long long wi;
  f4s_warp_argmax_f32(v, index, &wv, &wi);
  __syncthreads();
  if (lane == 0) {
    scratch_v[warp] = wv;
    scratch_i[warp] = wi;
  }
  __syncthreads();
  if (warp == 0) {
    float bv;
    long long bi;
    f4s_warp_argmax_f32(lane < warps ? scratch_v[lane] : 0.0f, lane < warps ? scratch_i[lane] : -1, &bv, &bi);
    if (lane == 0) {
      scratch_v[0] = bv;
      scratch_i[0] = bi;
    }
  }
  __syncthreads();
  *out_value = scratch_v[0];
  *out_index = scratch_i[0];
}

/* --------------------------------------------------------------- cluster */

F4S_DEVICE unsigned f4s_cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

F4S_DEVICE unsigned f4s_cluster_size() {
  unsigned n;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
  return n;
}

F4S_DEVICE void f4s_cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

/* Address of `p` (this CTA's shared memory) in CTA `rank` of the cluster. */
F4S_DEVICE unsigned f4s_cluster_map(const void* p, unsigned rank) {
  const unsigned local = static_cast<unsigned>(__cvta_generic_to_shared(p));
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}

/* `scratch`: 32 floats of shared memory (as for f4s_block_sum_f32);
 * `slots`: 16 floats of shared memory at the same offset in every CTA
 * (declare it the same way in each). */
F4S_DEVICE float f4s_cluster_sum_f32(float v, float* scratch, float* slots) {
  const float block = f4s_block_sum_f32(v, scratch);
  const unsigned rank = f4s_cluster_rank(), n = f4s_cluster_size();
  if (threadIdx.x == 0) {
    const unsigned dst = f4s_cluster_map(&slots[rank], 0);
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst), "f"(block) : "memory");
  }
  f4s_cluster_barrier();  /* every partial is in the leader's slots */
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (unsigned r = 0; r < n; ++r) {
      float x;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(f4s_cluster_map(&slots[r], 0)) : "memory");
      total += x;
    }
    scratch[0] = total;
  }
  f4s_cluster_barrier();  /* the leader's slots stay alive until every CTA has read them */
  const float total = scratch[0];
  __syncthreads();
  return total;
}

/* ------------------------------------------------------------------ math */

F4S_DEVICE float f4s_exp_f32(float x) { return expf(x); }
F4S_DEVICE float f4s_rsqrt_f32(float x) { return rsqrtf(x); }

#undef F4S_DEVICE

#endif /* FLIGHT4S_B200_DEVICE_CUH */
