// Test kernels for include/flight4s_b200_device.cuh, compiled by NVRTC the
// way a generated kernel is (no other includes).  Every thread writes what
// it received, so the tests check that all lanes / threads / CTAs agree.
#include "flight4s_b200_device.cuh"

// one warp per 32 inputs: out[i] = warp sum seen by thread i
extern "C" __global__ void warp_sum_f32(const float* x, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out[i] = f4s_warp_sum_f32(x[i]);
}

extern "C" __global__ void warp_sum_f64(const double* x, double* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out[i] = f4s_warp_sum_f64(x[i]);
}

extern "C" __global__ void warp_sum_i32(const int* x, int* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out[i] = f4s_warp_sum_i32(x[i]);
}

extern "C" __global__ void warp_max_f32(const float* x, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out[i] = f4s_warp_max_f32(x[i]);
}

// lanes with index[i] < 0 hold no element
extern "C" __global__ void warp_argmax_f32(const float* x, const long long* index, float* out_v,
                                           long long* out_i) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  f4s_warp_argmax_f32(x[i], index[i], &out_v[i], &out_i[i]);
}

extern "C" __global__ void block_sum_f32(const float* x, float* out) {
  __shared__ float scratch[32];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const float first = f4s_block_sum_f32(x[i], scratch);
  const float second = f4s_block_sum_f32(-x[i], scratch);  // reusing the scratch: exact negation
  out[i] = first == -second ? first : __int_as_float(0x7fc00001);
}

extern "C" __global__ void block_argmax_f32(const float* x, float* out_v, long long* out_i) {
  __shared__ float sv[32];
  __shared__ long long si[32];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  f4s_block_argmax_f32(x[i], i, sv, si, &out_v[i], &out_i[i]);
}

// launch with a cluster dimension (x): every thread of every CTA of a
// cluster writes the cluster's sum
extern "C" __global__ void cluster_sum_f32(const float* x, float* out) {
  __shared__ float scratch[32];
  __shared__ float slots[16];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out[i] = f4s_cluster_sum_f32(x[i], scratch, slots);
}

extern "C" __global__ void math_f32(const float* x, float* out_exp, float* out_rsqrt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out_exp[i] = f4s_exp_f32(x[i]);
  out_rsqrt[i] = f4s_rsqrt_f32(x[i]);
}

// the same math through CUDA's own functions, for comparison
extern "C" __global__ void math_f32_cuda(const float* x, float* out_exp, float* out_rsqrt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  out_exp[i] = expf(x[i]);
  out_rsqrt[i] = rsqrtf(x[i]);
}
