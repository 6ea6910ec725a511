// Single translation unit for every sm_100a kernel of the hot path.  It is
// compiled to one cubin that the native layer loads with cuModuleLoadData and
// launches through cuLaunchKernelEx, the same route the reference takes for
// its generated kernels (native/src/cuda_driver.cpp:209-261,
// native/src/cuda_launcher.cpp:8-62).
#include "reduce.cuh"
#include "reduce_ordered.cuh"
#include "block_sum.cuh"
#include "elementwise.cuh"
#include "rowwise.cuh"
#include "fp8.cuh"
#include "convert.cuh"
#include "synthetic.cuh"
