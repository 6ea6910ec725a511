// Allocation-free block sum over a per-device static workspace
// (noalloc_scratch.cu).
#pragma once

#include <cuda.h>

#include <cstdint>

#include "hotpath.hpp"

namespace flight4s::cuda {

std::int64_t noalloc_block_sum_max_elements();

CUresult block_sum_f32_noalloc(Hotpath& hp, CUstream stream, CUdeviceptr in, std::int32_t n,
                               CUdeviceptr partials, CUdeviceptr out);

}  // namespace flight4s::cuda
