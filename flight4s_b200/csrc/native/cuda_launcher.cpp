#include "cuda_launcher.hpp"

#include <stdexcept>

namespace flight4s::cuda {

namespace {

void validate(const CudaLaunchRequest& request) {
  if (request.context == nullptr) throw std::invalid_argument("CUDA context handle must not be null");
  if (request.function == nullptr) throw std::invalid_argument("CUDA function handle must not be null");
  if (auto e = validate_launch_geometry(request.geometry)) throw std::invalid_argument(*e);
  if (auto e = validate_argument_layout(request.arguments)) throw std::invalid_argument(*e);
}

}  // namespace

CUresult launch_in_current_context(const DriverApi& api, const CudaLaunchRequest& request, bool programmatic) {
  validate(request);
  auto pointers = build_argument_pointers(request.arguments);
  const LaunchGeometry& g = request.geometry;
  CUlaunchConfig config{};
  config.gridDimX = static_cast<unsigned>(g.grid_x);
  config.gridDimY = static_cast<unsigned>(g.grid_y);
  config.gridDimZ = static_cast<unsigned>(g.grid_z);
  config.blockDimX = static_cast<unsigned>(g.block_x);
  config.blockDimY = static_cast<unsigned>(g.block_y);
  config.blockDimZ = static_cast<unsigned>(g.block_z);
  config.sharedMemBytes = static_cast<unsigned>(g.dynamic_shared_memory_bytes);
  config.hStream = request.stream;
  CUlaunchAttribute attrs[2]{};
  unsigned count = 0;
  if (g.uses_cluster) {
    attrs[count].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attrs[count].value.clusterDim.x = static_cast<unsigned>(g.cluster_x);
    attrs[count].value.clusterDim.y = static_cast<unsigned>(g.cluster_y);
    attrs[count].value.clusterDim.z = static_cast<unsigned>(g.cluster_z);
    ++count;
  }
  if (programmatic) {
    attrs[count].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attrs[count].value.programmaticStreamSerializationAllowed = 1;
    ++count;
  }
  if (count > 0) {
    config.attrs = attrs;
    config.numAttrs = count;
  }
  return api.cuLaunchKernelEx(&config, request.function, pointers.empty() ? nullptr : pointers.data(),
                              nullptr);
}

CudaDriverStatus CudaLauncher::launch(const CudaLaunchRequest& request) const {
  validate(request);
  const DriverApi& api = require_driver();
  CurrentContextScope scope(request.context);
  if (scope.push_result() != CUDA_SUCCESS) return make_driver_status(scope.push_result());
  const CUresult r = launch_in_current_context(api, request);
  const CUresult pop = scope.close();
  return make_driver_status(r == CUDA_SUCCESS ? pop : r);
}

}  // namespace flight4s::cuda
