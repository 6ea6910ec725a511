// Kernel launch through cuLaunchKernelEx with an optional thread-block
// cluster attribute.  Same request shape and behaviour as the reference's
// launcher (native/include/flight4s/cuda/cuda_launcher.hpp:10-22,
// native/src/cuda_launcher.cpp:8-62): invalid requests throw
// std::invalid_argument, driver failures are returned, the caller's current
// context is restored, and nothing synchronizes.
#pragma once

#include <cuda.h>

#include "cuda_driver.hpp"
#include "launch_contract.hpp"

namespace flight4s::cuda {

struct CudaLaunchRequest {
  CUcontext context;
  CUfunction function;
  CUstream stream;
  LaunchGeometry geometry;
  ArgumentLayout arguments;
};

class CudaLauncher final {
 public:
  [[nodiscard]] CudaDriverStatus launch(const CudaLaunchRequest& request) const;
};

// The same launch without the context push/pop, for callers that already
// made `request.context` current (the hot-path entry points do, once per
// call).  Returns the raw CUresult.  `programmatic` adds programmatic
// stream serialization (the kernel may start while the previous kernel on
// the stream finishes; it must wait with griddepcontrol.wait before using
// anything that kernel writes).
CUresult launch_in_current_context(const DriverApi& api, const CudaLaunchRequest& request,
                                   bool programmatic = false);

}  // namespace flight4s::cuda
