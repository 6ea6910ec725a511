// Late-bound CUDA Driver API.
//
// The library resolves libcuda at first use (dlopen + cuGetProcAddress)
// instead of linking it, so it loads, and reports a clean error, on hosts
// that have no NVIDIA driver.  FLIGHT4S_CUDA_DRIVER, when set, names the
// driver library to open instead of libcuda.so.1.  Function-pointer types come from <cuda.h>, so
// every entry has the exact versioned prototype the driver hands back.
#pragma once

#include <cuda.h>

#include <string>

namespace flight4s::cuda {

struct DriverApi {
#define F4S_DRIVER_FN(name) decltype(&::name) name = nullptr;
#include "driver_functions.inc"
#undef F4S_DRIVER_FN
};

// nullptr when no usable driver is present; `why` then explains.
const DriverApi* driver_api(std::string* why = nullptr);

// Status code returned by the boundary when libcuda cannot be loaded.
constexpr int kDriverUnavailable = -3;

}  // namespace flight4s::cuda
