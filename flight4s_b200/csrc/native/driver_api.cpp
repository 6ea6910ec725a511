#include "driver_api.hpp"

#include <dlfcn.h>

#include <cstdlib>
#include <mutex>

namespace flight4s::cuda {
namespace {

using GetProcAddress = CUresult (*)(const char*, void**, int, cuuint64_t,
                                    CUdriverProcAddressQueryResult*);

struct Loaded {
  DriverApi api;
  bool ok = false;
  std::string why;
};

Loaded load() {
  Loaded l;
  // FLIGHT4S_CUDA_DRIVER names another driver library (the tests point it
  // at a fake that records launches and injects errors).
  const char* override_path = std::getenv("FLIGHT4S_CUDA_DRIVER");
  const std::string name = (override_path && *override_path) ? override_path : "libcuda.so.1";
  void* lib = dlopen(name.c_str(), RTLD_NOW | RTLD_GLOBAL);
  if (lib == nullptr) {
    const char* err = dlerror();
    l.why = "cannot load " + name + ": " + (err ? err : "unknown dlopen error");
    return l;
  }
  auto get = reinterpret_cast<GetProcAddress>(dlsym(lib, "cuGetProcAddress_v2"));
  if (get == nullptr) {
    l.why = name + " does not export cuGetProcAddress_v2 (driver older than CUDA 12)";
    return l;
  }
#define F4S_DRIVER_FN(name)                                                                \
  {                                                                                        \
    void* fn = nullptr;                                                                    \
    CUdriverProcAddressQueryResult found{};                                                \
    if (get(#name, &fn, CUDA_VERSION, CU_GET_PROC_ADDRESS_DEFAULT, &found) != CUDA_SUCCESS || \
        fn == nullptr) {                                                                   \
      l.why = std::string("CUDA driver lacks ") + #name;                                   \
      return l;                                                                            \
    }                                                                                      \
    l.api.name = reinterpret_cast<decltype(l.api.name)>(fn);                               \
  }
#include "driver_functions.inc"
#undef F4S_DRIVER_FN
  l.ok = true;
  return l;
}

}  // namespace

const DriverApi* driver_api(std::string* why) {
  static const Loaded loaded = load();
  if (!loaded.ok) {
    if (why) *why = loaded.why;
    return nullptr;
  }
  return &loaded.api;
}

}  // namespace flight4s::cuda
