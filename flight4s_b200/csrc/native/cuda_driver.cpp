#include "cuda_driver.hpp"

#include <algorithm>
#include <array>
#include <limits>

namespace flight4s::cuda {

const DriverApi& require_driver() {
  std::string why;
  const DriverApi* api = driver_api(&why);
  if (api == nullptr) throw DriverUnavailable(why);
  return *api;
}

CudaDriverStatus make_driver_status(CUresult result, std::string info_log, std::string error_log) {
  const char* name = nullptr;
  const char* description = nullptr;
  if (const DriverApi* api = driver_api()) {
    api->cuGetErrorName(result, &name);
    api->cuGetErrorString(result, &description);
  }
  return {result, name ? name : "CUDA_ERROR_UNKNOWN",
          description ? description : "no CUDA error description", std::move(info_log),
          std::move(error_log)};
}

CurrentContextScope::CurrentContextScope(CUcontext context)
    : api_(require_driver()),
      context_(context),
      push_result_(api_.cuCtxPushCurrent(context)),
      active_(push_result_ == CUDA_SUCCESS) {}

CurrentContextScope::~CurrentContextScope() {
  if (active_) {
    CUcontext popped = nullptr;
    api_.cuCtxPopCurrent(&popped);
  }
}

CUresult CurrentContextScope::close() noexcept {
  if (!active_) return push_result_;
  CUcontext popped = nullptr;
  const CUresult r = api_.cuCtxPopCurrent(&popped);
  active_ = false;
  if (r != CUDA_SUCCESS) return r;
  return popped == context_ ? CUDA_SUCCESS : CUDA_ERROR_INVALID_CONTEXT;
}

namespace {

constexpr std::size_t kJitLogBytes = 64 * 1024;

void require(const void* handle, const char* what) {
  if (handle == nullptr) throw std::invalid_argument(std::string(what) + " must not be null");
}

void require_address(CUdeviceptr address, const char* what) {
  if (address == 0) throw std::invalid_argument(std::string(what) + " must not be null");
}

std::size_t checked_size(std::uint64_t size_bytes, const char* what) {
  if (size_bytes == 0) throw std::invalid_argument(std::string(what) + " must be positive");
  if (size_bytes > std::numeric_limits<std::size_t>::max())
    throw std::overflow_error(std::string(what) + " exceeds the native size limit");
  return static_cast<std::size_t>(size_bytes);
}

CUdeviceptr checked_range(CUdeviceptr address, std::uint64_t offset, std::uint64_t size,
                          const char* what) {
  const auto top = std::numeric_limits<CUdeviceptr>::max();
  if (offset > top - address)
    throw std::overflow_error(std::string(what) + " exceeds the device address range");
  const CUdeviceptr start = address + offset;
  if (size - 1 > top - start)
    throw std::overflow_error(std::string(what) + " extent exceeds the device address range");
  return start;
}

std::string log_text(const std::vector<char>& buffer) {
  return std::string(buffer.begin(), std::find(buffer.begin(), buffer.end(), '\0'));
}

// Push `context`, run `op` (which returns a CUresult), pop, and fold the
// pop outcome into the status the way the reference does: the operation's
// error wins, otherwise a failed/mismatched pop is reported.
template <class Op>
CudaDriverStatus in_context(CUcontext context, Op&& op, std::string* info = nullptr,
                            std::string* error = nullptr) {
  CurrentContextScope scope(context);
  if (scope.push_result() != CUDA_SUCCESS) return make_driver_status(scope.push_result());
  const CUresult r = op();
  const CUresult pop = scope.close();
  return make_driver_status(r == CUDA_SUCCESS ? pop : r, info ? std::move(*info) : std::string(),
                            error ? std::move(*error) : std::string());
}

CudaModuleResult load_with_logs(CUcontext context, const void* image) {
  const DriverApi& api = require_driver();
  std::vector<char> info(kJitLogBytes, '\0');
  std::vector<char> error(kJitLogBytes, '\0');
  std::array<CUjit_option, 4> options{CU_JIT_INFO_LOG_BUFFER, CU_JIT_INFO_LOG_BUFFER_SIZE_BYTES,
                                      CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
  std::array<void*, 4> values{info.data(), reinterpret_cast<void*>(static_cast<std::uintptr_t>(info.size())),
                              error.data(), reinterpret_cast<void*>(static_cast<std::uintptr_t>(error.size()))};
  CUmodule module = nullptr;
  CurrentContextScope scope(context);
  if (scope.push_result() != CUDA_SUCCESS) return {make_driver_status(scope.push_result()), nullptr};
  const CUresult r = api.cuModuleLoadDataEx(&module, image, static_cast<unsigned>(options.size()),
                                            options.data(), values.data());
  const CUresult pop = scope.close();
  auto status = make_driver_status(r == CUDA_SUCCESS ? pop : r, log_text(info), log_text(error));
  const bool ok = status.succeeded();
  return {std::move(status), ok ? module : nullptr};
}

}  // namespace

CudaContextResult CudaDriver::retain_primary_context(std::int32_t ordinal) const {
  if (ordinal < 0) throw std::invalid_argument("CUDA device ordinal must not be negative");
  const DriverApi& api = require_driver();
  CUresult r = api.cuInit(0);
  if (r != CUDA_SUCCESS) return {make_driver_status(r), nullptr, ordinal, 0, 0};
  CUdevice device = 0;
  if ((r = api.cuDeviceGet(&device, ordinal)) != CUDA_SUCCESS)
    return {make_driver_status(r), nullptr, ordinal, 0, 0};
  int major = 0, minor = 0;
  if ((r = api.cuDeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, device)) !=
      CUDA_SUCCESS)
    return {make_driver_status(r), nullptr, ordinal, 0, 0};
  if ((r = api.cuDeviceGetAttribute(&minor, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, device)) !=
      CUDA_SUCCESS)
    return {make_driver_status(r), nullptr, ordinal, major, 0};
  CUcontext context = nullptr;
  r = api.cuDevicePrimaryCtxRetain(&context, device);
  return {make_driver_status(r), r == CUDA_SUCCESS ? context : nullptr, ordinal, major, minor};
}

CudaDriverStatus CudaDriver::release_primary_context(std::int32_t ordinal) const {
  if (ordinal < 0) throw std::invalid_argument("CUDA device ordinal must not be negative");
  const DriverApi& api = require_driver();
  CUdevice device = 0;
  const CUresult r = api.cuDeviceGet(&device, ordinal);
  if (r != CUDA_SUCCESS) return make_driver_status(r);
  return make_driver_status(api.cuDevicePrimaryCtxRelease(device));
}

CudaDriverStatus CudaDriver::synchronize_context(CUcontext context) const {
  require(context, "CUDA context");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuCtxSynchronize(); });
}

CudaAttributeResult CudaDriver::device_attribute(CUcontext context, CUdevice_attribute attribute) const {
  require(context, "CUDA context handle");
  const DriverApi& api = require_driver();
  int value = 0;
  auto status = in_context(context, [&] {
    CUdevice device = 0;
    CUresult r = api.cuCtxGetDevice(&device);
    if (r == CUDA_SUCCESS) r = api.cuDeviceGetAttribute(&value, attribute, device);
    return r;
  });
  return {std::move(status), value};
}

CudaModuleResult CudaDriver::load_ptx(CUcontext context, const std::vector<std::uint8_t>& ptx) const {
  require(context, "CUDA context handle");
  if (ptx.empty()) throw std::invalid_argument("PTX must not be empty");
  if (std::find(ptx.begin(), ptx.end(), std::uint8_t{0}) != ptx.end())
    throw std::invalid_argument("PTX must not contain a null byte");
  std::vector<char> text(ptx.begin(), ptx.end());
  text.push_back('\0');
  return load_with_logs(context, text.data());
}

CudaModuleResult CudaDriver::load_module_image(CUcontext context, const void* image,
                                               std::size_t size_bytes) const {
  require(context, "CUDA context handle");
  require(image, "module image");
  if (size_bytes == 0) throw std::invalid_argument("module image must not be empty");
  return load_with_logs(context, image);
}

CudaDriverStatus CudaDriver::unload_module(CUcontext context, CUmodule module) const {
  require(context, "CUDA context handle");
  require(module, "CUDA module handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuModuleUnload(module); });
}

CudaFunctionResult CudaDriver::resolve_function(CUcontext context, CUmodule module,
                                                const std::string& name) const {
  require(context, "CUDA context handle");
  require(module, "CUDA module handle");
  if (name.empty()) throw std::invalid_argument("CUDA function name must not be empty");
  if (name.find('\0') != std::string::npos)
    throw std::invalid_argument("CUDA function name must not contain a null byte");
  const DriverApi& api = require_driver();
  CUfunction function = nullptr;
  auto status = in_context(context, [&] { return api.cuModuleGetFunction(&function, module, name.c_str()); });
  const bool ok = status.succeeded();
  return {std::move(status), ok ? function : nullptr};
}

CudaFunctionAttributesResult CudaDriver::function_attributes(CUcontext context, CUfunction function) const {
  require(context, "CUDA context handle");
  require(function, "CUDA function handle");
  const DriverApi& api = require_driver();
  CudaFunctionAttributes a{};
  auto status = in_context(context, [&] {
    const std::pair<CUfunction_attribute, std::int32_t*> queries[] = {
        {CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, &a.max_threads_per_block},
        {CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, &a.static_shared_memory_bytes},
        {CU_FUNC_ATTRIBUTE_CONST_SIZE_BYTES, &a.constant_memory_bytes},
        {CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, &a.local_memory_bytes},
        {CU_FUNC_ATTRIBUTE_NUM_REGS, &a.registers_per_thread},
    };
    for (const auto& [attribute, slot] : queries) {
      const CUresult r = api.cuFuncGetAttribute(slot, attribute, function);
      if (r != CUDA_SUCCESS) return r;
    }
    return CUDA_SUCCESS;
  });
  const bool ok = status.succeeded();
  return {std::move(status), ok ? a : CudaFunctionAttributes{}};
}

CudaStreamResult CudaDriver::create_stream(CUcontext context, std::uint32_t flags) const {
  require(context, "CUDA context handle");
  if (flags != CU_STREAM_DEFAULT && flags != CU_STREAM_NON_BLOCKING)
    throw std::invalid_argument("unsupported CUDA stream flags");
  const DriverApi& api = require_driver();
  CUstream stream = nullptr;
  auto status = in_context(context, [&] { return api.cuStreamCreate(&stream, flags); });
  const bool ok = status.succeeded();
  return {std::move(status), ok ? stream : nullptr};
}

CudaDriverStatus CudaDriver::destroy_stream(CUcontext context, CUstream stream) const {
  require(context, "CUDA context handle");
  require(stream, "CUDA stream handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuStreamDestroy(stream); });
}

CudaDriverStatus CudaDriver::synchronize_stream(CUcontext context, CUstream stream) const {
  require(context, "CUDA context handle");
  require(stream, "CUDA stream handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuStreamSynchronize(stream); });
}

CudaEventResult CudaDriver::create_event(CUcontext context, std::uint32_t flags) const {
  require(context, "CUDA context handle");
  if ((flags & ~static_cast<std::uint32_t>(CU_EVENT_BLOCKING_SYNC | CU_EVENT_DISABLE_TIMING)) != 0)
    throw std::invalid_argument("unsupported CUDA event flags");
  const DriverApi& api = require_driver();
  CUevent event = nullptr;
  auto status = in_context(context, [&] { return api.cuEventCreate(&event, flags); });
  const bool ok = status.succeeded();
  return {std::move(status), ok ? event : nullptr};
}

CudaDriverStatus CudaDriver::destroy_event(CUcontext context, CUevent event) const {
  require(context, "CUDA context handle");
  require(event, "CUDA event handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuEventDestroy(event); });
}

CudaDriverStatus CudaDriver::record_event(CUcontext context, CUevent event, CUstream stream) const {
  require(context, "CUDA context handle");
  require(event, "CUDA event handle");
  require(stream, "CUDA stream handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuEventRecord(event, stream); });
}

CudaEventQueryResult CudaDriver::query_event(CUcontext context, CUevent event) const {
  require(context, "CUDA context handle");
  require(event, "CUDA event handle");
  const DriverApi& api = require_driver();
  bool complete = false;
  auto status = in_context(context, [&] {
    const CUresult r = api.cuEventQuery(event);
    if (r == CUDA_ERROR_NOT_READY) return CUDA_SUCCESS;
    if (r == CUDA_SUCCESS) complete = true;
    return r;
  });
  return {std::move(status), complete};
}

CudaDriverStatus CudaDriver::synchronize_event(CUcontext context, CUevent event) const {
  require(context, "CUDA context handle");
  require(event, "CUDA event handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuEventSynchronize(event); });
}

CudaDriverStatus CudaDriver::wait_for_event(CUcontext context, CUstream stream, CUevent event) const {
  require(context, "CUDA context handle");
  require(stream, "CUDA stream handle");
  require(event, "CUDA event handle");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuStreamWaitEvent(stream, event, 0); });
}

CudaElapsedResult CudaDriver::elapsed_time(CUcontext context, CUevent start, CUevent end) const {
  require(context, "CUDA context handle");
  require(start, "CUDA start event handle");
  require(end, "CUDA end event handle");
  const DriverApi& api = require_driver();
  float ms = 0.0f;
  auto status = in_context(context, [&] { return api.cuEventElapsedTime(&ms, start, end); });
  return {std::move(status), ms};
}

CudaPinnedMemoryResult CudaDriver::allocate_pinned_memory(CUcontext context, std::uint64_t size_bytes) const {
  require(context, "CUDA context handle");
  const std::size_t size = checked_size(size_bytes, "CUDA pinned allocation size");
  const DriverApi& api = require_driver();
  void* address = nullptr;
  auto status = in_context(context, [&] { return api.cuMemHostAlloc(&address, size, 0); });
  const bool ok = status.succeeded();
  return {std::move(status), ok ? address : nullptr};
}

CudaDriverStatus CudaDriver::free_pinned_memory(CUcontext context, void* address) const {
  require(context, "CUDA context handle");
  require(address, "CUDA pinned host address");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuMemFreeHost(address); });
}

CudaDeviceMemoryResult CudaDriver::allocate_device_memory(CUcontext context, std::uint64_t size_bytes) const {
  require(context, "CUDA context handle");
  const std::size_t size = checked_size(size_bytes, "CUDA allocation size");
  const DriverApi& api = require_driver();
  CUdeviceptr address = 0;
  auto status = in_context(context, [&] { return api.cuMemAlloc(&address, size); });
  const bool ok = status.succeeded();
  return {std::move(status), ok ? address : 0};
}

CudaDriverStatus CudaDriver::free_device_memory(CUcontext context, CUdeviceptr address) const {
  require(context, "CUDA context handle");
  require_address(address, "CUDA device address");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuMemFree(address); });
}

CudaDriverStatus CudaDriver::copy_host_to_device(CUcontext context, CUdeviceptr destination,
                                                 std::uint64_t offset, const void* source,
                                                 std::uint64_t size_bytes) const {
  require(context, "CUDA context handle");
  require_address(destination, "CUDA destination address");
  require(source, "host source address");
  const std::size_t size = checked_size(size_bytes, "CUDA copy size");
  const CUdeviceptr dst = checked_range(destination, offset, size_bytes, "CUDA destination offset");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuMemcpyHtoD(dst, source, size); });
}

CudaDriverStatus CudaDriver::copy_host_to_device_async(CUcontext context, CUdeviceptr destination,
                                                       std::uint64_t offset, const void* source,
                                                       std::uint64_t size_bytes, CUstream stream) const {
  require(context, "CUDA context handle");
  require_address(destination, "CUDA destination address");
  require(source, "host source address");
  require(stream, "CUDA stream handle");
  const std::size_t size = checked_size(size_bytes, "CUDA copy size");
  const CUdeviceptr dst = checked_range(destination, offset, size_bytes, "CUDA destination offset");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuMemcpyHtoDAsync(dst, source, size, stream); });
}

CudaDriverStatus CudaDriver::copy_device_to_host(CUcontext context, void* destination, CUdeviceptr source,
                                                 std::uint64_t offset, std::uint64_t size_bytes) const {
  require(context, "CUDA context handle");
  require(destination, "host destination address");
  require_address(source, "CUDA source address");
  const std::size_t size = checked_size(size_bytes, "CUDA copy size");
  const CUdeviceptr src = checked_range(source, offset, size_bytes, "CUDA source offset");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuMemcpyDtoH(destination, src, size); });
}

CudaDriverStatus CudaDriver::copy_device_to_host_async(CUcontext context, void* destination,
                                                       CUdeviceptr source, std::uint64_t offset,
                                                       std::uint64_t size_bytes, CUstream stream) const {
  require(context, "CUDA context handle");
  require(destination, "host destination address");
  require_address(source, "CUDA source address");
  require(stream, "CUDA stream handle");
  const std::size_t size = checked_size(size_bytes, "CUDA copy size");
  const CUdeviceptr src = checked_range(source, offset, size_bytes, "CUDA source offset");
  const DriverApi& api = require_driver();
  return in_context(context, [&] { return api.cuMemcpyDtoHAsync(destination, src, size, stream); });
}

}  // namespace flight4s::cuda
