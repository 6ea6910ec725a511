// extern "C" facade over the native layer (declarations and the reference
// interface each entry replaces: include/flight4s_b200.h).
//
// Error mapping follows the reference's JNI adapters
// (native/src/jni_cuda_launcher.cpp:154-203, native/src/jni_cuda_driver.cpp):
// std::invalid_argument -> F4S_STATUS_INVALID_ARGUMENT (Java
// IllegalArgumentException), std::overflow_error -> F4S_STATUS_OVERFLOW,
// driver failures -> their CUresult with name/description/logs kept for
// f4s_last_status_*().
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../../include/flight4s_b200.h"
#include "cuda_driver.hpp"
#include "cuda_launcher.hpp"
#include "hotpath.hpp"
#include "launch_contract.hpp"
#include "noalloc_scratch.hpp"

using flight4s::cuda::CudaDriver;
using flight4s::cuda::CudaDriverStatus;
using flight4s::cuda::Hotpath;
using flight4s::cuda::ReduceOp;
using flight4s::cuda::kReduceOpCount;
using flight4s::cuda::ReducePolicy;
using flight4s::cuda::sum_op_for_type_code;
using flight4s::cuda::argmax_op_for_type_code;

struct f4s_hotpath {
  Hotpath* impl;
};

namespace {

struct LastStatus {
  int code = 0;
  std::string name = "CUDA_SUCCESS";
  std::string description;
  std::string info_log;
  std::string error_log;
};

thread_local LastStatus last;

int set_status(int code, std::string name, std::string description, std::string info = {},
               std::string error = {}) {
  last.code = code;
  last.name = std::move(name);
  last.description = std::move(description);
  last.info_log = std::move(info);
  last.error_log = std::move(error);
  return code;
}

int from_driver(const CudaDriverStatus& s) {
  return set_status(static_cast<int>(s.result_code), s.result_name, s.result_description, s.info_log,
                    s.error_log);
}

int from_result(CUresult r) { return from_driver(flight4s::cuda::make_driver_status(r)); }

// Runs `body` (returning an int status) and maps exceptions.
template <class Body>
int guarded(Body&& body) {
  try {
    return body();
  } catch (const flight4s::cuda::DriverUnavailable& e) {
    return set_status(F4S_STATUS_DRIVER_UNAVAILABLE, "DRIVER_UNAVAILABLE", e.what());
  } catch (const std::invalid_argument& e) {
    return set_status(F4S_STATUS_INVALID_ARGUMENT, "INVALID_ARGUMENT", e.what());
  } catch (const std::overflow_error& e) {
    return set_status(F4S_STATUS_OVERFLOW, "OVERFLOW", e.what());
  } catch (const std::exception& e) {
    return set_status(F4S_STATUS_INTERNAL, "INTERNAL", e.what());
  } catch (...) {
    return set_status(F4S_STATUS_INTERNAL, "INTERNAL", "unknown native failure");
  }
}

template <class T>
T* as_ptr(std::uint64_t handle) {
  return reinterpret_cast<T*>(static_cast<std::uintptr_t>(handle));
}
CUcontext ctx(std::uint64_t h) { return as_ptr<CUctx_st>(h); }
CUstream stream_of(std::uint64_t h) { return as_ptr<CUstream_st>(h); }
CUevent event_of(std::uint64_t h) { return as_ptr<CUevent_st>(h); }
CUmodule module_of(std::uint64_t h) { return as_ptr<CUmod_st>(h); }
CUfunction function_of(std::uint64_t h) { return as_ptr<CUfunc_st>(h); }
std::uint64_t handle(const void* p) { return static_cast<std::uint64_t>(reinterpret_cast<std::uintptr_t>(p)); }

template <class T>
void require_out(T* p, const char* what) {
  if (p == nullptr) throw std::invalid_argument(std::string(what) + " output pointer must not be null");
}

Hotpath& hot(f4s_hotpath* h) {
  if (h == nullptr || h->impl == nullptr) throw std::invalid_argument("hotpath handle must not be null");
  return *h->impl;
}

int op_status(CUresult r) { return from_result(r); }

const CudaDriver driver;

}  // namespace

extern "C" {

int f4s_abi_version(void) { return 1000; }

int f4s_last_status_code(void) { return last.code; }
const char* f4s_last_status_name(void) { return last.name.c_str(); }
const char* f4s_last_status_description(void) { return last.description.c_str(); }
const char* f4s_last_info_log(void) { return last.info_log.c_str(); }
const char* f4s_last_error_log(void) { return last.error_log.c_str(); }

int f4s_driver_available(void) {
  std::string why;
  if (flight4s::cuda::driver_api(&why) == nullptr) {
    set_status(F4S_STATUS_DRIVER_UNAVAILABLE, "DRIVER_UNAVAILABLE", why);
    return 0;
  }
  set_status(0, "CUDA_SUCCESS", "");
  return 1;
}

int f4s_validate_launch_geometry(int32_t gx, int32_t gy, int32_t gz, int32_t bx, int32_t by, int32_t bz,
                                 int32_t smem, int32_t uses_cluster, int32_t cx, int32_t cy, int32_t cz) {
  const flight4s::cuda::LaunchGeometry g{gx, gy, gz, bx, by, bz, smem, uses_cluster != 0, cx, cy, cz};
  if (auto e = flight4s::cuda::validate_launch_geometry(g))
    return set_status(F4S_STATUS_INVALID_ARGUMENT, "INVALID_ARGUMENT", *e);
  return set_status(0, "SUCCESS", "");
}

int f4s_validate_argument_layout(const void* storage, int64_t size, const int32_t* offsets, size_t offset_count,
                                 const int8_t* codes, size_t code_count) {
  const flight4s::cuda::ArgumentLayout l{const_cast<void*>(storage), size, offsets, offset_count, codes,
                                         code_count};
  if (auto e = flight4s::cuda::validate_argument_layout(l))
    return set_status(F4S_STATUS_INVALID_ARGUMENT, "INVALID_ARGUMENT", *e);
  return set_status(0, "SUCCESS", "");
}

int f4s_launch_kernel(uint64_t context, uint64_t function, uint64_t stream, int32_t gx, int32_t gy, int32_t gz,
                      int32_t bx, int32_t by, int32_t bz, int32_t smem, int32_t uses_cluster, int32_t cx,
                      int32_t cy, int32_t cz, void* storage, int64_t storage_size, const int32_t* offsets,
                      const int8_t* codes, size_t count) {
  return guarded([&] {
    const flight4s::cuda::CudaLaunchRequest request{
        ctx(context), function_of(function), stream_of(stream),
        flight4s::cuda::LaunchGeometry{gx, gy, gz, bx, by, bz, smem, uses_cluster != 0, cx, cy, cz},
        flight4s::cuda::ArgumentLayout{storage, storage_size, offsets, count, codes, count}};
    return from_driver(flight4s::cuda::CudaLauncher{}.launch(request));
  });
}

int f4s_retain_primary_context(int32_t ordinal, uint64_t* context, int32_t* major, int32_t* minor) {
  return guarded([&] {
    require_out(context, "context");
    auto r = driver.retain_primary_context(ordinal);
    *context = handle(r.context);
    if (major) *major = r.compute_capability_major;
    if (minor) *minor = r.compute_capability_minor;
    return from_driver(r.status);
  });
}

int f4s_release_primary_context(int32_t ordinal) {
  return guarded([&] { return from_driver(driver.release_primary_context(ordinal)); });
}

int f4s_synchronize_context(uint64_t context) {
  return guarded([&] { return from_driver(driver.synchronize_context(ctx(context))); });
}

int f4s_device_attribute(uint64_t context, int32_t attribute, int32_t* value) {
  return guarded([&] {
    require_out(value, "attribute value");
    auto r = driver.device_attribute(ctx(context), static_cast<CUdevice_attribute>(attribute));
    *value = r.value;
    return from_driver(r.status);
  });
}

int f4s_load_ptx(uint64_t context, const uint8_t* ptx, size_t size, uint64_t* module) {
  return guarded([&] {
    require_out(module, "module");
    if (ptx == nullptr && size > 0) throw std::invalid_argument("PTX bytes must not be null");
    std::vector<std::uint8_t> bytes(ptx, ptx + size);
    auto r = driver.load_ptx(ctx(context), bytes);
    *module = handle(r.module);
    return from_driver(r.status);
  });
}

int f4s_load_module_image(uint64_t context, const void* image, size_t size, uint64_t* module) {
  return guarded([&] {
    require_out(module, "module");
    auto r = driver.load_module_image(ctx(context), image, size);
    *module = handle(r.module);
    return from_driver(r.status);
  });
}

int f4s_unload_module(uint64_t context, uint64_t module) {
  return guarded([&] { return from_driver(driver.unload_module(ctx(context), module_of(module))); });
}

int f4s_resolve_function(uint64_t context, uint64_t module, const char* name, uint64_t* function) {
  return guarded([&] {
    require_out(function, "function");
    if (name == nullptr) throw std::invalid_argument("CUDA function name must not be null");
    auto r = driver.resolve_function(ctx(context), module_of(module), name);
    *function = handle(r.function);
    return from_driver(r.status);
  });
}

int f4s_query_function_attributes(uint64_t context, uint64_t function, int32_t attributes[5]) {
  return guarded([&] {
    require_out(attributes, "attributes");
    auto r = driver.function_attributes(ctx(context), function_of(function));
    attributes[0] = r.attributes.max_threads_per_block;
    attributes[1] = r.attributes.static_shared_memory_bytes;
    attributes[2] = r.attributes.constant_memory_bytes;
    attributes[3] = r.attributes.local_memory_bytes;
    attributes[4] = r.attributes.registers_per_thread;
    return from_driver(r.status);
  });
}

int f4s_create_stream(uint64_t context, int32_t flags, uint64_t* stream) {
  return guarded([&] {
    require_out(stream, "stream");
    auto r = driver.create_stream(ctx(context), static_cast<std::uint32_t>(flags));
    *stream = handle(r.stream);
    return from_driver(r.status);
  });
}

int f4s_destroy_stream(uint64_t context, uint64_t stream) {
  return guarded([&] { return from_driver(driver.destroy_stream(ctx(context), stream_of(stream))); });
}

int f4s_synchronize_stream(uint64_t context, uint64_t stream) {
  return guarded([&] { return from_driver(driver.synchronize_stream(ctx(context), stream_of(stream))); });
}

int f4s_create_event(uint64_t context, int32_t flags, uint64_t* event) {
  return guarded([&] {
    require_out(event, "event");
    auto r = driver.create_event(ctx(context), static_cast<std::uint32_t>(flags));
    *event = handle(r.event);
    return from_driver(r.status);
  });
}

int f4s_destroy_event(uint64_t context, uint64_t event) {
  return guarded([&] { return from_driver(driver.destroy_event(ctx(context), event_of(event))); });
}

int f4s_record_event(uint64_t context, uint64_t event, uint64_t stream) {
  return guarded([&] {
    return from_driver(driver.record_event(ctx(context), event_of(event), stream_of(stream)));
  });
}

int f4s_query_event(uint64_t context, uint64_t event, int32_t* complete) {
  return guarded([&] {
    require_out(complete, "completion flag");
    auto r = driver.query_event(ctx(context), event_of(event));
    *complete = r.complete ? 1 : 0;
    return from_driver(r.status);
  });
}

int f4s_synchronize_event(uint64_t context, uint64_t event) {
  return guarded([&] { return from_driver(driver.synchronize_event(ctx(context), event_of(event))); });
}

int f4s_wait_for_event(uint64_t context, uint64_t stream, uint64_t event) {
  return guarded([&] {
    return from_driver(driver.wait_for_event(ctx(context), stream_of(stream), event_of(event)));
  });
}

int f4s_event_elapsed_ms(uint64_t context, uint64_t start, uint64_t end, float* ms) {
  return guarded([&] {
    require_out(ms, "elapsed time");
    auto r = driver.elapsed_time(ctx(context), event_of(start), event_of(end));
    *ms = r.milliseconds;
    return from_driver(r.status);
  });
}

int f4s_allocate_pinned_memory(uint64_t context, uint64_t size, void** host) {
  return guarded([&] {
    require_out(host, "host address");
    auto r = driver.allocate_pinned_memory(ctx(context), size);
    *host = r.address;
    return from_driver(r.status);
  });
}

int f4s_free_pinned_memory(uint64_t context, void* host) {
  return guarded([&] { return from_driver(driver.free_pinned_memory(ctx(context), host)); });
}

int f4s_allocate_device_memory(uint64_t context, uint64_t size, uint64_t* device) {
  return guarded([&] {
    require_out(device, "device address");
    auto r = driver.allocate_device_memory(ctx(context), size);
    *device = static_cast<std::uint64_t>(r.address);
    return from_driver(r.status);
  });
}

int f4s_free_device_memory(uint64_t context, uint64_t device) {
  return guarded([&] { return from_driver(driver.free_device_memory(ctx(context), device)); });
}

int f4s_copy_host_to_device(uint64_t context, uint64_t dst, uint64_t off, const void* src, uint64_t size) {
  return guarded([&] { return from_driver(driver.copy_host_to_device(ctx(context), dst, off, src, size)); });
}

int f4s_copy_host_to_device_async(uint64_t context, uint64_t dst, uint64_t off, const void* src, uint64_t size,
                                  uint64_t stream) {
  return guarded([&] {
    return from_driver(driver.copy_host_to_device_async(ctx(context), dst, off, src, size, stream_of(stream)));
  });
}

int f4s_copy_device_to_host(uint64_t context, uint64_t src, uint64_t off, void* dst, uint64_t size) {
  return guarded([&] { return from_driver(driver.copy_device_to_host(ctx(context), dst, src, off, size)); });
}

int f4s_copy_device_to_host_async(uint64_t context, uint64_t src, uint64_t off, void* dst, uint64_t size,
                                  uint64_t stream) {
  return guarded([&] {
    return from_driver(driver.copy_device_to_host_async(ctx(context), dst, src, off, size, stream_of(stream)));
  });
}

int f4s_hotpath_open(uint64_t context, f4s_hotpath** hotpath) {
  return guarded([&] {
    require_out(hotpath, "hotpath");
    *hotpath = nullptr;
    Hotpath* impl = Hotpath::open(ctx(context));
    *hotpath = new f4s_hotpath{impl};
    return set_status(0, "CUDA_SUCCESS", "");
  });
}

int f4s_hotpath_close(f4s_hotpath* hotpath) {
  return guarded([&] {
    if (hotpath == nullptr) throw std::invalid_argument("hotpath handle must not be null");
    delete hotpath->impl;
    delete hotpath;
    return set_status(0, "CUDA_SUCCESS", "");
  });
}

uint64_t f4s_hotpath_module(const f4s_hotpath* hotpath) {
  return (hotpath && hotpath->impl) ? handle(hotpath->impl->module()) : 0;
}

int f4s_hotpath_sm_count(const f4s_hotpath* hotpath) {
  return (hotpath && hotpath->impl) ? hotpath->impl->sm_count() : 0;
}

int f4s_hotpath_set_reduce_cluster(f4s_hotpath* hotpath, int32_t cluster) {
  return guarded([&] { return op_status(hot(hotpath).set_reduce_cluster(cluster)); });
}

int f4s_hotpath_set_launch_overlap(f4s_hotpath* hotpath, int32_t enable) {
  return guarded([&] {
    hot(hotpath).set_launch_overlap(enable != 0);
    return 0;
  });
}

int f4s_hotpath_wait_timeouts(f4s_hotpath* hotpath, uint32_t* count, int32_t reset) {
  return guarded([&] {
    require_out(count, "timeout count");
    return op_status(hot(hotpath).wait_timeouts(count, reset != 0));
  });
}

int f4s_hotpath_check_bounded_wait(f4s_hotpath* hotpath, uint32_t polls) {
  return guarded([&] { return op_status(hot(hotpath).check_bounded_wait(polls)); });
}

uint64_t f4s_reduce_workspace_bytes(const f4s_hotpath* hotpath) {
  return (hotpath && hotpath->impl) ? hotpath->impl->reduce_workspace_bytes() : 0;
}

int f4s_reduce_sum_f32(f4s_hotpath* hp, uint64_t stream, uint64_t in, uint64_t n, uint64_t out, uint64_t ws,
                       uint64_t ws_bytes, int32_t accumulate) {
  return guarded([&] {
    return op_status(hot(hp).reduce(ReduceOp::kSumF32, stream_of(stream), in, n, out, ws, ws_bytes, 0, accumulate));
  });
}

int f4s_reduce_sum_i32(f4s_hotpath* hp, uint64_t stream, uint64_t in, uint64_t n, uint64_t out, uint64_t ws,
                       uint64_t ws_bytes, int32_t accumulate) {
  return guarded([&] {
    return op_status(hot(hp).reduce(ReduceOp::kSumI32, stream_of(stream), in, n, out, ws, ws_bytes, 0, accumulate));
  });
}

int f4s_reduce_argmax_f32(f4s_hotpath* hp, uint64_t stream, uint64_t in, uint64_t n, uint64_t out, uint64_t ws,
                          uint64_t ws_bytes, uint64_t index_base, int32_t accumulate) {
  return guarded([&] {
    return op_status(
        hot(hp).reduce(ReduceOp::kArgmaxF32, stream_of(stream), in, n, out, ws, ws_bytes, index_base, accumulate));
  });
}

int f4s_reduce_sum(f4s_hotpath* hp, uint64_t stream, int32_t input_type, uint64_t in, uint64_t n, uint64_t out,
                   uint64_t ws, uint64_t ws_bytes, int32_t accumulate) {
  return guarded([&] {
    return op_status(
        hot(hp).reduce(sum_op_for_type_code(input_type), stream_of(stream), in, n, out, ws, ws_bytes, 0, accumulate));
  });
}

namespace {

ReducePolicy policy_of(int32_t policy) {
  if (policy < 0 || policy > 2) throw std::invalid_argument("unknown reduction policy " + std::to_string(policy));
  return static_cast<ReducePolicy>(policy);
}

bool uses_ordered(ReduceOp op, ReducePolicy policy) {
  return policy != ReducePolicy::kFast && Hotpath::has_ordered_kernel(op);
}

}  // namespace

int f4s_reduce_argmax(f4s_hotpath* hp, uint64_t stream, int32_t input_type, uint64_t in, uint64_t n, uint64_t out,
                      uint64_t ws, uint64_t ws_bytes, uint64_t index_base, int32_t accumulate) {
  return guarded([&] {
    return op_status(hot(hp).reduce(argmax_op_for_type_code(input_type), stream_of(stream), in, n, out, ws, ws_bytes,
                                    index_base, accumulate));
  });
}

int f4s_reduce_sum_policy(f4s_hotpath* hp, uint64_t stream, int32_t input_type, int32_t policy, uint64_t in,
                          uint64_t n, uint64_t out, uint64_t ws, uint64_t ws_bytes, int32_t accumulate) {
  return guarded([&] {
    const ReduceOp op = sum_op_for_type_code(input_type);
    if (uses_ordered(op, policy_of(policy)))
      return op_status(hot(hp).reduce_ordered(op, stream_of(stream), in, n, out, ws, ws_bytes, accumulate));
    return op_status(hot(hp).reduce(op, stream_of(stream), in, n, out, ws, ws_bytes, 0, accumulate));
  });
}

int f4s_reduce_policy_workspace_bytes(const f4s_hotpath* hp, int32_t input_type, int32_t policy, uint64_t n,
                                      uint64_t* bytes) {
  return guarded([&] {
    if (hp == nullptr || hp->impl == nullptr) throw std::invalid_argument("hotpath handle must not be null");
    if (bytes == nullptr) throw std::invalid_argument("output pointer must not be null");
    const ReduceOp op = sum_op_for_type_code(input_type);
    *bytes = uses_ordered(op, policy_of(policy)) ? Hotpath::ordered_workspace_bytes(op, n)
                                                 : hp->impl->reduce_workspace_bytes();
    return 0;
  });
}

int f4s_reduce_ordered_groups(int32_t input_type, uint64_t in, uint64_t n, uint64_t* groups) {
  return guarded([&] {
    if (groups == nullptr) throw std::invalid_argument("output pointer must not be null");
    *groups = Hotpath::ordered_groups(sum_op_for_type_code(input_type), in, n);
    return 0;
  });
}

int f4s_reduce_ordered_final(f4s_hotpath* hp, uint64_t stream, uint64_t groups, uint64_t count, uint64_t out,
                             int32_t accumulate) {
  return guarded([&] {
    return op_status(hot(hp).reduce_ordered_final(stream_of(stream), groups, count, out, accumulate));
  });
}

int f4s_convert(f4s_hotpath* hp, uint64_t stream, int32_t from_type, int32_t to_type, int32_t rounding,
                int32_t saturation, uint64_t in, uint64_t out, uint64_t n) {
  return guarded([&] {
    return op_status(hot(hp).convert(stream_of(stream), from_type, to_type, rounding, saturation, in, out, n));
  });
}

int f4s_reduce_host(f4s_hotpath* hp, int32_t op, const void* host_in, uint64_t n, uint64_t index_base,
                    void* host_out, uint64_t staging, uint64_t staging_bytes, uint64_t ws, uint64_t ws_bytes,
                    uint64_t copy_stream, uint64_t compute_stream) {
  return guarded([&] {
    if (op < 0 || op >= kReduceOpCount) throw std::invalid_argument("unknown reduction op " + std::to_string(op));
    return op_status(hot(hp).reduce_host(static_cast<ReduceOp>(op), host_in, n, index_base, host_out, staging,
                                         staging_bytes, ws, ws_bytes, stream_of(copy_stream),
                                         stream_of(compute_stream)));
  });
}

int f4s_reduce_host_sum_policy(f4s_hotpath* hp, int32_t input_type, int32_t policy, const void* host_in, uint64_t n,
                               void* host_out, uint64_t staging, uint64_t staging_bytes, uint64_t ws,
                               uint64_t ws_bytes, uint64_t copy_stream, uint64_t compute_stream) {
  return guarded([&] {
    const ReduceOp op = sum_op_for_type_code(input_type);
    if (uses_ordered(op, policy_of(policy)))
      return op_status(hot(hp).reduce_host_ordered(op, host_in, n, host_out, staging, staging_bytes, ws, ws_bytes,
                                                   stream_of(copy_stream), stream_of(compute_stream)));
    return op_status(hot(hp).reduce_host(op, host_in, n, 0, host_out, staging, staging_bytes, ws, ws_bytes,
                                         stream_of(copy_stream), stream_of(compute_stream)));
  });
}

int f4s_reduce_host_sum_argmax_f32(f4s_hotpath* hp, const void* host_in, uint64_t n, uint64_t index_base,
                                   void* host_sum_out, void* host_argmax_out, uint64_t staging,
                                   uint64_t staging_bytes, uint64_t ws, uint64_t ws_bytes, uint64_t copy_stream,
                                   uint64_t compute_stream) {
  return guarded([&] {
    return op_status(hot(hp).reduce_host_sum_argmax(host_in, n, index_base, host_sum_out, host_argmax_out, staging,
                                                    staging_bytes, ws, ws_bytes, stream_of(copy_stream),
                                                    stream_of(compute_stream)));
  });
}

uint64_t f4s_block_reduce_workspace_bytes(int32_t n) {
  return Hotpath::block_sum_workspace_bytes(n < 0 ? 0 : n);
}

int f4s_block_reduce_sum_f32(f4s_hotpath* hp, uint64_t stream, uint64_t in, int32_t n, uint64_t partials,
                             uint64_t out, uint64_t ws, uint64_t ws_bytes) {
  return guarded(
      [&] { return op_status(hot(hp).block_sum_f32(stream_of(stream), in, n, partials, out, ws, ws_bytes)); });
}

int f4s_block_reduce_sum_f32_noalloc(f4s_hotpath* hp, uint64_t stream, uint64_t in, int32_t n, uint64_t partials,
                                     uint64_t out) {
  return guarded([&] {
    return op_status(flight4s::cuda::block_sum_f32_noalloc(hot(hp), stream_of(stream), in, n, partials, out));
  });
}

int f4s_vector_add_f32(f4s_hotpath* hp, uint64_t stream, uint64_t a, uint64_t b, uint64_t c, int32_t n) {
  return guarded([&] { return op_status(hot(hp).vector_add(false, stream_of(stream), a, b, c, n)); });
}

int f4s_vector_add_bf16(f4s_hotpath* hp, uint64_t stream, uint64_t a, uint64_t b, uint64_t c, int32_t n) {
  return guarded([&] { return op_status(hot(hp).vector_add(true, stream_of(stream), a, b, c, n)); });
}

int f4s_vector_add(f4s_hotpath* hp, uint64_t stream, int32_t type_code, uint64_t a, uint64_t b, uint64_t c,
                   int32_t n) {
  return guarded([&] { return op_status(hot(hp).vector_add_typed(type_code, stream_of(stream), a, b, c, n)); });
}

int f4s_softmax_rows_bf16(f4s_hotpath* hp, uint64_t stream, uint64_t in, uint64_t out, int32_t rows, int32_t cols) {
  return guarded([&] { return op_status(hot(hp).softmax_rows(stream_of(stream), in, out, rows, cols)); });
}

int f4s_rmsnorm_rows_bf16(f4s_hotpath* hp, uint64_t stream, uint64_t in, uint64_t weight, uint64_t out,
                          int32_t rows, int32_t cols, float eps) {
  return guarded(
      [&] { return op_status(hot(hp).rmsnorm_rows(stream_of(stream), in, weight, out, rows, cols, eps)); });
}

int f4s_fp8_quantize_e4m3(f4s_hotpath* hp, uint64_t stream, uint64_t x, uint64_t codes, uint64_t scales,
                          int32_t rows, int32_t cols) {
  return guarded(
      [&] { return op_status(hot(hp).fp8_quantize(stream_of(stream), x, codes, scales, rows, cols)); });
}

int f4s_fp8_dequantize_e4m3(f4s_hotpath* hp, uint64_t stream, uint64_t codes, uint64_t scales, uint64_t y,
                            int32_t rows, int32_t cols) {
  return guarded(
      [&] { return op_status(hot(hp).fp8_dequantize(stream_of(stream), codes, scales, y, rows, cols)); });
}

int f4s_fill_synthetic(f4s_hotpath* hp, uint64_t stream, uint64_t out, uint64_t n, uint64_t offset, uint64_t seed,
                       uint32_t stream_id, int32_t kind, float p0, float p1, float p2, float p3, int32_t ilo,
                       int32_t ihi) {
  return guarded([&] {
    return op_status(hot(hp).fill_synthetic(stream_of(stream), out, n, offset, seed, stream_id, kind, p0, p1, p2,
                                            p3, ilo, ihi));
  });
}

}  // extern "C"
