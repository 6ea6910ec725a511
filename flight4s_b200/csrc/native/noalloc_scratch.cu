// Allocation-free block sum: f4s_block_reduce_sum_f32_noalloc.
//
// Why it exists: some callers of this library cannot allocate device
// memory when they need a result.  Examples are hosts whose device memory
// is owned by another allocator and must not be bypassed with a raw
// cudaMalloc (a JVM or Python runtime that hands out pooled buffers), code
// running where allocation is not allowed or too costly (a real-time loop
// that must not block on the allocator, a CUDA host callback), and caller
// code that has no way to size or keep a workspace.  The regular block sum
// needs a small caller-provided workspace; this entry point needs none.
//
// How: the workspace lives in the file-scope device array below, 64 KiB
// per GPU, created when this library's device code is first loaded on a GPU
// and held by that GPU until the process exits.  Host code cannot use the
// array's name as a device address (on the host it names a stand-in), so the
// first call on each device makes that device's context current and asks
// cudaGetSymbolAddress for the real address, which is cached per device.
// Make that first call outside any stream capture.  The block-sum kernel is
// the same one the regular entry point launches; only the workspace differs.
//
// Limits and sharing: the workspace holds 256 bytes of header plus one
// 4-byte partial per 65536-element cluster, so n may be at most
// 16320 * 65536 = 1,069,547,520 elements; larger n is rejected with
// F4S_STATUS_INVALID_ARGUMENT.  Every call on a device shares the one
// array and the array keeps the last call's contents: each call first
// zeroes the ticket counter with cudaMemsetAsync on its own stream, and
// calls whose execution overlaps on the GPU (different streams, no
// ordering between them) race on the array and give wrong results.
// Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda.h>
#include <cuda_runtime_api.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "cuda_driver.hpp"
#include "hotpath.hpp"

namespace {

constexpr std::size_t kNoallocWorkspaceBytes = 64 * 1024;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char f4s_noalloc_block_sum_workspace[kNoallocWorkspaceBytes];

std::mutex g_setup_mutex;
void* g_workspace_address[kMaxDevices] = {};

// Device address of this device's workspace; `context` must be current.
void* workspace_for_current_device() {
  const flight4s::cuda::DriverApi& api = flight4s::cuda::require_driver();
  CUdevice device = 0;
  if (api.cuCtxGetDevice(&device) != CUDA_SUCCESS || device < 0 || device >= kMaxDevices)
    throw std::runtime_error("no usable current CUDA device for the allocation-free workspace");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_workspace_address[device] == nullptr) {
    void* address = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&address, f4s_noalloc_block_sum_workspace);
    if (err != cudaSuccess || address == nullptr) {
      throw std::runtime_error(std::string("cudaGetSymbolAddress of the allocation-free workspace failed: ") +
                               cudaGetErrorString(err));
    }
    g_workspace_address[device] = address;
  }
  return g_workspace_address[device];
}

}  // namespace

namespace flight4s::cuda {

// Largest n the static workspace can serve.
std::int64_t noalloc_block_sum_max_elements() {
  return static_cast<std::int64_t>((kNoallocWorkspaceBytes - 256) / 4) * 65536;
}

CUresult block_sum_f32_noalloc(Hotpath& hp, CUstream stream, CUdeviceptr in, std::int32_t n,
                               CUdeviceptr partials, CUdeviceptr out) {
  if (n < 0) throw std::invalid_argument("element count must not be negative: " + std::to_string(n));
  if (static_cast<std::int64_t>(n) > noalloc_block_sum_max_elements()) {
    throw std::invalid_argument("allocation-free block sum supports at most " +
                                std::to_string(noalloc_block_sum_max_elements()) + " elements (got " +
                                std::to_string(n) + "); use f4s_block_reduce_sum_f32 with a workspace");
  }
  CurrentContextScope scope(hp.context());
  if (scope.push_result() != CUDA_SUCCESS) return scope.push_result();
  void* ws = workspace_for_current_device();
  // The kernel leaves the ticket at zero, but a call that never finished
  // could not; clear it, ordered on this call's stream.
  const cudaError_t err = cudaMemsetAsync(ws, 0, 256, reinterpret_cast<cudaStream_t>(stream));
  if (err != cudaSuccess)
    throw std::runtime_error(std::string("clearing the allocation-free workspace failed: ") + cudaGetErrorString(err));
  const CUresult r = hp.block_sum_f32(stream, in, n, partials, out, reinterpret_cast<CUdeviceptr>(ws),
                                      kNoallocWorkspaceBytes);
  const CUresult pop = scope.close();
  return r == CUDA_SUCCESS ? pop : r;
}

}  // namespace flight4s::cuda
