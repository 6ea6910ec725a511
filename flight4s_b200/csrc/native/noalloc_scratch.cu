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
// per GPU, created when this library's device code is first loaded into a
// CUDA context and held until that context is destroyed (for the primary
// context, until the process exits).  Host code cannot use the array's name
// as a device address (on the host it names a stand-in), so the first call
// in each context makes that context current and asks cudaGetSymbolAddress
// for the real address, which is then cached under the context's unique id
// (cuCtxGetId).  One device can carry several contexts (its primary context
// and contexts made with cuCtxCreate), each with its own copy of the array,
// and a destroyed context's id is never reused, so an address is only ever
// used in the context it was looked up in.  That first call per context may
// load this file's device code, which a stream capture cannot record: it is
// rejected with F4S_STATUS_INVALID_ARGUMENT while `stream` is capturing, so
// make it before any capture.  The block-sum kernels are the same ones the
// regular entry point launches; only the workspace differs (arrays of up to
// 2^23 elements take the two-launch form, which reads no workspace, so only
// larger arrays use the array's ticket and partials).
//
// Limits and sharing: the workspace holds 256 bytes of header plus one
// 4-byte partial per 65536-element cluster, so n may be at most
// 16320 * 65536 = 1,069,547,520 elements; larger n is rejected with
// F4S_STATUS_INVALID_ARGUMENT.  Every call in a context shares the one
// array and the array keeps the last call's contents: each call first
// zeroes the header (the ticket counter) on its own stream, and calls
// whose execution overlaps on the GPU (different streams, no ordering
// between them) race on the array and give wrong results.  Nothing here
// calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda.h>
#include <cuda_runtime_api.h>

#include <limits>
#include <mutex>
#include <stdexcept>
#include <string>

#include "cuda_driver.hpp"
#include "hotpath.hpp"

namespace {

constexpr std::size_t kNoallocWorkspaceBytes = 64 * 1024;

static __device__ __align__(256) unsigned char f4s_noalloc_block_sum_workspace[kNoallocWorkspaceBytes];

// Workspace addresses by context id.  A fixed table (no host allocation
// either): when it is full the oldest entry is replaced, which only costs
// that context one more symbol lookup on its next call.
struct CachedAddress {
  unsigned long long context_id = 0;
  void* address = nullptr;
};
constexpr int kCachedContexts = 64;
std::mutex g_setup_mutex;
CachedAddress g_cache[kCachedContexts];
int g_next_slot = 0;

// Device address of the workspace in the current context (the caller has
// made the hot path's context current).  `stream` is the call's stream.
void* workspace_for_current_context(CUstream stream) {
  const flight4s::cuda::DriverApi& api = flight4s::cuda::require_driver();
  CUcontext context = nullptr;
  unsigned long long id = 0;
  if (api.cuCtxGetCurrent(&context) != CUDA_SUCCESS || context == nullptr ||
      api.cuCtxGetId(context, &id) != CUDA_SUCCESS)
    throw std::runtime_error("no usable current CUDA context for the allocation-free workspace");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  for (const CachedAddress& entry : g_cache) {
    if (entry.address != nullptr && entry.context_id == id) return entry.address;
  }
  CUstreamCaptureStatus capture = CU_STREAM_CAPTURE_STATUS_NONE;
  if (api.cuStreamIsCapturing(stream, &capture) != CUDA_SUCCESS || capture != CU_STREAM_CAPTURE_STATUS_NONE) {
    throw std::invalid_argument(
        "the first allocation-free block sum in a CUDA context looks up its workspace, which a stream capture "
        "cannot record: make one call in this context before capturing");
  }
  void* address = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&address, f4s_noalloc_block_sum_workspace);
  if (err != cudaSuccess || address == nullptr) {
    throw std::runtime_error(std::string("cudaGetSymbolAddress of the allocation-free workspace failed: ") +
                             cudaGetErrorString(err));
  }
  g_cache[g_next_slot] = CachedAddress{id, address};
  g_next_slot = (g_next_slot + 1) % kCachedContexts;
  return address;
}

}  // namespace

namespace flight4s::cuda {

// Largest n whose block-sum workspace fits the static array (the
// workspace size grows with n).
std::int64_t noalloc_block_sum_max_elements() {
  static const std::int64_t largest = [] {
    std::int64_t lo = 0, hi = std::numeric_limits<std::int32_t>::max();
    while (lo < hi) {
      const std::int64_t mid = lo + (hi - lo + 1) / 2;
      if (Hotpath::block_sum_workspace_bytes(mid) <= kNoallocWorkspaceBytes) lo = mid; else hi = mid - 1;
    }
    return lo;
  }();
  return largest;
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
  void* ws = workspace_for_current_context(stream);
  // The kernel leaves the ticket at zero, but a call that never finished
  // could not; clear the header, ordered on this call's stream.
  const CUresult cleared = require_driver().cuMemsetD8Async(reinterpret_cast<CUdeviceptr>(ws), 0, 256, stream);
  if (cleared != CUDA_SUCCESS) {
    scope.close();
    return cleared;
  }
  const CUresult r = hp.block_sum_f32(stream, in, n, partials, out, reinterpret_cast<CUdeviceptr>(ws),
                                      kNoallocWorkspaceBytes);
  const CUresult pop = scope.close();
  return r == CUDA_SUCCESS ? pop : r;
}

}  // namespace flight4s::cuda
