// Hot-path operators: the B200 lowering targets of the reference's
// reduction node and of the elementwise / row-wise / FP8 kernels.
//
// A Hotpath binds one CUDA context to the embedded sm_100a module (loaded
// with cuModuleLoadDataEx, as the reference loads its generated modules,
// native/src/cuda_driver.cpp:209-261) and to launch shapes sized for the
// device (SM count x resident CTAs, cluster occupancy).  Every operator
// packs its kernel arguments with the reference's descriptor codes and goes
// through the same cuLaunchKernelEx launcher as user kernels
// (native/src/cuda_launcher.cpp:8-62).  Operators are asynchronous on the
// given stream and never allocate: device buffers, including the small
// reduction workspace, belong to the caller.
#pragma once

#include <cuda.h>

#include <cstdint>
#include <string>

#include "cuda_driver.hpp"
#include "launch_contract.hpp"

namespace flight4s::cuda {

// Full-array reductions.  0..2 are the original f32 / i32 operators; the
// rest sum the other AccumulatorType inputs of the reference's ReduceSum
// (core/src/main/scala/flight4s/core/types/CudaType.scala:199-230).
enum class ReduceOp : int {
  kSumF32 = 0,
  kSumI32 = 1,
  kArgmaxF32 = 2,
  kSumU32 = 3,
  kSumF16 = 4,
  kSumBf16 = 5,
  kSumF64 = 6,
  kSumE4m3 = 7,
  kSumE5m2 = 8,
  // max / argmax over the other OrderedTypes (CudaType.scala:182-188)
  kArgmaxI32 = 9,
  kArgmaxU32 = 10,
  kArgmaxF16 = 11,
  kArgmaxBf16 = 12,
  kArgmaxF64 = 13,
};
constexpr int kReduceOpCount = 14;

// Bytes of one input element and of the result record of `op`.
int reduce_input_bytes(ReduceOp op);
int reduce_output_bytes(ReduceOp op);
// The sum operator for a launch-ABI type code
// (core/src/main/scala/flight4s/core/abi/CudaAbi.scala:11-20: 2 i32, 3 u32,
// 4 f16, 5 bf16, 6 f32, 7 f64, 8 fp8 e4m3, 9 fp8 e5m2); throws
// std::invalid_argument for codes without an accumulator (bool, pointer).
ReduceOp sum_op_for_type_code(int code);
// The max / argmax operator for an OrderedType code (2 i32, 3 u32, 4 f16,
// 5 bf16, 6 f32, 7 f64); std::invalid_argument otherwise.
ReduceOp argmax_op_for_type_code(int code);
bool is_argmax(ReduceOp op);

// The reference's ReductionPolicy (core/src/main/scala/flight4s/core/ir/IR.scala:79-82).
// Fast: the geometry-sized kernels (reproducible on one device and launch
// shape).  Deterministic and Strict: the order-fixed kernels, whose
// floating-point result depends on the elements only (any grid, cluster,
// device or GPU count); the reference's serial loop order itself cannot be
// kept by a parallel sum, so Strict gets the same fixed order.
enum class ReducePolicy : int { kStrict = 0, kDeterministic = 1, kFast = 2 };

struct HotpathShape {
  int reduce_cluster = 4;       // CTAs per cluster in the full-array reductions
  int reduce_max_clusters[kReduceOpCount] = {};  // co-resident clusters per op (occupancy query)
  int add_grid = 0;
  int fp8_grid = 0;
  int fill_grid = 0;
  int ordered_ctas_per_sm[kReduceOpCount] = {};  // order-fixed sums (float ops only)
};

class Hotpath {
 public:
  // Loads the module into `context` and sizes launch shapes.
  static Hotpath* open(CUcontext context);
  ~Hotpath();

  CUcontext context() const { return context_; }
  CUmodule module() const { return module_; }
  int sm_count() const { return sm_count_; }
  const HotpathShape& shape() const { return shape_; }
  // Re-size the full-array reduction grid for a cluster size in [1, 8].
  CUresult set_reduce_cluster(int cluster);
  // Let each full-array reduction start streaming its input while the
  // kernel launched before it on the same stream finishes (programmatic
  // dependent launch); it waits for that kernel before touching its
  // workspace or output.  Off by default; only for callers whose reduction
  // inputs are never written by the kernel launched right before them.
  void set_launch_overlap(bool enable) { overlap_ = enable; }
  bool launch_overlap() const { return overlap_; }

  std::uint64_t reduce_workspace_bytes() const;
  static std::uint64_t block_sum_workspace_bytes(std::int64_t n);

  CUresult reduce(ReduceOp op, CUstream stream, CUdeviceptr in, std::uint64_t n, CUdeviceptr out,
                  CUdeviceptr workspace, std::uint64_t workspace_bytes, std::uint64_t index_base,
                  int accumulate) {
    return reduce_launch(op, stream, in, n, out, workspace, workspace_bytes, index_base, accumulate, overlap_);
  }
  // Order-fixed floating-point sums: 256 KiB groups of the 16-byte-aligned
  // body, group partials in `workspace` from byte 256 (f64 each, readable
  // after the launch), total = fixed tree over the group partials + the
  // unaligned head.  f32/f16/bf16/f64/e4m3/e5m2 sum ops only.
  static bool has_ordered_kernel(ReduceOp op);
  static std::uint64_t ordered_groups(ReduceOp op, CUdeviceptr in, std::uint64_t n);
  static std::uint64_t ordered_workspace_bytes(ReduceOp op, std::uint64_t n);  // any alignment
  CUresult reduce_ordered(ReduceOp op, CUstream stream, CUdeviceptr in, std::uint64_t n, CUdeviceptr out,
                          CUdeviceptr workspace, std::uint64_t workspace_bytes, int accumulate);
  // The same fixed tree over `count` group partials (several GPUs' partials
  // concatenated in array order).
  CUresult reduce_ordered_final(CUstream stream, CUdeviceptr groups, std::uint64_t count, CUdeviceptr out,
                                int accumulate);
  // Elementwise Convert (the reference's Convert node) of n elements from
  // one launch-ABI type to another: f32 -> f16 / bf16 under a rounding
  // mode (0 nearest-even, 1 toward zero, 2 toward +inf, 3 toward -inf),
  // f32 -> FP8 E4M3 / E5M2 under a saturation mode (0 none, 1 finite),
  // f16 / bf16 / FP8 -> f32, or the same type (a copy).
  CUresult convert(CUstream stream, int from_type, int to_type, int rounding, int saturation, CUdeviceptr in,
                   CUdeviceptr out, std::uint64_t n);
  CUresult block_sum_f32(CUstream stream, CUdeviceptr in, std::int32_t n, CUdeviceptr partials,
                         CUdeviceptr out, CUdeviceptr workspace, std::uint64_t workspace_bytes);
  // c = a + b for an AdditiveType by launch-ABI code: 2 i32, 3 u32 (32-bit
  // wrap), 4 f16, 5 bf16 (nearest-even), 6 f32, 7 f64.
  CUresult vector_add_typed(int type_code, CUstream stream, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c,
                            std::int32_t n);
  CUresult vector_add(bool bf16, CUstream stream, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c,
                      std::int32_t n);
  CUresult softmax_rows(CUstream stream, CUdeviceptr in, CUdeviceptr out, std::int32_t rows,
                        std::int32_t cols);
  CUresult rmsnorm_rows(CUstream stream, CUdeviceptr in, CUdeviceptr weight, CUdeviceptr out,
                        std::int32_t rows, std::int32_t cols, float eps);
  CUresult fp8_quantize(CUstream stream, CUdeviceptr x, CUdeviceptr codes, CUdeviceptr scales,
                        std::int32_t rows, std::int32_t cols);
  CUresult fp8_dequantize(CUstream stream, CUdeviceptr codes, CUdeviceptr scales, CUdeviceptr y,
                          std::int32_t rows, std::int32_t cols);
  CUresult fill_synthetic(CUstream stream, CUdeviceptr out, std::uint64_t n, std::uint64_t offset,
                          std::uint64_t seed, std::uint32_t stream_id, int kind, float p0, float p1,
                          float p2, float p3, std::int32_t ilo, std::int32_t ihi);

  // End-to-end reduction of a HOST buffer: chunked host->device copies on
  // `copy_stream` overlapped with per-chunk reductions on `compute_stream`
  // (double-buffered in `staging`), result copied back to `host_out`, and
  // both streams synchronized before returning.
  CUresult reduce_host(ReduceOp op, const void* host_in, std::uint64_t n, std::uint64_t index_base, void* host_out,
                       CUdeviceptr staging, std::uint64_t staging_bytes, CUdeviceptr workspace,
                       std::uint64_t workspace_bytes, CUstream copy_stream, CUstream compute_stream);

  // Same pipeline computing the f32 sum and the argmax from one host->device
  // transfer of each chunk (8-byte sum and 16-byte argmax record out).
  CUresult reduce_host_sum_argmax(const void* host_in, std::uint64_t n, std::uint64_t index_base,
                                  void* host_sum_out, void* host_argmax_out, CUdeviceptr staging,
                                  std::uint64_t staging_bytes, CUdeviceptr workspace, std::uint64_t workspace_bytes,
                                  CUstream copy_stream, CUstream compute_stream);

  // Order-fixed sum of a HOST buffer: the same pipeline with chunks of
  // whole 256 KiB groups, each chunk's group partials written to their
  // place in `workspace` (ordered_workspace_bytes(op, n) bytes), then F over
  // all of them.  The f64 result is bit-identical to reduce_ordered() of
  // the same array at a 16-byte-aligned device address.
  CUresult reduce_host_ordered(ReduceOp op, const void* host_in, std::uint64_t n, void* host_out,
                               CUdeviceptr staging, std::uint64_t staging_bytes, CUdeviceptr workspace,
                               std::uint64_t workspace_bytes, CUstream copy_stream, CUstream compute_stream);

  // Bounded device-side waits that gave up since the last reset (read after
  // synchronizing the context); non-zero means some output was not written.
  CUresult wait_timeouts(std::uint32_t* count, bool reset);
  // Launches a one-thread kernel whose wait can never be satisfied, bounded
  // to `polls` polls: exercises the give-up path on the device.
  CUresult check_bounded_wait(std::uint32_t polls);

  CUfunction function(const std::string& name) const;

 private:
  Hotpath() = default;
  CUresult launch(CUfunction fn, CUstream stream, int grid, int block, int cluster, ArgumentPack& args,
                  bool programmatic = false);
  // reduce(); `programmatic` launches it as a programmatic dependent of the
  // previous kernel on `stream` (the host-buffer pipelines never do: their
  // inputs arrive by copies).
  CUresult reduce_launch(ReduceOp op, CUstream stream, CUdeviceptr in, std::uint64_t n, CUdeviceptr out,
                         CUdeviceptr workspace, std::uint64_t workspace_bytes, std::uint64_t index_base,
                         int accumulate, bool programmatic);
  // Chunked, double-buffered host->device pipeline shared by the host-buffer
  // reductions: every op in `ops` reduces each staged chunk, op i into
  // `host_outs[i]`.
  CUresult reduce_host_ops(const ReduceOp* ops, int nops, const void* host_in, std::uint64_t n,
                           std::uint64_t index_base, void* const* host_outs, CUdeviceptr staging,
                           std::uint64_t staging_bytes, CUdeviceptr workspace, std::uint64_t workspace_bytes,
                           CUstream copy_stream, CUstream compute_stream);
  // The pipeline itself: chunks of `chunk` elements (> 0) of `elem` bytes
  // copied into the two halves of the staging area on `copy_stream`;
  // `on_chunk(k, buffer, first, count)` enqueues chunk k's work on
  // `compute_stream` (called once with count 0 when n == 0), `on_done()`
  // the work after the last chunk; then both streams are synchronized.
  template <class OnChunk, class OnDone>
  CUresult stream_chunks(const void* host_in, std::uint64_t n, int elem, std::uint64_t chunk,
                         const CUdeviceptr buffers[2], CUstream copy_stream, CUstream compute_stream,
                         OnChunk&& on_chunk, OnDone&& on_done);

  CUcontext context_ = nullptr;
  CUmodule module_ = nullptr;
  int sm_count_ = 0;
  HotpathShape shape_;
  bool overlap_ = false;
};

}  // namespace flight4s::cuda
