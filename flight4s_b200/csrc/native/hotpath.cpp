#include "hotpath.hpp"

#include <algorithm>
#include <stdexcept>
#include <string>

#include "cuda_launcher.hpp"
#include "launch_contract.hpp"

// The sm_100a cubin, embedded at build time (kernel_image.S).
extern "C" const unsigned char f4s_kernel_image_begin[];
extern "C" const unsigned char f4s_kernel_image_end[];

namespace flight4s::cuda {
namespace {

// Launch constants shared with the kernels (csrc/kernels/*.cuh).
constexpr int kReduceBlock = 512;
constexpr int kReduceUnroll = 8;
constexpr int kReduceWaves = 8;
constexpr std::uint64_t kReducePartialOffset = 256;
constexpr std::uint64_t kReducePartialBytes = 16;
constexpr int kOrderedBlock = 512;
constexpr std::uint64_t kOrderedGroupBytes = 256 * 1024;  // 64 tiles of 256 16-byte vectors
constexpr std::uint64_t kOrderedGroupOffset = 256;
constexpr int kBlockSumThreads = 1024;
constexpr int kBlockSumCluster = 8;
constexpr std::int64_t kBlockSumElemsPerCluster = 256LL * 256LL;
constexpr std::int64_t kBlockSumWarps = kBlockSumThreads / 32;
// Arrays of at most this many 256-element tiles (2^23 elements) take the
// two-launch form (csrc/kernels/block_sum.cuh: kBlockSumSmallMaxTiles).
constexpr std::int64_t kBlockSumSmallMaxTiles = 128LL * 256LL;
constexpr int kBlockSumUpperThreads = 512;
constexpr int kAddBlock = 256;
constexpr int kRowBlock = 256;
constexpr int kFp8Threads = 256;
constexpr int kFp8Block = 128;
constexpr int kQuantUnroll = 4;
constexpr int kDequantUnroll = 2;

void check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error(std::string(what) + " failed with CUDA error " + std::to_string(r));
  }
}

const char* ordered_kernel_name(ReduceOp op) {
  switch (op) {
    case ReduceOp::kSumF32: return "f4s_reduce_ordered_f32";
    case ReduceOp::kSumF16: return "f4s_reduce_ordered_f16";
    case ReduceOp::kSumBf16: return "f4s_reduce_ordered_bf16";
    case ReduceOp::kSumF64: return "f4s_reduce_ordered_f64";
    case ReduceOp::kSumE4m3: return "f4s_reduce_ordered_e4m3";
    case ReduceOp::kSumE5m2: return "f4s_reduce_ordered_e5m2";
    default: return nullptr;
  }
}

void require_ptr(CUdeviceptr p, const char* what) {
  if (p == 0) throw std::invalid_argument(std::string(what) + " must not be null");
}

void require_nonnegative(std::int64_t v, const char* what) {
  if (v < 0) throw std::invalid_argument(std::string(what) + " must not be negative: " + std::to_string(v));
}

// RAII push of the hotpath's context around one operator call.
class Current {
 public:
  explicit Current(CUcontext c) : scope_(c) {
    if (scope_.push_result() != CUDA_SUCCESS) result_ = scope_.push_result();
  }
  CUresult result() const { return result_; }
  CUresult finish(CUresult r) {
    const CUresult pop = scope_.close();
    return r == CUDA_SUCCESS ? pop : r;
  }

 private:
  CurrentContextScope scope_;
  CUresult result_ = CUDA_SUCCESS;
};

}  // namespace

Hotpath* Hotpath::open(CUcontext context) {
  if (context == nullptr) throw std::invalid_argument("CUDA context handle must not be null");
  const DriverApi& api = require_driver();
  CurrentContextScope scope(context);
  check(scope.push_result(), "cuCtxPushCurrent");
  auto* hp = new Hotpath();
  hp->context_ = context;
  try {
    check(api.cuModuleLoadDataEx(&hp->module_, f4s_kernel_image_begin, 0, nullptr, nullptr),
          "loading the sm_100a kernel image (cuModuleLoadDataEx)");
    CUdevice device = 0;
    check(api.cuCtxGetDevice(&device), "cuCtxGetDevice");
    check(api.cuDeviceGetAttribute(&hp->sm_count_, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, device),
          "cuDeviceGetAttribute(MULTIPROCESSOR_COUNT)");
    auto occupancy = [&](const char* name, int block) {
      int blocks = 0;
      check(api.cuOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, hp->function(name), block, 0),
            "cuOccupancyMaxActiveBlocksPerMultiprocessor");
      return std::max(1, blocks);
    };
    hp->shape_.add_grid = hp->sm_count_ * occupancy("f4s_vector_add_f32", kAddBlock);
    hp->shape_.fp8_grid = hp->sm_count_ * occupancy("f4s_fp8_quant_flat", kFp8Threads);
    hp->shape_.fill_grid = hp->sm_count_ * occupancy("f4s_fill_synthetic", 256);
    for (int op = 0; op < kReduceOpCount; ++op) {
      if (const char* name = ordered_kernel_name(static_cast<ReduceOp>(op)))
        hp->shape_.ordered_ctas_per_sm[op] = occupancy(name, kOrderedBlock);
    }
    check(hp->set_reduce_cluster(4), "sizing the reduction grid");
  } catch (...) {
    if (hp->module_ != nullptr) api.cuModuleUnload(hp->module_);
    delete hp;
    throw;
  }
  return hp;
}

Hotpath::~Hotpath() {
  if (module_ != nullptr) {
    if (const DriverApi* api = driver_api()) {
      CurrentContextScope scope(context_);
      if (scope.push_result() == CUDA_SUCCESS) api->cuModuleUnload(module_);
    }
  }
}

CUresult Hotpath::wait_timeouts(std::uint32_t* count, bool reset) {
  const DriverApi& api = require_driver();
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  CUdeviceptr addr = 0;
  std::size_t bytes = 0;
  CUresult r = api.cuModuleGetGlobal(&addr, &bytes, module_, "f4s_wait_timeouts");
  if (r == CUDA_SUCCESS && bytes != sizeof(std::uint32_t)) r = CUDA_ERROR_INVALID_VALUE;
  if (r == CUDA_SUCCESS) r = api.cuCtxSynchronize();
  if (r == CUDA_SUCCESS) r = api.cuMemcpyDtoH(count, addr, sizeof(std::uint32_t));
  if (r == CUDA_SUCCESS && reset) {
    const std::uint32_t zero = 0;
    r = api.cuMemcpyHtoD(addr, &zero, sizeof(zero));
  }
  return cur.finish(r);
}

CUresult Hotpath::check_bounded_wait(std::uint32_t polls) {
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.u32(polls);
  return cur.finish(launch(function("f4s_check_bounded_wait"), nullptr, 1, 32, 0, args));
}

CUfunction Hotpath::function(const std::string& name) const {
  const DriverApi& api = require_driver();
  CUfunction fn = nullptr;
  const CUresult r = api.cuModuleGetFunction(&fn, module_, name.c_str());
  if (r != CUDA_SUCCESS) throw std::invalid_argument("no kernel named " + name + " in the hot-path module");
  return fn;
}

namespace {

const char* reduce_kernel_name(ReduceOp op) {
  switch (op) {
    case ReduceOp::kSumF32: return "f4s_reduce_sum_f32";
    case ReduceOp::kSumI32:
    case ReduceOp::kSumU32: return "f4s_reduce_sum_i32";  // same bits: 32-bit wrap
    case ReduceOp::kArgmaxF32: return "f4s_reduce_argmax_f32";
    case ReduceOp::kSumF16: return "f4s_reduce_sum_f16";
    case ReduceOp::kSumBf16: return "f4s_reduce_sum_bf16";
    case ReduceOp::kSumF64: return "f4s_reduce_sum_f64";
    case ReduceOp::kSumE4m3: return "f4s_reduce_sum_e4m3";
    case ReduceOp::kSumE5m2: return "f4s_reduce_sum_e5m2";
    case ReduceOp::kArgmaxI32: return "f4s_reduce_argmax_i32";
    case ReduceOp::kArgmaxU32: return "f4s_reduce_argmax_u32";
    case ReduceOp::kArgmaxF16:
    case ReduceOp::kArgmaxBf16: return "f4s_reduce_argmax_half";  // same 16-bit order key
    case ReduceOp::kArgmaxF64: return "f4s_reduce_argmax_f64";
  }
  throw std::invalid_argument("unknown reduction op " + std::to_string(static_cast<int>(op)));
}

}  // namespace

int reduce_input_bytes(ReduceOp op) {
  switch (op) {
    case ReduceOp::kSumF32:
    case ReduceOp::kSumI32:
    case ReduceOp::kArgmaxF32:
    case ReduceOp::kSumU32: return 4;
    case ReduceOp::kSumF16:
    case ReduceOp::kSumBf16: return 2;
    case ReduceOp::kSumF64: return 8;
    case ReduceOp::kSumE4m3:
    case ReduceOp::kSumE5m2: return 1;
    case ReduceOp::kArgmaxI32:
    case ReduceOp::kArgmaxU32: return 4;
    case ReduceOp::kArgmaxF16:
    case ReduceOp::kArgmaxBf16: return 2;
    case ReduceOp::kArgmaxF64: return 8;
  }
  throw std::invalid_argument("unknown reduction op " + std::to_string(static_cast<int>(op)));
}

int reduce_output_bytes(ReduceOp op) {
  switch (op) {
    case ReduceOp::kSumI32:
    case ReduceOp::kSumU32: return 4;
    case ReduceOp::kArgmaxF32:
    case ReduceOp::kArgmaxI32:
    case ReduceOp::kArgmaxU32:
    case ReduceOp::kArgmaxF16:
    case ReduceOp::kArgmaxBf16:
    case ReduceOp::kArgmaxF64: return 16;
    case ReduceOp::kSumF32:
    case ReduceOp::kSumF16:
    case ReduceOp::kSumBf16:
    case ReduceOp::kSumF64:
    case ReduceOp::kSumE4m3:
    case ReduceOp::kSumE5m2: return 8;  // f64
  }
  throw std::invalid_argument("unknown reduction op " + std::to_string(static_cast<int>(op)));
}

bool is_argmax(ReduceOp op) {
  return op == ReduceOp::kArgmaxF32 || static_cast<int>(op) >= static_cast<int>(ReduceOp::kArgmaxI32);
}

ReduceOp argmax_op_for_type_code(int code) {
  switch (code) {
    case 2: return ReduceOp::kArgmaxI32;
    case 3: return ReduceOp::kArgmaxU32;
    case 4: return ReduceOp::kArgmaxF16;
    case 5: return ReduceOp::kArgmaxBf16;
    case 6: return ReduceOp::kArgmaxF32;
    case 7: return ReduceOp::kArgmaxF64;
    default:
      throw std::invalid_argument("no max/argmax order for argument type code " + std::to_string(code));
  }
}

ReduceOp sum_op_for_type_code(int code) {
  switch (code) {
    case 2: return ReduceOp::kSumI32;
    case 3: return ReduceOp::kSumU32;
    case 4: return ReduceOp::kSumF16;
    case 5: return ReduceOp::kSumBf16;
    case 6: return ReduceOp::kSumF32;
    case 7: return ReduceOp::kSumF64;
    case 8: return ReduceOp::kSumE4m3;
    case 9: return ReduceOp::kSumE5m2;
    default:
      throw std::invalid_argument("no ReduceSum accumulator for argument type code " + std::to_string(code));
  }
}

CUresult Hotpath::set_reduce_cluster(int cluster) {
  if (cluster < 1 || cluster > 8) throw std::invalid_argument("reduction cluster size must be in [1, 8]");
  const DriverApi& api = require_driver();
  CurrentContextScope scope(context_);
  if (scope.push_result() != CUDA_SUCCESS) return scope.push_result();
  CUlaunchAttribute attr{};
  attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
  attr.value.clusterDim.x = static_cast<unsigned>(cluster);
  attr.value.clusterDim.y = 1;
  attr.value.clusterDim.z = 1;
  CUlaunchConfig config{};
  config.gridDimX = static_cast<unsigned>(cluster * sm_count_);
  config.gridDimY = config.gridDimZ = 1;
  config.blockDimX = kReduceBlock;
  config.blockDimY = config.blockDimZ = 1;
  config.attrs = &attr;
  config.numAttrs = 1;
  int clusters[kReduceOpCount] = {};
  for (int op = 0; op < kReduceOpCount; ++op) {
    const CUresult r =
        api.cuOccupancyMaxActiveClusters(&clusters[op], function(reduce_kernel_name(static_cast<ReduceOp>(op))), &config);
    if (r != CUDA_SUCCESS) return r;
    if (clusters[op] <= 0) return CUDA_ERROR_INVALID_CLUSTER_SIZE;
  }
  shape_.reduce_cluster = cluster;
  for (int op = 0; op < kReduceOpCount; ++op) shape_.reduce_max_clusters[op] = clusters[op];
  return scope.close();
}

namespace {

// 16-byte vectors per lane per step of each fast kernel (its Op::kUnroll in
// reduce.cuh): 8, except 6 for the f64 argmax.
int reduce_step_vectors(ReduceOp op) { return op == ReduceOp::kArgmaxF64 ? 6 : kReduceUnroll; }

// Waves of co-resident clusters in one launch: every fast kernel holds two
// CTAs per SM and is launched in twice kReduceWaves waves (~4544 CTAs;
// measured +0.5-6 % over 8 waves of 4-vector steps at 3-4 CTAs per SM, 2 to
// 16 GiB).  This stays within reduce_workspace_bytes(): at most 4 CTAs per
// SM x kReduceWaves.
constexpr int kReduceLaunchWaves = 2 * kReduceWaves;

}  // namespace

std::uint64_t Hotpath::reduce_workspace_bytes() const {
  // One partial slot per launched cluster; kReduceWaves waves of at most
  // 2048 / kReduceBlock co-resident CTAs per SM bound every cluster size.
  const std::uint64_t ctas = static_cast<std::uint64_t>(sm_count_) * (2048 / kReduceBlock) * kReduceWaves;
  return kReducePartialOffset + kReducePartialBytes * ctas;
}

std::uint64_t Hotpath::block_sum_workspace_bytes(std::int64_t n) {
  const std::int64_t clusters = std::max<std::int64_t>(1, (n + kBlockSumElemsPerCluster - 1) / kBlockSumElemsPerCluster);
  return 256 + 4 * static_cast<std::uint64_t>(clusters);
}

CUresult Hotpath::launch(CUfunction fn, CUstream stream, int grid, int block, int cluster, ArgumentPack& args,
                         bool programmatic) {
  const DriverApi& api = require_driver();
  CudaLaunchRequest request{
      context_, fn, stream,
      LaunchGeometry{grid, 1, 1, block, 1, 1, 0, cluster > 0, cluster > 0 ? cluster : 0,
                     cluster > 0 ? 1 : 0, cluster > 0 ? 1 : 0},
      args.layout()};
  return launch_in_current_context(api, request, programmatic);
}

CUresult Hotpath::reduce_launch(ReduceOp op, CUstream stream, CUdeviceptr in, std::uint64_t n, CUdeviceptr out,
                                CUdeviceptr workspace, std::uint64_t workspace_bytes, std::uint64_t index_base,
                                int accumulate, bool programmatic) {
  const char* name = reduce_kernel_name(op);
  const int elem = reduce_input_bytes(op);
  if (n > 0) require_ptr(in, "input buffer");
  require_ptr(out, "output buffer");
  require_ptr(workspace, "reduction workspace");
  if (in % elem != 0)
    throw std::invalid_argument("input buffer must be " + std::to_string(elem) + "-byte aligned");
  if (reduce_output_bytes(op) >= 8 && out % 8 != 0) throw std::invalid_argument("output must be 8-byte aligned");
  if (out % 4 != 0) throw std::invalid_argument("output must be 4-byte aligned");
  if (workspace % 16 != 0) throw std::invalid_argument("reduction workspace must be 16-byte aligned");
  const int cluster = shape_.reduce_cluster;
  // Enough clusters to give each thread >= one unrolled step of 16-byte
  // vectors, at most kReduceLaunchWaves waves of co-resident clusters
  // (several waves measured faster than one persistent wave: no idle tail).
  const std::uint64_t per_cluster =
      static_cast<std::uint64_t>(cluster) * kReduceBlock * (16 / elem) * reduce_step_vectors(op);
  const std::uint64_t wanted = std::max<std::uint64_t>(1, (n + per_cluster - 1) / per_cluster);
  const int clusters = static_cast<int>(
      std::min<std::uint64_t>(wanted, static_cast<std::uint64_t>(shape_.reduce_max_clusters[static_cast<int>(op)]) *
                                          kReduceLaunchWaves));
  const std::uint64_t need = kReducePartialOffset + kReducePartialBytes * static_cast<std::uint64_t>(clusters);
  if (workspace_bytes < need) {
    throw std::invalid_argument("reduction workspace too small: " + std::to_string(workspace_bytes) +
                                " bytes, need " + std::to_string(need));
  }
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(in).u32(static_cast<std::uint32_t>(n)).u32(static_cast<std::uint32_t>(n >> 32)).ptr(out).ptr(workspace)
      .u32(static_cast<std::uint32_t>(index_base)).u32(static_cast<std::uint32_t>(index_base >> 32))
      .i32(accumulate ? 1 : 0);
  return cur.finish(launch(function(name), stream, clusters * cluster, kReduceBlock, cluster, args, programmatic));
}

namespace {

// Bytes and the reference's CUDA spelling of each launch-ABI type that
// Convert can name (core/src/main/scala/flight4s/core/types/CudaType.scala:60-140).
int type_bytes(int code) {
  switch (code) {
    case 1: case 8: case 9: return 1;
    case 4: case 5: return 2;
    case 2: case 3: case 6: return 4;
    case 7: return 8;
    default: return 0;
  }
}

const char* cuda_type_name(int code) {
  switch (code) {
    case 1: return "bool";
    case 2: return "int";
    case 3: return "unsigned int";
    case 4: return "__half";
    case 5: return "__nv_bfloat16";
    case 6: return "float";
    case 7: return "double";
    case 8: return "__nv_fp8_e4m3";
    case 9: return "__nv_fp8_e5m2";
    default: return nullptr;
  }
}

std::string convert_kernel_name(int from, int to, int rounding, int saturation) {
  if (cuda_type_name(from) == nullptr || cuda_type_name(to) == nullptr)
    throw std::invalid_argument("unknown Convert type code " + std::to_string(cuda_type_name(from) ? to : from));
  if (rounding < 0 || rounding > 3) throw std::invalid_argument("unknown rounding mode " + std::to_string(rounding));
  if (saturation < 0 || saturation > 1)
    throw std::invalid_argument("unknown saturation mode " + std::to_string(saturation));
  static const char* const kRound[] = {"rn", "rz", "ru", "rd"};
  if (from == to) return "f4s_convert_copy_" + std::to_string(type_bytes(from));
  if (from == 6 && to == 4) return std::string("f4s_convert_f32_f16_") + kRound[rounding];
  if (from == 6 && to == 5) return std::string("f4s_convert_f32_bf16_") + kRound[rounding];
  // FP8 conversion rounds to nearest-even whatever the mode (the reference's
  // lowering passes no rounding to __nv_cvt_float_to_fp8)
  if (from == 6 && to == 8) return saturation ? "f4s_convert_f32_e4m3_sat" : "f4s_convert_f32_e4m3_nosat";
  if (from == 6 && to == 9) return saturation ? "f4s_convert_f32_e5m2_sat" : "f4s_convert_f32_e5m2_nosat";
  if (to == 6 && from == 4) return "f4s_convert_f16_f32";
  if (to == 6 && from == 5) return "f4s_convert_bf16_f32";
  if (to == 6 && from == 8) return "f4s_convert_e4m3_f32";
  if (to == 6 && from == 9) return "f4s_convert_e5m2_f32";
  // CudaCodegen.scala:440-449 (UnsupportedConversion, CudaArtifacts.scala:84-91)
  throw std::invalid_argument(std::string("cannot emit a conversion from ") + cuda_type_name(from) + " to " +
                              cuda_type_name(to));
}

}  // namespace

CUresult Hotpath::convert(CUstream stream, int from_type, int to_type, int rounding, int saturation, CUdeviceptr in,
                          CUdeviceptr out, std::uint64_t n) {
  const std::string name = convert_kernel_name(from_type, to_type, rounding, saturation);
  const int in_bytes = type_bytes(from_type), out_bytes = type_bytes(to_type);
  if (n > 0) {
    require_ptr(in, "input buffer");
    require_ptr(out, "output buffer");
  }
  if (in % in_bytes != 0 || out % out_bytes != 0)
    throw std::invalid_argument("Convert buffers must be aligned to their element sizes");
  constexpr std::uint64_t kElemsPerBlock = 256 * 16;
  const std::uint64_t blocks = std::max<std::uint64_t>(1, (n + kElemsPerBlock - 1) / kElemsPerBlock);
  const int grid = static_cast<int>(std::min<std::uint64_t>(blocks, 1u << 20));
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(in).ptr(out).u32(static_cast<std::uint32_t>(n)).u32(static_cast<std::uint32_t>(n >> 32));
  return cur.finish(launch(function(name), stream, grid, 256, 0, args));
}

bool Hotpath::has_ordered_kernel(ReduceOp op) { return ordered_kernel_name(op) != nullptr; }

std::uint64_t Hotpath::ordered_groups(ReduceOp op, CUdeviceptr in, std::uint64_t n) {
  if (!has_ordered_kernel(op)) throw std::invalid_argument("no order-fixed kernel for this reduction");
  const std::uint64_t elem = static_cast<std::uint64_t>(reduce_input_bytes(op));
  const std::uint64_t head = std::min<std::uint64_t>(((16 - in % 16) % 16) / elem, n);
  const std::uint64_t body_bytes = (n - head) * elem;
  return (body_bytes + kOrderedGroupBytes - 1) / kOrderedGroupBytes;
}

std::uint64_t Hotpath::ordered_workspace_bytes(ReduceOp op, std::uint64_t n) {
  return kOrderedGroupOffset + 8 * ordered_groups(op, 0, n);
}

CUresult Hotpath::reduce_ordered(ReduceOp op, CUstream stream, CUdeviceptr in, std::uint64_t n, CUdeviceptr out,
                                 CUdeviceptr workspace, std::uint64_t workspace_bytes, int accumulate) {
  const char* name = ordered_kernel_name(op);
  if (name == nullptr) throw std::invalid_argument("no order-fixed kernel for this reduction");
  const int elem = reduce_input_bytes(op);
  if (n > 0) require_ptr(in, "input buffer");
  require_ptr(out, "output buffer");
  require_ptr(workspace, "reduction workspace");
  if (in % elem != 0)
    throw std::invalid_argument("input buffer must be " + std::to_string(elem) + "-byte aligned");
  if (out % 8 != 0) throw std::invalid_argument("output must be 8-byte aligned");
  if (workspace % 16 != 0) throw std::invalid_argument("reduction workspace must be 16-byte aligned");
  const std::uint64_t groups = ordered_groups(op, in, n);
  const std::uint64_t need = kOrderedGroupOffset + 8 * groups;
  if (workspace_bytes < need) {
    throw std::invalid_argument("reduction workspace too small: " + std::to_string(workspace_bytes) +
                                " bytes, need " + std::to_string(need));
  }
  const std::uint64_t resident =
      static_cast<std::uint64_t>(sm_count_) * static_cast<std::uint64_t>(shape_.ordered_ctas_per_sm[static_cast<int>(op)]);
  const int grid = static_cast<int>(std::max<std::uint64_t>(1, std::min<std::uint64_t>(groups, resident)));
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(in).u32(static_cast<std::uint32_t>(n)).u32(static_cast<std::uint32_t>(n >> 32)).ptr(out).ptr(workspace)
      .ptr(workspace + kOrderedGroupOffset).i32(accumulate ? 1 : 0);
  return cur.finish(launch(function(name), stream, grid, kOrderedBlock, 0, args));
}

CUresult Hotpath::reduce_ordered_final(CUstream stream, CUdeviceptr groups, std::uint64_t count, CUdeviceptr out,
                                       int accumulate) {
  if (count > 0) require_ptr(groups, "group partials");
  require_ptr(out, "output buffer");
  if (groups % 8 != 0 || out % 8 != 0) throw std::invalid_argument("group partials and output must be 8-byte aligned");
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(groups).u32(static_cast<std::uint32_t>(count)).u32(static_cast<std::uint32_t>(count >> 32)).ptr(out)
      .i32(accumulate ? 1 : 0);
  return cur.finish(launch(function("f4s_reduce_ordered_final"), stream, 1, kOrderedBlock, 0, args));
}

CUresult Hotpath::block_sum_f32(CUstream stream, CUdeviceptr in, std::int32_t n, CUdeviceptr partials,
                                CUdeviceptr out, CUdeviceptr workspace, std::uint64_t workspace_bytes) {
  require_nonnegative(n, "element count");
  if (n > 0) {
    require_ptr(in, "input buffer");
    require_ptr(partials, "partials buffer");
  }
  require_ptr(out, "output buffer");
  require_ptr(workspace, "block-sum workspace");
  if (in % 4 != 0 || partials % 4 != 0 || out % 4 != 0 || workspace % 16 != 0)
    throw std::invalid_argument("block-sum buffers must be 4-byte aligned (workspace 16-byte)");
  if (workspace_bytes < block_sum_workspace_bytes(n))
    throw std::invalid_argument("block-sum workspace too small: " + std::to_string(workspace_bytes) +
                                " bytes, need " + std::to_string(block_sum_workspace_bytes(n)));
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  const std::int64_t tiles = (static_cast<std::int64_t>(n) + 255) / 256;
  if (tiles <= kBlockSumSmallMaxTiles) {
    // small arrays: the tiles kernel, then the one-CTA upper pass as its
    // programmatic dependent (same tree, same bits; the workspace is unused)
    const int ctas = static_cast<int>(std::max<std::int64_t>(1, (tiles + kBlockSumWarps - 1) / kBlockSumWarps));
    ArgumentPack tiles_args;
    tiles_args.ptr(in).i32(n).ptr(partials);
    const CUresult r = launch(function("f4s_block_sum_tiles_f32"), stream, ctas, kBlockSumThreads, 0, tiles_args);
    if (r != CUDA_SUCCESS) return cur.finish(r);
    ArgumentPack upper_args;
    upper_args.ptr(partials).i32(n).ptr(out);
    return cur.finish(launch(function("f4s_block_sum_upper_f32"), stream, 1, kBlockSumUpperThreads, 0, upper_args,
                             true));
  }
  ArgumentPack args;
  args.ptr(in).i32(n).ptr(partials).ptr(out).ptr(workspace);
  const int clusters = static_cast<int>(std::max<std::int64_t>(1, (static_cast<std::int64_t>(n) + kBlockSumElemsPerCluster - 1) / kBlockSumElemsPerCluster));
  return cur.finish(launch(function("f4s_block_reduce_sum_f32"), stream, clusters * kBlockSumCluster,
                           kBlockSumThreads, kBlockSumCluster, args));
}

CUresult Hotpath::vector_add(bool bf16, CUstream stream, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c,
                             std::int32_t n) {
  return vector_add_typed(bf16 ? 5 : 6, stream, a, b, c, n);
}

CUresult Hotpath::vector_add_typed(int type_code, CUstream stream, CUdeviceptr a, CUdeviceptr b, CUdeviceptr c,
                                   std::int32_t n) {
  // AdditiveType (core/src/main/scala/flight4s/core/types/CudaType.scala:154-160)
  const char* name = nullptr;
  std::uint64_t elem = 0;
  switch (type_code) {
    case 2: case 3: name = "f4s_vector_add_i32"; elem = 4; break;
    case 4: name = "f4s_vector_add_f16"; elem = 2; break;
    case 5: name = "f4s_vector_add_bf16"; elem = 2; break;
    case 6: name = "f4s_vector_add_f32"; elem = 4; break;
    case 7: name = "f4s_vector_add_f64"; elem = 8; break;
    default:
      throw std::invalid_argument("no addition for argument type code " + std::to_string(type_code));
  }
  require_nonnegative(n, "element count");
  if (n == 0) return CUDA_SUCCESS;
  require_ptr(a, "left buffer");
  require_ptr(b, "right buffer");
  require_ptr(c, "output buffer");
  if (a % elem != 0 || b % elem != 0 || c % elem != 0)
    throw std::invalid_argument("vectorAdd buffers must be aligned to their element size");
  // one thread per 32-byte vector (the kernel loops for any other grid)
  const std::int64_t per_cta = static_cast<std::int64_t>(kAddBlock) * static_cast<std::int64_t>(32 / elem);
  const int grid = static_cast<int>((n + per_cta - 1) / per_cta);
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(a).ptr(b).ptr(c).i32(n);
  return cur.finish(launch(function(name), stream, std::max(grid, 1), kAddBlock, 0, args));
}

namespace {

// Register-resident variant for a row width, or "" for the looped kernel.
int row_vectors_per_thread(std::int32_t cols, std::uint64_t in, std::uint64_t out) {
  if (cols % 8 != 0 || (in % 16) != 0 || (out % 16) != 0) return 0;
  const int nvec = cols / 8;
  for (int vpt : {1, 2, 4, 8}) {
    if (nvec <= vpt * kRowBlock) return vpt;
  }
  return 0;
}

}  // namespace

CUresult Hotpath::softmax_rows(CUstream stream, CUdeviceptr in, CUdeviceptr out, std::int32_t rows,
                               std::int32_t cols) {
  require_nonnegative(rows, "row count");
  require_nonnegative(cols, "column count");
  if (rows == 0 || cols == 0) return CUDA_SUCCESS;
  require_ptr(in, "input buffer");
  require_ptr(out, "output buffer");
  if (in % 2 != 0 || out % 2 != 0) throw std::invalid_argument("bf16 buffers must be 2-byte aligned");
  const int vpt = row_vectors_per_thread(cols, in, out);
  const std::string name = vpt ? "f4s_softmax_rows_bf16_v" + std::to_string(vpt) : "f4s_softmax_rows_bf16_any";
  const CUfunction fn = function(name);
  // two rows per CTA for rows of up to 8192 elements (VPT <= 4), one row per
  // CTA for wider ones (no persistent tail either way)
  const int grid = (vpt >= 1 && vpt <= 4) ? (rows + 1) / 2 : rows;
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(in).ptr(out).i32(rows).i32(cols);
  return cur.finish(launch(fn, stream, grid, kRowBlock, 0, args));
}

CUresult Hotpath::rmsnorm_rows(CUstream stream, CUdeviceptr in, CUdeviceptr weight, CUdeviceptr out,
                               std::int32_t rows, std::int32_t cols, float eps) {
  require_nonnegative(rows, "row count");
  require_nonnegative(cols, "column count");
  if (rows == 0 || cols == 0) return CUDA_SUCCESS;
  require_ptr(in, "input buffer");
  require_ptr(weight, "weight buffer");
  require_ptr(out, "output buffer");
  if (in % 2 != 0 || out % 2 != 0 || weight % 2 != 0)
    throw std::invalid_argument("bf16 buffers must be 2-byte aligned");
  if (!(eps >= 0.0f)) throw std::invalid_argument("eps must be a non-negative number");
  int vpt = row_vectors_per_thread(cols, in, out);
  if (weight % 16 != 0) vpt = 0;
  if (vpt == 4) {
    // 2049..8192-wide rows: TMA-staged kernel, 2 persistent CTAs per SM
    // (the measured optimum; rows are 16-byte aligned because cols % 8 == 0).
    Current cur(context_);
    if (cur.result() != CUDA_SUCCESS) return cur.result();
    ArgumentPack args;
    args.ptr(in).ptr(weight).ptr(out).i32(rows).i32(cols).f32(eps);
    const int grid = static_cast<int>(std::min<std::int64_t>(rows, static_cast<std::int64_t>(sm_count_) * 2));
    return cur.finish(launch(function("f4s_rmsnorm_rows_bf16_tma"), stream, grid, kRowBlock, 0, args));
  }
  const std::string name = vpt ? "f4s_rmsnorm_rows_bf16_v" + std::to_string(vpt) : "f4s_rmsnorm_rows_bf16_any";
  const CUfunction fn = function(name);
  // Persistent CTAs (8 per SM, measured flat between 2 and 8 for 8192-wide
  // rows), each keeping its weight slice in registers across its rows.
  const int grid = static_cast<int>(std::min<std::int64_t>(rows, static_cast<std::int64_t>(sm_count_) * 8));
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(in).ptr(weight).ptr(out).i32(rows).i32(cols).f32(eps);
  return cur.finish(launch(fn, stream, grid, kRowBlock, 0, args));
}

CUresult Hotpath::fp8_quantize(CUstream stream, CUdeviceptr x, CUdeviceptr codes, CUdeviceptr scales,
                               std::int32_t rows, std::int32_t cols) {
  require_nonnegative(rows, "row count");
  require_nonnegative(cols, "column count");
  if (rows == 0 || cols == 0) return CUDA_SUCCESS;
  require_ptr(x, "input buffer");
  require_ptr(codes, "code buffer");
  require_ptr(scales, "scale buffer");
  if (x % 2 != 0 || scales % 4 != 0) throw std::invalid_argument("fp8 quantize buffers are misaligned");
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  const std::int64_t total = static_cast<std::int64_t>(rows) * cols;
  if (cols % kFp8Block == 0 && x % 32 == 0 && codes % 16 == 0 && total / kFp8Block <= INT32_MAX) {
    // one warp per kQuantUnroll 4-block steps: the loop runs about once
    const std::int64_t blocks = total / kFp8Block;
    const std::int64_t warps = (blocks + 4 * kQuantUnroll - 1) / (4 * kQuantUnroll);
    const std::int64_t ctas = (warps + kFp8Threads / 32 - 1) / (kFp8Threads / 32);
    ArgumentPack args;
    args.ptr(x).ptr(codes).ptr(scales).i32(static_cast<std::int32_t>(blocks));
    return cur.finish(launch(function("f4s_fp8_quant_flat"), stream, static_cast<int>(std::max<std::int64_t>(ctas, 1)),
                             kFp8Threads, 0, args));
  }
  ArgumentPack args;
  args.ptr(x).ptr(codes).ptr(scales).i32(rows).i32(cols);
  return cur.finish(launch(function("f4s_fp8_quant_rows"), stream, shape_.fp8_grid, kFp8Threads, 0, args));
}

CUresult Hotpath::fp8_dequantize(CUstream stream, CUdeviceptr codes, CUdeviceptr scales, CUdeviceptr y,
                                 std::int32_t rows, std::int32_t cols) {
  require_nonnegative(rows, "row count");
  require_nonnegative(cols, "column count");
  if (rows == 0 || cols == 0) return CUDA_SUCCESS;
  require_ptr(codes, "code buffer");
  require_ptr(scales, "scale buffer");
  require_ptr(y, "output buffer");
  if (y % 2 != 0 || scales % 4 != 0) throw std::invalid_argument("fp8 dequantize buffers are misaligned");
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  const std::int64_t total = static_cast<std::int64_t>(rows) * cols;
  if (cols % kFp8Block == 0 && codes % 16 == 0 && y % 32 == 0 && total / kFp8Block <= INT32_MAX) {
    const std::int64_t blocks = total / kFp8Block;
    const std::int64_t warps = (blocks + 4 * kDequantUnroll - 1) / (4 * kDequantUnroll);
    const std::int64_t ctas = (warps + kFp8Threads / 32 - 1) / (kFp8Threads / 32);
    ArgumentPack args;
    args.ptr(codes).ptr(scales).ptr(y).i32(static_cast<std::int32_t>(blocks));
    return cur.finish(launch(function("f4s_fp8_dequant_flat"), stream,
                             static_cast<int>(std::max<std::int64_t>(ctas, 1)), kFp8Threads, 0, args));
  }
  ArgumentPack args;
  args.ptr(codes).ptr(scales).ptr(y).i32(rows).i32(cols);
  return cur.finish(launch(function("f4s_fp8_dequant_rows"), stream, shape_.fp8_grid, kFp8Threads, 0, args));
}

CUresult Hotpath::fill_synthetic(CUstream stream, CUdeviceptr out, std::uint64_t n, std::uint64_t offset,
                                 std::uint64_t seed, std::uint32_t stream_id, int kind, float p0, float p1,
                                 float p2, float p3, std::int32_t ilo, std::int32_t ihi) {
  if (n == 0) return CUDA_SUCCESS;
  require_ptr(out, "output buffer");
  if (kind < 0 || kind > 5) throw std::invalid_argument("unknown synthetic distribution kind");
  if (kind == 4 && (ilo > ihi)) throw std::invalid_argument("integer range must satisfy lo <= hi");
  if (kind == 4 && static_cast<std::int64_t>(ihi) - ilo >= 0xFFFFFFFFLL)
    throw std::invalid_argument("integer range too wide");
  if (kind == 5 && !(p2 >= 0.0f && p2 < 1.0f)) throw std::invalid_argument("outlier probability must be in [0, 1)");
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  ArgumentPack args;
  args.ptr(out).u32(static_cast<std::uint32_t>(n)).u32(static_cast<std::uint32_t>(n >> 32))
      .u32(static_cast<std::uint32_t>(offset)).u32(static_cast<std::uint32_t>(offset >> 32))
      .u32(static_cast<std::uint32_t>(seed)).u32(static_cast<std::uint32_t>(seed >> 32)).u32(stream_id)
      .i32(kind).f32(p0).f32(p1).f32(p2).f32(p3).i32(ilo).i32(ihi);
  return cur.finish(launch(function("f4s_fill_synthetic"), stream, shape_.fill_grid, 256, 0, args));
}

CUresult Hotpath::reduce_host(ReduceOp op, const void* host_in, std::uint64_t n, std::uint64_t index_base,
                              void* host_out, CUdeviceptr staging, std::uint64_t staging_bytes,
                              CUdeviceptr workspace, std::uint64_t workspace_bytes, CUstream copy_stream,
                              CUstream compute_stream) {
  void* outs[1] = {host_out};
  return reduce_host_ops(&op, 1, host_in, n, index_base, outs, staging, staging_bytes, workspace, workspace_bytes,
                         copy_stream, compute_stream);
}

CUresult Hotpath::reduce_host_sum_argmax(const void* host_in, std::uint64_t n, std::uint64_t index_base,
                                         void* host_sum_out, void* host_argmax_out, CUdeviceptr staging,
                                         std::uint64_t staging_bytes, CUdeviceptr workspace,
                                         std::uint64_t workspace_bytes, CUstream copy_stream,
                                         CUstream compute_stream) {
  const ReduceOp ops[2] = {ReduceOp::kSumF32, ReduceOp::kArgmaxF32};
  void* outs[2] = {host_sum_out, host_argmax_out};
  return reduce_host_ops(ops, 2, host_in, n, index_base, outs, staging, staging_bytes, workspace, workspace_bytes,
                         copy_stream, compute_stream);
}

template <class OnChunk, class OnDone>
CUresult Hotpath::stream_chunks(const void* host_in, std::uint64_t n, int elem, std::uint64_t chunk,
                                const CUdeviceptr buffers[2], CUstream copy_stream, CUstream compute_stream,
                                OnChunk&& on_chunk, OnDone&& on_done) {
  const DriverApi& api = require_driver();
  Current cur(context_);
  if (cur.result() != CUDA_SUCCESS) return cur.result();
  CUevent copied[2] = {nullptr, nullptr};
  CUevent consumed[2] = {nullptr, nullptr};
  CUresult r = CUDA_SUCCESS;
  for (int i = 0; i < 2 && r == CUDA_SUCCESS; ++i) {
    r = api.cuEventCreate(&copied[i], CU_EVENT_DISABLE_TIMING);
    if (r == CUDA_SUCCESS) r = api.cuEventCreate(&consumed[i], CU_EVENT_DISABLE_TIMING);
  }
  const std::uint64_t chunks = n == 0 ? 1 : (n + chunk - 1) / chunk;
  for (std::uint64_t k = 0; k < chunks && r == CUDA_SUCCESS; ++k) {
    const int b = static_cast<int>(k % 2);
    const std::uint64_t first = k * chunk;
    const std::uint64_t count = n == 0 ? 0 : std::min(chunk, n - first);
    if (k >= 2) r = api.cuStreamWaitEvent(copy_stream, consumed[b], 0);
    if (r == CUDA_SUCCESS && count > 0)
      r = api.cuMemcpyHtoDAsync(buffers[b], static_cast<const unsigned char*>(host_in) + first * elem, count * elem,
                                copy_stream);
    if (r == CUDA_SUCCESS) r = api.cuEventRecord(copied[b], copy_stream);
    if (r == CUDA_SUCCESS) r = api.cuStreamWaitEvent(compute_stream, copied[b], 0);
    // the ops push the same context again: harmless
    if (r == CUDA_SUCCESS) r = on_chunk(k, buffers[b], first, count);
    if (r == CUDA_SUCCESS) r = api.cuEventRecord(consumed[b], compute_stream);
  }
  if (r == CUDA_SUCCESS) r = on_done();
  if (r == CUDA_SUCCESS) r = api.cuStreamSynchronize(compute_stream);
  if (r == CUDA_SUCCESS) r = api.cuStreamSynchronize(copy_stream);
  for (int i = 0; i < 2; ++i) {
    if (copied[i]) api.cuEventDestroy(copied[i]);
    if (consumed[i]) api.cuEventDestroy(consumed[i]);
  }
  return cur.finish(r);
}

namespace {

// Common checks of the host-buffer entry points; returns the byte size of
// each staging half (a multiple of 256): staging = [256 B of device-side
// results (32 B per op) | half 0 | half 1].
std::uint64_t staging_half(const void* host_in, std::uint64_t n, CUdeviceptr staging, std::uint64_t staging_bytes,
                           CUstream copy_stream, CUstream compute_stream) {
  if (n > 0 && host_in == nullptr) throw std::invalid_argument("host input must not be null");
  require_ptr(staging, "staging buffer");
  if (staging % 256 != 0) throw std::invalid_argument("staging buffer must be 256-byte aligned");
  if (copy_stream == nullptr || compute_stream == nullptr || copy_stream == compute_stream)
    throw std::invalid_argument("host-buffer reductions need two distinct non-null streams");
  const std::uint64_t half = ((staging_bytes > 256 ? staging_bytes - 256 : 0) / 2) / 256 * 256;
  if (half < 256) throw std::invalid_argument("staging buffer too small (need >= 768 bytes)");
  return half;
}

}  // namespace

CUresult Hotpath::reduce_host_ops(const ReduceOp* ops, int nops, const void* host_in, std::uint64_t n,
                                  std::uint64_t index_base, void* const* host_outs, CUdeviceptr staging,
                                  std::uint64_t staging_bytes, CUdeviceptr workspace, std::uint64_t workspace_bytes,
                                  CUstream copy_stream, CUstream compute_stream) {
  for (int i = 0; i < nops; ++i)
    if (host_outs[i] == nullptr) throw std::invalid_argument("host output must not be null");
  const std::uint64_t half = staging_half(host_in, n, staging, staging_bytes, copy_stream, compute_stream);
  const int elem = reduce_input_bytes(ops[0]);
  for (int i = 1; i < nops; ++i)
    if (reduce_input_bytes(ops[i]) != elem) throw std::invalid_argument("fused host reductions need one input type");
  const CUdeviceptr buffers[2] = {staging + 256, staging + 256 + half};
  auto result_slot = [&](int i) { return staging + 32 * static_cast<CUdeviceptr>(i); };
  const DriverApi& api = require_driver();
  return stream_chunks(
      host_in, n, elem, half / static_cast<std::uint64_t>(elem), buffers, copy_stream, compute_stream,
      [&](std::uint64_t k, CUdeviceptr buf, std::uint64_t first, std::uint64_t count) {
        // every op reduces the same staged chunk (one transfer, nops kernels)
        CUresult r = CUDA_SUCCESS;
        for (int i = 0; i < nops && r == CUDA_SUCCESS; ++i)
          r = reduce_launch(ops[i], compute_stream, buf, count, result_slot(i), workspace, workspace_bytes,
                            index_base + first, k > 0 ? 1 : 0, false);
        return r;
      },
      [&] {
        CUresult r = CUDA_SUCCESS;
        for (int i = 0; i < nops && r == CUDA_SUCCESS; ++i)
          r = api.cuMemcpyDtoHAsync(host_outs[i], result_slot(i), reduce_output_bytes(ops[i]), compute_stream);
        return r;
      });
}

CUresult Hotpath::reduce_host_ordered(ReduceOp op, const void* host_in, std::uint64_t n, void* host_out,
                                      CUdeviceptr staging, std::uint64_t staging_bytes, CUdeviceptr workspace,
                                      std::uint64_t workspace_bytes, CUstream copy_stream, CUstream compute_stream) {
  const char* name = ordered_kernel_name(op);
  if (name == nullptr) throw std::invalid_argument("no order-fixed kernel for this reduction");
  if (host_out == nullptr) throw std::invalid_argument("host output must not be null");
  const std::uint64_t half = staging_half(host_in, n, staging, staging_bytes, copy_stream, compute_stream);
  // chunks of whole groups: every chunk starts on a group boundary of the
  // array, so its group partials are the array's own
  const std::uint64_t chunk_bytes = half / kOrderedGroupBytes * kOrderedGroupBytes;
  if (chunk_bytes == 0) {
    throw std::invalid_argument("staging buffer too small for an order-fixed sum: need >= " +
                                std::to_string(256 + 2 * kOrderedGroupBytes) + " bytes");
  }
  require_ptr(workspace, "reduction workspace");
  if (workspace % 16 != 0) throw std::invalid_argument("reduction workspace must be 16-byte aligned");
  const std::uint64_t need = ordered_workspace_bytes(op, n);
  if (workspace_bytes < need) {
    throw std::invalid_argument("reduction workspace too small: " + std::to_string(workspace_bytes) +
                                " bytes, need " + std::to_string(need));
  }
  const std::uint64_t elem = static_cast<std::uint64_t>(reduce_input_bytes(op));
  const std::uint64_t chunk = chunk_bytes / elem;
  const std::uint64_t groups_per_chunk = chunk_bytes / kOrderedGroupBytes;
  const CUdeviceptr buffers[2] = {staging + 256, staging + 256 + half};
  const CUfunction fn = function(name);
  const std::uint64_t resident =
      static_cast<std::uint64_t>(sm_count_) * static_cast<std::uint64_t>(shape_.ordered_ctas_per_sm[static_cast<int>(op)]);
  const DriverApi& api = require_driver();
  return stream_chunks(
      host_in, n, static_cast<int>(elem), chunk, buffers, copy_stream, compute_stream,
      [&](std::uint64_t k, CUdeviceptr buf, std::uint64_t, std::uint64_t count) {
        if (count == 0) return CUDA_SUCCESS;
        const std::uint64_t groups = (count * elem + kOrderedGroupBytes - 1) / kOrderedGroupBytes;
        const int grid = static_cast<int>(std::max<std::uint64_t>(1, std::min<std::uint64_t>(groups, resident)));
        // the chunk total lands in the result slot and is overwritten by F
        ArgumentPack args;
        args.ptr(buf).u32(static_cast<std::uint32_t>(count)).u32(static_cast<std::uint32_t>(count >> 32))
            .ptr(staging).ptr(workspace).ptr(workspace + kOrderedGroupOffset + 8 * k * groups_per_chunk).i32(0);
        return launch(fn, compute_stream, grid, kOrderedBlock, 0, args);
      },
      [&] {
        CUresult r = reduce_ordered_final(compute_stream, workspace + kOrderedGroupOffset, ordered_groups(op, 0, n),
                                          staging, 0);
        if (r == CUDA_SUCCESS) r = api.cuMemcpyDtoHAsync(host_out, staging, 8, compute_stream);
        return r;
      });
}

}  // namespace flight4s::cuda
