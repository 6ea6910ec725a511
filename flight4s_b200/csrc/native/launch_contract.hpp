// Launch geometry and descriptor-coded argument layouts.
//
// Same data model and validation rules as the reference's launch contract
// (native/include/flight4s/cuda/launch_contract.hpp:11-44,
// native/src/launch_contract.cpp:14-209), so requests built by its Scala
// side (`NativeLaunchRequest`, `NativeArgumentStorage`) are accepted or
// rejected identically, with the same messages.
#pragma once

#include <cstddef>
#include <cstdint>
#include <optional>
#include <string>
#include <vector>

namespace flight4s::cuda {

struct LaunchGeometry {
  std::int32_t grid_x;
  std::int32_t grid_y;
  std::int32_t grid_z;
  std::int32_t block_x;
  std::int32_t block_y;
  std::int32_t block_z;
  std::int32_t dynamic_shared_memory_bytes;
  bool uses_cluster;
  std::int32_t cluster_x;
  std::int32_t cluster_y;
  std::int32_t cluster_z;
};

struct ArgumentLayout {
  void* storage;
  std::int64_t storage_size_bytes;
  const std::int32_t* offsets;
  std::size_t offset_count;
  const std::int8_t* descriptor_codes;
  std::size_t descriptor_count;
};

// Stable ABI descriptor codes (core/src/main/scala/flight4s/core/abi/CudaAbi.scala:12-21).
enum DescriptorCode : std::int8_t {
  kBool8 = 1,
  kSignedInt32 = 2,
  kUnsignedInt32 = 3,
  kFloat16 = 4,
  kBFloat16 = 5,
  kFloat32 = 6,
  kFloat64 = 7,
  kFloat8E4M3 = 8,
  kFloat8E5M2 = 9,
  kDevicePointer64 = 10,
  // Addition (not one of the reference's codes): a signed 64-bit value, so
  // element counts and offsets above 2^31 - 1 pass as one argument.
  kSignedInt64 = 11,
};

struct DescriptorLayout {
  std::size_t size_bytes;
  std::size_t alignment_bytes;
};

std::optional<DescriptorLayout> descriptor_layout(std::int8_t code);

std::optional<std::string> validate_launch_geometry(const LaunchGeometry& geometry);

std::optional<std::string> validate_argument_layout(const ArgumentLayout& layout);

std::vector<void*> build_argument_pointers(const ArgumentLayout& layout);

// Packs typed kernel arguments the way the Scala side's
// NativeArgumentStorage does: each argument at the next offset aligned to
// its own alignment, storage size = end of the last argument.
class ArgumentPack {
 public:
  ArgumentPack& ptr(std::uint64_t device_address) { return put(kDevicePointer64, &device_address); }
  ArgumentPack& i32(std::int32_t v) { return put(kSignedInt32, &v); }
  ArgumentPack& i64(std::int64_t v) { return put(kSignedInt64, &v); }
  ArgumentPack& u32(std::uint32_t v) { return put(kUnsignedInt32, &v); }
  ArgumentPack& f32(float v) { return put(kFloat32, &v); }
  ArgumentPack& f64(double v) { return put(kFloat64, &v); }
  ArgumentLayout layout();

 private:
  ArgumentPack& put(DescriptorCode code, const void* value);
  alignas(16) unsigned char storage_[256] = {};
  std::int64_t size_ = 0;
  std::int32_t offsets_[32] = {};
  std::int8_t codes_[32] = {};
  std::size_t count_ = 0;
};

}  // namespace flight4s::cuda
