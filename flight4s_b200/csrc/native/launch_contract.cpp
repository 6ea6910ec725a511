#include "launch_contract.hpp"

#include <cstring>
#include <sstream>
#include <stdexcept>

namespace flight4s::cuda {

std::optional<DescriptorLayout> descriptor_layout(std::int8_t code) {
  switch (static_cast<std::uint8_t>(code)) {
    case kBool8:
    case kFloat8E4M3:
    case kFloat8E5M2:
      return DescriptorLayout{1, 1};
    case kFloat16:
    case kBFloat16:
      return DescriptorLayout{2, 2};
    case kSignedInt32:
    case kUnsignedInt32:
    case kFloat32:
      return DescriptorLayout{4, 4};
    case kFloat64:
    case kDevicePointer64:
    case kSignedInt64:
      return DescriptorLayout{8, 8};
    default:
      return std::nullopt;
  }
}

namespace {

std::optional<std::string> positive(const char* what, std::int32_t value) {
  if (value > 0) return std::nullopt;
  std::ostringstream m;
  m << what << " must be positive: " << value;
  return m.str();
}

}  // namespace

std::optional<std::string> validate_launch_geometry(const LaunchGeometry& g) {
  const std::pair<const char*, std::int32_t> dims[] = {
      {"grid x dimension", g.grid_x},   {"grid y dimension", g.grid_y},
      {"grid z dimension", g.grid_z},   {"block x dimension", g.block_x},
      {"block y dimension", g.block_y}, {"block z dimension", g.block_z},
  };
  for (const auto& [what, value] : dims) {
    if (auto e = positive(what, value)) return e;
  }
  if (g.dynamic_shared_memory_bytes < 0) {
    std::ostringstream m;
    m << "dynamic shared memory must not be negative: " << g.dynamic_shared_memory_bytes;
    return m.str();
  }
  if (!g.uses_cluster) {
    if (g.cluster_x != 0 || g.cluster_y != 0 || g.cluster_z != 0)
      return std::string("cluster dimensions must be zero when clusters are disabled");
    return std::nullopt;
  }
  const struct {
    const char* axis;
    std::int32_t grid;
    std::int32_t cluster;
  } axes[] = {{"x", g.grid_x, g.cluster_x}, {"y", g.grid_y, g.cluster_y}, {"z", g.grid_z, g.cluster_z}};
  for (const auto& a : axes) {
    const std::string what = std::string("cluster ") + a.axis + " dimension";
    if (auto e = positive(what.c_str(), a.cluster)) return e;
    if (a.grid % a.cluster != 0) {
      std::ostringstream m;
      m << "grid " << a.axis << " dimension " << a.grid << " must be divisible by cluster " << a.axis
        << " dimension " << a.cluster;
      return m.str();
    }
  }
  return std::nullopt;
}

std::optional<std::string> validate_argument_layout(const ArgumentLayout& l) {
  if (l.storage_size_bytes < 0) return std::string("argument storage must be a direct buffer");
  if (l.storage_size_bytes > 0 && l.storage == nullptr)
    return std::string("argument storage address must not be null");
  if (l.offset_count != l.descriptor_count) {
    std::ostringstream m;
    m << "argument metadata count mismatch: " << l.offset_count << " offsets and "
      << l.descriptor_count << " descriptors";
    return m.str();
  }
  if (l.offset_count > 0 && (l.offsets == nullptr || l.descriptor_codes == nullptr))
    return std::string("argument metadata arrays must not be null");

  std::vector<DescriptorLayout> layouts(l.descriptor_count);
  std::size_t widest = 1;
  for (std::size_t i = 0; i < l.descriptor_count; ++i) {
    const auto d = descriptor_layout(l.descriptor_codes[i]);
    if (!d) {
      std::ostringstream m;
      m << "unknown descriptor code at argument " << i << ": "
        << static_cast<int>(static_cast<std::uint8_t>(l.descriptor_codes[i]));
      return m.str();
    }
    layouts[i] = *d;
    if (d->alignment_bytes > widest) widest = d->alignment_bytes;
  }
  if (l.storage_size_bytes > 0 && reinterpret_cast<std::uintptr_t>(l.storage) % widest != 0) {
    std::ostringstream m;
    m << "argument storage base is not aligned to " << widest << " bytes";
    return m.str();
  }
  std::int64_t end = 0;
  for (std::size_t i = 0; i < l.offset_count; ++i) {
    const std::int64_t off = l.offsets[i];
    const auto align = static_cast<std::int64_t>(layouts[i].alignment_bytes);
    std::ostringstream m;
    if (off < 0) {
      m << "argument " << i << " has negative offset " << off;
      return m.str();
    }
    if (off % align != 0) {
      m << "argument " << i << " offset " << off << " is not aligned to " << align << " bytes";
      return m.str();
    }
    if (off < end) {
      m << "argument " << i << " overlaps the previous argument";
      return m.str();
    }
    const std::int64_t arg_end = off + static_cast<std::int64_t>(layouts[i].size_bytes);
    if (arg_end > l.storage_size_bytes) {
      m << "argument " << i << " ends at " << arg_end << " beyond storage size " << l.storage_size_bytes;
      return m.str();
    }
    end = arg_end;
  }
  if (end != l.storage_size_bytes) {
    std::ostringstream m;
    m << "argument layout ends at " << end << " but storage size is " << l.storage_size_bytes;
    return m.str();
  }
  return std::nullopt;
}

std::vector<void*> build_argument_pointers(const ArgumentLayout& l) {
  std::vector<void*> out(l.offset_count);
  auto* base = static_cast<unsigned char*>(l.storage);
  for (std::size_t i = 0; i < l.offset_count; ++i) out[i] = base + l.offsets[i];
  return out;
}

ArgumentPack& ArgumentPack::put(DescriptorCode code, const void* value) {
  const auto d = *descriptor_layout(code);
  const auto align = static_cast<std::int64_t>(d.alignment_bytes);
  const std::int64_t off = (size_ + align - 1) / align * align;
  if (count_ >= 32 || off + static_cast<std::int64_t>(d.size_bytes) > static_cast<std::int64_t>(sizeof storage_))
    throw std::length_error("kernel argument pack is full");
  std::memcpy(storage_ + off, value, d.size_bytes);
  offsets_[count_] = static_cast<std::int32_t>(off);
  codes_[count_] = code;
  ++count_;
  size_ = off + static_cast<std::int64_t>(d.size_bytes);
  return *this;
}

ArgumentLayout ArgumentPack::layout() {
  return ArgumentLayout{storage_, size_, offsets_, count_, codes_, count_};
}

}  // namespace flight4s::cuda
