// Generates the conversion golden vectors and runs the exhaustive check.
//
// The reference's generated CUDA converts with
//   __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)   (f32 -> E4M3)
//   __float2bfloat16_rn(v)                                 (f32 -> bf16)
// (core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:518-538).
// Both are __host__ __device__ functions of the CUDA 12.9 headers
// (cuda_fp8.h / cuda_bf16.h); this program calls their host forms.
//
//   golden:     writes conversions.bin = for each input of the fixed set
//               below: u32 fp32 bits, u8 e4m3 code, u16 bf16 bits
//   exhaustive: compares the oracle's encoders with those functions over all
//               2^32 fp32 bit patterns and prints the mismatch counts
//   decoders:   writes the f32 bits (u32 little-endian) of every E4M3 code,
//               then every E5M2 code, then every f16 code, widened the way
//               the reference's ReduceSum widens its inputs (__half2float,
//               static_cast<float> of __nv_fp8_e4m3 / __nv_fp8_e5m2;
//               CudaCodegen.scala:451-466), NaNs written as 0x7fc00000 (only
//               NaN-ness is pinned), and prints the oracle decoders' mismatch
//               count on all 66048 codes
//
// Build + run (from tests/golden):
//   gcc -O2 -std=c11 -ffp-contract=off -c ../../oracle/oracle.c -o /tmp/oracle.o
//   g++ -O2 -std=c++17 -ffp-contract=off -I/usr/local/cuda/include \
//       make_golden_conversions.cpp /tmp/oracle.o -o /tmp/mkconv -lpthread -lm
//   /tmp/mkconv golden conversions.bin ; /tmp/mkconv exhaustive
//   /tmp/mkconv decoders /tmp/decoders.bin && xz -9e -c /tmp/decoders.bin > decoders.bin.xz
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cmath>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

extern "C" {
#include "../../oracle/oracle.h"
}

static float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

static uint8_t cuda_e4m3(float v) { return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)); }
static uint16_t cuda_bf16(float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  uint16_t r;
  std::memcpy(&r, &b, 2);
  return r;
}

// Fixed input set: every sign/exponent/top-3-mantissa combination with the
// low 20 mantissa bits at {0, just below half, half, just above half, max}
// (the E4M3 rounding boundaries), the same for bf16's boundary (low 16 bits),
// plus 4096 seeded random patterns.
static std::vector<uint32_t> inputs() {
  std::vector<uint32_t> v;
  const uint32_t low20[] = {0x00000u, 0x7FFFFu, 0x80000u, 0x80001u, 0xFFFFFu};
  for (uint32_t top = 0; top < (1u << 12); ++top)
    for (uint32_t lo : low20) v.push_back((top << 20) | lo);
  const uint32_t low16[] = {0x7FFFu, 0x8000u, 0x8001u};
  for (uint32_t top = 0; top < (1u << 16); top += 61)
    for (uint32_t lo : low16) v.push_back((top << 16) | lo);
  std::mt19937 gen(0x5EED);
  for (int i = 0; i < 4096; ++i) v.push_back(gen());
  return v;
}

static uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static uint32_t canon(float f) { return std::isnan(f) ? 0x7fc00000u : f2u(f); }

static float cuda_f16(uint16_t bits) {
  __half_raw raw;
  raw.x = bits;
  return __half2float(__half(raw));
}
static float cuda_e4m3_dec(uint8_t code) {
  __nv_fp8_e4m3 v;
  v.__x = code;
  return static_cast<float>(v);
}
static float cuda_e5m2_dec(uint8_t code) {
  __nv_fp8_e5m2 v;
  v.__x = code;
  return static_cast<float>(v);
}

static void write_table(FILE* f, unsigned n, float (*dec)(unsigned)) {
  for (unsigned c = 0; c < n; ++c) {
    const uint32_t u = canon(dec(c));
    std::fwrite(&u, 4, 1, f);
  }
}

int main(int argc, char** argv) {
  if (argc >= 3 && std::strcmp(argv[1], "decoders") == 0) {
    FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 1;
    write_table(f, 256, [](unsigned c) { return cuda_e4m3_dec(static_cast<uint8_t>(c)); });
    write_table(f, 256, [](unsigned c) { return cuda_e5m2_dec(static_cast<uint8_t>(c)); });
    write_table(f, 65536, [](unsigned c) { return cuda_f16(static_cast<uint16_t>(c)); });
    std::fclose(f);
    unsigned bad = 0;
    for (unsigned c = 0; c < 256; ++c) {
      bad += canon(orc_e4m3_to_f32(static_cast<uint8_t>(c))) != canon(cuda_e4m3_dec(static_cast<uint8_t>(c)));
      bad += canon(orc_e5m2_to_f32(static_cast<uint8_t>(c))) != canon(cuda_e5m2_dec(static_cast<uint8_t>(c)));
    }
    for (unsigned c = 0; c < 65536; ++c)
      bad += canon(orc_f16_to_f32(static_cast<uint16_t>(c))) != canon(cuda_f16(static_cast<uint16_t>(c)));
    std::printf("decoder codes checked: 66048, oracle mismatches: %u\n", bad);
    return bad == 0 ? 0 : 2;
  }
  if (argc >= 3 && std::strcmp(argv[1], "golden") == 0) {
    const auto in = inputs();
    FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 1;
    const uint32_t n = static_cast<uint32_t>(in.size());
    std::fwrite(&n, 4, 1, f);
    std::fwrite(in.data(), 4, in.size(), f);
    for (uint32_t u : in) { const uint8_t c = cuda_e4m3(u2f(u)); std::fwrite(&c, 1, 1, f); }
    for (uint32_t u : in) { const uint16_t b = cuda_bf16(u2f(u)); std::fwrite(&b, 2, 1, f); }
    std::fclose(f);
    std::printf("wrote %u vectors to %s\n", n, argv[2]);
    return 0;
  }
  if (argc >= 2 && std::strcmp(argv[1], "exhaustive") == 0) {
    const unsigned threads = std::max(1u, std::thread::hardware_concurrency());
    std::vector<uint64_t> e4m3_bad(threads), bf16_bad(threads), bf16_nan_bad(threads);
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < threads; ++t) {
      pool.emplace_back([&, t] {
        const uint64_t begin = (1ull << 32) * t / threads, end = (1ull << 32) * (t + 1) / threads;
        for (uint64_t i = begin; i < end; ++i) {
          const float v = u2f(static_cast<uint32_t>(i));
          if (orc_f32_to_e4m3_satfinite(v) != cuda_e4m3(v)) ++e4m3_bad[t];
          const uint16_t ob = orc_f32_to_bf16_rn(v), cb = cuda_bf16(v);
          if (ob != cb) {
            const bool both_nan = ((ob & 0x7F80) == 0x7F80 && (ob & 0x7F)) && ((cb & 0x7F80) == 0x7F80 && (cb & 0x7F));
            if (both_nan) ++bf16_nan_bad[t]; else ++bf16_bad[t];
          }
        }
      });
    }
    for (auto& th : pool) th.join();
    uint64_t e = 0, b = 0, bn = 0;
    for (unsigned t = 0; t < threads; ++t) { e += e4m3_bad[t]; b += bf16_bad[t]; bn += bf16_nan_bad[t]; }
    std::printf("fp32 patterns checked: 4294967296\n");
    std::printf("e4m3 satfinite rn mismatches: %llu\n", (unsigned long long)e);
    std::printf("bf16 rn mismatches (non-NaN): %llu\n", (unsigned long long)b);
    std::printf("bf16 rn NaN payload differences: %llu\n", (unsigned long long)bn);
    return (e == 0 && b == 0) ? 0 : 2;
  }
  std::fprintf(stderr, "usage: %s golden <out.bin> | exhaustive | decoders <out.json>\n", argv[0]);
  return 1;
}
