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
//   modes:      compares the oracle's moded conversions (f16 and bf16 under
//               the four rounding modes, E4M3 without and E5M2 with and
//               without saturation) with __float2half_{rn,rz,ru,rd},
//               __float2bfloat16_{rn,rz,ru,rd} and __nv_cvt_float_to_fp8
//               over all 2^32 fp32 patterns and prints the mismatch counts
//   modes-golden: writes those conversions' outputs on a fixed input set
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
//   /tmp/mkconv modes > conversions_modes_exhaustive.txt
//   /tmp/mkconv modes-golden /tmp/modes.bin && xz -9e -c /tmp/modes.bin > conversions_modes.bin.xz
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

// The conversions of the reference's Convert node with rounding and
// saturation modes (CudaCodegen.scala:405-449,506-538), host forms.
static uint16_t half_bits(__half h) { __half_raw r = h; return r.x; }
static uint16_t bf16_bits(__nv_bfloat16 b) { uint16_t r; std::memcpy(&r, &b, 2); return r; }
static uint16_t cuda_f16(float v, int rounding) {
  switch (rounding) {
    case 0: return half_bits(__float2half_rn(v));
    case 1: return half_bits(__float2half_rz(v));
    case 2: return half_bits(__float2half_ru(v));
    default: return half_bits(__float2half_rd(v));
  }
}
static uint16_t cuda_bf16_mode(float v, int rounding) {
  switch (rounding) {
    case 0: return bf16_bits(__float2bfloat16_rn(v));
    case 1: return bf16_bits(__float2bfloat16_rz(v));
    case 2: return bf16_bits(__float2bfloat16_ru(v));
    default: return bf16_bits(__float2bfloat16_rd(v));
  }
}
static uint8_t cuda_fp8(float v, bool e4m3, bool saturate) {
  return static_cast<uint8_t>(
      __nv_cvt_float_to_fp8(v, saturate ? __NV_SATFINITE : __NV_NOSAT, e4m3 ? __NV_E4M3 : __NV_E5M2));
}

// The eleven moded conversions, in fixture order: f16 rn/rz/ru/rd, bf16
// rn/rz/ru/rd, e4m3 nosat, e5m2 nosat, e5m2 satfinite (e4m3 satfinite is
// in conversions.bin).
constexpr int kModed = 11;
static uint32_t cuda_moded(int c, float v) {
  if (c < 4) return cuda_f16(v, c);
  if (c < 8) return cuda_bf16_mode(v, c - 4);
  if (c == 8) return cuda_fp8(v, true, false);
  return cuda_fp8(v, false, c == 10);
}
static uint32_t oracle_moded(int c, float v) {
  if (c < 4) return orc_f32_to_f16(v, c);
  if (c < 8) return orc_f32_to_bf16(v, c - 4);
  if (c == 8) return orc_f32_to_e4m3(v, 0);
  return orc_f32_to_e5m2(v, c == 10);
}
static bool is_nan_code(int c, uint32_t bits) {
  if (c < 4) return (bits & 0x7C00) == 0x7C00 && (bits & 0x3FF);
  if (c < 8) return (bits & 0x7F80) == 0x7F80 && (bits & 0x7F);
  if (c == 8) return (bits & 0x7F) == 0x7F;
  return (bits & 0x7C) == 0x7C && (bits & 0x3);
}
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
  if (argc >= 2 && std::strcmp(argv[1], "modes") == 0) {
    // exhaustive: every fp32 pattern through the eleven moded conversions
    const unsigned threads = std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::vector<uint64_t>> bad(threads, std::vector<uint64_t>(kModed)),
        nan_bad(threads, std::vector<uint64_t>(kModed));
    std::vector<std::vector<uint32_t>> first(threads, std::vector<uint32_t>(kModed, 0xFFFFFFFFu));
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < threads; ++t) {
      pool.emplace_back([&, t] {
        const uint64_t begin = (1ull << 32) * t / threads, end = (1ull << 32) * (t + 1) / threads;
        for (uint64_t i = begin; i < end; ++i) {
          const float v = u2f(static_cast<uint32_t>(i));
          for (int c = 0; c < kModed; ++c) {
            const uint32_t a = oracle_moded(c, v), b = cuda_moded(c, v);
            if (a == b) continue;
            if (is_nan_code(c, a) && is_nan_code(c, b)) ++nan_bad[t][c];
            else {
              if (!bad[t][c]) first[t][c] = static_cast<uint32_t>(i);
              ++bad[t][c];
            }
          }
        }
      });
    }
    for (auto& th : pool) th.join();
    const char* names[kModed] = {"f16 rn", "f16 rz", "f16 ru", "f16 rd", "bf16 rn", "bf16 rz", "bf16 ru",
                                 "bf16 rd", "e4m3 nosat", "e5m2 nosat", "e5m2 satfinite"};
    std::printf("fp32 patterns checked: 4294967296\n");
    int rc = 0;
    for (int c = 0; c < kModed; ++c) {
      uint64_t b = 0, nb = 0;
      uint32_t f = 0xFFFFFFFFu;
      for (unsigned t = 0; t < threads; ++t) {
        b += bad[t][c];
        nb += nan_bad[t][c];
        if (bad[t][c] && f == 0xFFFFFFFFu) f = first[t][c];
      }
      std::printf("%s mismatches (non-NaN): %llu; NaN payload differences: %llu", names[c],
                  (unsigned long long)b, (unsigned long long)nb);
      if (b) std::printf("; first at 0x%08x (oracle 0x%x, cuda 0x%x)", f, oracle_moded(c, u2f(f)), cuda_moded(c, u2f(f)));
      std::printf("\n");
      if (b || nb) rc = 2;
    }
    return rc;
  }
  if (argc >= 3 && std::strcmp(argv[1], "modes-golden") == 0) {
    // fixture: the fixed input set below plus f16 rounding boundaries,
    // then each moded conversion's output bits (u16 for f16/bf16, u8 fp8)
    auto in = inputs();
    const uint32_t low13[] = {0x0000u, 0x0FFFu, 0x1000u, 0x1001u, 0x1FFFu};
    for (uint32_t top = 0; top < (1u << 19); top += 101)
      for (uint32_t lo : low13) in.push_back((top << 13) | lo);
    FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 1;
    const uint32_t n = static_cast<uint32_t>(in.size());
    std::fwrite(&n, 4, 1, f);
    std::fwrite(in.data(), 4, in.size(), f);
    for (int c = 0; c < kModed; ++c) {
      for (uint32_t u : in) {
        const uint32_t b = cuda_moded(c, u2f(u));
        if (c < 8) { const uint16_t h = static_cast<uint16_t>(b); std::fwrite(&h, 2, 1, f); }
        else { const uint8_t q = static_cast<uint8_t>(b); std::fwrite(&q, 1, 1, f); }
      }
    }
    std::fclose(f);
    std::printf("wrote %u inputs x %d conversions to %s\n", n, kModed, argv[2]);
    return 0;
  }
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
  std::fprintf(stderr, "usage: %s golden <out.bin> | exhaustive | decoders <out.bin> | modes | modes-golden <out.bin>\n",
               argv[0]);
  return 1;
}
