/*
 * CPU oracle for the flight4s hot path — TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C restatement of the reference's CPU-side checks and of the
 * arithmetic the hot-path kernels define.  Only the test suite, the smoke
 * check and the benchmark's CPU-baseline leg load this library; the
 * product path never does.
 *
 * Pinning (what each part is checked against):
 *   - vectorAdd and the sequential fp32 fold restate the reference's own CPU
 *     checks: Array.tabulate(n)(i => l(i) + r(i)) and `inputValues.sum`
 *     (runtime/src/test/scala/flight4s/runtime/cuda/CudaResourcesJniSuite.scala:114-122,235-238),
 *     pinned by that suite's known answers (c[i] = 3i for n = 1024; 896.0
 *     for x[i] = i % 8, n = 256);
 *   - the block tree restates the generated blockReduceSum text
 *     (core/src/test/scala/flight4s/core/codegen/CudaCodegenSuite.scala:133-216);
 *   - E4M3 and bf16 conversions are written from the OCP FP8 and IEEE-754
 *     definitions and pinned against the conversion functions the
 *     reference's generated code calls (__nv_cvt_float_to_fp8 with
 *     __NV_SATFINITE/__NV_E4M3 and __float2bfloat16_rn,
 *     core/src/main/scala/flight4s/core/codegen/CudaCodegen.scala:518-538),
 *     run on the host by tests/golden/make_golden_conversions.cpp;
 *   - the f16, E4M3 and E5M2 decoders (ReduceSum's widening of its 16-bit
 *     and 8-bit inputs: __half2float and static_cast<float>,
 *     CudaCodegen.scala:451-466) are pinned on every code against the same
 *     functions' host forms (tests/golden/decoders.bin.xz);
 *   - max/argmax, softmax, RMSNorm and the FP8 block scaling have no
 *     reference implementation: parity unpinned for those, the oracle is
 *     their definition.
 *
 * Compile with -ffp-contract=off: every float operation here is one IEEE
 * single or double rounding, in source order.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------- bit casts */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* --------------------------------------------------------------- Philox
 * Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): 10 rounds of
 * (hi0,lo0) = M0*c0, (hi1,lo1) = M1*c2,
 * c = (hi1^c1^k0, lo1, hi0^c3^k1, lo0), key += (W0, W1). */
void orc_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
    c0 = n0;
    c1 = (uint32_t)p1;
    c2 = n2;
    c3 = (uint32_t)p0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static uint32_t philox_word(uint64_t index, uint32_t stream, uint64_t seed) {
  const uint64_t g = index / 4;
  const uint32_t ctr[4] = {(uint32_t)g, (uint32_t)(g >> 32), stream, 0u};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t w[4];
  orc_philox4x32_10(ctr, key, w);
  return w[index % 4];
}

void orc_fill_uniform_f32(float* out, uint64_t n, uint64_t offset, uint64_t seed, uint32_t stream) {
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t w = philox_word(offset + i, stream, seed);
    out[i] = (float)(w >> 8) * 0x1p-23f - 1.0f;
  }
}

void orc_fill_uniform_i32(int32_t* out, uint64_t n, uint64_t offset, uint64_t seed, uint32_t stream,
                          int32_t lo, int32_t hi) {
  const uint32_t span = (uint32_t)(hi - lo) + 1u;
  for (uint64_t i = 0; i < n; ++i) out[i] = lo + (int32_t)(philox_word(offset + i, stream, seed) % span);
}

/* ----------------------------------------------------------------- bf16
 * IEEE-754 round-to-nearest-even of the top 16 bits; NaN -> 0x7FFF. */
uint16_t orc_f32_to_bf16_rn(float f) {
  const uint32_t u = f2u(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF;
  const uint32_t bias = 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)((u + bias) >> 16);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* ----------------------------------------------------------------- E4M3
 * OCP 8-bit floating point, E4M3: bias 7, 3 mantissa bits, no infinities,
 * NaN = S.1111.111, max finite 448 = 1.75 * 2^8, min normal 2^-6,
 * subnormals m * 2^-9.  Round to nearest even; with saturation, every
 * finite or infinite magnitude above 448 becomes 448; NaN -> 0x7F. */
uint8_t orc_f32_to_e4m3_satfinite(float f) {
  if (isnan(f)) return 0x7F;
  const uint8_t sign = (f2u(f) >> 31) ? 0x80 : 0x00;
  const double a = fabs((double)f);
  if (a > 448.0) return sign | 0x7E;
  if (a < 0x1p-6) {
    /* subnormal grid m * 2^-9, m in [0, 8]; m == 8 is the min normal 0x08 */
    const double m = nearbyint(a * 512.0);
    return sign | (uint8_t)m;
  }
  int k;
  const double frac = frexp(a, &k); /* a = frac * 2^k, frac in [0.5, 1) */
  int e = k - 1;                    /* a = (2 * frac) * 2^e */
  double q = nearbyint(frac * 16.0); /* (2*frac) * 8, in [8, 16] */
  if (q == 16.0) {
    q = 8.0;
    e += 1;
  }
  /* a <= 448 guarantees e <= 8 and (e == 8 => q <= 14) */
  return sign | (uint8_t)(((e + 7) << 3) | ((int)q - 8));
}

float orc_e4m3_to_f32(uint8_t c) {
  const int s = c >> 7, e = (c >> 3) & 0xF, m = c & 7;
  if (e == 0xF && m == 7) return s ? -NAN : NAN;
  const double v = e == 0 ? ldexp((double)m, -9) : ldexp(1.0 + m / 8.0, e - 7);
  return (float)(s ? -v : v);
}

/* ----------------------------------------------------------------- E5M2
 * OCP 8-bit floating point, E5M2: the IEEE-754 layout with bias 15 and 2
 * mantissa bits; exponent 31 holds infinities (m == 0) and NaNs. */
float orc_e5m2_to_f32(uint8_t c) {
  const int s = c >> 7, e = (c >> 2) & 0x1F, m = c & 3;
  double v;
  if (e == 0x1F) v = m ? NAN : INFINITY;
  else v = e == 0 ? ldexp((double)m, -16) : ldexp(1.0 + m / 4.0, e - 15);
  return (float)(s ? -v : v);
}

/* --------------------------------------------------------------- binary16
 * IEEE-754 binary16: bias 15, 10 mantissa bits, subnormals m * 2^-24,
 * exponent 31 holds infinities and NaNs.  Widening to f32 is exact. */
float orc_f16_to_f32(uint16_t h) {
  const int s = h >> 15, e = (h >> 10) & 0x1F, m = h & 0x3FF;
  double v;
  if (e == 0x1F) v = m ? NAN : INFINITY;
  else v = e == 0 ? ldexp((double)m, -24) : ldexp(1.0 + m / 1024.0, e - 15);
  return (float)(s ? -v : v);
}

/* Decode n elements of a ReduceSum input type (launch-ABI type code
 * 4 f16, 5 bf16, 6 f32, 8 e4m3, 9 e5m2) to f32. */
int orc_decode_to_f32(int type_code, const void* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    switch (type_code) {
      case 4: out[i] = orc_f16_to_f32(((const uint16_t*)x)[i]); break;
      case 5: out[i] = orc_bf16_to_f32(((const uint16_t*)x)[i]); break;
      case 6: out[i] = ((const float*)x)[i]; break;
      case 8: out[i] = orc_e4m3_to_f32(((const uint8_t*)x)[i]); break;
      case 9: out[i] = orc_e5m2_to_f32(((const uint8_t*)x)[i]); break;
      default: return -1;
    }
  }
  return 0;
}

/* ------------------------------------------------ Convert with modes
 * The reference's Convert node (core/src/main/scala/flight4s/core/ir/IR.scala:54-70)
 * carries a RoundingMode {NearestEven, TowardZero, TowardPositive,
 * TowardNegative} (ordinals 0..3) and a SaturationMode {NoSaturation,
 * SaturateFinite} (0, 1); its codegen calls __float2half_{rn,rz,ru,rd},
 * __float2bfloat16_{rn,rz,ru,rd} and __nv_cvt_float_to_fp8(v, sat, kind)
 * (CudaCodegen.scala:405-449,506-538).  Restated here from IEEE-754 (f16,
 * bf16) and the OCP FP8 definitions; FP8 conversion always rounds to
 * nearest-even (the call has no rounding argument). */

/* Round the non-negative quotient m (exact in double) to an integer:
 * 0 nearest-even, 1 toward zero, 2 away from zero. */
static double round_magnitude(double m, int mode_on_magnitude) {
  const double fl = floor(m);
  switch (mode_on_magnitude) {
    case 0: return nearbyint(m);           /* default FE_TONEAREST: ties to even */
    case 1: return fl;
    default: return fl == m ? m : fl + 1;  /* away from zero */
  }
}

/* magnitude rounding for a signed value: RU rounds positive magnitudes up
 * and negative magnitudes toward zero; RD the reverse */
static int magnitude_mode(int rounding, int negative) {
  switch (rounding) {
    case 0: return 0;
    case 1: return 1;
    case 2: return negative ? 1 : 2;
    default: return negative ? 2 : 1;
  }
}

uint16_t orc_f32_to_f16(float f, int rounding) {
  const uint32_t u = f2u(f);
  const uint16_t sign = (u >> 31) ? 0x8000 : 0;
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF;
  if ((u & 0x7FFFFFFFu) == 0x7F800000u) return sign | 0x7C00;
  const double a = fabs((double)f);
  if (a == 0.0) return sign;
  int k;
  frexp(a, &k);                  /* a in [2^(k-1), 2^k) */
  int e = k - 1;
  if (e < -14) e = -14;          /* subnormal quantum 2^-24 */
  if (e > 15) e = 15;            /* overflow handled below */
  const double q = ldexp(1.0, e - 10);
  const double r = round_magnitude(a / q, magnitude_mode(rounding, sign != 0)) * q;
  if (r > 65504.0) {
    const int mm = magnitude_mode(rounding, sign != 0);
    return sign | (mm == 1 ? 0x7BFF : 0x7C00);   /* toward zero: max finite; else inf */
  }
  if (r < 0x1p-14) return sign | (uint16_t)(r / 0x1p-24);
  int kr;
  const double fr = frexp(r, &kr);
  return sign | (uint16_t)(((kr - 1 + 15) << 10) | (uint16_t)((2.0 * fr - 1.0) * 1024.0));
}

uint16_t orc_f32_to_bf16(float f, int rounding) {
  if (rounding == 0) return orc_f32_to_bf16_rn(f);
  const uint32_t u = f2u(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF;
  const uint16_t t = (uint16_t)(u >> 16);
  const int inexact = (u & 0xFFFFu) != 0;
  const int mm = magnitude_mode(rounding, (u >> 31) != 0);
  /* magnitude + 1 ulp carries into the exponent (and to inf) by itself */
  return (mm == 2 && inexact) ? (uint16_t)(t + 1) : t;
}

uint8_t orc_f32_to_e4m3(float f, int saturate) {
  if (saturate) return orc_f32_to_e4m3_satfinite(f);
  const uint8_t sign = (f2u(f) >> 31) ? 0x80 : 0x00;
  if (isnan(f)) return 0x7F;
  /* beyond 448 the next step would be 480 = the NaN code: values that round
   * above 448 (|x| > 464; 464 ties to the even 448) become NaN */
  if (fabs((double)f) > 464.0) return sign | 0x7F;
  return orc_f32_to_e4m3_satfinite(f);
}

/* E5M2: bias 15, 2 mantissa bits, subnormals m * 2^-16, max finite 57344. */
uint8_t orc_f32_to_e5m2(float f, int saturate) {
  const uint32_t u = f2u(f);
  const uint8_t sign = (u >> 31) ? 0x80 : 0x00;
  if (isnan(f)) return 0x7F;
  const double a = fabs((double)f);
  if (isinf(f)) return saturate ? (sign | 0x7B) : (sign | 0x7C);
  if (a == 0.0) return sign;
  int k;
  frexp(a, &k);
  int e = k - 1;
  if (e < -14) e = -14;
  if (e > 15) e = 15;
  const double q = ldexp(1.0, e - 2);
  const double r = nearbyint(a / q) * q;
  if (r > 57344.0) return saturate ? (sign | 0x7B) : (sign | 0x7C);
  if (r < 0x1p-14) return sign | (uint8_t)(r / 0x1p-16);
  int kr;
  const double fr = frexp(r, &kr);
  return sign | (uint8_t)(((kr - 1 + 15) << 2) | (uint8_t)((2.0 * fr - 1.0) * 4.0));
}

/* Elementwise Convert over n elements (launch-ABI type codes 4 f16, 5 bf16,
 * 6 f32, 8 e4m3, 9 e5m2: f32 <-> the others; or any type 1..9 to itself).
 * Returns 0, or -1 for a pair the reference's codegen rejects. */
int orc_convert(int from, int to, int rounding, int saturation, const void* in, void* out, int64_t n) {
  if (from == to) {  /* the reference emits the value unchanged (CudaCodegen.scala:440-441) */
    static const int kBytes[10] = {0, 1, 4, 4, 2, 2, 4, 8, 1, 1};
    const int eb = (from >= 1 && from <= 9) ? kBytes[from] : 0;
    if (eb == 0) return -1;
    memcpy(out, in, (size_t)(n * eb));
    return 0;
  }
  if (from == 6) {
    const float* x = (const float*)in;
    for (int64_t i = 0; i < n; ++i) {
      switch (to) {
        case 4: ((uint16_t*)out)[i] = orc_f32_to_f16(x[i], rounding); break;
        case 5: ((uint16_t*)out)[i] = orc_f32_to_bf16(x[i], rounding); break;
        case 8: ((uint8_t*)out)[i] = orc_f32_to_e4m3(x[i], saturation); break;
        case 9: ((uint8_t*)out)[i] = orc_f32_to_e5m2(x[i], saturation); break;
        default: return -1;
      }
    }
    return 0;
  }
  if (to == 6 && (from == 4 || from == 5 || from == 8 || from == 9))
    return orc_decode_to_f32(from, in, n, (float*)out);
  return -1;
}

/* ----------------------------------------------------------- vectorAdd
 * Array.tabulate(n)(i => l(i) + r(i)) (CudaResourcesJniSuite.scala:120-122). */
void orc_vector_add_f32(const float* a, const float* b, float* c, int64_t n) {
  for (int64_t i = 0; i < n; ++i) c[i] = a[i] + b[i];
}

/* bf16: widen exactly, add in f32 (one rounding), round to nearest-even. */
void orc_vector_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n) {
  for (int64_t i = 0; i < n; ++i) c[i] = orc_f32_to_bf16_rn(orc_bf16_to_f32(a[i]) + orc_bf16_to_f32(b[i]));
}

/* `+` over every AdditiveType (CudaType.scala:154-160), by launch-ABI code:
 * 2/3 32-bit wrap, 4 f16 and 5 bf16 (the f32 sum of the widened operands
 * rounded to nearest-even once more: f32's 24 bits >= 2 * 11 + 2, so this
 * equals the correctly rounded 16-bit sum), 6 f32, 7 f64.  -1 otherwise. */
int orc_vector_add_typed(int type_code, const void* a, const void* b, void* c, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    switch (type_code) {
      case 2: case 3:
        ((uint32_t*)c)[i] = ((const uint32_t*)a)[i] + ((const uint32_t*)b)[i];
        break;
      case 4:
        ((uint16_t*)c)[i] = orc_f32_to_f16(orc_f16_to_f32(((const uint16_t*)a)[i]) +
                                           orc_f16_to_f32(((const uint16_t*)b)[i]), 0);
        break;
      case 5:
        ((uint16_t*)c)[i] = orc_f32_to_bf16_rn(orc_bf16_to_f32(((const uint16_t*)a)[i]) +
                                               orc_bf16_to_f32(((const uint16_t*)b)[i]));
        break;
      case 6: ((float*)c)[i] = ((const float*)a)[i] + ((const float*)b)[i]; break;
      case 7: ((double*)c)[i] = ((const double*)a)[i] + ((const double*)b)[i]; break;
      default: return -1;
    }
  }
  return 0;
}

/* ---------------------------------------------------------- reductions
 * Scala's Array[Float].sum: a left fold in Float from 0.0f
 * (CudaResourcesJniSuite.scala:238). */
float orc_sum_f32_sequential(const float* x, int64_t n) {
  return orc_sum_f32_sequential_from(x, n, 0.0f);
}

/* The same fold continued from a running Float accumulator, so an array
 * can be folded chunk by chunk with the exact bits of one pass. */
float orc_sum_f32_sequential_from(const float* x, int64_t n, float acc) {
  for (int64_t i = 0; i < n; ++i) acc += x[i];
  return acc;
}

/* Ground truth: compensated (Neumaier) summation in long double. */
double orc_sum_f32_exactish(const float* x, int64_t n, double* abs_sum) {
  long double s = 0.0L, c = 0.0L, a = 0.0L;
  for (int64_t i = 0; i < n; ++i) {
    const long double v = x[i];
    const long double t = s + v;
    if (fabsl(s) >= fabsl(v)) c += (s - t) + v; else c += (v - t) + s;
    s = t;
    a += fabsl(v);
  }
  if (abs_sum) *abs_sum = (double)a;
  return (double)(s + c);
}

/* Ground truth of a floating-point ReduceSum over any accumulator input
 * type (launch-ABI code 4 f16, 5 bf16, 6 f32, 7 f64, 8 e4m3, 9 e5m2):
 * every element widened exactly, then compensated summation in long double.
 * The reference accumulates the 16-bit and 8-bit types in F32
 * (core/src/main/scala/flight4s/core/types/CudaType.scala:212-230); this is
 * the exact value both it and a wider accumulator approximate. */
double orc_sum_typed_exactish(int type_code, const void* x, int64_t n, double* abs_sum) {
  long double s = 0.0L, c = 0.0L, a = 0.0L;
  for (int64_t i = 0; i < n; ++i) {
    long double v;
    switch (type_code) {
      case 4: v = orc_f16_to_f32(((const uint16_t*)x)[i]); break;
      case 5: v = orc_bf16_to_f32(((const uint16_t*)x)[i]); break;
      case 6: v = ((const float*)x)[i]; break;
      case 7: v = ((const double*)x)[i]; break;
      case 8: v = orc_e4m3_to_f32(((const uint8_t*)x)[i]); break;
      case 9: v = orc_e5m2_to_f32(((const uint8_t*)x)[i]); break;
      default: return NAN;
    }
    const long double t = s + v;
    if (fabsl(s) >= fabsl(v)) c += (s - t) + v; else c += (v - t) + s;
    s = t;
    a += fabsl(v);
  }
  if (abs_sum) *abs_sum = (double)a;
  return (double)(s + c);
}

/* ------------------------------------------------- order-fixed sums
 * The order-fixed ("Deterministic") sum the B200 kernels define for the
 * reference's ReductionPolicy (core/src/main/scala/flight4s/core/ir/IR.scala:79-82),
 * restated operation by operation so results compare bit for bit:
 *   body = elements from the first 16-byte boundary (`head` elements before
 *   it), cut into 16-byte vectors (the last zero-padded); tile = 256
 *   vectors, lane l of 32 takes vectors l + 32u (u < 8); group = 64 tiles.
 *   vector value: f32 (a+b)+(c+d); f16/bf16 ((((0+h0)+h1)+h2)+h3) +
 *   ((((0+h4)+h5)+h6)+h7) in f32; FP8 the same over bytes 0..7 and 8..15;
 *   f64 d0+d1.  Lane: the 8 vector values (zero past the end) folded
 *   pairwise (s0+=s1, s2+=s3, ...; s0+=s2, ...; s0+=s4) -- in f32 then
 *   widened for f32 input, in f64 otherwise -- added to 0.0.  Tile: warp
 *   tree v[l] += v[l+o], o = 16..1.  Group: the warp tree of
 *   tile[l] + tile[l+32].  Total: thread t of 512 adds groups t, t+512, ...
 *   in order from 0.0; warp trees; the 16 warp values (16 zeros after
 *   them) through one more warp tree; then + the head elements, each widened
 *   and added in order to 0.0. */
static int elem_bytes(int type_code) {
  switch (type_code) {
    case 4: case 5: return 2;
    case 6: return 4;
    case 7: return 8;
    case 8: case 9: return 1;
    default: return 0;
  }
}

static double widen(int type_code, const unsigned char* p) {
  switch (type_code) {
    case 4: { uint16_t h; memcpy(&h, p, 2); return orc_f16_to_f32(h); }
    case 5: { uint16_t h; memcpy(&h, p, 2); return orc_bf16_to_f32(h); }
    case 6: { float f; memcpy(&f, p, 4); return f; }
    case 7: { double d; memcpy(&d, p, 8); return d; }
    case 8: return orc_e4m3_to_f32(*p);
    default: return orc_e5m2_to_f32(*p);
  }
}

static float widen_f(int type_code, const unsigned char* p) { return (float)widen(type_code, p); }

/* value of one 16-byte vector; f32-valued types return the f32 widened */
static double vector_value(int type_code, const unsigned char* v, int* is_f32) {
  *is_f32 = type_code != 7;
  if (type_code == 6) {
    const float a = widen_f(6, v), b = widen_f(6, v + 4), c = widen_f(6, v + 8), d = widen_f(6, v + 12);
    return (double)((a + b) + (c + d));
  }
  if (type_code == 7) return widen(7, v) + widen(7, v + 8);
  const int eb = elem_bytes(type_code), half = 8 / eb;
  float a = 0.0f, b = 0.0f;
  for (int k = 0; k < half; ++k) a = a + widen_f(type_code, v + k * eb);
  for (int k = 0; k < half; ++k) b = b + widen_f(type_code, v + 8 + k * eb);
  return (double)(a + b);
}

static double warp_tree(double* v) {
  for (int o = 16; o > 0; o >>= 1)
    for (int l = 0; l < o; ++l) v[l] = v[l] + v[l + o];
  return v[0];
}

double orc_ordered_final(const double* groups, int64_t count) {
  double acc[512], warps[32];
  for (int t = 0; t < 512; ++t) {
    double a = 0.0;
    for (int64_t g = t; g < count; g += 512) a = a + groups[g];
    acc[t] = a;
  }
  for (int w = 0; w < 16; ++w) warps[w] = warp_tree(acc + 32 * w);
  for (int w = 16; w < 32; ++w) warps[w] = 0.0;
  return warp_tree(warps);
}

double orc_sum_ordered(int type_code, const void* x, int64_t n, int64_t head, double* groups_out,
                       int64_t* ngroups_out) {
  const int eb = elem_bytes(type_code);
  if (eb == 0 || head < 0 || head > n) return NAN;
  const unsigned char* in = (const unsigned char*)x;
  const unsigned char* body = in + head * eb;
  const int per = 16 / eb;
  const int64_t nvec_full = (n - head) / per;
  const int tail = (int)((n - head) % per);
  const int64_t nvec = nvec_full + (tail > 0);
  const int64_t ntiles = (nvec + 255) / 256, ngroups = (ntiles + 63) / 64;
  unsigned char tailv[16];
  memset(tailv, 0, 16);
  if (tail > 0) memcpy(tailv, body + nvec_full * 16, (size_t)tail * eb);
  double* groups = (double*)malloc(sizeof(double) * (size_t)(ngroups > 0 ? ngroups : 1));
  for (int64_t g = 0; g < ngroups; ++g) {
    double tiles[64];
    for (int local = 0; local < 64; ++local) {
      const int64_t tile = g * 64 + local;
      double lanes[32];
      for (int l = 0; l < 32; ++l) {
        double sd[8];
        float sf[8];
        int is_f32 = 1;
        for (int u = 0; u < 8; ++u) {
          const int64_t idx = tile * 256 + l + 32 * u;
          double val = 0.0;
          if (tile < ntiles && idx < nvec) val = vector_value(type_code, idx < nvec_full ? body + idx * 16 : tailv, &is_f32);
          sd[u] = val;
          sf[u] = (float)val;
        }
        double folded;
        if (type_code == 6) {
          for (int w = 1; w < 8; w <<= 1)
            for (int u = 0; u + w < 8; u += 2 * w) sf[u] = sf[u] + sf[u + w];
          folded = (double)sf[0];
        } else {
          for (int w = 1; w < 8; w <<= 1)
            for (int u = 0; u + w < 8; u += 2 * w) sd[u] = sd[u] + sd[u + w];
          folded = sd[0];
        }
        lanes[l] = tile < ntiles ? 0.0 + folded : 0.0;
      }
      tiles[local] = warp_tree(lanes);
    }
    double v[32];
    for (int l = 0; l < 32; ++l) v[l] = tiles[l] + tiles[l + 32];
    groups[g] = warp_tree(v);
  }
  double total = orc_ordered_final(groups, ngroups);
  double h = 0.0;
  for (int64_t i = 0; i < head; ++i) h = h + widen(type_code, in + i * eb);
  total = total + h;
  if (groups_out) memcpy(groups_out, groups, sizeof(double) * (size_t)ngroups);
  if (ngroups_out) *ngroups_out = ngroups;
  free(groups);
  return total;
}

/* U32 accumulates in U32 (CudaType.scala:208-210): wrap modulo 2^32. */
uint32_t orc_sum_u32(const uint32_t* x, int64_t n) {
  uint32_t acc = 0;
  for (int64_t i = 0; i < n; ++i) acc += x[i];
  return acc;
}

/* I32 accumulates in I32 with two's-complement wrap
 * (core/src/main/scala/flight4s/core/types/CudaType.scala:204-206). */
int32_t orc_sum_i32(const int32_t* x, int64_t n) {
  uint32_t acc = 0;
  for (int64_t i = 0; i < n; ++i) acc += (uint32_t)x[i];
  return (int32_t)acc;
}

/* Signed-int image of IEEE-754 totalOrder. */
static int32_t total_order_key(float v) {
  const int32_t b = (int32_t)f2u(v);
  return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}

/* max under totalOrder, first (lowest) index on ties; -1 when n == 0. */
int64_t orc_argmax_f32(const float* x, int64_t n, float* max_value) {
  int64_t best = -1;
  int32_t key = 0;
  for (int64_t i = 0; i < n; ++i) {
    const int32_t k = total_order_key(x[i]);
    if (best < 0 || k > key) {
      key = k;
      best = i;
    }
  }
  if (max_value) *max_value = best >= 0 ? x[best] : NAN;
  return best;
}

/* Packed cross-device key, compared as a signed 64-bit integer:
 * (signed totalOrder key << 32) | (0xFFFFFFFF - index). */
/* max / argmax over every OrderedType (CudaType.scala:182-188) by launch-ABI
 * code (2 i32, 3 u32, 4 f16, 5 bf16, 6 f32, 7 f64): the first index of the
 * largest element, integers by value, floats by IEEE totalOrder (the
 * signed-magnitude bits with the magnitude inverted for negatives); -1 when
 * n == 0 or the type has no order.  *key_out receives the order key. */
static int64_t order_key(int type_code, const unsigned char* p) {
  switch (type_code) {
    case 2: { int32_t v; memcpy(&v, p, 4); return v; }
    case 3: { uint32_t v; memcpy(&v, p, 4); return (int64_t)v - 2147483648LL; }
    case 4: case 5: {
      int16_t v; memcpy(&v, p, 2);
      return v < 0 ? (int64_t)(v ^ 0x7FFF) : (int64_t)v;
    }
    case 6: { int32_t v; memcpy(&v, p, 4); return v < 0 ? (int64_t)(v ^ 0x7FFFFFFF) : (int64_t)v; }
    default: { int64_t v; memcpy(&v, p, 8); return v < 0 ? (v ^ INT64_MAX) : v; }
  }
}

int64_t orc_argmax_typed(int type_code, const void* x, int64_t n, int64_t* key_out) {
  static const int kBytes[8] = {0, 0, 4, 4, 2, 2, 4, 8};
  if (type_code < 2 || type_code > 7 || n <= 0) return -1;
  const unsigned char* in = (const unsigned char*)x;
  const int eb = kBytes[type_code];
  int64_t best = 0, bk = order_key(type_code, in);
  for (int64_t i = 1; i < n; ++i) {
    const int64_t k = order_key(type_code, in + i * eb);
    if (k > bk) { bk = k; best = i; }
  }
  if (key_out) *key_out = bk;
  return best;
}

int64_t orc_argmax_packed_key(float value, int64_t index) {
  const uint64_t hi = (uint64_t)(uint32_t)total_order_key(value) << 32;
  return (int64_t)(hi | (uint64_t)(0xFFFFFFFFu - (uint32_t)index));
}

/* --------------------------------------------------------- block tree
 * One node = the reference's shared-memory tree over 256 values
 * (strides 128, 64, ..., 1: s[t] += s[t + stride] for t < stride). */
static float tree256(float s[256]) {
  for (int stride = 128; stride >= 1; stride >>= 1)
    for (int t = 0; t < stride; ++t) s[t] = s[t] + s[t + stride];
  return s[0];
}

/* partials[t] = node over tile t (zero padded); then nodes over runs of 256
 * partials, level by level, until one value remains (a single tile is the
 * result itself).  n == 0 gives +0.0. */
float orc_block_tree_sum_f32(const float* x, int64_t n, float* partials) {
  const int64_t tiles = (n + 255) / 256;
  if (tiles == 0) return 0.0f;
  float* level = (float*)malloc(sizeof(float) * (size_t)tiles);
  float s[256];
  for (int64_t t = 0; t < tiles; ++t) {
    for (int k = 0; k < 256; ++k) {
      const int64_t i = t * 256 + k;
      s[k] = i < n ? x[i] : 0.0f;
    }
    level[t] = tree256(s);
    if (partials) partials[t] = level[t];
  }
  int64_t count = tiles;
  while (count > 1) {
    const int64_t nodes = (count + 255) / 256;
    for (int64_t g = 0; g < nodes; ++g) {
      for (int k = 0; k < 256; ++k) {
        const int64_t i = g * 256 + k;
        s[k] = i < count ? level[i] : 0.0f;
      }
      level[g] = tree256(s);
    }
    count = nodes;
  }
  const float r = level[0];
  free(level);
  return r;
}

/* ------------------------------------------------------------ row ops
 * fp64 definitions of the row ops (no reference implementation exists). */
void orc_softmax_rows_f64(const uint16_t* x, double* y, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * cols;
    double m = -INFINITY;
    for (int64_t c = 0; c < cols; ++c) m = fmax(m, orc_bf16_to_f32(xr[c]));
    double s = 0.0;
    for (int64_t c = 0; c < cols; ++c) s += exp((double)orc_bf16_to_f32(xr[c]) - m);
    for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = exp((double)orc_bf16_to_f32(xr[c]) - m) / s;
  }
}

void orc_rmsnorm_rows_f64(const uint16_t* x, const uint16_t* w, double* y, int64_t rows, int64_t cols,
                          double eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * cols;
    double ss = 0.0;
    for (int64_t c = 0; c < cols; ++c) {
      const double v = orc_bf16_to_f32(xr[c]);
      ss += v * v;
    }
    const double inv = 1.0 / sqrt(ss / (double)cols + eps);
    for (int64_t c = 0; c < cols; ++c)
      y[r * cols + c] = (double)orc_bf16_to_f32(xr[c]) * inv * (double)orc_bf16_to_f32(w[c]);
  }
}

/* ------------------------------------------------------ FP8 block quant
 * amax = max |x| over the 128-element block (NaN ignored),
 * scale = amax / 448 (f32), inv = amax > 0 ? min(448 / amax, FLT_MAX) : 0,
 * code = e4m3_satfinite(x * inv) (one f32 rounding). */
void orc_fp8_quantize(const uint16_t* x, uint8_t* codes, float* scales, int64_t rows, int64_t cols) {
  const int64_t bpr = (cols + 127) / 128;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < bpr; ++b) {
      const int64_t c0 = b * 128, c1 = c0 + 128 < cols ? c0 + 128 : cols;
      float amax = 0.0f;
      for (int64_t c = c0; c < c1; ++c) amax = fmaxf(amax, fabsf(orc_bf16_to_f32(x[r * cols + c])));
      const float scale = amax / 448.0f;
      float inv = 0.0f;
      if (amax > 0.0f) {
        inv = 448.0f / amax;
        if (inv > FLT_MAX) inv = FLT_MAX;
      }
      scales[r * bpr + b] = scale;
      for (int64_t c = c0; c < c1; ++c) {
        const float v = orc_bf16_to_f32(x[r * cols + c]) * inv;
        codes[r * cols + c] = orc_f32_to_e4m3_satfinite(v);
      }
    }
  }
}

void orc_fp8_dequantize(const uint8_t* codes, const float* scales, uint16_t* y, int64_t rows, int64_t cols) {
  const int64_t bpr = (cols + 127) / 128;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const float v = orc_e4m3_to_f32(codes[r * cols + c]) * scales[r * bpr + c / 128];
      y[r * cols + c] = orc_f32_to_bf16_rn(v);
    }
}

/* ------------------------------------------- multi-threaded baselines
 * The same loops split over `threads` POSIX threads (contiguous chunks),
 * used to time the CPU baseline on all host cores. */
typedef struct {
  const void* a;
  const void* b;
  void* c;
  int64_t begin, end;
  int kind;
  double out_f;
  int64_t out_i;
  int32_t out_key;
} Job;

static void* run_job(void* p) {
  Job* j = (Job*)p;
  switch (j->kind) {
    case 0: { /* sequential f32 fold of a chunk */
      const float* x = (const float*)j->a;
      float acc = 0.0f;
      for (int64_t i = j->begin; i < j->end; ++i) acc += x[i];
      j->out_f = acc;
      break;
    }
    case 1: { /* i32 wrap sum */
      const int32_t* x = (const int32_t*)j->a;
      uint32_t acc = 0;
      for (int64_t i = j->begin; i < j->end; ++i) acc += (uint32_t)x[i];
      j->out_i = (int32_t)acc;
      break;
    }
    case 2: { /* argmax */
      const float* x = (const float*)j->a;
      int64_t best = -1;
      int32_t key = 0;
      for (int64_t i = j->begin; i < j->end; ++i) {
        const int32_t k = total_order_key(x[i]);
        if (best < 0 || k > key) { key = k; best = i; }
      }
      j->out_i = best;
      j->out_key = key;
      break;
    }
    case 3: { /* vectorAdd f32 */
      orc_vector_add_f32((const float*)j->a + j->begin, (const float*)j->b + j->begin, (float*)j->c + j->begin,
                         j->end - j->begin);
      break;
    }
    default:
      break;
  }
  return NULL;
}

static void run_parallel(Job* jobs, int threads) {
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, run_job, &jobs[t]);
  run_job(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
  free(tid);
}

static Job* split(const void* a, const void* b, void* c, int64_t n, int threads, int kind) {
  Job* jobs = (Job*)calloc((size_t)threads, sizeof(Job));
  for (int t = 0; t < threads; ++t) {
    jobs[t].a = a; jobs[t].b = b; jobs[t].c = c; jobs[t].kind = kind;
    jobs[t].begin = n * t / threads;
    jobs[t].end = n * (t + 1) / threads;
  }
  return jobs;
}

double orc_mt_sum_f32(const float* x, int64_t n, int threads) {
  if (threads < 1) threads = 1;
  Job* jobs = split(x, NULL, NULL, n, threads, 0);
  run_parallel(jobs, threads);
  double s = 0.0;
  for (int t = 0; t < threads; ++t) s += jobs[t].out_f;
  free(jobs);
  return s;
}

int32_t orc_mt_sum_i32(const int32_t* x, int64_t n, int threads) {
  if (threads < 1) threads = 1;
  Job* jobs = split(x, NULL, NULL, n, threads, 1);
  run_parallel(jobs, threads);
  uint32_t s = 0;
  for (int t = 0; t < threads; ++t) s += (uint32_t)jobs[t].out_i;
  free(jobs);
  return (int32_t)s;
}

int64_t orc_mt_argmax_f32(const float* x, int64_t n, int threads) {
  if (threads < 1) threads = 1;
  Job* jobs = split(x, NULL, NULL, n, threads, 2);
  run_parallel(jobs, threads);
  int64_t best = -1;
  int32_t key = 0;
  for (int t = 0; t < threads; ++t) {
    if (jobs[t].out_i >= 0 && (best < 0 || jobs[t].out_key > key)) {
      key = jobs[t].out_key;
      best = jobs[t].out_i;
    }
  }
  free(jobs);
  return best;
}

void orc_mt_vector_add_f32(const float* a, const float* b, float* c, int64_t n, int threads) {
  if (threads < 1) threads = 1;
  Job* jobs = split(a, b, c, n, threads, 3);
  run_parallel(jobs, threads);
  free(jobs);
}
