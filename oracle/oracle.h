/* CPU oracle for the flight4s hot path (test infrastructure only; see oracle.c). */
#ifndef FLIGHT4S_ORACLE_H_
#define FLIGHT4S_ORACLE_H_

#include <stdint.h>

void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
void orc_fill_uniform_f32(float* out, uint64_t n, uint64_t offset, uint64_t seed, uint32_t stream);
void orc_fill_uniform_i32(int32_t* out, uint64_t n, uint64_t offset, uint64_t seed, uint32_t stream,
                          int32_t lo, int32_t hi);

uint16_t orc_f32_to_bf16_rn(float f);
float orc_bf16_to_f32(uint16_t b);
uint8_t orc_f32_to_e4m3_satfinite(float f);
float orc_e4m3_to_f32(uint8_t c);
float orc_e5m2_to_f32(uint8_t c);
float orc_f16_to_f32(uint16_t h);
int orc_decode_to_f32(int type_code, const void* x, int64_t n, float* out);
uint16_t orc_f32_to_f16(float f, int rounding);
uint16_t orc_f32_to_bf16(float f, int rounding);
uint8_t orc_f32_to_e4m3(float f, int saturate);
uint8_t orc_f32_to_e5m2(float f, int saturate);
int orc_convert(int from, int to, int rounding, int saturation, const void* in, void* out, int64_t n);
double orc_sum_typed_exactish(int type_code, const void* x, int64_t n, double* abs_sum);
uint32_t orc_sum_u32(const uint32_t* x, int64_t n);
int orc_vector_add_typed(int type_code, const void* a, const void* b, void* c, int64_t n);
int64_t orc_argmax_typed(int type_code, const void* x, int64_t n, int64_t* key_out);
double orc_ordered_final(const double* groups, int64_t count);
double orc_sum_ordered(int type_code, const void* x, int64_t n, int64_t head, double* groups_out,
                       int64_t* ngroups_out);

void orc_vector_add_f32(const float* a, const float* b, float* c, int64_t n);
void orc_vector_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* c, int64_t n);

float orc_sum_f32_sequential(const float* x, int64_t n);
float orc_sum_f32_sequential_from(const float* x, int64_t n, float acc);
double orc_sum_f32_exactish(const float* x, int64_t n, double* abs_sum);
int32_t orc_sum_i32(const int32_t* x, int64_t n);
int64_t orc_argmax_f32(const float* x, int64_t n, float* max_value);
int64_t orc_argmax_packed_key(float value, int64_t index);
float orc_block_tree_sum_f32(const float* x, int64_t n, float* partials);

void orc_softmax_rows_f64(const uint16_t* x, double* y, int64_t rows, int64_t cols);
void orc_rmsnorm_rows_f64(const uint16_t* x, const uint16_t* w, double* y, int64_t rows, int64_t cols,
                          double eps);
void orc_fp8_quantize(const uint16_t* x, uint8_t* codes, float* scales, int64_t rows, int64_t cols);
void orc_fp8_dequantize(const uint8_t* codes, const float* scales, uint16_t* y, int64_t rows, int64_t cols);

double orc_mt_sum_f32(const float* x, int64_t n, int threads);
int32_t orc_mt_sum_i32(const int32_t* x, int64_t n, int threads);
int64_t orc_mt_argmax_f32(const float* x, int64_t n, int threads);
void orc_mt_vector_add_f32(const float* a, const float* b, float* c, int64_t n, int threads);

#endif
