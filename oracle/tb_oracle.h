/*
 * tb_oracle.h -- CPU oracle for the decode + GEMM path.  TEST INFRASTRUCTURE
 * ONLY (tests, smoke check, bench CPU baseline); see tb_oracle.c.
 */
#ifndef TB_ORACLE_H
#define TB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same numbering as tb_format in include/tensor_bridge_b200.h. */
enum {
    ORACLE_F16 = 0,
    ORACLE_E4M3 = 1,
    ORACLE_E5M2 = 2,
    ORACLE_E2M1 = 3,          /* packed, first value in the high nibble */
    ORACLE_E2M1_UNPACKED = 4, /* one value per byte */
    ORACLE_BF16 = 5,
    ORACLE_TF32 = 6,
    ORACLE_E2M1_HW = 7        /* packed, first value in the low nibble */
};

uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);

uint16_t oracle_e4m3_to_f16(uint8_t c);
uint16_t oracle_e5m2_to_f16(uint8_t c);
uint16_t oracle_e2m1_to_f16(uint8_t nibble);
uint16_t oracle_bf16_to_f16(uint16_t bf);
uint16_t oracle_tf32_to_f16(uint32_t t);

uint8_t oracle_f32_to_e4m3(float v);
uint8_t oracle_f32_to_e5m2(float v);
uint8_t oracle_f32_to_e2m1(float v);
uint16_t oracle_f32_to_bf16(float v);
uint32_t oracle_f32_to_tf32(float v);

uint16_t oracle_decode_one(int fmt, const void* src, size_t i);
void oracle_decode(int fmt, const void* src, uint16_t* dst, size_t n);
void oracle_quantize(int fmt, const float* src, void* dst, size_t n, float scale);
void oracle_gemm(int a_fmt, const void* A, int b_fmt, const void* B, void* D, int M, int N, int K, int row0, int row1,
                 float alpha, int out_f16, int nthreads);

/* INT8 path (src/gemm.cu:35-41, 58-70). */
int8_t oracle_e4m3_to_i8(uint8_t c, float scale);
void oracle_decode_e4m3_i8(const uint8_t* src, int8_t* dst, size_t n, float scale);
void oracle_gemm_i8(const int8_t* A, const int8_t* B, int32_t* D, int M, int N, int K, int nthreads);
float oracle_e4m3_scale_to_f32(uint8_t s);
uint16_t oracle_nvfp4_at(const uint8_t* q, const uint8_t* scales, size_t i);
void oracle_decode_nvfp4(const uint8_t* q, const uint8_t* scales, uint16_t* dst, size_t n);

#ifdef __cplusplus
}
#endif

#endif
