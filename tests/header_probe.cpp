// header_probe.cpp -- compiled by tests/test_headers.py (with g++ and with
// nvcc) to check that include/tensor_bridge/*.h, the source-compatible
// primitives, give bit-identical results to the reference on host code.
#include <cstddef>
#include <cstdint>
#include "tensor_bridge/fp8.h"
#include "tensor_bridge/fp4.h"
#include "tensor_bridge/bf16.h"
#include "tensor_bridge/tf32.h"

using namespace tensor_bridge;

extern "C" {

void p_e4m3_to_half(const uint8_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_bits(fp8_e4m3_to_half(in[i]));
}
void p_e5m2_to_half(const uint8_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_bits(fp8_e5m2_to_half(in[i]));
}
void p_fp4_to_half(const uint8_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_bits(fp4_e2m1_to_half(in[i]));
}
void p_fp4_byte_to_half2(const uint8_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        const half2 h = fp4_e2m1_byte_to_half2(in[i]);
        out[2 * i] = half_to_bits(h.x);
        out[2 * i + 1] = half_to_bits(h.y);
    }
}
void p_bf16_to_half(const uint16_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_bits(bf16_to_half(in[i]));
}
void p_tf32_to_half(const uint32_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_bits(tf32_to_half(in[i]));
}
void p_fp32_to_e4m3(const float* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_fp8_e4m3(in[i]);
}
void p_fp32_to_e5m2(const float* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_fp8_e5m2(in[i]);
}
void p_fp32_to_e2m1(const float* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_fp4_e2m1(in[i]);
}
void p_half_to_e2m1(const uint16_t* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_fp4_e2m1(bits_to_half(in[i]));
}
void p_fp32_to_bf16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_bf16(in[i]);
}
void p_half_to_bf16(const uint16_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = half_to_bf16(bits_to_half(in[i]));
}
void p_fp32_to_tf32(const float* in, uint32_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_tf32(in[i]);
}
// Scale helpers: quantize(v * scale) and dequant(q) = decode(q) / scale.
void p_e4m3_scaled(const float* in, uint8_t* out, size_t n, float scale) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_fp8_e4m3_scaled(in[i], scale);
}
void p_e4m3_dequant(const uint8_t* in, float* out, size_t n, float scale) {
    for (size_t i = 0; i < n; ++i) out[i] = fp8_e4m3_dequant(in[i], scale);
}
void p_e2m1_scaled(const float* in, uint8_t* out, size_t n, float scale) {
    for (size_t i = 0; i < n; ++i) out[i] = fp32_to_fp4_e2m1_scaled(in[i], scale);
}
void p_e2m1_dequant(const uint8_t* in, float* out, size_t n, float scale) {
    for (size_t i = 0; i < n; ++i) out[i] = fp4_e2m1_dequant(in[i], scale);
}

}  // extern "C"
