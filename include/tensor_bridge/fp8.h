/*
 * tensor_bridge/fp8.h -- FP8 (E4M3 / E5M2) <-> FP16 conversion primitives.
 *
 * Source-compatible with tensor-bridge's include/tensor_bridge/fp8.h: same
 * names, signatures and bit-exact results for every input.
 *
 *   E4M3 (NVIDIA "fn" flavour): 1 sign, 4 exponent (bias 7), 3 mantissa.
 *     No infinities; exponent 15 with mantissa 7 is NaN; max finite 448.
 *   E5M2: 1 sign, 5 exponent (bias 15), 2 mantissa -- the top byte of an FP16.
 *
 * Decode semantics pinned by the reference (fp8.h:23-39):
 *   - E4M3 codes with exponent field 0 (zero *and* subnormals) decode to a
 *     signed zero: subnormals are flushed.
 *   - E4M3 0x7F / 0xFF decode to the quiet FP16 NaN 0x7E00 with the sign kept.
 *   - E5M2 is a pure field shift; FP16 Inf/NaN patterns pass through.
 * Quantize semantics (fp8.h:43-81): clamp to the format max, round to FP16
 * with round-to-nearest-even, then round the FP16 mantissa to 3 (2) bits with
 * round-to-nearest-even again (so a value can be double rounded), flush
 * results below the smallest normal to a signed zero, saturate at the max.
 */
#ifndef TENSOR_BRIDGE_FP8_H
#define TENSOR_BRIDGE_FP8_H

#include "tensor_bridge/common.h"

namespace tensor_bridge {

// ---- decode, raw-bit forms (host + device) ----------------------------------

// E4M3 byte -> FP16 bits.  Follows fp8.h:23-31 of the reference.
TB_HD uint16_t e4m3_to_half_bits(uint8_t code) {
    const uint16_t s = static_cast<uint16_t>(code & 0x80u) << 8;
    const uint16_t mag = code & 0x7Fu;
    if ((mag >> 3) == 0) return s;                 // exponent 0: flush to +-0
    if (mag == 0x7Fu) return s | 0x7E00u;          // exponent 15, mantissa 7: NaN
    // exponent field E (bias 7) becomes E + 8 (bias 15); mantissa moves up 7.
    return s | static_cast<uint16_t>((mag << 7) + (8u << 10));
}

// E5M2 byte -> FP16 bits.  Follows fp8.h:34-39: the byte is the FP16 top byte.
TB_HD uint16_t e5m2_to_half_bits(uint8_t code) {
    return static_cast<uint16_t>(code) << 8;
}

// ---- decode, reference names -----------------------------------------------

TB_HD half fp8_e4m3_to_half(uint8_t f8) { return bits_to_half(e4m3_to_half_bits(f8)); }

TB_HD half fp8_e5m2_to_half(uint8_t f8) { return bits_to_half(e5m2_to_half_bits(f8)); }

// ---- quantize (host + device) ----------------------------------------------

namespace detail {
// Round an FP16 mantissa (10 bits) to `keep` bits, nearest-even on the dropped
// bits.  Returns the rounded mantissa, which may equal 1 << keep (a carry).
TB_HD uint16_t round_half_mantissa(uint16_t man10, int keep) {
    const int drop = 10 - keep;
    const uint16_t half_ulp = static_cast<uint16_t>(1u << (drop - 1));
    const uint16_t rest = man10 & static_cast<uint16_t>((1u << drop) - 1u);
    const uint16_t odd = (man10 >> drop) & 1u;
    const bool up = rest > half_ulp || (rest == half_ulp && odd);
    return static_cast<uint16_t>((man10 >> drop) + (up ? 1u : 0u));
}
}  // namespace detail

// FP32 -> E4M3.  Follows fp8.h:43-61: clamp to +-448 (a NaN input clamps to
// +448), FP16 round, mantissa round to 3 bits, flush below 2^-6, saturate.
TB_HD uint8_t fp32_to_fp8_e4m3(float v) {
    const float c = fmaxf(-448.0f, fminf(448.0f, v));
    const uint16_t h = half_to_bits(__float2half(c));
    const uint8_t s = static_cast<uint8_t>((h >> 8) & 0x80u);
    uint16_t m = detail::round_half_mantissa(h & 0x3FFu, 3);
    int e = static_cast<int>((h >> 10) & 0x1Fu) - 8;  // bias 15 -> bias 7
    if (m >= 8u) { m = 0; ++e; }
    if (e <= 0) return s;
    if (e > 15) { e = 15; m = 6; }
    return static_cast<uint8_t>(s | (e << 3) | m);
}

// FP32 -> E5M2.  Follows fp8.h:64-81: clamp to +-57344, FP16 round, mantissa
// round to 2 bits, flush FP16 subnormals, exponent clamp at 31.
TB_HD uint8_t fp32_to_fp8_e5m2(float v) {
    const float c = fmaxf(-57344.0f, fminf(57344.0f, v));
    const uint16_t h = half_to_bits(__float2half(c));
    const uint8_t s = static_cast<uint8_t>((h >> 8) & 0x80u);
    uint16_t m = detail::round_half_mantissa(h & 0x3FFu, 2);
    int e = static_cast<int>((h >> 10) & 0x1Fu);
    if (m >= 4u) { m = 0; ++e; }
    if (e <= 0) return s;
    if (e >= 31) e = 31;
    return static_cast<uint8_t>(s | (e << 2) | m);
}

// ---- per-tensor scale helpers ------------------------------------------------
// The reference applies a per-tensor scale in its harness
// (bench/bench_formats.cu:128-132,164): scale = FORMAT_MAX / maxabs,
// q = Q(x * scale), and the GEMM result is divided by the scale.
constexpr float kE4M3Max = 448.0f;
constexpr float kE5M2Max = 57344.0f;

TB_HD uint8_t fp32_to_fp8_e4m3_scaled(float v, float scale) { return fp32_to_fp8_e4m3(v * scale); }
TB_HD uint8_t fp32_to_fp8_e5m2_scaled(float v, float scale) { return fp32_to_fp8_e5m2(v * scale); }
TB_HD float fp8_e4m3_dequant(uint8_t q, float scale) { return __half2float(fp8_e4m3_to_half(q)) / scale; }
TB_HD float fp8_e5m2_dequant(uint8_t q, float scale) { return __half2float(fp8_e5m2_to_half(q)) / scale; }

}  // namespace tensor_bridge

#endif  // TENSOR_BRIDGE_FP8_H
