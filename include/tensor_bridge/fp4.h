/*
 * tensor_bridge/fp4.h -- FP4 E2M1 <-> FP16 conversion primitives.
 *
 * Source-compatible with tensor-bridge's include/tensor_bridge/fp4.h: same
 * names and bit-exact results.  Additions: the decode is also callable from
 * host code (the reference's is device-only, fp4.h:33-43), and packed-byte
 * helpers in both directions.
 *
 * E2M1: 1 sign, 2 exponent (bias 1), 1 mantissa.  A nibble [s e1 e0 m0]
 * encodes +-{0, 0.5, 1, 1.5, 2, 3, 4, 6}; there is no Inf or NaN.  Code 8 is
 * -0 (FP16 0x8000).
 *
 * Packed storage (fp4.h:37-43): two values per byte, the FIRST value in the
 * HIGH nibble and the second in the low nibble.
 *
 * Quantize semantics (fp4.h:46-53): nearest of the 8 magnitudes by a linear
 * scan with a strict '<' in FP32 arithmetic, so ties go to the smaller
 * magnitude (0.25 -> 0, 2.5 -> 2, 5 -> 4); the sign bit is set only for v < 0
 * (so -0 and NaN give code 0); values so large that every FP32 distance
 * |v| - g rounds to the same number (above about 2^27, and Inf) give
 * magnitude code 0.
 */
#ifndef TENSOR_BRIDGE_FP4_H
#define TENSOR_BRIDGE_FP4_H

#include "tensor_bridge/common.h"

namespace tensor_bridge {

// FP16 bit patterns of the 16 E2M1 codes.  Every entry has a zero low byte.
constexpr uint16_t kFp4E2M1HalfBits[16] = {
    0x0000, 0x3800, 0x3C00, 0x3E00, 0x4000, 0x4200, 0x4400, 0x4600,
    0x8000, 0xB800, 0xBC00, 0xBE00, 0xC000, 0xC200, 0xC400, 0xC600,
};

#if defined(__CUDACC__)
// Reference-named device table (fp4.h:27-30), declared as the reference
// declares it (external linkage, so a translation unit that extern-declares
// the table links against it).  Kept for source compatibility; the
// conversion functions below do not read it.
__device__ __constant__ unsigned short kFp4E2M1LUT[16] = {
    0x0000, 0x3800, 0x3C00, 0x3E00, 0x4000, 0x4200, 0x4400, 0x4600,
    0x8000, 0xB800, 0xBC00, 0xBE00, 0xC000, 0xC200, 0xC400, 0xC600,
};
#endif

// E2M1 nibble -> FP16 bits, computed (no table): magnitude code c >= 2 maps to
// (c << 9) + 0x3800; c = 1 is 0.5 (0x3800); c = 0 is zero.
TB_HD uint16_t e2m1_to_half_bits(uint8_t nibble) {
    const uint16_t c = nibble & 0x7u;
    const uint16_t s = static_cast<uint16_t>(nibble & 0x8u) << 12;
    const uint16_t mag = c >= 2 ? static_cast<uint16_t>((c << 9) + 0x3800u)
                                : static_cast<uint16_t>(c ? 0x3800u : 0u);
    return s | mag;
}

// FP4 nibble (low 4 bits of the argument) -> FP16.  Host and device.
TB_HD half fp4_e2m1_to_half(uint8_t nibble) { return bits_to_half(e2m1_to_half_bits(nibble & 0x0Fu)); }

// Packed byte -> two FP16 values: .x from the high nibble (first element),
// .y from the low nibble (second element).
TB_HD half2 fp4_e2m1_byte_to_half2(uint8_t packed) {
    half2 r;
    r.x = fp4_e2m1_to_half(static_cast<uint8_t>(packed >> 4));
    r.y = fp4_e2m1_to_half(static_cast<uint8_t>(packed & 0x0Fu));
    return r;
}

// FP32 -> E2M1 nibble, nearest-of-8 magnitudes as in fp4.h:46-53.
TB_HD uint8_t fp32_to_fp4_e2m1(float v) {
    const float grid[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const uint8_t neg = v < 0.0f ? 1u : 0u;
    const float a = fabsf(v);
    uint8_t pick = 0;
    float best = fabsf(a - grid[0]);
    for (int i = 1; i < 8; ++i) {
        const float d = fabsf(a - grid[i]);
        if (d < best) { best = d; pick = static_cast<uint8_t>(i); }
    }
    return static_cast<uint8_t>((neg << 3) | pick);
}

// FP16 -> E2M1 nibble (fp4.h:58-60): widen to FP32 and quantize.
TB_HD uint8_t half_to_fp4_e2m1(half h) { return fp32_to_fp4_e2m1(__half2float(h)); }

// Two nibbles -> one packed byte in the reference order (first in high nibble).
TB_HD uint8_t fp4_e2m1_pack(uint8_t first, uint8_t second) {
    return static_cast<uint8_t>(((first & 0x0Fu) << 4) | (second & 0x0Fu));
}

// ---- per-tensor scale helpers ------------------------------------------------
constexpr float kE2M1Max = 6.0f;

TB_HD uint8_t fp32_to_fp4_e2m1_scaled(float v, float scale) { return fp32_to_fp4_e2m1(v * scale); }
TB_HD float fp4_e2m1_dequant(uint8_t q, float scale) { return __half2float(fp4_e2m1_to_half(q)) / scale; }

}  // namespace tensor_bridge

#endif  // TENSOR_BRIDGE_FP4_H
