/*
 * tensor_bridge/bf16.h -- BF16 <-> FP16 conversion primitives.
 *
 * Source-compatible with tensor-bridge's include/tensor_bridge/bf16.h: same
 * names and bit-exact results for every input.
 *
 * BF16 (bias 127, 7-bit mantissa) -> FP16 (bias 15, 10-bit mantissa), as in
 * bf16.h:22-34 of the reference:
 *   - re-bias the exponent by -112 and shift the mantissa up 3 bits;
 *   - a re-biased exponent <= 0 (every BF16 value below 2^-14, subnormals
 *     included) becomes a signed zero;
 *   - a re-biased exponent >= 31 becomes a signed Inf, except that a BF16 NaN
 *     becomes the quiet FP16 NaN 0x7E00 with the sign kept.
 * FP32 -> BF16 (bf16.h:37-48): add 0x7FFF plus the kept LSB, keep the top 16
 * bits (round-to-nearest-even); Inf and NaN are truncated, so a NaN whose
 * payload lies only in the low 16 bits becomes Inf.
 */
#ifndef TENSOR_BRIDGE_BF16_H
#define TENSOR_BRIDGE_BF16_H

#include "tensor_bridge/common.h"

namespace tensor_bridge {

TB_HD uint16_t bf16_to_half_bits(uint16_t bf) {
    const uint16_t s = bf & 0x8000u;
    const uint32_t ebf = (bf >> 7) & 0xFFu;
    const int e = static_cast<int>(ebf) - 112;
    if (e <= 0) return s;
    if (e >= 31) return s | ((ebf == 0xFFu && (bf & 0x7Fu)) ? 0x7E00u : 0x7C00u);
    return static_cast<uint16_t>(s | (e << 10) | ((bf & 0x7Fu) << 3));
}

TB_HD half bf16_to_half(uint16_t bf) { return bits_to_half(bf16_to_half_bits(bf)); }

TB_HD uint16_t fp32_to_bf16(float v) {
    uint32_t u = f2u(v);
    if ((u & 0x7F800000u) != 0x7F800000u) u += 0x7FFFu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

// FP16 -> BF16 through FP32 (bf16.h:53-55).
TB_HD uint16_t half_to_bf16(half h) { return fp32_to_bf16(__half2float(h)); }

// BF16 bits -> FP32 (exact widening).
TB_HD float bf16_to_fp32(uint16_t bf) { return u2f(static_cast<uint32_t>(bf) << 16); }

}  // namespace tensor_bridge

#endif  // TENSOR_BRIDGE_BF16_H
