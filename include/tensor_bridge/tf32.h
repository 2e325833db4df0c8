/*
 * tensor_bridge/tf32.h -- TF32 <-> FP16 conversion primitives.
 *
 * Source-compatible with tensor-bridge's include/tensor_bridge/tf32.h: same
 * names and bit-exact results for every input.
 *
 * A TF32 value is carried in a 32-bit word laid out like FP32 (sign, 8-bit
 * exponent with bias 127, mantissa) whose low 13 mantissa bits are normally
 * zero.  TF32 -> FP16 (tf32.h:22-34): re-bias by -112, keep mantissa bits
 * 22..13; a re-biased exponent <= 0 gives a signed zero; >= 31 gives a signed
 * Inf, or the quiet NaN 0x7E00 (sign kept) when the word is a NaN (the NaN
 * test looks at all 23 mantissa bits).
 * FP32 -> TF32 (tf32.h:37-44): Inf/NaN are masked to the TF32 bits, otherwise
 * add 0xFFF plus the kept LSB and mask (round-to-nearest-even).
 */
#ifndef TENSOR_BRIDGE_TF32_H
#define TENSOR_BRIDGE_TF32_H

#include "tensor_bridge/common.h"

namespace tensor_bridge {

TB_HD uint16_t tf32_to_half_bits(uint32_t t) {
    const uint16_t s = static_cast<uint16_t>((t >> 16) & 0x8000u);
    const uint32_t et = (t >> 23) & 0xFFu;
    const int e = static_cast<int>(et) - 112;
    if (e <= 0) return s;
    if (e >= 31) return s | ((et == 0xFFu && (t & 0x7FFFFFu)) ? 0x7E00u : 0x7C00u);
    return static_cast<uint16_t>(s | (e << 10) | ((t >> 13) & 0x3FFu));
}

TB_HD half tf32_to_half(uint32_t tf32) { return bits_to_half(tf32_to_half_bits(tf32)); }

TB_HD uint32_t fp32_to_tf32(float v) {
    uint32_t u = f2u(v);
    if ((u & 0x7F800000u) != 0x7F800000u) u += 0xFFFu + ((u >> 13) & 1u);
    return u & 0xFFFFE000u;
}

}  // namespace tensor_bridge

#endif  // TENSOR_BRIDGE_TF32_H
