// tb_decode.cuh -- vectorised, bit-exact decoders from the stored formats to
// FP16, used by the streaming decode kernels and by the decode warps of the
// fused GEMM.  Every function reproduces the reference primitive of its format
// (include/tensor_bridge/{fp8,fp4,bf16,tf32}.h of tensor-bridge) on every
// input bit pattern; the exhaustive decode tests compare them code by code.
//
// Output packing: a uint32_t holds two FP16 values, the lower-addressed
// (earlier) element in the low 16 bits, so words can be stored as-is.
#pragma once

#include <cstdint>
#include "tensor_bridge/fp8.h"
#include "tensor_bridge/fp4.h"
#include "tensor_bridge/bf16.h"
#include "tensor_bridge/tf32.h"

namespace tb {

// prmt.b32 in its default mode.  Each selector nibble picks byte [2:0] of the
// pair {b, a} (a = bytes 0-3); if bit 3 of the nibble is set the byte's sign
// bit is replicated instead (0x00 or 0xFF).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Two E4M3 codes (low byte = first) -> two FP16 values by the hardware
// converter.  Exact for every code whose exponent field is non-zero and that
// is not a NaN; the callers route the other codes through the scalar path.
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint16_t pair) {
    uint32_t r;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(pair));
    return r;
}

__device__ __forceinline__ uint32_t pack2(uint16_t lo, uint16_t hi) {
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// ---- E4M3 --------------------------------------------------------------------------

// Bit 7 of each byte set where the E4M3 code is not reproduced by the
// hardware converter alone: exponent field 0 with a non-zero mantissa (a
// subnormal, flushed by the reference) or magnitude 0x7F (NaN, which the
// reference encodes as sign | 0x7E00).  With m = code & 0x7F (no byte carries
// out of its lane): m + 0x7F has bit 7 iff m >= 1;  m + 0x78 iff m >= 8;
// m + 0x01 iff m == 0x7F.
__device__ __forceinline__ uint32_t e4m3_special_bits(uint32_t w) {
    const uint32_t m = w & 0x7F7F7F7Fu;
    const uint32_t ge1 = m + 0x7F7F7F7Fu, ge8 = m + 0x78787878u, nan = m + 0x01010101u;
    return (ge1 & ~ge8) | nan;  // only bit 7 of each byte is meaningful
}
__device__ __forceinline__ uint32_t e4m3_special_mask(uint32_t w) { return e4m3_special_bits(w) & 0x80808080u; }

// Bit 7 of each byte set where the code is a NaN (magnitude 0x7F).
__device__ __forceinline__ uint32_t e4m3_nan_bits(uint32_t w) {
    return ((w & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u;
}

// Four E4M3 codes (byte 0 first) -> four FP16 values in o0, o1.  Fast path:
// valid when e4m3_special_mask(w) == 0.
__device__ __forceinline__ void decode_e4m3_x4_fast(uint32_t w, uint32_t& o0, uint32_t& o1) {
    o0 = cvt_e4m3x2(static_cast<uint16_t>(w & 0xFFFFu));
    o1 = cvt_e4m3x2(static_cast<uint16_t>(w >> 16));
}

// Valid for every code but NaN (e4m3_nan_bits(w) == 0): the converter's
// result with the codes whose exponent field is zero masked to a signed zero
// (the converter keeps the code's sign in bit 15).  Bit 7 of each byte of
// (w & 0x78787878) + 0x78787878 is set iff that code's exponent field is
// non-zero; prmt replicates it over the code's FP16 lane.
__device__ __forceinline__ void decode_e4m3_x4_flush(uint32_t w, uint32_t& o0, uint32_t& o1) {
    const uint32_t nz = (w & 0x78787878u) + 0x78787878u;
    o0 = cvt_e4m3x2(static_cast<uint16_t>(w & 0xFFFFu)) & (prmt(nz, 0u, 0x9988u) | 0x80008000u);
    o1 = cvt_e4m3x2(static_cast<uint16_t>(w >> 16)) & (prmt(nz, 0u, 0xBBAAu) | 0x80008000u);
}

// Scalar path: the reference rule code by code (valid for every code).
__device__ __forceinline__ void decode_e4m3_x4_scalar(uint32_t w, uint32_t& o0, uint32_t& o1) {
    using tensor_bridge::e4m3_to_half_bits;
    o0 = pack2(e4m3_to_half_bits(w & 0xFFu), e4m3_to_half_bits((w >> 8) & 0xFFu));
    o1 = pack2(e4m3_to_half_bits((w >> 16) & 0xFFu), e4m3_to_half_bits(w >> 24));
}

__device__ __forceinline__ void decode_e4m3_x4(uint32_t w, uint32_t& o0, uint32_t& o1) {
    if (e4m3_special_mask(w) == 0u) decode_e4m3_x4_fast(w, o0, o1);
    else if (e4m3_nan_bits(w) == 0u) decode_e4m3_x4_flush(w, o0, o1);
    else decode_e4m3_x4_scalar(w, o0, o1);
}

// For operands that only feed a tensor core whose accumulators are scaled
// back by 2^8 (GemmArgs::acc_shift): the reference decoder's value of every
// code times 2^-8, with no branch.  The hardware converter gives every code's
// exact value (subnormal codes included); the multiplication by 2^-8 with
// flush-to-zero is exact for the normal codes (at least 2^-6, which land at
// 2^-14 or above) and sends the subnormal codes (below 2^-6) under FP16's
// normal range, where .ftz makes them the signed zero the reference decoder
// gives them.  A NaN code becomes an FP16 NaN of another payload than the
// reference's 0x7E00 | sign, which changes nothing downstream: any product
// with it is NaN.  Scaling every product by 2^-8 and the FP32 sum back by 2^8
// is exact (no product of an FP16 value at least 2^-14 with an FP16 operand
// comes near FP32's subnormal range), so D does not change.
__device__ __forceinline__ void decode_e4m3_x4_scaled(uint32_t w, uint32_t& o0, uint32_t& o1) {
    uint32_t h0, h1;
    decode_e4m3_x4_fast(w, h0, h1);
    asm("mul.rn.ftz.f16x2 %0, %1, %2;" : "=r"(o0) : "r"(h0), "r"(0x1C001C00u));  // 2^-8 in both halves
    asm("mul.rn.ftz.f16x2 %0, %1, %2;" : "=r"(o1) : "r"(h1), "r"(0x1C001C00u));
}
constexpr int kE4M3AccShift = 8;

// ---- E5M2: each code is the top byte of its FP16 value -------------------------------

__device__ __forceinline__ void decode_e5m2_x4(uint32_t w, uint32_t& o0, uint32_t& o1) {
    o0 = prmt(w, 0u, 0x1404u);  // bytes {0, b0, 0, b1}
    o1 = prmt(w, 0u, 0x3424u);  // bytes {0, b2, 0, b3}
}

// ---- E2M1 ----------------------------------------------------------------------------
// Every E2M1 value (0, 0.5, 1, 1.5, 2, 3, 4, 6 and their negatives, code 8
// being -0) is an FP16 value, so the hardware conversion reproduces the
// reference table (fp4.h:27-30) code for code.

// Four bytes, each holding two E2M1 codes -> four FP16 pairs by the hardware
// converter (cvt.rn.f16x2.e2m1x2: the low nibble of a byte becomes the low
// half).  Exact for all 16 codes (code 8 is -0, as the reference table).
__device__ __forceinline__ void cvt_e2m1x2_x4(uint32_t w, uint32_t (&o)[4]) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
        : "r"(w));
}

// Packed, reference order: byte j holds element 2j in its HIGH nibble and
// element 2j+1 in its low nibble.  Eight elements -> o[0..3]: swap the
// nibbles of every byte (element 2j to the low half), then convert.
__device__ __forceinline__ void decode_e2m1_packed_x8(uint32_t w, uint32_t (&o)[4]) {
    cvt_e2m1x2_x4(((w >> 4) & 0x0F0F0F0Fu) | ((w << 4) & 0xF0F0F0F0u), o);
}

// Unpacked (one value per byte, low nibble; high nibble ignored as in the
// reference's `nibble & 0x0F`).  Four elements -> o0, o1.
__device__ __forceinline__ void decode_e2m1_unpacked_x4(uint32_t w, uint32_t& o0, uint32_t& o1) {
    const uint32_t t = w & 0x0F0F0F0Fu;
    // byte 0 = code1 << 4 | code0, byte 2 = code3 << 4 | code2
    uint32_t o[4];
    cvt_e2m1x2_x4(t | (t >> 4), o);
    o0 = o[0];
    o1 = o[2];
}

// Tensor-core packing (element 2j in the LOW nibble): a nibble swap of the
// reference order.
__device__ __forceinline__ uint32_t swap_nibbles(uint32_t w) {
    return ((w >> 4) & 0x0F0F0F0Fu) | ((w << 4) & 0xF0F0F0F0u);
}

// ---- BF16 ---------------------------------------------------------------------------

// Two FP16 values times 1 with flush-to-zero: a subnormal becomes the zero of
// its sign, every other value (zeros, normals, Inf) is unchanged.
__device__ __forceinline__ uint32_t f16x2_flush_subnormal(uint32_t h) {
    uint32_t r;
    asm("mul.rn.ftz.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x3C003C00u));
    return r;
}

// Two BF16 values (low lane first) -> two FP16 values.  Fast path: widen to
// FP32 (exact), convert with the hardware FP32->FP16x2 converter (exact for
// BF16 values in FP16 range, Inf beyond, as the reference), then flush FP16
// subnormal results to a signed zero (the reference maps every BF16 value
// below 2^-14 to zero; no BF16 value below 2^-14 rounds up to 2^-14).  BF16
// NaN lanes take the scalar path (the reference encodes them as 0x7E00).
__device__ __forceinline__ uint32_t bf16_nan_lanes(uint32_t w) {
    return ((w & 0x7FFF7FFFu) + 0x007F007Fu) & 0x80008000u;
}

__device__ __forceinline__ uint32_t decode_bf16_x2_scalar(uint32_t w) {
    return pack2(tensor_bridge::bf16_to_half_bits(w & 0xFFFFu), tensor_bridge::bf16_to_half_bits(w >> 16));
}

// Fast path, valid when bf16_nan_lanes(w) == 0.
__device__ __forceinline__ uint32_t decode_bf16_x2_fast(uint32_t w) {
    const float lo = __uint_as_float(w << 16);
    const float hi = __uint_as_float(w & 0xFFFF0000u);
    uint32_t h;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
    return f16x2_flush_subnormal(h);
}

__device__ __forceinline__ uint32_t decode_bf16_x2(uint32_t w) {
    return bf16_nan_lanes(w) != 0u ? decode_bf16_x2_scalar(w) : decode_bf16_x2_fast(w);
}

// ---- TF32 ---------------------------------------------------------------------------

// One TF32 word -> FP16 bits, the reference rule (tf32.h:22-34) written with
// selects: re-biased exponent <= 0 -> signed zero, >= 31 -> Inf or NaN.
__device__ __forceinline__ uint32_t decode_tf32_x1(uint32_t t) {
    const uint32_t s = (t >> 16) & 0x8000u;
    const uint32_t mag = t & 0x7FFFFFFFu;
    uint32_t h = (mag >> 13) - (112u << 10);          // valid when 113 <= exp <= 142
    h = mag < (113u << 23) ? 0u : h;                  // exponent - 112 <= 0
    const uint32_t big = mag > 0x7F800000u ? 0x7E00u : 0x7C00u;
    h = mag >= (143u << 23) ? big : h;                // exponent - 112 >= 31
    return s | h;
}

__device__ __forceinline__ uint32_t decode_tf32_x2_scalar(uint32_t t0, uint32_t t1) {
    return decode_tf32_x1(t0) | (decode_tf32_x1(t1) << 16);
}

// Largest magnitude of a pair; at or above 2^16 (0x47800000, which includes
// Inf and NaN) a word needs the scalar path.
__device__ __forceinline__ uint32_t tf32_max_mag(uint32_t t0, uint32_t t1) {
    return max(t0 & 0x7FFFFFFFu, t1 & 0x7FFFFFFFu);
}
constexpr uint32_t kTf32ScalarFrom = 143u << 23;

// Fast path, valid when both magnitudes are below 2^16.  Converting with
// round-toward-zero drops the 13 low bits exactly as the reference's
// truncation does and cannot round a value below 2^-14 up into the normal
// range; FP16 subnormal results are then flushed to a signed zero (the
// reference flushes every value below 2^-14).
__device__ __forceinline__ uint32_t decode_tf32_x2_fast(uint32_t t0, uint32_t t1) {
    uint32_t h;
    asm("cvt.rz.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(__uint_as_float(t1)), "f"(__uint_as_float(t0)));
    return f16x2_flush_subnormal(h);
}

__device__ __forceinline__ uint32_t decode_tf32_x2(uint32_t t0, uint32_t t1) {
    return tf32_max_mag(t0, t1) >= kTf32ScalarFrom ? decode_tf32_x2_scalar(t0, t1) : decode_tf32_x2_fast(t0, t1);
}

}  // namespace tb
