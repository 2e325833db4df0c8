/*
 * tb_oracle.c -- CPU oracle for the decode + GEMM path.  TEST INFRASTRUCTURE
 * ONLY: the tests, the smoke check and the CPU-baseline leg of bench.py call
 * it to check or time the CUDA path; nothing in the product links it.
 *
 * A plain-C restatement of tensor-bridge's conversion primitives and of the
 * decode -> FP16 -> FP32-accumulate GEMM the reference runs.  Each function
 * names the reference lines it follows.  The restatement is pinned against the
 * reference itself: tests/golden holds tables generated from the reference's
 * own headers (oracle/ref_shim.cu, built into oracle/_ref), and the known-answer
 * vectors of tests/test_conversions.cu are replayed in tests/test_oracle.py.
 *
 * FP32 -> FP16 rounding (the reference calls CUDA's __float2half) is written
 * here from the IEEE 754 round-to-nearest-even rule.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "tb_oracle.h"

/* ---- FP16 helpers ----------------------------------------------------------- */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest, ties to even. */
uint16_t oracle_f32_to_f16(float f) {
    const uint32_t x = f2u(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t mag = x & 0x7FFFFFFFu;
    if (mag > 0x7F800000u) return (uint16_t)(sign | 0x7FFFu);  /* NaN */
    if (mag >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 (and Inf) -> Inf */
    if (mag < 0x38800000u) {                                   /* below 2^-14: subnormal result */
        if (mag <= 0x33000000u) return sign;                    /* <= 2^-25 rounds to zero */
        const uint32_t e = mag >> 23;
        const uint32_t m = (mag & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e;                         /* 14..24 */
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((((mag >> 23) - 112u) << 10) | ((mag & 0x7FFFFFu) >> 13));
    const uint32_t rem = mag & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
}

/* binary16 -> binary32 (exact).  Like CUDA's __half2float, which the
 * reference uses (bf16.h:54, fp4.h:59), every NaN becomes 0x7FFFFFFF. */
float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        const float v = (float)m * 5.9604644775390625e-8f; /* m * 2^-24, exact */
        return u2f(f2u(v) | sign);
    }
    if (e == 31) return m ? u2f(0x7FFFFFFFu) : u2f(sign | 0x7F800000u);
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* ---- decode (reference include/tensor_bridge/*.h) ---------------------------- */

/* fp8.h:23-31 */
uint16_t oracle_e4m3_to_f16(uint8_t c) {
    const uint16_t sign = (uint16_t)((c & 0x80u) << 8);
    const uint8_t e = (c >> 3) & 0x0Fu;
    const uint16_t m = (uint16_t)((c & 0x07u) << 7);
    if (e == 0) return sign;
    if (e == 15 && (c & 0x07u) == 0x07u) return (uint16_t)(sign | 0x7E00u);
    return (uint16_t)(sign | ((uint16_t)(e + 8) << 10) | m);
}

/* fp8.h:34-39 */
uint16_t oracle_e5m2_to_f16(uint8_t c) {
    return (uint16_t)(((uint16_t)(c & 0x80u) << 8) | ((uint16_t)((c >> 2) & 0x1Fu) << 10) | ((uint16_t)(c & 0x03u) << 8));
}

/* fp4.h:27-35 (the LUT, restated) */
static const uint16_t kE2M1[16] = {0x0000, 0x3800, 0x3C00, 0x3E00, 0x4000, 0x4200, 0x4400, 0x4600,
                                   0x8000, 0xB800, 0xBC00, 0xBE00, 0xC000, 0xC200, 0xC400, 0xC600};
uint16_t oracle_e2m1_to_f16(uint8_t nibble) { return kE2M1[nibble & 0x0Fu]; }

/* bf16.h:22-34 */
uint16_t oracle_bf16_to_f16(uint16_t bf) {
    const uint16_t sign = bf & 0x8000u;
    const int e = (int)((bf >> 7) & 0xFFu) - 112;
    const uint16_t m = (uint16_t)((bf & 0x7Fu) << 3);
    if (e <= 0) return sign;
    if (e >= 31) {
        if (((bf >> 7) & 0xFFu) == 0xFFu && (bf & 0x7Fu)) return (uint16_t)(sign | 0x7E00u);
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | (uint16_t)(e << 10) | m);
}

/* tf32.h:22-34 */
uint16_t oracle_tf32_to_f16(uint32_t t) {
    const uint16_t sign = (uint16_t)((t >> 16) & 0x8000u);
    const int e = (int)((t >> 23) & 0xFFu) - 112;
    const uint16_t m = (uint16_t)((t >> 13) & 0x3FFu);
    if (e <= 0) return sign;
    if (e >= 31) {
        if (((t >> 23) & 0xFFu) == 0xFFu && (t & 0x7FFFFFu)) return (uint16_t)(sign | 0x7E00u);
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | (uint16_t)(e << 10) | m);
}

/* ---- quantize -------------------------------------------------------------------- */

/* The reference clamps with fminf/fmaxf (fp8.h:44,65).  Its host build calls
 * glibc's, which follow IEEE 754-2008 minNum/maxNum: a quiet NaN operand yields
 * the other operand, a signaling NaN yields a quiet NaN.  Restated here so the
 * result does not depend on how this compiler folds the builtins. */
static int is_snan(float x) { const uint32_t u = f2u(x); return (u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu) && !(u & 0x400000u); }
static float min_num(float a, float b) {
    if (is_snan(a) || is_snan(b)) return u2f(0x7FC00000u);
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a < b ? a : b;
}
static float max_num(float a, float b) {
    if (is_snan(a) || is_snan(b)) return u2f(0x7FC00000u);
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* fp8.h:43-61 */
uint8_t oracle_f32_to_e4m3(float v) {
    const float clip = max_num(-448.0f, min_num(448.0f, v));
    const uint16_t u = oracle_f32_to_f16(clip);
    const uint16_t man = u & 0x03FFu;
    const uint16_t lsb = (man >> 7) & 1u, sticky = man & 0x007Fu;
    const uint16_t r = (sticky > 0x40u || (sticky == 0x40u && lsb)) ? 0x80u : 0u;
    uint16_t man3 = (uint16_t)((man + r) >> 7);
    const uint8_t sign = (uint8_t)((u >> 8) & 0x80u);
    int e = (int)((u >> 10) & 0x1Fu) - 15 + 7;
    if (man3 >= 8) { man3 = 0; e++; }
    if (e <= 0) return sign;
    if (e > 15) { e = 15; man3 = 6; }
    return (uint8_t)(sign | (uint8_t)(e << 3) | (uint8_t)man3);
}

/* fp8.h:64-81 */
uint8_t oracle_f32_to_e5m2(float v) {
    const float clip = max_num(-57344.0f, min_num(57344.0f, v));
    const uint16_t u = oracle_f32_to_f16(clip);
    const uint16_t man = u & 0x03FFu;
    const uint16_t lsb = (man >> 8) & 1u, sticky = man & 0x00FFu;
    const uint16_t r = (sticky > 0x80u || (sticky == 0x80u && lsb)) ? 0x100u : 0u;
    uint16_t man2 = (uint16_t)((man + r) >> 8);
    const uint8_t sign = (uint8_t)((u >> 8) & 0x80u);
    int e = (u >> 10) & 0x1Fu;
    if (man2 >= 4) { man2 = 0; e++; }
    if (e <= 0) return sign;
    if (e >= 31) e = 31;
    return (uint8_t)(sign | (uint8_t)(e << 2) | (uint8_t)man2);
}

/* fp4.h:46-53: nearest of 8 magnitudes, strict '<' so ties keep the smaller. */
uint8_t oracle_f32_to_e2m1(float v) {
    static const float vals[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const int sign = v < 0.0f ? 1 : 0;
    const float a = fabsf(v);
    int best = 0;
    float bd = fabsf(a - vals[0]);
    for (int i = 1; i < 8; i++) {
        const float d = fabsf(a - vals[i]);
        if (d < bd) { bd = d; best = i; }
    }
    return (uint8_t)((sign << 3) | best);
}

/* bf16.h:37-48 */
uint16_t oracle_f32_to_bf16(float v) {
    uint32_t u = f2u(v);
    if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)(u >> 16);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* tf32.h:37-44 */
uint32_t oracle_f32_to_tf32(float v) {
    uint32_t u = f2u(v);
    if ((u & 0x7F800000u) == 0x7F800000u) return u & 0xFFFFE000u;
    u += 0x00000FFFu + ((u >> 13) & 1u);
    return u & 0xFFFFE000u;
}

/* ---- array forms -------------------------------------------------------------------- */

uint16_t oracle_decode_one(int fmt, const void* src, size_t i) {
    switch (fmt) {
        case ORACLE_F16: return ((const uint16_t*)src)[i];
        case ORACLE_E4M3: return oracle_e4m3_to_f16(((const uint8_t*)src)[i]);
        case ORACLE_E5M2: return oracle_e5m2_to_f16(((const uint8_t*)src)[i]);
        case ORACLE_E2M1: {
            /* fp4.h:37-43: first value in the high nibble */
            const uint8_t b = ((const uint8_t*)src)[i >> 1];
            return oracle_e2m1_to_f16((i & 1) ? (b & 0x0Fu) : (uint8_t)(b >> 4));
        }
        case ORACLE_E2M1_UNPACKED: return oracle_e2m1_to_f16(((const uint8_t*)src)[i]);
        case ORACLE_BF16: return oracle_bf16_to_f16(((const uint16_t*)src)[i]);
        case ORACLE_TF32: return oracle_tf32_to_f16(((const uint32_t*)src)[i]);
        case ORACLE_E2M1_HW: {
            const uint8_t b = ((const uint8_t*)src)[i >> 1];
            return oracle_e2m1_to_f16((i & 1) ? (uint8_t)(b >> 4) : (b & 0x0Fu));
        }
        default: return 0;
    }
}

void oracle_decode(int fmt, const void* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = oracle_decode_one(fmt, src, i);
}

/* Quantize n floats (each multiplied by `scale` first, as the reference
 * harness does: bench/bench_formats.cu:132; scale 1 quantizes the value
 * itself, as RUN_FORMAT does at :64-65).  Packed FP4 writes (n+1)/2 bytes,
 * first value in the high nibble. */
static float scaled(float v, float scale) { return scale == 1.0f ? v : v * scale; }

void oracle_quantize(int fmt, const float* src, void* dst, size_t n, float scale) {
    switch (fmt) {
        case ORACLE_F16:
            for (size_t i = 0; i < n; i++) ((uint16_t*)dst)[i] = oracle_f32_to_f16(scaled(src[i], scale));
            break;
        case ORACLE_E4M3:
            for (size_t i = 0; i < n; i++) ((uint8_t*)dst)[i] = oracle_f32_to_e4m3(scaled(src[i], scale));
            break;
        case ORACLE_E5M2:
            for (size_t i = 0; i < n; i++) ((uint8_t*)dst)[i] = oracle_f32_to_e5m2(scaled(src[i], scale));
            break;
        case ORACLE_E2M1_UNPACKED:
            for (size_t i = 0; i < n; i++) ((uint8_t*)dst)[i] = oracle_f32_to_e2m1(scaled(src[i], scale));
            break;
        case ORACLE_E2M1:
        case ORACLE_E2M1_HW: {
            uint8_t* d = (uint8_t*)dst;
            const int hi_first = fmt == ORACLE_E2M1;
            for (size_t i = 0; i < n; i += 2) {
                const uint8_t a = oracle_f32_to_e2m1(scaled(src[i], scale));
                const uint8_t b = i + 1 < n ? oracle_f32_to_e2m1(scaled(src[i + 1], scale)) : 0;
                d[i >> 1] = hi_first ? (uint8_t)((a << 4) | b) : (uint8_t)((b << 4) | a);
            }
            break;
        }
        case ORACLE_BF16:
            for (size_t i = 0; i < n; i++) ((uint16_t*)dst)[i] = oracle_f32_to_bf16(scaled(src[i], scale));
            break;
        case ORACLE_TF32:
            for (size_t i = 0; i < n; i++) ((uint32_t*)dst)[i] = oracle_f32_to_tf32(scaled(src[i], scale));
            break;
        default: break;
    }
}

/* ---- GEMM ------------------------------------------------------------------------------ */

/* D[M x N] = alpha * decode(A)[M x K] * decode(B)[N x K]^T, FP32 products of
 * the decoded FP16 values summed in FP32 in ascending k, which is the
 * arithmetic of the reference's CPU check loop (bench/bench_formats.cu:183-186)
 * applied to the decoded operands.  Rows [row0, row1) only (row sampling);
 * D holds (row1 - row0) x N.  out_f16: round the scaled result to FP16 and
 * store FP16 bits; otherwise store FP32.  Threads split the rows. */
void oracle_gemm(int a_fmt, const void* A, int b_fmt, const void* B, void* D, int M, int N, int K, int row0, int row1,
                 float alpha, int out_f16, int nthreads) {
    (void)M;
    float* bf = (float*)malloc((size_t)N * K * sizeof(float));
    if (!bf) return;
    for (size_t i = 0; i < (size_t)N * K; i++) bf[i] = oracle_f16_to_f32(oracle_decode_one(b_fmt, B, i));
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
    {
        float* arow = (float*)malloc((size_t)K * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int r = row0; r < row1; r++) {
            for (int k = 0; k < K; k++) arow[k] = oracle_f16_to_f32(oracle_decode_one(a_fmt, A, (size_t)r * K + k));
            for (int n = 0; n < N; n++) {
                const float* b = bf + (size_t)n * K;
                float s = 0.0f;
                for (int k = 0; k < K; k++) s += arow[k] * b[k];
                const float v = s * alpha;
                const size_t o = (size_t)(r - row0) * N + n;
                if (out_f16) ((uint16_t*)D)[o] = oracle_f32_to_f16(v);
                else ((float*)D)[o] = v;
            }
        }
        free(arow);
    }
    free(bf);
}

/* ---- INT8 path -------------------------------------------------------------------------- */

/* decode_fp8_to_int8, src/gemm.cu:35-41, per element:
 * (int8_t)__float2int_rn(__half2float(fp8_e4m3_to_half(c)) * scale).  The FP16
 * decode is the reference primitive (fp8.h:23-31) and widens exactly; the
 * product is one FP32 multiply; __float2int_rn rounds to nearest even and the
 * conversion it compiles to (cvt.rni.s32.f32) clamps to the int32 range and
 * gives 0 for NaN; the int8_t cast keeps the low byte. */
int8_t oracle_e4m3_to_i8(uint8_t c, float scale) {
    const float v = oracle_f16_to_f32(oracle_e4m3_to_f16(c)) * scale;
    int32_t r;
    if (v != v) r = 0;
    else if (v >= 2147483648.0f) r = INT32_MAX;
    else if (v <= -2147483648.0f) r = INT32_MIN;
    else r = (int32_t)nearbyintf(v); /* default rounding: nearest, ties to even */
    return (int8_t)(uint8_t)((uint32_t)r & 0xFFu);
}

void oracle_decode_e4m3_i8(const uint8_t* src, int8_t* dst, size_t n, float scale) {
    for (size_t i = 0; i < n; i++) dst[i] = oracle_e4m3_to_i8(src[i], scale);
}

/* ---- block-scaled FP4 (the NVFP4 layout fp4.h:6 names; no reference kernel) -- */

/* A scale byte read as OCP E4M3 with subnormals (exponent 0: m * 2^-9);
 * 0x7F and 0xFF are NaN.  Unlike fp8_e4m3_to_half (fp8.h:23-31) nothing is
 * flushed: block scales use the whole E4M3 range. */
float oracle_e4m3_scale_to_f32(uint8_t s) {
    const uint32_t e = (s >> 3) & 0x0Fu, m = s & 0x07u;
    float v;
    if (e == 15 && m == 7) return u2f(0x7FFFFFFFu);
    if (e == 0) v = (float)m * 0.001953125f; /* m * 2^-9, exact */
    else v = u2f(((e + 120u) << 23) | (m << 20));
    return (s & 0x80u) ? -v : v;
}

/* Value i: the E2M1 code (packed two per byte, element 2j in the high nibble
 * of byte j, fp4.h:37-43; values from the table of fp4.h:27-30) times the
 * scale of its 16-value block, rounded to FP16 -- exact, every product being
 * an FP16 value.  A NaN scale gives 0x7E00. */
uint16_t oracle_nvfp4_at(const uint8_t* q, const uint8_t* scales, size_t i) {
    const uint8_t s = scales[i / 16];
    if ((s & 0x7Fu) == 0x7Fu) return 0x7E00u;
    const uint8_t b = q[i / 2];
    const uint16_t x = kE2M1[(i & 1) ? (b & 0x0Fu) : (b >> 4)];
    return oracle_f32_to_f16(oracle_f16_to_f32(x) * oracle_e4m3_scale_to_f32(s));
}

void oracle_decode_nvfp4(const uint8_t* q, const uint8_t* scales, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = oracle_nvfp4_at(q, scales, i);
}

/* gemm_int8_wmma, src/gemm.cu:58-70: D[M x N] = sum_k A8[m][k] * B8[n][k] with
 * 32-bit integer accumulation (B8 is the reference's column-major B, [N x K]
 * row-major).  Summed in 64 bits and wrapped to 32, as a 32-bit accumulator
 * wraps. */
void oracle_gemm_i8(const int8_t* A, const int8_t* B, int32_t* D, int M, int N, int K, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int m = 0; m < M; m++) {
        for (int n = 0; n < N; n++) {
            int64_t s = 0;
            for (int k = 0; k < K; k++) s += (int64_t)A[(size_t)m * K + k] * (int64_t)B[(size_t)n * K + k];
            D[(size_t)m * N + n] = (int32_t)(uint32_t)(uint64_t)s;
        }
    }
    (void)nthreads;
}
