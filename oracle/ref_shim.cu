/*
 * ref_shim.cu -- exposes tensor-bridge's OWN conversion primitives (its
 * include/tensor_bridge/{fp8,fp4,bf16,tf32}.h, compiled from where they lie in
 * the reference checkout) and its CPU decode + FP32 GEMM loop through a C ABI,
 * as oracle/_ref/libtbref.so.  TEST INFRASTRUCTURE ONLY: it generates the
 * golden tables under tests/golden (tests/golden/make_golden.py), pins the
 * oracle restatement, and is the CPU baseline of bench.py --impl reference.
 *
 * Built by oracle/Makefile with nvcc as HOST code (the reference headers need
 * cuda_fp16.h and do not compile with a plain host compiler: fp8.h:44 uses
 * fminf without <cmath>).  The reference's FP4 decode reads a __constant__
 * table and is device-only (fp4.h:27-35); the host baseline restates that
 * 16-entry table.
 */
#include <cmath>
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <omp.h>

#include "tensor_bridge/fp8.h"
#include "tensor_bridge/fp4.h"
#include "tensor_bridge/bf16.h"
#include "tensor_bridge/tf32.h"

namespace {
inline uint16_t bits(half h) { return __half_as_ushort(h); }
const uint16_t kFp4Host[16] = {0x0000, 0x3800, 0x3C00, 0x3E00, 0x4000, 0x4200, 0x4400, 0x4600,
                               0x8000, 0xB800, 0xBC00, 0xBE00, 0xC000, 0xC200, 0xC400, 0xC600};

// Reference decode of element i of a stored operand (format ids as in
// include/tensor_bridge_b200.h), as FP32.
inline float ref_decode_f32(int fmt, const void* src, size_t i) {
    using namespace tensor_bridge;
    switch (fmt) {
        case 0: return __half2float(__ushort_as_half(static_cast<const uint16_t*>(src)[i]));
        case 1: return __half2float(fp8_e4m3_to_half(static_cast<const uint8_t*>(src)[i]));
        case 2: return __half2float(fp8_e5m2_to_half(static_cast<const uint8_t*>(src)[i]));
        case 3: {
            const uint8_t b = static_cast<const uint8_t*>(src)[i >> 1];
            return __half2float(__ushort_as_half(kFp4Host[(i & 1) ? (b & 0xF) : (b >> 4)]));
        }
        case 4: return __half2float(__ushort_as_half(kFp4Host[static_cast<const uint8_t*>(src)[i] & 0xF]));
        case 5: return __half2float(bf16_to_half(static_cast<const uint16_t*>(src)[i]));
        case 6: return __half2float(tf32_to_half(static_cast<const uint32_t*>(src)[i]));
        default: return 0.0f;
    }
}
}  // namespace

extern "C" {

void ref_e4m3_to_half(const uint8_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = bits(tensor_bridge::fp8_e4m3_to_half(in[i]));
}
void ref_e5m2_to_half(const uint8_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = bits(tensor_bridge::fp8_e5m2_to_half(in[i]));
}
void ref_bf16_to_half(const uint16_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = bits(tensor_bridge::bf16_to_half(in[i]));
}
void ref_tf32_to_half(const uint32_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = bits(tensor_bridge::tf32_to_half(in[i]));
}
void ref_fp32_to_e4m3(const float* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::fp32_to_fp8_e4m3(in[i]);
}
void ref_fp32_to_e5m2(const float* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::fp32_to_fp8_e5m2(in[i]);
}
void ref_fp32_to_e2m1(const float* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::fp32_to_fp4_e2m1(in[i]);
}
void ref_half_to_e2m1(const uint16_t* in, uint8_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::half_to_fp4_e2m1(__ushort_as_half(in[i]));
}
void ref_fp32_to_bf16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::fp32_to_bf16(in[i]);
}
void ref_half_to_bf16(const uint16_t* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::half_to_bf16(__ushort_as_half(in[i]));
}
void ref_fp32_to_tf32(const float* in, uint32_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tensor_bridge::fp32_to_tf32(in[i]);
}
void ref_fp32_to_half(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = bits(__float2half(in[i]));
}

/* The reference's CPU path for one weight-only GEMM, rows [row0, row1):
 * decode A with the reference primitives, widen the FP16 B [N x K] with
 * __half2float, and run the reference's FP32 loop `s += a * b`
 * (bench/bench_formats.cu:183-186).  D is (row1 - row0) x N FP32, times alpha.
 * The rows are split over `nthreads` host threads. */
void ref_cpu_decode_gemm(int a_fmt, const void* A, const uint16_t* B, float* D, int M, int N, int K, int row0,
                         int row1, float alpha, int nthreads) {
    (void)M;
    if (nthreads > 0) omp_set_num_threads(nthreads);
    // B is widened once per call, split over the threads like the rows (a
    // fixed cost that a single thread would make dominate short row samples).
    const long long nk = static_cast<long long>(N) * K;
    float* bf = new float[static_cast<size_t>(nk)];
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < nk; ++i) bf[i] = __half2float(__ushort_as_half(B[i]));
#pragma omp parallel
    {
        float* arow = new float[K];
#pragma omp for schedule(dynamic, 1)
        for (int r = row0; r < row1; ++r) {
            for (int k = 0; k < K; ++k) arow[k] = ref_decode_f32(a_fmt, A, static_cast<size_t>(r) * K + k);
            for (int n = 0; n < N; ++n) {
                const float* b = bf + static_cast<size_t>(n) * K;
                float s = 0.0f;
                for (int k = 0; k < K; ++k) s += arow[k] * b[k];
                D[static_cast<size_t>(r - row0) * N + n] = s * alpha;
            }
        }
        delete[] arow;
    }
    delete[] bf;
}

/* The reference's own CPU check product (bench/bench_formats.cu:183-186), one
 * thread: D[i][j] = sum_k a[i][k] * b[k][j] in ascending k with B in its
 * [K x N] row-major layout, after decoding A [M x K] with the reference
 * primitives (row by row) and widening B [K x N] FP16 with __half2float.
 * The naive loop whose timing the build's GPU path is set against at the
 * sizes where it is tractable (256^3, 512^3). */
void ref_naive_decode_gemm(int a_fmt, const void* A, const uint16_t* B_kn, float* D, int M, int N, int K,
                           float alpha) {
    float* b = new float[static_cast<size_t>(K) * N];
    for (size_t i = 0; i < static_cast<size_t>(K) * N; ++i) b[i] = __half2float(__ushort_as_half(B_kn[i]));
    float* a = new float[static_cast<size_t>(M) * K];
    for (size_t i = 0; i < static_cast<size_t>(M) * K; ++i) a[i] = ref_decode_f32(a_fmt, A, i);
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float s = 0.0f;
            for (int k = 0; k < K; ++k) s += a[static_cast<size_t>(i) * K + k] * b[static_cast<size_t>(k) * N + j];
            D[static_cast<size_t>(i) * N + j] = s * alpha;
        }
    delete[] a;
    delete[] b;
}

}  // extern "C"
