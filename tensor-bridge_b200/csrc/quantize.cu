// quantize.cu -- device-side per-tensor quantization: FP32 -> stored format
// with the reference's quantizers (include/tensor_bridge/*.h of tensor-bridge:
// fp32_to_fp8_e4m3 fp8.h:43-61, fp32_to_fp8_e5m2 fp8.h:64-81,
// fp32_to_fp4_e2m1 fp4.h:46-53, fp32_to_bf16 bf16.h:37-48,
// fp32_to_tf32 tf32.h:37-44), applied to x * scale as the reference harness
// does (bench/bench_formats.cu:132), plus the max-|x| reduction that gives the
// per-tensor scale FORMAT_MAX / maxabs (bench/bench_formats.cu:128-130).
#include <cstdint>
#include <cuda_runtime.h>
#include "tensor_bridge/fp8.h"
#include "tensor_bridge/fp4.h"
#include "tensor_bridge/bf16.h"
#include "tensor_bridge/tf32.h"
#include "gemm_kernel.cuh"
#include "tb_host.h"

namespace tb {


template <int FMT>
__device__ __forceinline__ uint32_t quant1(float v) {
    using namespace tensor_bridge;
    if constexpr (FMT == kE4M3) return fp32_to_fp8_e4m3(v);
    else if constexpr (FMT == kE5M2) return fp32_to_fp8_e5m2(v);
    else if constexpr (FMT == kE2M1U || FMT == kE2M1 || FMT == kE2M1HW) return fp32_to_fp4_e2m1(v);
    else if constexpr (FMT == kBF16) return fp32_to_bf16(v);
    else if constexpr (FMT == kTF32) return fp32_to_tf32(v);
    else return half_to_bits(__float2half_rn(v));
}

// One thread per group of 4 values (vector path when src is 16-byte aligned).
// SCALED = false quantizes the values themselves: a multiply by 1.0 would be
// folded away by the compiler only sometimes, and GPU multiplies return a
// canonical NaN, so scale 1 gets its own instance with no multiply at all.
template <int FMT, bool SCALED>
__global__ void __launch_bounds__(256) k_quantize(const float* __restrict__ src, void* __restrict__ dst, size_t n,
                                                  float scale) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t groups = (n + 3) / 4;
    const bool vec = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
    for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += stride) {
        const size_t i0 = g * 4;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (vec && i0 + 4 <= n) {
            const float4 t = reinterpret_cast<const float4*>(src)[g];
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
            for (int j = 0; j < 4; ++j)
                if (i0 + j < n) v[j] = src[i0 + j];
        }
        uint32_t q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = quant1<FMT>(SCALED ? v[j] * scale : v[j]);
        const int cnt = static_cast<int>(n - i0 < 4 ? n - i0 : 4);
        if constexpr (FMT == kE2M1 || FMT == kE2M1HW) {
            // Two bytes per group; the reference packs the first value high.
            uint8_t* d = static_cast<uint8_t*>(dst) + i0 / 2;
            for (int j = 0; j < cnt; j += 2) {
                const uint32_t a = q[j], b = j + 1 < cnt ? q[j + 1] : 0u;
                d[j / 2] = FMT == kE2M1 ? static_cast<uint8_t>((a << 4) | b) : static_cast<uint8_t>((b << 4) | a);
            }
        } else if constexpr (FMT == kBF16 || FMT == kF16) {
            uint16_t* d = static_cast<uint16_t*>(dst) + i0;
            for (int j = 0; j < cnt; ++j) d[j] = static_cast<uint16_t>(q[j]);
        } else if constexpr (FMT == kTF32) {
            uint32_t* d = static_cast<uint32_t*>(dst) + i0;
            for (int j = 0; j < cnt; ++j) d[j] = q[j];
        } else {
            uint8_t* d = static_cast<uint8_t*>(dst) + i0;
            for (int j = 0; j < cnt; ++j) d[j] = static_cast<uint8_t>(q[j]);
        }
    }
}

// max |x| over non-NaN values (NaN is skipped, as fmaxf does), as FP32 bits in
// *out (which the launcher zeroes first).  Non-negative floats order like
// their bit patterns, so an integer atomicMax gives the float maximum.
__global__ void __launch_bounds__(256) k_absmax(const float* __restrict__ src, size_t n, unsigned int* out) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    float m = 0.0f;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float a = fabsf(src[i]);
        m = a > m ? a : m;  // false for NaN: skipped
    }
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

template <int FMT>
static cudaError_t launch_q(const float* src, void* dst, size_t n, float scale, cudaStream_t st, int sms) {
    const size_t groups = (n + 3) / 4;
    const size_t blocks = std::max<size_t>(1, std::min<size_t>((groups + 255) / 256, static_cast<size_t>(sms) * 8));
    if (scale == 1.0f) k_quantize<FMT, false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(src, dst, n, scale);
    else k_quantize<FMT, true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(src, dst, n, scale);
    return cudaGetLastError();
}

cudaError_t quantize_launch(int fmt, const float* src, void* dst, size_t n, float scale, cudaStream_t st, int sms) {
    switch (fmt) {
        case kF16: return launch_q<kF16>(src, dst, n, scale, st, sms);
        case kE4M3: return launch_q<kE4M3>(src, dst, n, scale, st, sms);
        case kE5M2: return launch_q<kE5M2>(src, dst, n, scale, st, sms);
        case kE2M1: return launch_q<kE2M1>(src, dst, n, scale, st, sms);
        case kE2M1U: return launch_q<kE2M1U>(src, dst, n, scale, st, sms);
        case kBF16: return launch_q<kBF16>(src, dst, n, scale, st, sms);
        case kTF32: return launch_q<kTF32>(src, dst, n, scale, st, sms);
        case kE2M1HW: return launch_q<kE2M1HW>(src, dst, n, scale, st, sms);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t absmax_launch(const float* src, size_t n, float* out, cudaStream_t st, int sms) {
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float), st);
    if (e != cudaSuccess || n == 0) return e;
    const size_t blocks = std::max<size_t>(1, std::min<size_t>((n + 255) / 256, static_cast<size_t>(sms) * 4));
    k_absmax<<<static_cast<unsigned>(blocks), 256, 0, st>>>(src, n, reinterpret_cast<unsigned int*>(out));
    return cudaGetLastError();
}

}  // namespace tb
