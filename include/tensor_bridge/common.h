/*
 * tensor_bridge/common.h -- shared helpers for the conversion primitives.
 *
 * Source-compatible with tensor-bridge's include/tensor_bridge/common.h:13-27
 * (f2u / u2f).  Header-only; compiles under nvcc (host and device) and under a
 * plain host C++ compiler that can see cuda_fp16.h.
 */
#ifndef TENSOR_BRIDGE_COMMON_H
#define TENSOR_BRIDGE_COMMON_H

#include <cstdint>
#include <cstring>
#include <cmath>
#include <cuda_fp16.h>

#if defined(__CUDACC__)
#define TB_HD __host__ __device__ __forceinline__
#define TB_D __device__ __forceinline__
#else
#define TB_HD inline
#define TB_D inline
#endif

namespace tensor_bridge {

// Reinterpret the bits of a float as uint32 (and back).  Device code uses the
// intrinsic; host code goes through memcpy, which is the portable bit cast.
TB_HD uint32_t f2u(float v) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(v);
#else
    uint32_t u;
    std::memcpy(&u, &v, sizeof u);
    return u;
#endif
}

TB_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float v;
    std::memcpy(&v, &u, sizeof v);
    return v;
#endif
}

// Raw FP16 bits <-> half, usable on host and device.
TB_HD half bits_to_half(uint16_t b) {
    __half_raw r;
    r.x = b;
    return half(r);
}

TB_HD uint16_t half_to_bits(half h) {
    __half_raw r = static_cast<__half_raw>(h);
    return r.x;
}

}  // namespace tensor_bridge

#endif  // TENSOR_BRIDGE_COMMON_H
