// decode.cu -- standalone decode kernels (stored format -> FP16 in HBM).
//
// These replace the reference's one-element-per-thread decode kernels
// (src/gemm.cu:25-30, bench/bench_formats.cu:33-56).  The straight kernel is
// a grid-stride HBM streamer: each warp step reads 32 x kRep consecutive
// items (4-16 bytes each, one load per item) and writes their decoded FP16
// chunks (8 or 16 bytes, one store per item), kRep items in flight per thread,
// so every warp-wide load and store covers whole contiguous 32-byte sectors.  The transposed kernel (the reference's B operand,
// B16[col*K + k] = decode(B[k*N + col])) goes through a 32 x 64 shared-memory
// tile so both the reads and the writes are coalesced.
#include <cstdint>
#include <cuda_runtime.h>
#include "tb_decode.cuh"
#include "gemm_kernel.cuh"
#include "tb_host.h"

namespace tb {

// Per-format geometry of one item: the input bytes that decode to one output
// chunk.  Every item is a single aligned load and a single aligned store, and
// the 32 lanes of a warp touch 32 consecutive items, so both the loads and the
// stores of a warp are contiguous (no half-written 32-byte sectors).
template <int FMT> struct Item;
template <> struct Item<kE4M3> { using In = uint2; using Out = uint4; static constexpr int kElems = 8, kRep = 16; };
template <> struct Item<kE5M2> { using In = uint2; using Out = uint4; static constexpr int kElems = 8, kRep = 16; };
template <> struct Item<kE2M1U> { using In = uint2; using Out = uint4; static constexpr int kElems = 8, kRep = 16; };
template <> struct Item<kE2M1> { using In = uint32_t; using Out = uint4; static constexpr int kElems = 8, kRep = 16; };
template <> struct Item<kBF16> { using In = uint4; using Out = uint4; static constexpr int kElems = 8, kRep = 4; };
template <> struct Item<kTF32> { using In = uint4; using Out = uint2; static constexpr int kElems = 4, kRep = 4; };
template <> struct Item<kF16> { using In = uint4; using Out = uint4; static constexpr int kElems = 8, kRep = 4; };

template <int FMT>
__device__ __forceinline__ typename Item<FMT>::Out decode_item(const typename Item<FMT>::In& in) {
    typename Item<FMT>::Out out;
    if constexpr (FMT == kE4M3) {
        decode_e4m3_x4(in.x, out.x, out.y); decode_e4m3_x4(in.y, out.z, out.w);
    } else if constexpr (FMT == kE5M2) {
        decode_e5m2_x4(in.x, out.x, out.y); decode_e5m2_x4(in.y, out.z, out.w);
    } else if constexpr (FMT == kE2M1U) {
        decode_e2m1_unpacked_x4(in.x, out.x, out.y); decode_e2m1_unpacked_x4(in.y, out.z, out.w);
    } else if constexpr (FMT == kE2M1) {
        uint32_t o[4];
        decode_e2m1_packed_x8(in, o);
        out = make_uint4(o[0], o[1], o[2], o[3]);
    } else if constexpr (FMT == kBF16) {
        out = make_uint4(decode_bf16_x2(in.x), decode_bf16_x2(in.y), decode_bf16_x2(in.z), decode_bf16_x2(in.w));
    } else if constexpr (FMT == kTF32) {
        out = make_uint2(decode_tf32_x2(in.x, in.y), decode_tf32_x2(in.z, in.w));
    } else {
        out = in;
    }
    return out;
}

// Scalar decode of element i (used for tails and misaligned buffers).
template <int FMT>
__device__ __forceinline__ uint16_t decode_at(const void* src, size_t i) {
    if constexpr (FMT == kE4M3) return tensor_bridge::e4m3_to_half_bits(static_cast<const uint8_t*>(src)[i]);
    else if constexpr (FMT == kE5M2) return tensor_bridge::e5m2_to_half_bits(static_cast<const uint8_t*>(src)[i]);
    else if constexpr (FMT == kE2M1U) return tensor_bridge::e2m1_to_half_bits(static_cast<const uint8_t*>(src)[i] & 0xFu);
    else if constexpr (FMT == kE2M1) {
        const uint8_t b = static_cast<const uint8_t*>(src)[i >> 1];
        return tensor_bridge::e2m1_to_half_bits((i & 1) ? (b & 0xFu) : (b >> 4));
    } else if constexpr (FMT == kBF16) return tensor_bridge::bf16_to_half_bits(static_cast<const uint16_t*>(src)[i]);
    else if constexpr (FMT == kTF32) return tensor_bridge::tf32_to_half_bits(static_cast<const uint32_t*>(src)[i]);
    else return static_cast<const uint16_t*>(src)[i];
}

// Grid-stride over warp chunks of 32 x kRep consecutive items.  Each thread
// issues its kRep loads (lane, lane + 32, ...) before any decode, then stores
// the kRep outputs with streaming (evict-first) stores -- the outputs are not
// re-read from L2 by this kernel; the last partial chunk is bounds-checked
// per item.  (16 one-byte or FP4 items in flight per thread and the streaming
// stores: 14336 x 4096 E4M3 5.55 -> 5.99 TB/s, E2M1 5.23 -> 5.80 TB/s.)
template <int FMT>
__global__ void __launch_bounds__(256) k_decode_stream(const typename Item<FMT>::In* __restrict__ src,
                                                       typename Item<FMT>::Out* __restrict__ dst, size_t items,
                                                       const void* __restrict__ tail_src,
                                                       uint16_t* __restrict__ tail_dst, size_t tail_begin,
                                                       size_t n) {
    using I = Item<FMT>;
    constexpr size_t kChunk = 32 * I::kRep;
    const int lane = threadIdx.x & 31;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const size_t nwarps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    for (size_t base = warp * kChunk; base < items; base += nwarps * kChunk) {
        typename I::In in[I::kRep];
        if (base + kChunk <= items) {
#pragma unroll
            for (int j = 0; j < I::kRep; ++j) in[j] = __ldcs(src + base + j * 32 + lane);
#pragma unroll
            for (int j = 0; j < I::kRep; ++j) __stcs(dst + base + j * 32 + lane, decode_item<FMT>(in[j]));
        } else {
#pragma unroll
            for (int j = 0; j < I::kRep; ++j)
                if (base + j * 32 + lane < items) in[j] = __ldcs(src + base + j * 32 + lane);
#pragma unroll
            for (int j = 0; j < I::kRep; ++j)
                if (base + j * 32 + lane < items) dst[base + j * 32 + lane] = decode_item<FMT>(in[j]);
        }
    }
    // Elements past the last whole item (fewer than one item).
    const size_t gt = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (tail_begin + gt < n) tail_dst[tail_begin + gt] = decode_at<FMT>(tail_src, tail_begin + gt);
}

template <int FMT>
__global__ void __launch_bounds__(256) k_decode_scalar(const void* __restrict__ src, uint16_t* __restrict__ dst,
                                                       size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        dst[i] = decode_at<FMT>(src, i);
}

// src [rows x cols] -> dst [cols x rows].  Block = 256 threads handles a
// 64-row x 32-column source tile: reads run along columns (contiguous in
// src), writes along rows (contiguous in dst).
template <int FMT>
__global__ void __launch_bounds__(256) k_decode_transposed(const void* __restrict__ src, uint16_t* __restrict__ dst,
                                                           int rows, int cols) {
    __shared__ uint16_t tile[32][64 + 2];
    const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int r = r0 + ty + 8 * k, c = c0 + tx;
        if (r < rows && c < cols) tile[tx][ty + 8 * k] = decode_at<FMT>(src, static_cast<size_t>(r) * cols + c);
    }
    __syncthreads();
    // Write: each warp writes 64 consecutive rows of one output row as 32 half2.
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int oc = ty + 8 * k;  // output row = source column c0 + oc
        const int c = c0 + oc;
        const int r = r0 + 2 * tx;
        if (c < cols) {
            uint16_t* out = dst + static_cast<size_t>(c) * rows + r;
            if (r + 1 < rows && ((reinterpret_cast<uintptr_t>(out) & 3u) == 0)) {
                *reinterpret_cast<uint32_t*>(out) =
                    static_cast<uint32_t>(tile[oc][2 * tx]) | (static_cast<uint32_t>(tile[oc][2 * tx + 1]) << 16);
            } else {
                if (r < rows) out[0] = tile[oc][2 * tx];
                if (r + 1 < rows) out[1] = tile[oc][2 * tx + 1];
            }
        }
    }
}

// 16 consecutive stored values at `p` (16-byte aligned) -> 16 FP16 values,
// two per word, first value in the low half.
template <int FMT>
__device__ __forceinline__ void decode16_vec(const uint8_t* p, uint32_t (&h)[8]) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    if constexpr (FMT == kBF16) {
        const uint4 a = q[0], b = q[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) h[k] = decode_bf16_x2(w[k]);
    } else if constexpr (FMT == kTF32) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 a = q[k];
            h[2 * k] = decode_tf32_x2(a.x, a.y);
            h[2 * k + 1] = decode_tf32_x2(a.z, a.w);
        }
    } else {
        const uint4 a = q[0];
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if constexpr (FMT == kE4M3) decode_e4m3_x4(w[k], h[2 * k], h[2 * k + 1]);
            else if constexpr (FMT == kE5M2) decode_e5m2_x4(w[k], h[2 * k], h[2 * k + 1]);
            else decode_e2m1_unpacked_x4(w[k], h[2 * k], h[2 * k + 1]);
        }
    }
}

// Formats of one value per 1, 2 or 4 bytes (E4M3, E5M2, unpacked E2M1, BF16,
// TF32): 64 x 64-value tiles, each thread reading 16 values of a source row
// with 16-byte loads (whole tiles, 16-byte aligned rows), converting them,
// and scattering the FP16 values into the transposed shared-memory tile; each
// thread then writes 16 values (32 bytes) of one output row.  Edge tiles go
// element by element.
template <int FMT>
__global__ void __launch_bounds__(256) k_decode_transposed_vec(const uint8_t* __restrict__ src,
                                                               uint16_t* __restrict__ dst, int rows, int cols) {
    constexpr int VB = FMT == kBF16 ? 2 : FMT == kTF32 ? 4 : 1;  // bytes per stored value
    constexpr int PITCH = 72;  // halves per tile row: 64 + 8 keeps rows 16-byte aligned
    __shared__ __align__(16) uint16_t tile[64 * PITCH];
    const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
    const int t = threadIdx.x;
    const bool whole = r0 + 64 <= rows && c0 + 64 <= cols;
    {
        const int lr = t >> 2, v = t & 3;  // source row r0 + lr, columns c0 + 16 v ..
        const int r = r0 + lr, c = c0 + 16 * v;
        uint32_t h[8];
        if (whole && ((cols * VB) & 15) == 0 && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
            decode16_vec<FMT>(src + (static_cast<size_t>(r) * cols + c) * VB, h);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int ca = c + 2 * k;
                const uint32_t lo = (r < rows && ca < cols) ? decode_at<FMT>(src, static_cast<size_t>(r) * cols + ca) : 0u;
                const uint32_t hi =
                    (r < rows && ca + 1 < cols) ? decode_at<FMT>(src, static_cast<size_t>(r) * cols + ca + 1) : 0u;
                h[k] = lo | (hi << 16);
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
            tile[(16 * v + j) * PITCH + lr] = static_cast<uint16_t>(h[j >> 1] >> (16 * (j & 1)));
    }
    __syncthreads();
    {
        const int oc = t >> 2, v = t & 3;  // output row c0 + oc, its values r0 + 16 v ..
        const int c = c0 + oc, r = r0 + 16 * v;
        if (c < cols) {
            uint16_t* out = dst + static_cast<size_t>(c) * rows + r;
            const uint16_t* row = tile + oc * PITCH + 16 * v;
            if (whole && (rows & 7) == 0 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
                reinterpret_cast<uint4*>(out)[0] = reinterpret_cast<const uint4*>(row)[0];
                reinterpret_cast<uint4*>(out)[1] = reinterpret_cast<const uint4*>(row)[1];
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (r + j < rows) out[j] = row[j];
            }
        }
    }
}

// ---- FP8 E4M3 -> INT8 (the reference's integer tensor-core path) ----------------

// One E4M3 code -> INT8 as src/gemm.cu:35-41 computes it:
// (int8_t)__float2int_rn(__half2float(fp8_e4m3_to_half(c)) * scale) -- the FP16
// decode, an FP32 product, round to nearest even into an int32 (the conversion
// clamps to the int32 range and gives 0 for NaN), and the low byte of that.
__device__ __forceinline__ uint32_t e4m3_to_i8_byte(uint16_t h, float scale) {
    return static_cast<uint32_t>(__float2int_rn(__half2float(__ushort_as_half(h)) * scale)) & 0xFFu;
}

// Four codes (byte 0 first) -> four INT8 values in the same byte order.
__device__ __forceinline__ uint32_t e4m3x4_to_i8x4(uint32_t w, float scale) {
    uint32_t h01, h23;
    decode_e4m3_x4(w, h01, h23);
    return e4m3_to_i8_byte(static_cast<uint16_t>(h01), scale) |
           (e4m3_to_i8_byte(static_cast<uint16_t>(h01 >> 16), scale) << 8) |
           (e4m3_to_i8_byte(static_cast<uint16_t>(h23), scale) << 16) |
           (e4m3_to_i8_byte(static_cast<uint16_t>(h23 >> 16), scale) << 24);
}

// Four E4M3 codes with the reference decoder's subnormal rule applied in the
// code domain: a code whose exponent field is zero becomes the signed zero
// (sign bit kept), every other code (NaN included) stays.  The tensor core
// then reads the codes with the values the reference's decode gives them.
// Bit 7 of each byte of (w & 0x78787878) + 0x78787878 is set iff that code's
// exponent is non-zero; times 0xFF per byte it becomes a byte mask.
__device__ __forceinline__ uint32_t e4m3x4_flush_subnormals(uint32_t w) {
    const uint32_t nz = ((w & 0x78787878u) + 0x78787878u) & 0x80808080u;
    return w & (((nz >> 7) * 0xFFu) | 0x80808080u);
}

// Byte maps of the one-byte conversion kernels below: word() maps four codes,
// byte() one code (in the low byte).
struct ByteMapI8 {  // E4M3 -> INT8 of the reference's integer path
    float scale;
    __device__ __forceinline__ uint32_t word(uint32_t w) const { return e4m3x4_to_i8x4(w, scale); }
    __device__ __forceinline__ uint32_t byte(uint8_t c) const {
        return e4m3_to_i8_byte(tensor_bridge::e4m3_to_half_bits(c), scale);
    }
};
struct ByteMapFlush {  // E4M3 -> E4M3 with the subnormal codes flushed
    __device__ __forceinline__ uint32_t word(uint32_t w) const { return e4m3x4_flush_subnormals(w); }
    __device__ __forceinline__ uint32_t byte(uint8_t c) const { return e4m3x4_flush_subnormals(c); }
};

// Streamer: 16 codes -> 16 bytes per item, warp chunks of 32 x 4 consecutive
// items (contiguous 16-byte loads and stores); elements past the last whole
// item one per thread.
template <class Map>
__global__ void __launch_bounds__(256) k_e4m3_bytes(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                    size_t items, const uint8_t* __restrict__ tail_src,
                                                    uint8_t* __restrict__ tail_dst, size_t tail_begin, size_t n,
                                                    Map map) {
    constexpr int kRep = 4;
    constexpr size_t kChunk = 32 * kRep;
    const int lane = threadIdx.x & 31;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const size_t nwarps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    for (size_t base = warp * kChunk; base < items; base += nwarps * kChunk) {
        uint4 in[kRep];
#pragma unroll
        for (int j = 0; j < kRep; ++j)
            if (base + j * 32 + lane < items) in[j] = __ldcs(src + base + j * 32 + lane);
#pragma unroll
        for (int j = 0; j < kRep; ++j)
            if (base + j * 32 + lane < items)
                dst[base + j * 32 + lane] =
                    make_uint4(map.word(in[j].x), map.word(in[j].y), map.word(in[j].z), map.word(in[j].w));
    }
    const size_t gt = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (tail_begin + gt < n) tail_dst[tail_begin + gt] = static_cast<uint8_t>(map.byte(tail_src[tail_begin + gt]));
}

// src [rows x cols] -> dst [cols x rows] (the reference's B8[col * K + k]),
// through a 64 x 64-byte shared-memory tile: each thread reads 16 codes of a
// source row (one 16-byte load when the tile lies inside the matrix and rows
// are 16-byte aligned), converts them, scatters the bytes into the transposed
// tile, and then writes 16 bytes of one output row.  Edge tiles take bytes one
// at a time.
template <class Map>
__global__ void __launch_bounds__(256) k_e4m3_bytes_transposed(const uint8_t* __restrict__ src,
                                                               uint8_t* __restrict__ dst, int rows, int cols, Map map) {
    constexpr int PITCH = 80;  // 64 bytes + 16: keeps 16-byte alignment of tile rows
    __shared__ __align__(16) uint8_t tile[64 * PITCH];
    const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
    const int t = threadIdx.x;
    const bool whole = r0 + 64 <= rows && c0 + 64 <= cols;
    {
        const int lr = t >> 2, v = t & 3;  // source row r0 + lr, columns c0 + 16 v ..
        const int r = r0 + lr, c = c0 + 16 * v;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        const uint8_t* in = src + static_cast<size_t>(r) * cols + c;
        if (whole && (cols & 15) == 0 && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
            const uint4 q = *reinterpret_cast<const uint4*>(in);
            w[0] = map.word(q.x);
            w[1] = map.word(q.y);
            w[2] = map.word(q.z);
            w[3] = map.word(q.w);
        } else if (r < rows) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (c + j < cols) w[j >> 2] |= (map.byte(in[j]) & 0xFFu) << (8 * (j & 3));
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) tile[(16 * v + j) * PITCH + lr] = static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)));
    }
    __syncthreads();
    {
        const int oc = t >> 2, v = t & 3;  // output row c0 + oc, its bytes r0 + 16 v ..
        const int c = c0 + oc, r = r0 + 16 * v;
        if (c < cols) {
            uint8_t* out = dst + static_cast<size_t>(c) * rows + r;
            const uint8_t* row = tile + oc * PITCH + 16 * v;
            if (whole && (rows & 15) == 0 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
                *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(row);
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (r + j < rows) out[j] = row[j];
            }
        }
    }
}

// Nibble swap (reference FP4 packing <-> tensor-core packing).
__global__ void __launch_bounds__(256) k_fp4_repack(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                    size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t n16 = n / 16;
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0;
    size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        for (size_t u = i; u < n16; u += stride) {
            uint4 v = reinterpret_cast<const uint4*>(src)[u];
            v.x = swap_nibbles(v.x); v.y = swap_nibbles(v.y); v.z = swap_nibbles(v.z); v.w = swap_nibbles(v.w);
            reinterpret_cast<uint4*>(dst)[u] = v;
        }
        for (size_t k = n16 * 16 + i; k < n; k += stride) {
            const uint8_t b = src[k];
            dst[k] = static_cast<uint8_t>((b >> 4) | (b << 4));
        }
    } else {
        for (size_t k = i; k < n; k += stride) {
            const uint8_t b = src[k];
            dst[k] = static_cast<uint8_t>((b >> 4) | (b << 4));
        }
    }
}

// ---------------------------------------------------------------------------------
// Block-scaled FP4 (NVFP4 layout): packed E2M1 codes in the reference order
// (fp4.h:37-43, element 2j in the high nibble of byte j) and one E4M3 scale
// byte per 16 consecutive values.  value = e2m1(code) * e4m3(scale).  Scale
// bytes are read as OCP E4M3 with subnormals (exponent 0: m * 2^-9); 0x7F and
// 0xFF are NaN and give 0x7E00.  Every product is an FP16 value (|v| in
// [2^-10, 2688], at most six significant bits), so the FP16 multiply rounds
// nothing and -0 follows the IEEE sign rule.

// A scale byte as FP16 bits, duplicated into both halves.
__device__ __forceinline__ uint32_t nvfp4_scale_x2(uint32_t s) {
    const uint32_t e = (s >> 3) & 0xFu, m = s & 7u;
    uint32_t h = e ? (((e + 8u) << 10) | (m << 7))
                   : static_cast<uint32_t>(__half_as_ushort(__float2half_rn(static_cast<float>(m) * 0x1p-9f)));
    h |= (s & 0x80u) << 8;
    return h | (h << 16);
}

__device__ __forceinline__ uint32_t mul_f16x2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ bool nvfp4_scale_is_nan(uint32_t s) { return (s & 0x7Fu) == 0x7Fu; }

// One item = 8 values: 4 packed bytes -> 16 bytes of FP16; items 2b and 2b+1
// share scale byte b.  Same streaming scheme as k_decode_stream (16 items in
// flight per thread, each warp instruction covering contiguous bytes).  The
// 256 scale bytes of a warp's 512-item chunk come in as one 8-byte load per
// lane (lane l holds chunk bytes 8l..8l+7); item j of lane l needs chunk byte
// 16j + l/2, which lane 2j + l/16 holds at offset (l/2) % 8.
__global__ void __launch_bounds__(256) k_decode_nvfp4(const uint32_t* __restrict__ src,
                                                      const uint8_t* __restrict__ scales, uint4* __restrict__ dst,
                                                      size_t items) {
    constexpr int kRep = 16;
    constexpr size_t kChunk = 32 * kRep;
    const int lane = threadIdx.x & 31;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const size_t nwarps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    const size_t nsc = items >> 1;
    for (size_t base = warp * kChunk; base < items; base += nwarps * kChunk) {
        uint32_t in[kRep], sc[kRep];
        const size_t s0 = (base >> 1) + 8 * lane;
        uint32_t wx = 0, wy = 0;
        if (s0 + 8 <= nsc) {
            const uint2 w = __ldcs(reinterpret_cast<const uint2*>(scales + s0));
            wx = w.x;
            wy = w.y;
        } else {
#pragma unroll
            for (int b = 0; b < 8; ++b)
                if (s0 + b < nsc) {
                    const uint32_t v = __ldcs(scales + s0 + b);
                    if (b < 4) wx |= v << (8 * b);
                    else wy |= v << (8 * (b - 4));
                }
        }
#pragma unroll
        for (int j = 0; j < kRep; ++j) {
            const size_t it = base + j * 32 + lane;
            if (it < items) in[j] = __ldcs(src + it);
        }
        const int byte = (lane >> 1) & 7;
#pragma unroll
        for (int j = 0; j < kRep; ++j) {
            const int from = 2 * j + (lane >> 4);
            const uint32_t x = __shfl_sync(0xFFFFFFFFu, wx, from);
            const uint32_t y = __shfl_sync(0xFFFFFFFFu, wy, from);
            sc[j] = ((byte < 4 ? x : y) >> (8 * (byte & 3))) & 0xFFu;
        }
#pragma unroll
        for (int j = 0; j < kRep; ++j) {
            const size_t it = base + j * 32 + lane;
            if (it < items) {
                uint32_t o[4];
                if (nvfp4_scale_is_nan(sc[j])) {
                    o[0] = o[1] = o[2] = o[3] = 0x7E007E00u;
                } else {
                    decode_e2m1_packed_x8(in[j], o);
                    const uint32_t s2 = nvfp4_scale_x2(sc[j]);
#pragma unroll
                    for (int k = 0; k < 4; ++k) o[k] = mul_f16x2(o[k], s2);
                }
                __stcs(dst + it, make_uint4(o[0], o[1], o[2], o[3]));
            }
        }
    }
}

// Any alignment: one value per thread, grid-stride.
__global__ void __launch_bounds__(256) k_decode_nvfp4_scalar(const uint8_t* __restrict__ src,
                                                             const uint8_t* __restrict__ scales,
                                                             uint16_t* __restrict__ dst, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t s = scales[i >> 4];
        if (nvfp4_scale_is_nan(s)) {
            dst[i] = 0x7E00u;
            continue;
        }
        const uint8_t b = src[i >> 1];
        const uint32_t x = tensor_bridge::e2m1_to_half_bits((i & 1) ? (b & 0xFu) : (b >> 4));
        dst[i] = static_cast<uint16_t>(mul_f16x2(x, nvfp4_scale_x2(s)) & 0xFFFFu);
    }
}

// ---------------------------------------------------------------------------------
// Host launchers

static size_t in_bytes_of(int fmt, size_t n) {
    switch (fmt) {
        case kE2M1: return (n + 1) / 2;
        case kBF16: case kF16: return n * 2;
        case kTF32: return n * 4;
        default: return n;
    }
}

template <int FMT>
static cudaError_t launch_decode(const void* src, uint16_t* dst, size_t n, cudaStream_t st, int sms) {
    using I = Item<FMT>;
    const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0;
    if (!aligned) {
        const size_t blocks = std::min<size_t>((n + 255) / 256, static_cast<size_t>(sms) * 8);
        k_decode_scalar<FMT><<<static_cast<unsigned>(std::max<size_t>(blocks, 1)), 256, 0, st>>>(src, dst, n);
        return cudaGetLastError();
    }
    const size_t items = n / I::kElems;
    const size_t tail_begin = items * I::kElems;
    const size_t want = (items + 8 * 32 * I::kRep - 1) / (8 * 32 * I::kRep);  // 8 warps per block
    size_t blocks = std::min<size_t>(want, static_cast<size_t>(sms) * 8);
    blocks = std::max<size_t>(blocks, 1);  // the tail needs at least one block (tail < 8 elements)
    k_decode_stream<FMT><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        static_cast<const typename I::In*>(src), reinterpret_cast<typename I::Out*>(dst), items, src, dst,
        tail_begin, n);
    return cudaGetLastError();
}

template <int FMT>
static cudaError_t launch_decode_t(const void* src, uint16_t* dst, int rows, int cols, cudaStream_t st) {
    if constexpr (FMT == kE4M3 || FMT == kE5M2 || FMT == kE2M1U || FMT == kBF16 || FMT == kTF32) {
        dim3 grid((cols + 63) / 64, (rows + 63) / 64);
        k_decode_transposed_vec<FMT><<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(src), dst, rows, cols);
    } else {
        dim3 grid((cols + 31) / 32, (rows + 63) / 64);
        k_decode_transposed<FMT><<<grid, 256, 0, st>>>(src, dst, rows, cols);
    }
    return cudaGetLastError();
}

cudaError_t decode_launch(int fmt, const void* src, uint16_t* dst, size_t n, cudaStream_t st, int sms) {
    switch (fmt) {
        case kF16: return launch_decode<kF16>(src, dst, n, st, sms);
        case kE4M3: return launch_decode<kE4M3>(src, dst, n, st, sms);
        case kE5M2: return launch_decode<kE5M2>(src, dst, n, st, sms);
        case kE2M1: return launch_decode<kE2M1>(src, dst, n, st, sms);
        case kE2M1U: return launch_decode<kE2M1U>(src, dst, n, st, sms);
        case kBF16: return launch_decode<kBF16>(src, dst, n, st, sms);
        case kTF32: return launch_decode<kTF32>(src, dst, n, st, sms);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t decode_transposed_launch(int fmt, const void* src, uint16_t* dst, int rows, int cols, cudaStream_t st) {
    switch (fmt) {
        case kF16: return launch_decode_t<kF16>(src, dst, rows, cols, st);
        case kE4M3: return launch_decode_t<kE4M3>(src, dst, rows, cols, st);
        case kE5M2: return launch_decode_t<kE5M2>(src, dst, rows, cols, st);
        case kE2M1: return launch_decode_t<kE2M1>(src, dst, rows, cols, st);
        case kE2M1U: return launch_decode_t<kE2M1U>(src, dst, rows, cols, st);
        case kBF16: return launch_decode_t<kBF16>(src, dst, rows, cols, st);
        case kTF32: return launch_decode_t<kTF32>(src, dst, rows, cols, st);
        default: return cudaErrorInvalidValue;
    }
}

template <class Map>
static cudaError_t launch_e4m3_bytes(const uint8_t* src, uint8_t* d, size_t n, Map map, cudaStream_t st, int sms) {
    const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(d)) & 15u) == 0;
    const size_t items = aligned ? n / 16 : 0;
    const size_t tail_begin = items * 16;
    // Without alignment every element is a tail element: one per thread.
    const size_t want = aligned ? (items + 1023) / 1024 : (n - tail_begin + 255) / 256;
    size_t blocks = std::min<size_t>(std::max<size_t>(want, 1), static_cast<size_t>(sms) * 8);
    if (!aligned) blocks = std::max<size_t>(want, 1);
    k_e4m3_bytes<Map><<<static_cast<unsigned>(blocks), 256, 0, st>>>(reinterpret_cast<const uint4*>(src),
                                                                     reinterpret_cast<uint4*>(d), items, src, d,
                                                                     tail_begin, n, map);
    return cudaGetLastError();
}

template <class Map>
static cudaError_t launch_e4m3_bytes_transposed(const uint8_t* src, uint8_t* dst, int rows, int cols, Map map,
                                                cudaStream_t st) {
    dim3 grid((cols + 63) / 64, (rows + 63) / 64);
    k_e4m3_bytes_transposed<Map><<<grid, 256, 0, st>>>(src, dst, rows, cols, map);
    return cudaGetLastError();
}

cudaError_t decode_e4m3_i8_launch(const uint8_t* src, int8_t* dst, size_t n, float scale, cudaStream_t st, int sms) {
    return launch_e4m3_bytes(src, reinterpret_cast<uint8_t*>(dst), n, ByteMapI8{scale}, st, sms);
}

cudaError_t decode_e4m3_i8_transposed_launch(const uint8_t* src, int8_t* dst, int rows, int cols, float scale,
                                             cudaStream_t st) {
    return launch_e4m3_bytes_transposed(src, reinterpret_cast<uint8_t*>(dst), rows, cols, ByteMapI8{scale}, st);
}

cudaError_t e4m3_flush_launch(const uint8_t* src, uint8_t* dst, size_t n, cudaStream_t st, int sms) {
    return launch_e4m3_bytes(src, dst, n, ByteMapFlush{}, st, sms);
}

cudaError_t e4m3_flush_transposed_launch(const uint8_t* src, uint8_t* dst, int rows, int cols, cudaStream_t st) {
    return launch_e4m3_bytes_transposed(src, dst, rows, cols, ByteMapFlush{}, st);
}

cudaError_t fp4_repack_launch(const uint8_t* src, uint8_t* dst, size_t n, cudaStream_t st, int sms) {
    const size_t blocks = std::max<size_t>(1, std::min<size_t>((n / 16 + 255) / 256, static_cast<size_t>(sms) * 8));
    k_fp4_repack<<<static_cast<unsigned>(blocks), 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t decode_nvfp4_launch(const uint8_t* src, const uint8_t* scales, uint16_t* dst, size_t n,
                                cudaStream_t st, int sms) {
    const bool aligned = (reinterpret_cast<uintptr_t>(src) & 3u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0 &&
                         (reinterpret_cast<uintptr_t>(scales) & 7u) == 0;
    if (!aligned) {
        const size_t blocks = std::min<size_t>((n + 255) / 256, static_cast<size_t>(sms) * 8);
        k_decode_nvfp4_scalar<<<static_cast<unsigned>(std::max<size_t>(blocks, 1)), 256, 0, st>>>(src, scales, dst,
                                                                                                    n);
        return cudaGetLastError();
    }
    const size_t items = n / 8;  // n is a multiple of 16
    const size_t blocks = std::max<size_t>(1, std::min<size_t>((items + 8 * 32 * 16 - 1) / (8 * 32 * 16),
                                                               static_cast<size_t>(sms) * 8));
    k_decode_nvfp4<<<static_cast<unsigned>(blocks), 256, 0, st>>>(reinterpret_cast<const uint32_t*>(src), scales,
                                                                  reinterpret_cast<uint4*>(dst), items);
    return cudaGetLastError();
}

size_t stored_bytes(int fmt, size_t n) { return in_bytes_of(fmt, n); }

}  // namespace tb
