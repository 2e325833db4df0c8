// tb_host.h -- internal host-side declarations shared by the .cu files.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "tensor_bridge_b200.h"

namespace tb {

// Other GPUs a fused pair GEMM can copy its output tiles to (one box of 8).
constexpr int kMaxPeers = 7;

// decode.cu
cudaError_t decode_launch(int fmt, const void* src, uint16_t* dst, size_t n, cudaStream_t st, int sms);
cudaError_t decode_transposed_launch(int fmt, const void* src, uint16_t* dst, int rows, int cols, cudaStream_t st);
cudaError_t fp4_repack_launch(const uint8_t* src, uint8_t* dst, size_t n, cudaStream_t st, int sms);
cudaError_t decode_e4m3_i8_launch(const uint8_t* src, int8_t* dst, size_t n, float scale, cudaStream_t st, int sms);
cudaError_t decode_e4m3_i8_transposed_launch(const uint8_t* src, int8_t* dst, int rows, int cols, float scale,
                                             cudaStream_t st);
// E4M3 codes with the reference decoder's subnormal flush applied (a code
// with exponent field 0 becomes the signed zero), as a copy and as a
// transposed copy ([rows x cols] -> [cols x rows]).
cudaError_t e4m3_flush_launch(const uint8_t* src, uint8_t* dst, size_t n, cudaStream_t st, int sms);
cudaError_t e4m3_flush_transposed_launch(const uint8_t* src, uint8_t* dst, int rows, int cols, cudaStream_t st);
cudaError_t decode_nvfp4_launch(const uint8_t* src, const uint8_t* scales, uint16_t* dst, size_t n,
                                cudaStream_t st, int sms);
size_t stored_bytes(int fmt, size_t n);

// quantize.cu
cudaError_t quantize_launch(int fmt, const float* src, void* dst, size_t n, float scale, cudaStream_t st, int sms);
cudaError_t absmax_launch(const float* src, size_t n, float* out, cudaStream_t st, int sms);

// gemm.cu
enum class GemmKind { kF16, kFused, kNative, kInt8 };

struct GemmRequest {
    GemmKind kind;
    int a_fmt;          // stored format of A (decode / native) or kF16
    int b_fmt;          // native: stored format of B (E4M3, E5M2 or E2M1_HW)
    const void* A;
    const void* B;      // FP16 [N x K] (f16 / fused) or b_fmt [N x K] (native)
    void* D;
    long long ldd;      // row stride of D in elements (normally N)
    int M, N, K;
    int out_f16;
    float alpha;
    void* workspace;
    size_t workspace_bytes;
    int force_bn;       // 0 = choose automatically (for tests and tuning)
    int force_splits;   // 0 = choose automatically
    // Fused kind only: also copy every output tile to these other GPUs'
    // buffers at D's offset (fused pair kernel; no split).
    int n_peers;
    void* const* peer_D;
};

// Split-K workspace needed by a fused/f16 GEMM of this shape (0 if none).
size_t gemm_workspace_bytes(GemmKind kind, int a_fmt, int M, int N, int K, int sms);

// Validated launch.  Returns cudaSuccess or the failing CUDA error; sets
// *why to a static message when the request itself is unsupported.
cudaError_t gemm_launch(const GemmRequest& r, cudaStream_t st, const char** why);

// Block-scaled FP4 GEMM (kind::mxf4nvf4) on SM pairs; arguments validated by the caller.
cudaError_t nvfp4_gemm_launch(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb, void* D, int M,
                              int N, int K, int out_f16, float alpha, cudaStream_t st, const char** why);

// api.cu: validated fused GEMM (D row stride N, no split) whose pair-kernel
// epilogue also copies every output tile to the n_peers buffers peer_D, at
// D's offset (other GPUs' copies of the output, mapped into this process).
tb_status gemm_fused_to_peers(tb_format a_fmt, const void* A, const uint16_t* B, void* D, int M, int N, int K,
                              tb_out_type out, float alpha, int n_peers, void* const* peer_D, tb_stream_t stream);

// Device error word of the GEMM kernels (bounded-wait expiry).
cudaError_t device_error_read(int* v);
cudaError_t device_error_clear();

// api.cu: record "<what>: <detail>" as the calling thread's last error and
// return `s` (for entry points defined outside api.cu).
tb_status set_last_error(tb_status s, const char* what, const char* detail);

// Device properties cached per device.
struct DeviceInfo {
    int sms;
    int major, minor;
};
const DeviceInfo& device_info(int dev);
int current_device();

}  // namespace tb
