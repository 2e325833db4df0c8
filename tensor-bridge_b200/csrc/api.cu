// api.cu -- the extern "C" boundary (include/tensor_bridge_b200.h): argument
// checks, status codes, and dispatch to the decode and GEMM launchers.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <cuda_runtime.h>
#include "tensor_bridge_b200.h"
#include "tb_host.h"

namespace {

thread_local std::string g_last_error;

tb_status fail(tb_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
tb_status fail(tb_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

tb_status from_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TB_OK;
    return fail(TB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

tb_status check_device() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(TB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    const tb::DeviceInfo& d = tb::device_info(dev);
    if (d.major != 10 || d.minor != 0)
        return fail(TB_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", dev, d.major, d.minor);
    return TB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool known_format(int f) { return f >= TB_FMT_F16 && f <= TB_FMT_E2M1_HW; }

// Common GEMM shape checks.  K must be a multiple of 16 (32 for packed FP4)
// so that every operand row pitch is a multiple of 16 bytes (TMA rule).
tb_status check_gemm_shape(int M, int N, int K, int a_fmt) {
    if (M <= 0 || N <= 0 || K <= 0) return fail(TB_ERR_SHAPE, "M, N, K must be positive (got %d, %d, %d)", M, N, K);
    const int kmul = (a_fmt == TB_FMT_E2M1 || a_fmt == TB_FMT_E2M1_HW) ? 32 : 16;
    if (K % kmul != 0) return fail(TB_ERR_SHAPE, "K = %d must be a multiple of %d for this format", K, kmul);
    return TB_OK;
}

tb_status launch_gemm(const tb::GemmRequest& r, cudaStream_t st) {
    const char* why = nullptr;
    cudaError_t e = tb::gemm_launch(r, st, &why);
    if (e == cudaSuccess) return TB_OK;
    if (why) return fail(TB_ERR_UNSUPPORTED, "%s", why);
    return fail(TB_ERR_LAUNCH, "GEMM launch: %s", cudaGetErrorString(e));
}

}  // namespace

tb_status tb::set_last_error(tb_status s, const char* what, const char* detail) {
    return fail(s, "%s: %s", what, detail);
}

extern "C" {

const char* tb_status_string(tb_status s) {
    switch (s) {
        case TB_OK: return "TB_OK";
        case TB_ERR_INVALID_ARGUMENT: return "TB_ERR_INVALID_ARGUMENT";
        case TB_ERR_SHAPE: return "TB_ERR_SHAPE";
        case TB_ERR_ALIGNMENT: return "TB_ERR_ALIGNMENT";
        case TB_ERR_CUDA: return "TB_ERR_CUDA";
        case TB_ERR_LAUNCH: return "TB_ERR_LAUNCH";
        case TB_ERR_TIMEOUT: return "TB_ERR_TIMEOUT";
        case TB_ERR_UNSUPPORTED: return "TB_ERR_UNSUPPORTED";
        case TB_ERR_WORKSPACE: return "TB_ERR_WORKSPACE";
        case TB_ERR_NCCL: return "TB_ERR_NCCL";
    }
    return "TB_ERR_UNKNOWN";
}

const char* tb_last_error(void) { return g_last_error.c_str(); }

tb_status tb_device_supported(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
        return fail(TB_ERR_UNSUPPORTED, "no CUDA device %d", device);
    const tb::DeviceInfo& d = tb::device_info(device);
    if (d.major != 10 || d.minor != 0) return fail(TB_ERR_UNSUPPORTED, "device %d is sm_%d%d", device, d.major, d.minor);
    return TB_OK;
}

tb_status tb_device_error(int* code, int clear) {
    if (!code) return fail(TB_ERR_INVALID_ARGUMENT, "code is NULL");
    tb_status s = from_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    if (s != TB_OK) return s;
    int v = 0;
    s = from_cuda(tb::device_error_read(&v), "read device error word");
    if (s != TB_OK) return s;
    *code = v;
    if (clear && v) {
        s = from_cuda(tb::device_error_clear(), "clear device error word");
    }
    return s;
}

// ---- decode ------------------------------------------------------------------

tb_status tb_decode(tb_format fmt, const void* src, uint16_t* dst, size_t n, tb_stream_t stream) {
    if (!known_format(fmt) || fmt == TB_FMT_E2M1_HW) return fail(TB_ERR_INVALID_ARGUMENT, "bad format %d", (int)fmt);
    if (n == 0) return TB_OK;
    if (!src || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const int sms = tb::device_info(tb::current_device()).sms;
    return from_cuda(tb::decode_launch(fmt, src, dst, n, stream, sms), "decode launch");
}

tb_status tb_decode_transposed(tb_format fmt, const void* src, uint16_t* dst, int rows, int cols, tb_stream_t stream) {
    if (!known_format(fmt) || fmt == TB_FMT_E2M1_HW) return fail(TB_ERR_INVALID_ARGUMENT, "bad format %d", (int)fmt);
    if (rows < 0 || cols < 0) return fail(TB_ERR_SHAPE, "negative shape");
    if (rows == 0 || cols == 0) return TB_OK;
    if (fmt == TB_FMT_E2M1 && (cols & 1)) return fail(TB_ERR_SHAPE, "packed FP4 needs an even column count");
    if (!src || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    return from_cuda(tb::decode_transposed_launch(fmt, src, dst, rows, cols, stream), "transposed decode launch");
}

tb_status tb_decode_nvfp4(const uint8_t* src, const uint8_t* scales, uint16_t* dst, size_t n, tb_stream_t stream) {
    if (n % 16) return fail(TB_ERR_SHAPE, "block-scaled FP4 needs a multiple of 16 values, got %zu", n);
    if (n == 0) return TB_OK;
    if (!src || !scales || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const int sms = tb::device_info(tb::current_device()).sms;
    return from_cuda(tb::decode_nvfp4_launch(src, scales, dst, n, stream, sms), "block-scaled FP4 decode launch");
}

static tb_status decode_pair(tb_format fmt, const void* A, const void* B, uint16_t* A16, uint16_t* B16, int M, int N,
                             int K, tb_stream_t stream) {
    if (M < 0 || N < 0 || K < 0) return fail(TB_ERR_SHAPE, "negative shape");
    if ((A == nullptr) != (A16 == nullptr) || (B == nullptr) != (B16 == nullptr))
        return fail(TB_ERR_INVALID_ARGUMENT, "each operand needs both its source and destination");
    tb_status s = TB_OK;
    if (A) s = tb_decode(fmt, A, A16, static_cast<size_t>(M) * K, stream);
    if (s == TB_OK && B) s = tb_decode_transposed(fmt, B, B16, K, N, stream);
    return s;
}

tb_status tb_decode_fp8_to_half(const uint8_t* A, const uint8_t* B, uint16_t* A16, uint16_t* B16, int M, int N, int K,
                                tb_stream_t stream) {
    return decode_pair(TB_FMT_E4M3, A, B, A16, B16, M, N, K, stream);
}
tb_status tb_decode_bf16_to_half(const uint16_t* A, const uint16_t* B, uint16_t* A16, uint16_t* B16, int M, int N,
                                 int K, tb_stream_t stream) {
    return decode_pair(TB_FMT_BF16, A, B, A16, B16, M, N, K, stream);
}
tb_status tb_decode_tf32_to_half(const uint32_t* A, const uint32_t* B, uint16_t* A16, uint16_t* B16, int M, int N,
                                 int K, tb_stream_t stream) {
    return decode_pair(TB_FMT_TF32, A, B, A16, B16, M, N, K, stream);
}
tb_status tb_decode_fp4_to_half(const uint8_t* A, const uint8_t* B, uint16_t* A16, uint16_t* B16, int M, int N, int K,
                                tb_stream_t stream) {
    return decode_pair(TB_FMT_E2M1_UNPACKED, A, B, A16, B16, M, N, K, stream);
}

tb_status tb_fp4_repack_hw(const uint8_t* src, uint8_t* dst, size_t n_bytes, tb_stream_t stream) {
    if (n_bytes == 0) return TB_OK;
    if (!src || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const int sms = tb::device_info(tb::current_device()).sms;
    return from_cuda(tb::fp4_repack_launch(src, dst, n_bytes, stream, sms), "repack launch");
}

// ---- quantize ----------------------------------------------------------------

tb_status tb_quantize(tb_format fmt, const float* src, void* dst, size_t n, float scale, tb_stream_t stream) {
    if (!known_format(fmt)) return fail(TB_ERR_INVALID_ARGUMENT, "bad format %d", (int)fmt);
    if (n == 0) return TB_OK;
    if (!src || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const int sms = tb::device_info(tb::current_device()).sms;
    return from_cuda(tb::quantize_launch(fmt, src, dst, n, scale, stream, sms), "quantize launch");
}

tb_status tb_absmax(const float* src, size_t n, float* out, tb_stream_t stream) {
    if (!out || (n && !src)) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const int sms = tb::device_info(tb::current_device()).sms;
    return from_cuda(tb::absmax_launch(src, n, out, stream, sms), "absmax launch");
}

// ---- GEMMs -------------------------------------------------------------------

tb_status tb_gemm_f16(const uint16_t* A, const uint16_t* B, void* D, int M, int N, int K, tb_out_type out, float alpha,
                      tb_stream_t stream) {
    tb_status s = check_gemm_shape(M, N, K, TB_FMT_F16);
    if (s != TB_OK) return s;
    if (!A || !B || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    if (out != TB_OUT_F32 && out != TB_OUT_F16) return fail(TB_ERR_INVALID_ARGUMENT, "bad output type");
    if (!aligned16(A) || !aligned16(B)) return fail(TB_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
    s = check_device();
    if (s != TB_OK) return s;
    tb::GemmRequest r{};
    r.kind = tb::GemmKind::kF16;
    r.a_fmt = TB_FMT_F16;
    r.A = A; r.B = B; r.D = D; r.ldd = N;
    r.M = M; r.N = N; r.K = K;
    r.out_f16 = out == TB_OUT_F16;
    r.alpha = alpha;
    return launch_gemm(r, stream);
}

size_t tb_gemm_fused_workspace(tb_format a_fmt, int M, int N, int K) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    return tb::gemm_workspace_bytes(tb::GemmKind::kFused, a_fmt, M, N, K, tb::device_info(dev).sms);
}

static tb_status fused_request(tb_format a_fmt, const void* A, const uint16_t* B, void* D, long long ldd, int M, int N,
                               int K, tb_out_type out, float alpha, void* ws, size_t ws_bytes, tb_stream_t stream,
                               int n_peers = 0, void* const* peer_D = nullptr) {
    if (a_fmt != TB_FMT_E4M3 && a_fmt != TB_FMT_E5M2 && a_fmt != TB_FMT_E2M1 && a_fmt != TB_FMT_E2M1_UNPACKED &&
        a_fmt != TB_FMT_BF16 && a_fmt != TB_FMT_TF32 && a_fmt != TB_FMT_F16)
        return fail(TB_ERR_INVALID_ARGUMENT, "format %d is not a fused weight format", (int)a_fmt);
    tb_status s = check_gemm_shape(M, N, K, a_fmt);
    if (s != TB_OK) return s;
    if (!A || !B || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    if (out != TB_OUT_F32 && out != TB_OUT_F16) return fail(TB_ERR_INVALID_ARGUMENT, "bad output type");
    if (!aligned16(A) || !aligned16(B)) return fail(TB_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
    s = check_device();
    if (s != TB_OK) return s;
    tb::GemmRequest r{};
    r.kind = a_fmt == TB_FMT_F16 ? tb::GemmKind::kF16 : tb::GemmKind::kFused;
    r.a_fmt = a_fmt;
    r.A = A; r.B = B; r.D = D; r.ldd = ldd;
    r.M = M; r.N = N; r.K = K;
    r.out_f16 = out == TB_OUT_F16;
    r.alpha = alpha;
    r.workspace = ws;
    r.workspace_bytes = ws_bytes;
    r.n_peers = n_peers;
    r.peer_D = peer_D;
    return launch_gemm(r, stream);
}

tb_status tb_gemm_fused(tb_format a_fmt, const void* A, const uint16_t* B, void* D, int M, int N, int K,
                        tb_out_type out, float alpha, void* workspace, size_t workspace_bytes, tb_stream_t stream) {
    return fused_request(a_fmt, A, B, D, N, M, N, K, out, alpha, workspace, workspace_bytes, stream);
}

tb_status tb_gemm_nvfp4(const uint8_t* A, const uint8_t* A_scales, const uint8_t* B, const uint8_t* B_scales, void* D,
                        int M, int N, int K, tb_out_type out, float alpha, tb_stream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0) return fail(TB_ERR_SHAPE, "M, N, K must be positive (got %d, %d, %d)", M, N, K);
    if (K % 256 != 0) return fail(TB_ERR_SHAPE, "K = %d must be a multiple of 256 for the block-scaled FP4 GEMM", K);
    if (!A || !A_scales || !B || !B_scales || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    if (out != TB_OUT_F32 && out != TB_OUT_F16) return fail(TB_ERR_INVALID_ARGUMENT, "bad output type");
    if (!aligned16(A) || !aligned16(B) || !aligned16(A_scales) || !aligned16(B_scales))
        return fail(TB_ERR_ALIGNMENT, "A, B and both scale arrays must be 16-byte aligned");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const char* why = nullptr;
    cudaError_t e = tb::nvfp4_gemm_launch(A, A_scales, B, B_scales, D, M, N, K, out == TB_OUT_F16, alpha,
                                          reinterpret_cast<cudaStream_t>(stream), &why);
    if (e == cudaSuccess) return TB_OK;
    if (why) return fail(TB_ERR_UNSUPPORTED, "%s", why);
    return fail(TB_ERR_LAUNCH, "block-scaled FP4 GEMM launch: %s", cudaGetErrorString(e));
}

tb_status tb_gemm_native(tb_format a_fmt, const void* A, tb_format b_fmt, const void* B, void* D, int M, int N, int K,
                         tb_out_type out, float alpha, tb_stream_t stream) {
    auto native_ok = [](tb_format f) { return f == TB_FMT_E4M3 || f == TB_FMT_E5M2 || f == TB_FMT_E2M1_HW; };
    if (!native_ok(a_fmt) || !native_ok(b_fmt))
        return fail(TB_ERR_UNSUPPORTED, "native GEMM operands must be E4M3, E5M2 or E2M1_HW (got %d, %d)", (int)a_fmt,
                    (int)b_fmt);
    tb_status s = check_gemm_shape(M, N, K, a_fmt);
    if (s != TB_OK) return s;
    s = check_gemm_shape(M, N, K, b_fmt);
    if (s != TB_OK) return s;
    // Packed FP4 reaches the tensor core through the 16U4_ALIGN16B tensor-map
    // type, which needs a row length that is a multiple of 128 values and a
    // 32-byte aligned base.
    const bool fp4 = a_fmt == TB_FMT_E2M1_HW || b_fmt == TB_FMT_E2M1_HW;
    if (fp4 && K % 128 != 0) return fail(TB_ERR_SHAPE, "native FP4 needs K %% 128 == 0 (got K = %d)", K);
    if (!A || !B || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    if (out != TB_OUT_F32 && out != TB_OUT_F16) return fail(TB_ERR_INVALID_ARGUMENT, "bad output type");
    if (!aligned16(A) || !aligned16(B)) return fail(TB_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
    if ((a_fmt == TB_FMT_E2M1_HW && (reinterpret_cast<uintptr_t>(A) & 31u)) ||
        (b_fmt == TB_FMT_E2M1_HW && (reinterpret_cast<uintptr_t>(B) & 31u)))
        return fail(TB_ERR_ALIGNMENT, "native FP4 operands must be 32-byte aligned");
    s = check_device();
    if (s != TB_OK) return s;
    tb::GemmRequest r{};
    r.kind = tb::GemmKind::kNative;
    r.a_fmt = a_fmt;
    r.b_fmt = b_fmt;
    r.A = A; r.B = B; r.D = D; r.ldd = N;
    r.M = M; r.N = N; r.K = K;
    r.out_f16 = out == TB_OUT_F16;
    r.alpha = alpha;
    return launch_gemm(r, stream);
}

// Workspace of tb_gemm_fp8_fused_fp16: the flushed copy of A [M x K] and the
// flushed, transposed B [N x K], each 256-byte aligned.
static size_t fp8_pair_bytes(int M, int K) { return (static_cast<size_t>(M) * K + 255) / 256 * 256; }

size_t tb_gemm_fp8_fused_workspace(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return fp8_pair_bytes(M, K) + fp8_pair_bytes(N, K);
}

// ---- INT8 path -------------------------------------------------------------------

tb_status tb_decode_e4m3_to_i8(const uint8_t* src, int8_t* dst, size_t n, float scale, tb_stream_t stream) {
    if (n == 0) return TB_OK;
    if (!src || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    const int sms = tb::device_info(tb::current_device()).sms;
    return from_cuda(tb::decode_e4m3_i8_launch(src, dst, n, scale, stream, sms), "INT8 decode launch");
}

tb_status tb_decode_e4m3_to_i8_transposed(const uint8_t* src, int8_t* dst, int rows, int cols, float scale,
                                          tb_stream_t stream) {
    if (rows < 0 || cols < 0) return fail(TB_ERR_SHAPE, "negative shape");
    if (rows == 0 || cols == 0) return TB_OK;
    if (!src || !dst) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    tb_status s = check_device();
    if (s != TB_OK) return s;
    return from_cuda(tb::decode_e4m3_i8_transposed_launch(src, dst, rows, cols, scale, stream),
                     "transposed INT8 decode launch");
}

tb_status tb_decode_fp8_to_int8(const uint8_t* A, const uint8_t* B, int8_t* A8, int8_t* B8, int M, int N, int K,
                                float scale, tb_stream_t stream) {
    if (M < 0 || N < 0 || K < 0) return fail(TB_ERR_SHAPE, "negative shape");
    if ((A == nullptr) != (A8 == nullptr) || (B == nullptr) != (B8 == nullptr))
        return fail(TB_ERR_INVALID_ARGUMENT, "each operand needs both its source and destination");
    tb_status s = TB_OK;
    if (A) s = tb_decode_e4m3_to_i8(A, A8, static_cast<size_t>(M) * K, scale, stream);
    if (s == TB_OK && B) s = tb_decode_e4m3_to_i8_transposed(B, B8, K, N, scale, stream);
    return s;
}

tb_status tb_gemm_i8(const int8_t* A, const int8_t* B, int32_t* D, int M, int N, int K, tb_stream_t stream) {
    tb_status s = check_gemm_shape(M, N, K, TB_FMT_E4M3);
    if (s != TB_OK) return s;
    if (!A || !B || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    if (!aligned16(A) || !aligned16(B)) return fail(TB_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
    s = check_device();
    if (s != TB_OK) return s;
    tb::GemmRequest r{};
    r.kind = tb::GemmKind::kInt8;
    r.A = A; r.B = B; r.D = D; r.ldd = N;
    r.M = M; r.N = N; r.K = K;
    r.alpha = 1.0f;
    return launch_gemm(r, stream);
}

size_t tb_gemm_fp8_fused_int8_workspace(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return (static_cast<size_t>(M) * K + 255) / 256 * 256 + (static_cast<size_t>(N) * K + 255) / 256 * 256;
}

tb_status tb_gemm_fp8_fused_int8(const uint8_t* A, const uint8_t* B, int32_t* D, int M, int N, int K, float scale,
                                 void* workspace, size_t workspace_bytes, tb_stream_t stream) {
    tb_status s = check_gemm_shape(M, N, K, TB_FMT_E4M3);
    if (s != TB_OK) return s;
    if (!A || !B || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    const size_t need = tb_gemm_fp8_fused_int8_workspace(M, N, K);
    if (!workspace || workspace_bytes < need) return fail(TB_ERR_WORKSPACE, "workspace needs at least %zu bytes", need);
    if (!aligned16(workspace)) return fail(TB_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
    int8_t* A8 = static_cast<int8_t*>(workspace);
    int8_t* B8 = A8 + (static_cast<size_t>(M) * K + 255) / 256 * 256;
    s = tb_decode_fp8_to_int8(A, B, A8, B8, M, N, K, scale, stream);
    if (s != TB_OK) return s;
    return tb_gemm_i8(A8, B8, D, M, N, K, stream);
}

tb_status tb_gemm_fp8_fused_fp16(const uint8_t* A, const uint8_t* B, float* D, int M, int N, int K, void* workspace,
                                 size_t workspace_bytes, tb_stream_t stream) {
    tb_status s = check_gemm_shape(M, N, K, TB_FMT_E4M3);
    if (s != TB_OK) return s;
    if (!A || !B || !D) return fail(TB_ERR_INVALID_ARGUMENT, "null pointer");
    const size_t need = tb_gemm_fp8_fused_workspace(M, N, K);
    if (!workspace || workspace_bytes < need)
        return fail(TB_ERR_WORKSPACE, "workspace needs at least %zu bytes", need);
    if (!aligned16(A) || !aligned16(workspace)) return fail(TB_ERR_ALIGNMENT, "A and the workspace must be 16-byte aligned");
    s = check_device();
    if (s != TB_OK) return s;
    // Both operands are E4M3: the FP8 tensor cores multiply the codes
    // directly.  The reference decodes them to FP16 first, flushing the
    // subnormal codes to zero; the same flush applied to the codes (A copied,
    // B copied into [N x K]) makes the tensor core's exact products those of
    // the reference's FP16 operands.
    uint8_t* Af = static_cast<uint8_t*>(workspace);
    uint8_t* Bf = Af + fp8_pair_bytes(M, K);
    const int sms = tb::device_info(tb::current_device()).sms;
    s = from_cuda(tb::e4m3_flush_launch(A, Af, static_cast<size_t>(M) * K, stream, sms), "E4M3 flush launch");
    if (s != TB_OK) return s;
    s = from_cuda(tb::e4m3_flush_transposed_launch(B, Bf, K, N, stream), "E4M3 transposed flush launch");
    if (s != TB_OK) return s;
    return tb_gemm_native(TB_FMT_E4M3, Af, TB_FMT_E4M3, Bf, D, M, N, K, TB_OUT_F32, 1.0f, stream);
}

}  // extern "C"

tb_status tb::gemm_fused_to_peers(tb_format a_fmt, const void* A, const uint16_t* B, void* D, int M, int N, int K,
                                  tb_out_type out, float alpha, int n_peers, void* const* peer_D, tb_stream_t stream) {
    if (a_fmt == TB_FMT_F16) return fail(TB_ERR_INVALID_ARGUMENT, "peer copies need a stored weight format, not F16");
    return fused_request(a_fmt, A, B, D, N, M, N, K, out, alpha, nullptr, 0, stream, n_peers, peer_D);
}
