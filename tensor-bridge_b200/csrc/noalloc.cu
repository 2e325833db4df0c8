// noalloc.cu -- tb_gemm_fused_noalloc: the fused decode-in-shared-memory GEMM
// with its split-K partial sums kept in a fixed array compiled into this
// library instead of a caller-supplied workspace.
//
// Who needs it: a plugin hosted by a runtime that owns every byte of device
// memory (a serving engine that reserves HBM for weights and caches at start-up
// and routes all later allocations through its own pool) cannot call
// cudaMalloc behind the runtime's back, and often cannot hand a library a
// workspace pointer either because the plugin interface has no slot for one.
// cudaMalloc/cudaFree may also synchronise the device, which a latency-bound
// decode step cannot afford.  This entry point allocates nothing: no
// cudaMalloc, no cudaFree, no allocating library routine.
//
// The array is shared by every call on a device and keeps whatever the last
// call left in it.  Nothing in it has to start at zero: every split writes its
// whole M x N slice of partial sums before the reduction kernel reads it.
// Calls that overlap in time on one device (different streams with no ordering
// between them) race on the array; calls on one stream are ordered and safe.
#include <mutex>
#include <cuda_runtime.h>
#include "tensor_bridge_b200.h"
#include "tb_host.h"

namespace {

// 20 MiB.  On a 148-SM B200 the split heuristic keeps splits x tiles <= 148
// and one tile's partials are at most 128 x 256 FP32 (128 KiB), so every
// shape needs at most 148 x 128 KiB = 18.5 MiB; larger needs are rejected.
constexpr size_t kScratchBytes = size_t(20) << 20;

static __device__ __align__(256) unsigned char g_splitk_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's copy of g_splitk_scratch, looked up once per
// device with that device current.
tb_status scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return tb::set_last_error(TB_ERR_CUDA, "cudaGetDevice failed", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return tb::set_last_error(TB_ERR_UNSUPPORTED, "device ordinal out of range", "");
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_splitk_scratch);
        if (e != cudaSuccess || p == nullptr)
            return tb::set_last_error(TB_ERR_CUDA, "cudaGetSymbolAddress of the split-K scratch failed",
                                      cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return TB_OK;
}

}  // namespace

extern "C" {

tb_status tb_gemm_fused_noalloc(tb_format a_fmt, const void* A, const uint16_t* B, void* D, int M, int N, int K,
                                tb_out_type out, float alpha, tb_stream_t stream) {
    void* scratch = nullptr;
    tb_status s = scratch_for_current_device(&scratch);
    if (s != TB_OK) return s;
    const size_t need = tb_gemm_fused_workspace(a_fmt, M, N, K);
    if (need > kScratchBytes)
        return tb::set_last_error(TB_ERR_WORKSPACE, "split-K partial sums exceed the fixed 20 MiB scratch",
                                  "use tb_gemm_fused with a caller workspace");
    return tb_gemm_fused(a_fmt, A, B, D, M, N, K, out, alpha, scratch, kScratchBytes, stream);
}

}  // extern "C"
