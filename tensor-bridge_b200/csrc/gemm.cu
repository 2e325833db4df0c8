// gemm.cu -- instantiations and host-side planning of the tcgen05 GEMMs:
// tile width, split-K, TMA tensor maps, launch.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <cuda.h>
#include <cuda_runtime.h>
#include "fused_pair_kernel.cuh"
#include "fused_tmem_kernel.cuh"
#include "gemm_pair_kernel.cuh"
#include "gemm_nvfp4_kernel.cuh"
#include "gemm_kernel.cuh"
#include "tb_host.h"

namespace tb {

cudaError_t device_error_read(int* v) { return cudaMemcpyFromSymbol(v, g_tb_device_error, sizeof(int)); }

cudaError_t device_error_clear() {
    const int zero = 0;
    return cudaMemcpyToSymbol(g_tb_device_error, &zero, sizeof zero);
}

__global__ void k_splitk_reduce(const float* __restrict__ ws, void* D, long long ldd, int M, int N, int splits,
                                float alpha, int out_f16) {
    // Launched with programmatic stream serialisation: let the next GEMM start
    // streaming its weights, then wait for the partials of the GEMM before.
    grid_dep_launch_dependents();
    grid_dep_wait();
    const size_t total = static_cast<size_t>(M) * N;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        float s = 0.0f;
        for (int k = 0; k < splits; ++k) s += ws[static_cast<size_t>(k) * total + i];
        const size_t r = i / N, c = i % N;
        const size_t o = r * static_cast<size_t>(ldd) + c;
        if (out_f16) static_cast<__half*>(D)[o] = __float2half_rn(s * alpha);
        else static_cast<float*>(D)[o] = s * alpha;
    }
}

// ---------------------------------------------------------------------------------
// Device info

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

const DeviceInfo& device_info(int dev) {
    static DeviceInfo infos[64];
    static std::once_flag flags[64];
    dev = std::max(0, std::min(dev, 63));
    std::call_once(flags[dev], [dev]() {
        DeviceInfo& d = infos[dev];
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
        if (d.sms <= 0) d.sms = 148;
    });
    return infos[dev];
}

// ---------------------------------------------------------------------------------
// TMA tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = []() -> EncodeTiledFn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Row-major 2-D map: `inner` elements per row (contiguous), `outer` rows,
// `row_bytes` between rows; box of box_inner x box_outer elements.
static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    std::memset(m, 0, sizeof(*m));
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of a native-mode operand [rows x K]: one 128-element k-block per
// box row, 128-byte swizzle.  FP8 is one byte per element.  Packed FP4 (first
// value in the low nibble) uses the 16U4_ALIGN16B type: TMA expands every 16
// packed elements (8 bytes) to a 16-byte shared-memory chunk, the padded
// layout kind::f8f6f4 reads 4-bit operands from, so a box row is again 128
// bytes and the MMA descriptors match the FP8 case.
static bool make_native_map(CUtensorMap* m, int fmt, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows) {
    if (fmt == kE2M1HW)
        return make_map(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, base, K, rows, K / 2, 128, box_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, base, K, rows, K, 128, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// kind::f8f6f4 operand format codes of the instruction descriptor.
static int f8f6f4_code(int fmt) {
    switch (fmt) {
        case kE4M3: return 0;
        case kE5M2: return 1;
        case kE2M1HW: return 5;
        default: return -1;
    }
}

// Tensor map of a stored-format A [M x K] for the fused kernels: 128-byte
// boxes of 128 rows, 128-byte swizzle (the decode warps read that layout).
template <int FMT>
static bool make_raw_map(CUtensorMap* m, const void* A, uint64_t K, uint64_t M) {
    constexpr uint32_t bx = raw_box_elems(FMT);
    if constexpr (FMT == kE2M1)
        return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K / 2, M, K / 2, bx, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    else if constexpr (FMT == kBF16)
        return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, A, K, M, K * 2, bx, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    else if constexpr (FMT == kTF32)
        return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, A, K, M, K * 4, bx, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    else
        return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K, M, K, bx, 128, CU_TENSOR_MAP_SWIZZLE_128B);
}

// ---------------------------------------------------------------------------------
// Configurations

// Stage counts per configuration.  An operand-ring stage holds a B tile and
// an A tile; fused mode adds a raw-A ring (whose stages also carry the B tiles
// for narrow tiles, BN <= 64).  Fused: up to four operand stages and the rest
// (at least two, at most eight) raw stages.  The decode round DK is the raw
// stage's k-blocks, capped at two for wide tiles and four for narrow ones
// (and below S).
template <int BN, int MODE, int FMT>
struct Pick {
    static constexpr bool kDec = MODE == kModeDecode;
    static constexpr int A = 128 * 128, B = BN * 128;
    static constexpr int RK = kDec ? raw_kblocks(FMT) : 1;
    static constexpr int RA = kDec ? raw_stage_bytes(FMT) + (BN <= 64 ? RK * B : 0) : 0;
    static constexpr int S_MAX = kDec ? (BN >= 128 ? 4 : 8) : 12;
    static constexpr int S0 = (kSmemBudget - 2 * RA) / (A + B);
    static constexpr int S = S0 > S_MAX ? S_MAX : (S0 < 2 ? 2 : S0);
    static constexpr int SA0 = kDec ? (kSmemBudget - S * (A + B)) / RA : 0;
    static constexpr int SA = kDec ? (SA0 > 8 ? 8 : SA0) : 0;
    static constexpr int DK0 = RK < (BN >= 128 ? 2 : 4) ? RK : (BN >= 128 ? 2 : 4);
    // power of two dividing RK, at most S - 1
    static constexpr int DK = DK0 <= S - 1 ? DK0 : (DK0 / 2 <= S - 1 ? DK0 / 2 : 1);
    using Cfg = GemmCfg<BN, MODE, FMT, S, SA, DK>;
};

template <class C>
static cudaError_t launch_cfg(const CUtensorMap& ta, const CUtensorMap& tbm, const GemmArgs& args, cudaStream_t st,
                              int dev) {
    static std::atomic<uint64_t> attr_done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    const int sms = device_info(dev).sms;
    const int grid = std::min(args.num_units, sms);
    k_gemm<C><<<grid, C::NUM_THREADS, C::SMEM_ALLOC, st>>>(ta, tbm, args);
    return cudaGetLastError();
}

static int choose_bn(int N) {
    if (N <= 16) return 16;
    if (N <= 64) return 64;
    if (N <= 128) return 128;
    return 256;
}

static int choose_splits(int units, int num_kb, int sms) {
    if (units * 4 >= sms * 3) return 1;
    int s = sms / std::max(units, 1);
    s = std::min(s, 16);
    s = std::min(s, std::max(1, num_kb / 4));
    return std::max(s, 1);
}

static int kb_elems(GemmKind kind) { return kind == GemmKind::kNative || kind == GemmKind::kInt8 ? 128 : 64; }

size_t gemm_workspace_bytes(GemmKind kind, int a_fmt, int M, int N, int K, int sms) {
    (void)a_fmt;
    if (M <= 0 || N <= 0 || K <= 0 || kind == GemmKind::kNative || kind == GemmKind::kInt8) return 0;
    const int bn = choose_bn(N);
    const int units = ((M + 127) / 128) * ((N + bn - 1) / bn);
    const int num_kb = (K + kb_elems(kind) - 1) / kb_elems(kind);
    const int s = choose_splits(units, num_kb, sms);
    if (s <= 1) return 0;
    return static_cast<size_t>(s) * M * N * sizeof(float);
}

// ---- pairs of SMs (cta_group::2) for the operand-loading modes ------------------------

template <int MODE>
using PairOf = PairCfg<MODE, 6>;

// Clusters of two CTAs of `kernel` (configuration C) that fit on the device at
// once (0 if the query fails); also sets the kernel's shared-memory size.
template <class C, class Kern>
static int cluster_capacity(Kern kernel, int dev) {
    static std::atomic<int> cached[64] = {};
    if (dev < 0 || dev >= 64) return 0;
    int v = cached[dev].load();
    if (v) return v > 0 ? v : 0;
    int n = 0;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * 128, 1, 1);
    cfg.blockDim = dim3(C::NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_ALLOC;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_ALLOC) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    cached[dev].store(n > 0 ? n : -1);
    return n;
}

template <int MODE>
static int pair_clusters(int dev) {
    using C = PairOf<MODE>;
    return cluster_capacity<C>(k_gemm_pair<C>, dev);
}

// Launch of a two-CTA-cluster kernel over `units` pair tiles.
template <class C, class Kern>
static cudaError_t launch_pairs(Kern kernel, const CUtensorMap& ta, const CUtensorMap& tbm, const GemmArgs& args,
                                int units, int clusters, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * std::min(units, clusters), 1, 1);
    cfg.blockDim = dim3(C::NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_ALLOC;
    cfg.stream = st;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, ta, tbm, args);
}

template <int MODE>
static cudaError_t run_pair(const GemmRequest& r, const GemmArgs& args, int clusters, cudaStream_t st,
                            const char** why) {
    using C = PairOf<MODE>;
    CUtensorMap ta, tbm;
    const uint64_t K = static_cast<uint64_t>(r.K);
    bool ok;
    // B in 64-row boxes: one per CTA for a half tile, two for a whole one.
    if constexpr (MODE == kModeF16) {
        ok = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.A, K, r.M, K * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
             make_map(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.B, K, r.N, K * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
    } else if constexpr (MODE == kModeNative8) {
        ok = make_native_map(&ta, r.a_fmt, r.A, K, r.M, 128) && make_native_map(&tbm, r.b_fmt, r.B, K, r.N, 64);
    } else {
        ok = make_native_map(&ta, kE4M3, r.A, K, r.M, 128) && make_native_map(&tbm, kE4M3, r.B, K, r.N, 64);
    }
    if (!ok) {
        *why = "cuTensorMapEncodeTiled rejected the operand layout";
        return cudaErrorInvalidValue;
    }
    // Whole tiles for the full waves; the R tiles of a partial last wave as 2R
    // halves when those fit in one wave (the last wave then takes half a tile).
    const int tiles = ((r.M + C::BM - 1) / C::BM) * ((r.N + C::BN - 1) / C::BN);
    const int rem = tiles % clusters;
    GemmArgs a = args;
    a.pair_full = (rem > 0 && 2 * rem <= clusters) ? tiles - rem : tiles;
    const int units = a.pair_full + 2 * (tiles - a.pair_full);
    return launch_pairs<C>(k_gemm_pair<C>, ta, tbm, a, units, clusters, st);
}

template <int FMT>
static int fused_pair_clusters(int dev) {
    using C = typename PickFusedPair<FMT>::Cfg;
    return cluster_capacity<C>(k_fused_pair<C>, dev);
}

// Clusters of the fused pair kernel of this format that fit at once (0: none,
// or a format without a pair kernel).
static int fused_pair_capacity(int fmt, int dev) {
    switch (fmt) {
        case kE4M3: return fused_pair_clusters<kE4M3>(dev);
        case kE5M2: return fused_pair_clusters<kE5M2>(dev);
        case kE2M1: return fused_pair_clusters<kE2M1>(dev);
        case kE2M1U: return fused_pair_clusters<kE2M1U>(dev);
        case kBF16: return fused_pair_clusters<kBF16>(dev);
        case kTF32: return fused_pair_clusters<kTF32>(dev);
        default: return 0;
    }
}

// Throughput per SM of the fused pair kernel over the one-CTA fused kernel on
// whole waves (measured at 4096^3 on B200): the decode it halves per output
// bounds the one-byte and wider formats; packed FP4 is bound by the MMAs.
static double fused_pair_gain(int fmt) {
    switch (fmt) {
        case kE4M3: case kE5M2: return 1.19;
        case kBF16: return 1.40;
        case kTF32: return 1.57;
        default: return 1.0;
    }
}

// Pair tiles (256 x 512, on two SMs) against one-CTA tiles (128 x 256): a pair
// tile is twice an SM's work of a one-CTA tile, so compare the waves each
// needs, weighted by the pair kernel's gain; ties go to the pair kernel.
static bool fused_pair_wins(int fmt, int M, int N, int clusters, int sms) {
    const long long pair_tiles = static_cast<long long>((M + 255) / 256) * ((N + 511) / 512);
    const long long one_tiles = static_cast<long long>((M + 127) / 128) * ((N + 255) / 256);
    const long long pair_waves = (pair_tiles + clusters - 1) / clusters;
    const long long one_waves = (one_tiles + sms - 1) / sms;
    return 2.0 * static_cast<double>(pair_waves) / fused_pair_gain(fmt) <= static_cast<double>(one_waves) + 1e-9;
}

template <int FMT>
static cudaError_t run_fused_pair(const GemmRequest& r, const GemmArgs& args_in, int clusters, cudaStream_t st,
                                  const char** why) {
    using C = typename PickFusedPair<FMT>::Cfg;
    // Keep the smaller operand resident in L2 across waves (fused_pair_kernel.cuh):
    // N tiles fastest unless the stored A is smaller than B.  (Measured at
    // 4096^3: TF32 152 -> 149 us, BF16 133 -> 130; 8192^3 FP4 keeps M fastest,
    // 649 against 686 us.)
    GemmArgs args = args_in;
    const size_t a_bytes = stored_bytes(FMT, static_cast<size_t>(r.M) * r.K);
    const size_t b_bytes = static_cast<size_t>(r.N) * r.K * 2;
    args.n_fastest = a_bytes >= b_bytes ? 1 : 0;
    CUtensorMap ta, tbm;
    const uint64_t K = static_cast<uint64_t>(r.K);
    if (!make_raw_map<FMT>(&ta, r.A, K, r.M) ||
        !make_map(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.B, K, r.N, K * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) {
        *why = "cuTensorMapEncodeTiled rejected the operand layout";
        return cudaErrorInvalidValue;
    }
    const int units = ((r.M + C::BM - 1) / C::BM) * ((r.N + C::BN - 1) / C::BN);
    if (args.n_peers == 0) return launch_pairs<C>(k_fused_pair<C>, ta, tbm, args, units, clusters, st);
    // The instance with the peer copies: same shared memory and threads, so
    // the plain instance's cluster count holds for it.
    static std::atomic<uint64_t> attr_done{0};
    const uint64_t bit = 1ull << (current_device() & 63);
    if (!(attr_done.load() & bit)) {
        const cudaError_t e =
            cudaFuncSetAttribute(k_fused_pair<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    return launch_pairs<C>(k_fused_pair<C, true>, ta, tbm, args, units, clusters, st);
}

template <int BN, int MODE, int FMT>
static cudaError_t run(const GemmRequest& r, const GemmArgs& args, cudaStream_t st, int dev, const char** why) {
    using C = typename Pick<BN, MODE, FMT>::Cfg;
    CUtensorMap ta, tbm;
    bool ok;
    const uint64_t K = static_cast<uint64_t>(r.K);
    if constexpr (MODE == kModeF16) {
        ok = make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.A, K, r.M, K * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
        ok = ok && make_map(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.B, K, r.N, K * 2, 64, BN,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    } else if constexpr (MODE == kModeNative8) {
        ok = make_native_map(&ta, r.a_fmt, r.A, K, r.M, 128) && make_native_map(&tbm, r.b_fmt, r.B, K, r.N, BN);
    } else if constexpr (MODE == kModeInt8) {
        ok = make_native_map(&ta, kE4M3, r.A, K, r.M, 128) && make_native_map(&tbm, kE4M3, r.B, K, r.N, BN);
    } else {
        ok = make_raw_map<FMT>(&ta, r.A, K, r.M);
        ok = ok && make_map(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.B, K, r.N, K * 2, 64, BN,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (!ok) {
        *why = "cuTensorMapEncodeTiled rejected the operand layout";
        return cudaErrorInvalidValue;
    }
    return launch_cfg<C>(ta, tbm, args, st, dev);
}

template <int BN, int FMT>
static cudaError_t run_tmem(const GemmRequest& r, const GemmArgs& args, cudaStream_t st, int dev, const char** why) {
    using C = typename PickTmem<BN, FMT>::Cfg;
    CUtensorMap ta, tbm;
    const uint64_t K = static_cast<uint64_t>(r.K);
    bool ok = make_raw_map<FMT>(&ta, r.A, K, r.M);
    ok = ok && make_map(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT16, r.B, K, r.N, K * 2, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) {
        *why = "cuTensorMapEncodeTiled rejected the operand layout";
        return cudaErrorInvalidValue;
    }
    static std::atomic<uint64_t> attr_done{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_done.load() & bit)) {
        cudaError_t e = cudaFuncSetAttribute(k_fused_tmem<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_ALLOC);
        if (e != cudaSuccess) return e;
        attr_done.fetch_or(bit);
    }
    // Programmatic stream serialisation: the kernel may start while the
    // previous kernel in the stream is still running, if that kernel allows it
    // (another narrow GEMM does, right after its set-up); it waits for that
    // kernel before reading B and before storing D (k_fused_tmem).
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(std::min(args.num_units, device_info(dev).sms), 1, 1);
    cfg.blockDim = dim3(C::NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_ALLOC;
    cfg.stream = st;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_fused_tmem<C>, ta, tbm, args);
}

template <int MODE, int FMT>
static cudaError_t run_bn(int bn, const GemmRequest& r, const GemmArgs& a, cudaStream_t st, int dev, const char** why) {
    if constexpr (MODE == kModeDecode) {
        if (bn == 16) return run_tmem<16, FMT>(r, a, st, dev, why);
        if (bn == 64) return run_tmem<64, FMT>(r, a, st, dev, why);
        // 128 columns: the B tiles (64 KB a round) leave room for a raw ring of
        // two rounds only with the one-byte and half-byte formats.
        if constexpr (raw_row_bytes(FMT) <= 64)
            if (bn == 128) return run_tmem<128, FMT>(r, a, st, dev, why);
    }
    switch (bn) {
        case 16: return run<16, MODE, FMT>(r, a, st, dev, why);
        case 64: return run<64, MODE, FMT>(r, a, st, dev, why);
        case 128: return run<128, MODE, FMT>(r, a, st, dev, why);
        case 256: return run<256, MODE, FMT>(r, a, st, dev, why);
        default: *why = "unsupported tile width"; return cudaErrorInvalidValue;
    }
}

// ---- block-scaled FP4 (kind::mxf4nvf4) on SM pairs --------------------------------------

using Nvfp4Of = Nvfp4Cfg<5>;

cudaError_t nvfp4_gemm_launch(const void* A, const uint8_t* sfa, const void* B, const uint8_t* sfb, void* D, int M,
                              int N, int K, int out_f16, float alpha, cudaStream_t st, const char** why) {
    using C = Nvfp4Of;
    const int dev = current_device();
    const int clusters = cluster_capacity<C>(k_gemm_nvfp4<C>, dev);
    if (clusters <= 0) {
        *why = "no room for a two-CTA cluster of the block-scaled FP4 kernel";
        return cudaErrorInvalidConfiguration;
    }
    CUtensorMap ta, tbm, tsa, tsb;
    const uint64_t kb = static_cast<uint64_t>(K) / 2;   // code bytes per row
    const uint64_t ks = static_cast<uint64_t>(K) / 16;  // scale bytes per row
    if (!make_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, kb, M, kb, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tbm, CU_TENSOR_MAP_DATA_TYPE_UINT8, B, kb, N, kb, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, sfa, ks, M, ks, 16, 128, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, sfb, ks, N, ks, 16, 256, CU_TENSOR_MAP_SWIZZLE_NONE)) {
        *why = "cuTensorMapEncodeTiled rejected the operand layout";
        return cudaErrorInvalidValue;
    }
    GemmArgs a{};
    a.M = M; a.N = N; a.K = K;
    a.tiles_m = (M + C::BM - 1) / C::BM;
    a.tiles_n = (N + C::BN - 1) / C::BN;
    a.splits = 1;
    a.num_kb = K / C::KB_VALUES;
    a.kb_per_split = a.num_kb;
    a.num_units = a.tiles_m * a.tiles_n;
    a.half_from = a.num_units;
    a.pair_full = a.num_units;
    a.alpha = alpha;
    a.D = D; a.ldd = N;
    a.out_f16 = out_f16;
    const int vec_elems = out_f16 ? 8 : 4;
    a.vec_ok = ((reinterpret_cast<uintptr_t>(D) & 15u) == 0 && (N % vec_elems) == 0) ? 1 : 0;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * std::min(a.num_units, clusters), 1, 1);
    cfg.blockDim = dim3(C::NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_ALLOC;
    cfg.stream = st;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_gemm_nvfp4<C>, ta, tbm, tsa, tsb, a);
}

cudaError_t gemm_launch(const GemmRequest& r, cudaStream_t st, const char** why) {
    const int dev = current_device();
    const int sms = device_info(dev).sms;
    const int bn = r.force_bn ? r.force_bn : choose_bn(r.N);
    const int tiles_m = (r.M + 127) / 128;
    const int tiles_n = (r.N + bn - 1) / bn;
    const int num_kb = (r.K + kb_elems(r.kind) - 1) / kb_elems(r.kind);
    int splits = 1;
    if (r.kind != GemmKind::kNative && r.kind != GemmKind::kInt8) {
        splits = r.force_splits ? r.force_splits : choose_splits(tiles_m * tiles_n, num_kb, sms);
        splits = std::max(1, std::min(splits, num_kb));
    }
    // Each split starts on a round boundary (four k-blocks) of the fused kernels.
    const int rk = r.kind == GemmKind::kFused ? 4 : 1;
    int kb_per = (num_kb + splits - 1) / splits;
    kb_per = (kb_per + rk - 1) / rk * rk;
    splits = (num_kb + kb_per - 1) / kb_per;
    if (splits > 1) {
        const size_t need = static_cast<size_t>(splits) * r.M * r.N * sizeof(float);
        if (r.workspace == nullptr || r.workspace_bytes < need) {
            splits = 1;  // no room for partial sums: run unsplit
            kb_per = num_kb;
        }
    }

    GemmArgs a{};
    a.M = r.M; a.N = r.N; a.K = r.K;
    a.tiles_m = tiles_m; a.tiles_n = tiles_n; a.splits = splits;
    a.kb_per_split = kb_per; a.num_kb = num_kb;
    a.num_units = tiles_m * tiles_n * splits;
    a.half_from = a.num_units;  // no half tiles unless set below (one-CTA kernel)
    a.alpha = r.alpha;
    a.D = r.D; a.ldd = r.ldd;
    a.out_f16 = r.out_f16;
    a.out_i32 = r.kind == GemmKind::kInt8 ? 1 : 0;
    if (a.out_i32) a.tx_bytes = 128u * 128u + static_cast<uint32_t>(bn) * 128u;
    const int vec_elems = r.out_f16 ? 8 : 4;
    a.vec_ok = ((reinterpret_cast<uintptr_t>(r.D) & 15u) == 0 && (r.ldd % vec_elems) == 0) ? 1 : 0;
    a.ws = splits > 1 ? static_cast<float*>(r.workspace) : nullptr;
    if (r.kind == GemmKind::kFused && r.a_fmt == kE4M3) a.acc_shift = kE4M3AccShift;  // decode_e4m3_x4_scaled
    if (r.n_peers > 0) {
        // Tiles copied to other GPUs' D: the fused pair kernel's epilogue does it.
        if (r.kind != GemmKind::kFused || r.n_peers > kMaxPeers || splits != 1) {
            *why = "peer copies need an unsplit fused GEMM and at most 7 peers";
            return cudaErrorInvalidValue;
        }
        a.n_peers = r.n_peers;
        for (int i = 0; i < r.n_peers; ++i) a.peer_D[i] = r.peer_D[i];
        const int clusters = fused_pair_capacity(r.a_fmt, dev);
        switch (clusters > 0 ? r.a_fmt : -1) {
            case kE4M3: return run_fused_pair<kE4M3>(r, a, clusters, st, why);
            case kE5M2: return run_fused_pair<kE5M2>(r, a, clusters, st, why);
            case kE2M1: return run_fused_pair<kE2M1>(r, a, clusters, st, why);
            case kE2M1U: return run_fused_pair<kE2M1U>(r, a, clusters, st, why);
            case kBF16: return run_fused_pair<kBF16>(r, a, clusters, st, why);
            case kTF32: return run_fused_pair<kTF32>(r, a, clusters, st, why);
            default: *why = "the fused pair kernel cannot run this format on this device"; return cudaErrorInvalidValue;
        }
    }
    if (r.kind == GemmKind::kNative) {
        const int ca = f8f6f4_code(r.a_fmt), cb = f8f6f4_code(r.b_fmt);
        if (ca < 0 || cb < 0) { *why = "native GEMM operands must be E4M3, E5M2 or E2M1_HW"; return cudaErrorInvalidValue; }
        a.idesc_ab = (static_cast<uint32_t>(ca) << 7) | (static_cast<uint32_t>(cb) << 10);
        // A TMA box of 16U4_ALIGN16B data credits the packed bytes it reads
        // (64 per 128-value row), not the padded bytes it writes.
        auto row_bytes = [](int f) { return f == kE2M1HW ? 64u : 128u; };
        a.tx_bytes = 128u * row_bytes(r.a_fmt) + static_cast<uint32_t>(bn) * row_bytes(r.b_fmt);
    }

    // Pairs of SMs for the operand-loading kinds when the tiles are wide and
    // plentiful (256 x 256 tiles per cluster, those of a partial last wave as
    // 256 x 128 halves; no split).
    const bool loading = r.kind == GemmKind::kF16 || r.kind == GemmKind::kNative || r.kind == GemmKind::kInt8;
    if (loading && bn == 256 && splits == 1 && r.M >= 256 && !r.force_bn && !r.force_splits) {
        const int mode = r.kind == GemmKind::kF16 ? kModeF16 : r.kind == GemmKind::kNative ? kModeNative8 : kModeInt8;
        const int clusters = mode == kModeF16 ? pair_clusters<kModeF16>(dev)
                             : mode == kModeNative8 ? pair_clusters<kModeNative8>(dev)
                                                    : pair_clusters<kModeInt8>(dev);
        if (clusters > 0) {
            // Bytes each CTA stages per k-block: 128 rows of A and 128 of B.
            auto row_bytes = [&](int f) -> uint32_t {
                return r.kind == GemmKind::kF16 ? 128u : (f == kE2M1HW ? 64u : 128u);
            };
            a.tx_bytes = 128u * row_bytes(r.a_fmt) + 128u * row_bytes(r.kind == GemmKind::kNative ? r.b_fmt : r.a_fmt);
            a.tx_b_half = 64u * row_bytes(r.kind == GemmKind::kNative ? r.b_fmt : r.a_fmt);
            if (r.kind == GemmKind::kInt8) {
                a.tx_bytes = 2u * 128u * 128u;
                a.tx_b_half = 64u * 128u;
            }
            if (r.kind != GemmKind::kNative) a.idesc_ab = 0;
            cudaError_t e2 = mode == kModeF16 ? run_pair<kModeF16>(r, a, clusters, st, why)
                             : mode == kModeNative8 ? run_pair<kModeNative8>(r, a, clusters, st, why)
                                                    : run_pair<kModeInt8>(r, a, clusters, st, why);
            return e2;
        }
    }

    // Fused decode on SM pairs (256 x 512 tiles) for at least 512 columns,
    // tiles enough not to split K, and fewer waves' worth of work than the
    // one-CTA kernel.
    if (r.kind == GemmKind::kFused && r.N >= 512 && splits == 1 && r.M >= 256 && !r.force_bn && !r.force_splits) {
        const int clusters = fused_pair_capacity(r.a_fmt, dev);
        if (clusters > 0 && fused_pair_wins(r.a_fmt, r.M, r.N, clusters, sms)) {
            switch (r.a_fmt) {
                case kE4M3: return run_fused_pair<kE4M3>(r, a, clusters, st, why);
                case kE5M2: return run_fused_pair<kE5M2>(r, a, clusters, st, why);
                case kE2M1: return run_fused_pair<kE2M1>(r, a, clusters, st, why);
                case kE2M1U: return run_fused_pair<kE2M1U>(r, a, clusters, st, why);
                case kBF16: return run_fused_pair<kBF16>(r, a, clusters, st, why);
                case kTF32: return run_fused_pair<kTF32>(r, a, clusters, st, why);
                default: break;
            }
        }
    }

    // One-CTA kernel, 256-column tiles without a split: the R tiles of a
    // partial last wave (or all tiles, when fewer than the SMs) run as 2R
    // halves of 128 columns when those fit in one wave.
    if (bn == 256 && splits == 1) {
        const int tiles = a.num_units;
        const int rem = tiles > sms ? tiles % sms : tiles;
        if (rem > 0 && 2 * rem <= sms) {
            a.half_from = tiles - rem;
            a.num_units = tiles + rem;
        }
    }

    cudaError_t e;
    switch (r.kind) {
        case GemmKind::kF16: e = run_bn<kModeF16, kF16>(bn, r, a, st, dev, why); break;
        case GemmKind::kNative:
            if (bn == 16) e = run<16, kModeNative8, kE4M3>(r, a, st, dev, why);
            else if (bn == 64) e = run<64, kModeNative8, kE4M3>(r, a, st, dev, why);
            else if (bn == 128) e = run<128, kModeNative8, kE4M3>(r, a, st, dev, why);
            else e = run<256, kModeNative8, kE4M3>(r, a, st, dev, why);
            break;
        case GemmKind::kInt8:
            if (bn == 16) e = run<16, kModeInt8, kE4M3>(r, a, st, dev, why);
            else if (bn == 64) e = run<64, kModeInt8, kE4M3>(r, a, st, dev, why);
            else if (bn == 128) e = run<128, kModeInt8, kE4M3>(r, a, st, dev, why);
            else e = run<256, kModeInt8, kE4M3>(r, a, st, dev, why);
            break;
        case GemmKind::kFused:
            switch (r.a_fmt) {
                case kE4M3: e = run_bn<kModeDecode, kE4M3>(bn, r, a, st, dev, why); break;
                case kE5M2: e = run_bn<kModeDecode, kE5M2>(bn, r, a, st, dev, why); break;
                case kE2M1: e = run_bn<kModeDecode, kE2M1>(bn, r, a, st, dev, why); break;
                case kE2M1U: e = run_bn<kModeDecode, kE2M1U>(bn, r, a, st, dev, why); break;
                case kBF16: e = run_bn<kModeDecode, kBF16>(bn, r, a, st, dev, why); break;
                case kTF32: e = run_bn<kModeDecode, kTF32>(bn, r, a, st, dev, why); break;
                case kF16: e = run_bn<kModeF16, kF16>(bn, r, a, st, dev, why); break;
                default: *why = "unsupported weight format"; return cudaErrorInvalidValue;
            }
            break;
        default: *why = "unknown GEMM kind"; return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || splits <= 1) return e;
    const size_t total = static_cast<size_t>(r.M) * r.N;
    const int blocks = static_cast<int>(std::min<size_t>((total + 255) / 256, static_cast<size_t>(sms) * 8));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(std::max(blocks, 1), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_splitk_reduce, static_cast<const float*>(a.ws), r.D, static_cast<long long>(r.ldd),
                              r.M, r.N, splits, r.alpha, r.out_f16);
}

}  // namespace tb
