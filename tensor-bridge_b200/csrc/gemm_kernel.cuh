// gemm_kernel.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M x N] = alpha * A[M x K] * B[N x K]^T      (both operands K-major)
//
// One CTA per SM walks a static list of work units (128 x BN output tiles,
// optionally split along K).  Roles:
//   warp 0      TMA producer: raw A (or FP16 / FP8 A) and B tiles into an
//               R-stage ring of shared memory (one elected lane)
//   warp 1      TMEM allocator and MMA issuer: one lane issues
//               tcgen05.mma (M = 128, N = BN, 32 bytes of K per instruction)
//               into one of two TMEM accumulators
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns the
//               32 TMEM lanes = tile rows of its warp-id quarter), scale by
//               alpha, convert, store to global memory
//   warps 6..   (fused mode only) decode warps: read the raw A tile that TMA
//               staged, decode it to FP16 and write it, 128-byte swizzled,
//               into a D-stage ring the MMA reads directly
//
// Shared-memory operand tiles use the canonical K-major SWIZZLE_128B layout:
// 128-byte rows (64 FP16 or 128 FP8 values of K), 8-row groups of 1024 bytes,
// the 16-byte chunk c of row r stored at chunk position c ^ (r & 7).  TMA
// writes that layout itself; the decode warps write it explicitly.
//
// Every mbarrier wait is bounded (tb_ptx.cuh): on expiry the kernel sets the
// device error word, all roles leave their loops, and the TMEM allocation is
// released before the CTA exits.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include "tb_ptx.cuh"
#include "tb_decode.cuh"

namespace tb {

enum : int { kModeF16 = 0, kModeDecode = 1, kModeNative8 = 2 };

// Stored-format ids (same values as tb_format in the C header).
enum : int { kF16 = 0, kE4M3 = 1, kE5M2 = 2, kE2M1 = 3, kE2M1U = 4, kBF16 = 5, kTF32 = 6, kE2M1HW = 7 };

// Bytes of one 64-value K slice of one row, per stored format.
__host__ __device__ constexpr int raw_row_bytes(int fmt) {
    return fmt == kE2M1 ? 32 : fmt == kBF16 ? 128 : fmt == kTF32 ? 256 : fmt == kF16 ? 128 : 64;
}

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }
__host__ __device__ constexpr int pow2_at_least(int x) {
    return x <= 32 ? 32 : x <= 64 ? 64 : x <= 128 ? 128 : x <= 256 ? 256 : 512;
}

// Compile-time configuration of one kernel instance.
template <int BN_, int MODE_, int FMT_, int SR_, int SD_>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int MODE = MODE_;
    static constexpr int FMT = FMT_;
    static constexpr int SR = SR_;                          // R ring stages (A-or-raw + B)
    static constexpr int SD = MODE == kModeDecode ? SD_ : 0;  // D ring stages (decoded A)
    static constexpr int ND = MODE == kModeDecode ? 4 : 0;    // decode warps
    static constexpr int NUM_THREADS = 192 + ND * 32;
    static constexpr int DECODE_THREADS = ND * 32;

    static constexpr int A_BYTES = BM * 128;  // one swizzled 128 x 128-byte operand tile
    static constexpr int B_BYTES = BN * 128;
    static constexpr int RA_BYTES = MODE == kModeDecode ? BM * raw_row_bytes(FMT) : A_BYTES;
    // K elements per k-block and the TMA inner-coordinate step of A and B.
    static constexpr int KB_ELEMS = MODE == kModeNative8 ? 128 : 64;
    static constexpr int A_X_STEP = MODE == kModeDecode && FMT == kE2M1 ? 32 : KB_ELEMS;
    static constexpr int B_X_STEP = KB_ELEMS;

    static constexpr int OFF_B = 0;
    static constexpr int OFF_RA = OFF_B + SR * B_BYTES;
    static constexpr int OFF_D = OFF_RA + SR * RA_BYTES;
    static constexpr int OFF_BAR = OFF_D + SD * A_BYTES;
    static constexpr int NUM_BARS = 2 * SR + 2 * SD + 5;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to 1024-align the base

    static constexpr int TMEM_COLS = pow2_at_least(2 * BN);
    static constexpr int CW = BN < 32 ? BN : 32;  // epilogue column chunk

    // MMA formats: kind::f16 with FP16 operands, or kind::f8f6f4 with E4M3.
    static constexpr uint32_t IDESC = idesc_make(0u, 0u, BM, BN);

    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN");
    static_assert(B_BYTES % 1024 == 0 && RA_BYTES % 1024 == 0, "stage alignment");
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct GemmArgs {
    int M, N, K;
    int tiles_m, tiles_n, splits;
    int kb_per_split, num_kb;
    int num_units;
    float alpha;
    void* D;         // output (row stride ldd elements)
    long long ldd;
    int out_f16;     // 1: FP16 output, 0: FP32
    int vec_ok;      // 1: D rows allow 16-byte vector stores
    float* ws;       // split-K partials [splits][M][N] (FP32), when splits > 1
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a swizzled tile.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// Decode raw 16-byte unit q of a staged A tile into the swizzled FP16 tile.
template <int FMT>
__device__ __forceinline__ void decode_unit(const uint8_t* raw, uint8_t* dst, int q) {
    const uint4 in = *reinterpret_cast<const uint4*>(raw + q * 16);
    if constexpr (FMT == kE4M3 || FMT == kE5M2 || FMT == kE2M1U) {
        const int row = q >> 2, c0 = (q & 3) * 2;
        uint32_t o[8];
        if constexpr (FMT == kE4M3) {
            decode_e4m3_x4(in.x, o[0], o[1]); decode_e4m3_x4(in.y, o[2], o[3]);
            decode_e4m3_x4(in.z, o[4], o[5]); decode_e4m3_x4(in.w, o[6], o[7]);
        } else if constexpr (FMT == kE5M2) {
            decode_e5m2_x4(in.x, o[0], o[1]); decode_e5m2_x4(in.y, o[2], o[3]);
            decode_e5m2_x4(in.z, o[4], o[5]); decode_e5m2_x4(in.w, o[6], o[7]);
        } else {
            decode_e2m1_unpacked_x4(in.x, o[0], o[1]); decode_e2m1_unpacked_x4(in.y, o[2], o[3]);
            decode_e2m1_unpacked_x4(in.z, o[4], o[5]); decode_e2m1_unpacked_x4(in.w, o[6], o[7]);
        }
        *reinterpret_cast<uint4*>(dst + swz(row, c0)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(dst + swz(row, c0 + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    } else if constexpr (FMT == kE2M1) {
        const int row = q >> 1, c0 = (q & 1) * 4;
        uint32_t o[4];
        decode_e2m1_packed_x8(in.x, o);
        *reinterpret_cast<uint4*>(dst + swz(row, c0 + 0)) = make_uint4(o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.y, o);
        *reinterpret_cast<uint4*>(dst + swz(row, c0 + 1)) = make_uint4(o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.z, o);
        *reinterpret_cast<uint4*>(dst + swz(row, c0 + 2)) = make_uint4(o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.w, o);
        *reinterpret_cast<uint4*>(dst + swz(row, c0 + 3)) = make_uint4(o[0], o[1], o[2], o[3]);
    } else if constexpr (FMT == kBF16) {
        const int row = q >> 3, c = q & 7;
        *reinterpret_cast<uint4*>(dst + swz(row, c)) =
            make_uint4(decode_bf16_x2(in.x), decode_bf16_x2(in.y), decode_bf16_x2(in.z), decode_bf16_x2(in.w));
    } else if constexpr (FMT == kTF32) {
        const int row = q >> 4, c = (q & 15) >> 1;
        *reinterpret_cast<uint2*>(dst + swz(row, c) + (q & 1) * 8) =
            make_uint2(decode_tf32_x2(in.x, in.y), decode_tf32_x2(in.z, in.w));
    }
}

// Unit index -> (tile_m, tile_n, split).  M tiles vary fastest so that the
// CTAs running at the same time share B tiles.
__device__ __forceinline__ void unit_coords(const GemmArgs& p, int u, int& tm, int& tn, int& sp) {
    tm = u % p.tiles_m;
    const int r = u / p.tiles_m;
    tn = r % p.tiles_n;
    sp = r / p.tiles_n;
}

template <int CW>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&v)[CW]) {
    if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr, v);
    else tmem_ld_32x32b_x16(taddr, v);
}

// Store CW accumulator values of one row.
template <int CW>
__device__ __forceinline__ void store_row_chunk(const GemmArgs& p, int sp, int row, int col0, const uint32_t (&v)[CW]) {
    if (row >= p.M) return;
    const bool full = col0 + CW <= p.N;
    if (p.splits > 1) {
        float* dst = p.ws + (static_cast<size_t>(sp) * p.M + row) * static_cast<size_t>(p.N) + col0;
        if (full && (p.N & 3) == 0) {
#pragma unroll
            for (int j = 0; j < CW; j += 4)
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = __uint_as_float(v[j]);
        }
        return;
    }
    const float a = p.alpha;
    if (p.out_f16) {
        __half* dst = static_cast<__half*>(p.D) + static_cast<size_t>(row) * p.ldd + col0;
        if (full && p.vec_ok) {
#pragma unroll
            for (int j = 0; j < CW; j += 8) {
                uint32_t w[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const __half2 t = __floats2half2_rn(__uint_as_float(v[j + 2 * h]) * a,
                                                        __uint_as_float(v[j + 2 * h + 1]) * a);
                    w[h] = *reinterpret_cast<const uint32_t*>(&t);
                }
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = __float2half_rn(__uint_as_float(v[j]) * a);
        }
    } else {
        float* dst = static_cast<float*>(p.D) + static_cast<size_t>(row) * p.ldd + col0;
        if (full && p.vec_ok) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
                *reinterpret_cast<float4*>(dst + j) =
                    make_float4(__uint_as_float(v[j]) * a, __uint_as_float(v[j + 1]) * a,
                                __uint_as_float(v[j + 2]) * a, __uint_as_float(v[j + 3]) * a);
            }
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = __uint_as_float(v[j]) * a;
        }
    }
}

template <class C>
__global__ void __launch_bounds__(C::NUM_THREADS, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sbase = smem_addr(smem);

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* r_full = bars;
    uint64_t* r_empty = bars + C::SR;
    uint64_t* d_full = bars + 2 * C::SR;
    uint64_t* d_empty = d_full + C::SD;
    uint64_t* acc_full = d_empty + C::SD;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* fin_bar = acc_empty + 2;  // MMA drain on the abort path
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::SR; ++s) {
            mbar_init(&r_full[s], 1);
            mbar_init(&r_empty[s], C::MODE == kModeDecode ? 1 + C::DECODE_THREADS : 1);
        }
        for (int s = 0; s < C::SD; ++s) {
            mbar_init(&d_full[s], C::DECODE_THREADS);
            mbar_init(&d_empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 128);
        }
        mbar_init(fin_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                int tm, tn, sp;
                unit_coords(p, u, tm, tn, sp);
                const int kb0 = sp * p.kb_per_split;
                const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&r_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
                    mbar_arrive_expect_tx(&r_full[s], C::RA_BYTES + C::B_BYTES);
                    tma_load_2d(smem + C::OFF_RA + s * C::RA_BYTES, &tmA, &r_full[s], kb * C::A_X_STEP, tm * C::BM);
                    tma_load_2d(smem + C::OFF_B + s * C::B_BYTES, &tmB, &r_full[s], kb * C::B_X_STEP, tn * C::BN);
                    ++issued;
                    if (++s == C::SR) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) {
                // Abort path: let the copies already issued land before the
                // CTA's shared memory goes away.
                for (int st = 0; st < C::SR && st < issued; ++st) {
                    const long long last = st + (long long)C::SR * ((issued - 1 - st) / C::SR);
                    mbar_wait_drain(&r_full[st], static_cast<uint32_t>((last / C::SR) & 1));
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int rs = 0, ds = 0;
            uint32_t rph = 0, dph = 0;
            int t = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++t) {
                int tm, tn, sp;
                unit_coords(p, u, tm, tn, sp);
                const int kb0 = sp * p.kb_per_split;
                const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
                const int acc = t & 1;
                const uint32_t aph = (t >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&r_full[rs], rph, abort_flag)) { ok = false; break; }
                    uint32_t a_off;
                    if constexpr (C::MODE == kModeDecode) {
                        if (!mbar_wait(&d_full[ds], dph, abort_flag)) { ok = false; break; }
                        a_off = C::OFF_D + ds * C::A_BYTES;
                    } else {
                        a_off = C::OFF_RA + rs * C::RA_BYTES;
                    }
                    tc_fence_after();
                    const uint32_t b_off = C::OFF_B + rs * C::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = sdesc_k_sw128(sbase + a_off + kk * 32);
                        const uint64_t bd = sdesc_k_sw128(sbase + b_off + kk * 32);
                        const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
                        if constexpr (C::MODE == kModeNative8) mma_f8f6f4_ss(d_tmem, ad, bd, C::IDESC, accum);
                        else mma_f16_ss(d_tmem, ad, bd, C::IDESC, accum);
                    }
                    if constexpr (C::MODE == kModeDecode) {
                        mma_commit(&d_empty[ds]);
                        if (++ds == C::SD) { ds = 0; dph ^= 1u; }
                    }
                    mma_commit(&r_empty[rs]);
                    if (++rs == C::SR) { rs = 0; rph ^= 1u; }
                }
                if (!ok) break;
                mma_commit(&acc_full[acc]);
            }
            if (!ok || *abort_flag) {
                // Abort path: wait for the MMAs already issued before TMEM is freed.
                mma_commit(fin_bar);
                mbar_wait_drain(fin_bar, 0u);
            }
        }
    } else if (warp < 6) {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
        int t = 0;
        for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++t) {
            int tm, tn, sp;
            unit_coords(p, u, tm, tn, sp);
            const int acc = t & 1;
            const uint32_t aph = (t >> 1) & 1;
            const bool ok = mbar_wait(&acc_full[acc], aph, abort_flag);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            tc_fence_after();
            const int row = tm * C::BM + quarter * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * C::BN);
#pragma unroll 1
            for (int c = 0; c < C::BN; c += C::CW) {
                uint32_t v[C::CW];
                tmem_ld_chunk<C::CW>(t_row + c, v);
                tmem_wait_ld();
                store_row_chunk<C::CW>(p, sp, row, tn * C::BN + c, v);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
        }
    } else {
        // ---------------- decode warps (fused mode) ----------------
        if constexpr (C::MODE == kModeDecode) {
            constexpr int UNITS = C::RA_BYTES / 16;
            const int dt = threadIdx.x - 192;
            int rs = 0, ds = 0;
            uint32_t rph = 0, dph = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                int tm, tn, sp;
                unit_coords(p, u, tm, tn, sp);
                const int kb0 = sp * p.kb_per_split;
                const int kb1 = min(p.num_kb, kb0 + p.kb_per_split);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&r_full[rs], rph, abort_flag)) { ok = false; break; }
                    if (!mbar_wait(&d_empty[ds], dph ^ 1u, abort_flag)) { ok = false; break; }
                    const uint8_t* raw = smem + C::OFF_RA + rs * C::RA_BYTES;
                    uint8_t* dst = smem + C::OFF_D + ds * C::A_BYTES;
#pragma unroll 4
                    for (int q = dt; q < UNITS; q += C::DECODE_THREADS) decode_unit<C::FMT>(raw, dst, q);
                    fence_proxy_async_smem();
                    mbar_arrive(&d_full[ds]);
                    mbar_arrive(&r_empty[rs]);
                    if (++rs == C::SR) { rs = 0; rph ^= 1u; }
                    if (++ds == C::SD) { ds = 0; dph ^= 1u; }
                }
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// Split-K reduction: D = alpha * sum over splits of the FP32 partials.
__global__ void k_splitk_reduce(const float* __restrict__ ws, void* D, long long ldd, int M, int N, int splits,
                                float alpha, int out_f16);

}  // namespace tb
