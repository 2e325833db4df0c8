// gemm_kernel.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M x N] = alpha * A[M x K] * B[N x K]^T      (both operands K-major)
//
// One CTA per SM walks a static list of work units (128 x BN output tiles,
// optionally split along K).  Roles:
//   warp 0      TMA producer of B (and, when A needs no decode, of A) into
//               the operand ring (one elected lane)
//   warp 1      TMEM allocator and MMA issuer: one lane issues tcgen05.mma
//               (M = 128, N = BN, 32 bytes of K per instruction) into one of
//               two TMEM accumulators, so the epilogue of tile t overlaps the
//               main loop of tile t+1
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns the 32
//               TMEM lanes = tile rows of its warp-id quarter), scale by alpha,
//               convert, store to global memory
//   fused mode only:
//   warp 6      TMA producer of the raw (stored-format) A tiles into their own
//               ring, which the decode warps free as soon as they have read a
//               tile -- raw A is prefetched independently of the MMA
//   warps 7..   decode warps: read a staged raw A tile, decode it to FP16 and
//               write it, 128-byte swizzled, into the decoded-A ring the MMA
//               reads directly; decoded weights never leave shared memory
//
// Shared-memory operand tiles use the canonical K-major SWIZZLE_128B layout:
// 128-byte rows (64 FP16 or 128 FP8 values of K), 8-row groups of 1024 bytes,
// the 16-byte chunk c of row r stored at chunk position c ^ (r & 7).  TMA
// writes that layout itself; the decode warps write it explicitly.
//
// Every mbarrier wait is bounded (tb_ptx.cuh): on expiry the kernel sets the
// device error word, all roles leave their loops, asynchronous copies and
// MMAs already issued are drained, and the TMEM allocation is released before
// the CTA exits.
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

__host__ __device__ constexpr int pow2_at_least(int x) {
    return x <= 32 ? 32 : x <= 64 ? 64 : x <= 128 ? 128 : x <= 256 ? 256 : 512;
}

// Compile-time configuration of one kernel instance.
//   S_  operand-ring stages: B tiles (plus A tiles when A needs no decode)
//   SA_ raw-A ring stages (fused mode)
//   SD_ decoded-A ring stages (fused mode)
template <int BN_, int MODE_, int FMT_, int S_, int SA_, int SD_>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int MODE = MODE_;
    static constexpr int FMT = FMT_;
    static constexpr bool kDecode = MODE == kModeDecode;
    static constexpr int S = S_;
    static constexpr int SA = kDecode ? SA_ : 0;
    static constexpr int SD = kDecode ? SD_ : 0;
    static constexpr int ND = kDecode ? 8 : 0;  // decode warps
    static constexpr int DECODE_WARP0 = 7;
    static constexpr int NUM_THREADS = kDecode ? (DECODE_WARP0 + ND) * 32 : 192;
    static constexpr int DECODE_THREADS = ND * 32;

    static constexpr int A_BYTES = BM * 128;  // one swizzled 128-row x 128-byte operand tile
    static constexpr int B_BYTES = BN * 128;
    static constexpr int RA_BYTES = kDecode ? BM * raw_row_bytes(FMT) : 0;
    // K elements per k-block and the TMA inner-coordinate steps.
    static constexpr int KB_ELEMS = MODE == kModeNative8 ? 128 : 64;
    static constexpr int A_X_STEP = kDecode && FMT == kE2M1 ? 32 : KB_ELEMS;
    static constexpr int B_X_STEP = KB_ELEMS;

    // Shared-memory layout (offsets from a 1024-byte aligned base).
    static constexpr int OFF_B = 0;                              // S x B tile
    static constexpr int OFF_A = OFF_B + S * B_BYTES;            // S x A tile (non-fused modes)
    static constexpr int OFF_RA = OFF_A + (kDecode ? 0 : S * A_BYTES);  // SA x raw A tile
    static constexpr int OFF_D = OFF_RA + SA * RA_BYTES;         // SD x decoded A tile
    static constexpr int OFF_BAR = OFF_D + SD * A_BYTES;
    static constexpr int NUM_BARS = 2 * S + 2 * SA + 2 * SD + 5;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to 1024-align the base

    static constexpr int TMEM_COLS = pow2_at_least(2 * BN);
    static constexpr int CW = BN < 32 ? BN : 32;  // epilogue column chunk

    // MMA: kind::f16 with FP16 operands, or kind::f8f6f4 with E4M3 (same
    // format code 0), FP32 accumulation, K-major operands.
    static constexpr uint32_t IDESC = idesc_make(0u, 0u, BM, BN);

    // Raw A units (16 bytes) per k-block and per decode thread.
    static constexpr int UNITS = kDecode ? RA_BYTES / 16 : 0;
    static constexpr int UPT = kDecode ? UNITS / (DECODE_THREADS > 0 ? DECODE_THREADS : 1) : 0;

    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN");
    static_assert(B_BYTES % 1024 == 0 && RA_BYTES % 1024 == 0, "stage alignment");
    static_assert(!kDecode || (UNITS % (DECODE_THREADS > 0 ? DECODE_THREADS : 1) == 0 && UPT >= 1), "decode split");
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

// ---- explicit shared-memory accesses (32-bit shared addresses) ----------------------

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void sts64(uint32_t a, uint32_t x, uint32_t y) {
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a swizzled tile.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// True (warp-uniformly) if any lane's unit holds a code that the fast decode
// path does not reproduce; those units take the scalar reference path.
template <int FMT>
__device__ __forceinline__ bool unit_needs_scalar(const uint4& in) {
    if constexpr (FMT == kE4M3) {
        const uint32_t m = e4m3_special_mask(in.x) | e4m3_special_mask(in.y) | e4m3_special_mask(in.z) |
                           e4m3_special_mask(in.w);
        return __any_sync(0xFFFFFFFFu, m != 0u);
    } else if constexpr (FMT == kBF16) {
        const uint32_t m = bf16_nan_lanes(in.x) | bf16_nan_lanes(in.y) | bf16_nan_lanes(in.z) | bf16_nan_lanes(in.w);
        return __any_sync(0xFFFFFFFFu, m != 0u);
    } else {
        return false;
    }
}

// Decode raw 16-byte unit q (already loaded into `in`) of a staged A tile and
// store it into the swizzled FP16 tile at shared address `dst`.
template <int FMT>
__device__ __forceinline__ void decode_store_unit(const uint4& in, uint32_t dst, int q) {
    if constexpr (FMT == kE4M3 || FMT == kE5M2 || FMT == kE2M1U) {
        const int row = q >> 2, c0 = (q & 3) * 2;
        uint32_t o[8];
        if constexpr (FMT == kE4M3) {
            if (unit_needs_scalar<kE4M3>(in)) {
                decode_e4m3_x4_scalar(in.x, o[0], o[1]); decode_e4m3_x4_scalar(in.y, o[2], o[3]);
                decode_e4m3_x4_scalar(in.z, o[4], o[5]); decode_e4m3_x4_scalar(in.w, o[6], o[7]);
            } else {
                decode_e4m3_x4_fast(in.x, o[0], o[1]); decode_e4m3_x4_fast(in.y, o[2], o[3]);
                decode_e4m3_x4_fast(in.z, o[4], o[5]); decode_e4m3_x4_fast(in.w, o[6], o[7]);
            }
        } else if constexpr (FMT == kE5M2) {
            decode_e5m2_x4(in.x, o[0], o[1]); decode_e5m2_x4(in.y, o[2], o[3]);
            decode_e5m2_x4(in.z, o[4], o[5]); decode_e5m2_x4(in.w, o[6], o[7]);
        } else {
            decode_e2m1_unpacked_x4(in.x, o[0], o[1]); decode_e2m1_unpacked_x4(in.y, o[2], o[3]);
            decode_e2m1_unpacked_x4(in.z, o[4], o[5]); decode_e2m1_unpacked_x4(in.w, o[6], o[7]);
        }
        sts128(dst + swz(row, c0), o[0], o[1], o[2], o[3]);
        sts128(dst + swz(row, c0 + 1), o[4], o[5], o[6], o[7]);
    } else if constexpr (FMT == kE2M1) {
        const int row = q >> 1, c0 = (q & 1) * 4;
        uint32_t o[4];
        decode_e2m1_packed_x8(in.x, o);
        sts128(dst + swz(row, c0 + 0), o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.y, o);
        sts128(dst + swz(row, c0 + 1), o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.z, o);
        sts128(dst + swz(row, c0 + 2), o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.w, o);
        sts128(dst + swz(row, c0 + 3), o[0], o[1], o[2], o[3]);
    } else if constexpr (FMT == kBF16) {
        const int row = q >> 3, c = q & 7;
        if (unit_needs_scalar<kBF16>(in)) {
            sts128(dst + swz(row, c), decode_bf16_x2_scalar(in.x), decode_bf16_x2_scalar(in.y),
                   decode_bf16_x2_scalar(in.z), decode_bf16_x2_scalar(in.w));
        } else {
            sts128(dst + swz(row, c), decode_bf16_x2_fast(in.x), decode_bf16_x2_fast(in.y),
                   decode_bf16_x2_fast(in.z), decode_bf16_x2_fast(in.w));
        }
    } else if constexpr (FMT == kTF32) {
        const int row = q >> 4, c = (q & 15) >> 1;
        sts64(dst + swz(row, c) + (q & 1) * 8, decode_tf32_x2(in.x, in.y), decode_tf32_x2(in.z, in.w));
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

__device__ __forceinline__ void unit_kblocks(const GemmArgs& p, int sp, int& kb0, int& kb1) {
    kb0 = sp * p.kb_per_split;
    kb1 = min(p.num_kb, kb0 + p.kb_per_split);
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

// Abort path of a TMA producer: let the copies already issued into a ring of
// `stages` stages land before the CTA's shared memory goes away.
__device__ __forceinline__ void drain_ring(uint64_t* full, int stages, long long issued) {
    for (int st = 0; st < stages && st < issued; ++st) {
        const long long last = st + static_cast<long long>(stages) * ((issued - 1 - st) / stages);
        mbar_wait_drain(&full[st], static_cast<uint32_t>((last / stages) & 1));
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
    uint64_t* b_full = bars;                  // operand ring: TMA tx complete
    uint64_t* b_empty = b_full + C::S;        // operand ring: MMA done reading
    uint64_t* a_full = b_empty + C::S;        // raw-A ring: TMA tx complete
    uint64_t* a_empty = a_full + C::SA;       // raw-A ring: decode warps done reading
    uint64_t* d_full = a_empty + C::SA;       // decoded-A ring: decode warps done writing
    uint64_t* d_empty = d_full + C::SD;       // decoded-A ring: MMA done reading
    uint64_t* acc_full = d_empty + C::SD;     // accumulator ready for the epilogue
    uint64_t* acc_empty = acc_full + 2;       // accumulator drained by the epilogue
    uint64_t* fin_bar = acc_empty + 2;        // MMA drain on the abort path
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < C::SA; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], C::ND);
        }
        for (int s = 0; s < C::SD; ++s) {
            mbar_init(&d_full[s], C::ND);
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
        // ---------------- TMA producer: B (and A when no decode) ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            bool ok = true;
            constexpr uint32_t kTx = C::B_BYTES + (C::kDecode ? 0 : C::A_BYTES);
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                int tm, tn, sp, kb0, kb1;
                unit_coords(p, u, tm, tn, sp);
                unit_kblocks(p, sp, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&b_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
                    mbar_arrive_expect_tx(&b_full[s], kTx);
                    if constexpr (!C::kDecode)
                        tma_load_2d(smem + C::OFF_A + s * C::A_BYTES, &tmA, &b_full[s], kb * C::KB_ELEMS, tm * C::BM);
                    tma_load_2d(smem + C::OFF_B + s * C::B_BYTES, &tmB, &b_full[s], kb * C::B_X_STEP, tn * C::BN);
                    ++issued;
                    if (++s == C::S) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) drain_ring(b_full, C::S, issued);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int bs = 0, ds = 0;
            uint32_t bph = 0, dph = 0;
            int t = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++t) {
                int tm, tn, sp, kb0, kb1;
                unit_coords(p, u, tm, tn, sp);
                unit_kblocks(p, sp, kb0, kb1);
                const int acc = t & 1;
                const uint32_t aph = (t >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&b_full[bs], bph, abort_flag)) { ok = false; break; }
                    uint32_t a_off;
                    if constexpr (C::kDecode) {
                        if (!mbar_wait(&d_full[ds], dph, abort_flag)) { ok = false; break; }
                        a_off = C::OFF_D + ds * C::A_BYTES;
                    } else {
                        a_off = C::OFF_A + bs * C::A_BYTES;
                    }
                    tc_fence_after();
                    const uint32_t b_off = C::OFF_B + bs * C::B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = sdesc_k_sw128(sbase + a_off + kk * 32);
                        const uint64_t bd = sdesc_k_sw128(sbase + b_off + kk * 32);
                        const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
                        if constexpr (C::MODE == kModeNative8) mma_f8f6f4_ss(d_tmem, ad, bd, C::IDESC, accum);
                        else mma_f16_ss(d_tmem, ad, bd, C::IDESC, accum);
                    }
                    if constexpr (C::kDecode) {
                        mma_commit(&d_empty[ds]);
                        if (++ds == C::SD) { ds = 0; dph ^= 1u; }
                    }
                    mma_commit(&b_empty[bs]);
                    if (++bs == C::S) { bs = 0; bph ^= 1u; }
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
    } else if constexpr (C::kDecode) {
        if (warp == 6) {
            // ---------------- TMA producer: raw A ----------------
            if (lane == 0) {
                int s = 0;
                uint32_t ph = 0;
                long long issued = 0;
                bool ok = true;
                for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                    int tm, tn, sp, kb0, kb1;
                    unit_coords(p, u, tm, tn, sp);
                    unit_kblocks(p, sp, kb0, kb1);
                    for (int kb = kb0; kb < kb1; ++kb) {
                        if (!mbar_wait(&a_empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
                        mbar_arrive_expect_tx(&a_full[s], C::RA_BYTES);
                        tma_load_2d(smem + C::OFF_RA + s * C::RA_BYTES, &tmA, &a_full[s], kb * C::A_X_STEP, tm * C::BM);
                        ++issued;
                        if (++s == C::SA) { s = 0; ph ^= 1u; }
                    }
                }
                if (!ok) drain_ring(a_full, C::SA, issued);
            }
        } else {
            // ---------------- decode warps ----------------
            const int dt = threadIdx.x - C::DECODE_WARP0 * 32;
            int as = 0, ds = 0;
            uint32_t aph = 0, dph = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                int tm, tn, sp, kb0, kb1;
                unit_coords(p, u, tm, tn, sp);
                unit_kblocks(p, sp, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb) {
                    bool w_ok = mbar_wait(&a_full[as], aph, abort_flag);
                    w_ok = w_ok && mbar_wait(&d_empty[ds], dph ^ 1u, abort_flag);
                    if (!__all_sync(0xFFFFFFFFu, w_ok)) { ok = false; break; }
                    const uint32_t raw = sbase + C::OFF_RA + as * C::RA_BYTES;
                    const uint32_t dst = sbase + C::OFF_D + ds * C::A_BYTES;
                    uint4 in[C::UPT];
#pragma unroll
                    for (int j = 0; j < C::UPT; ++j) in[j] = lds128(raw + (dt + j * C::DECODE_THREADS) * 16);
                    // Raw tile fully read by this warp: release it to the raw-A producer.
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_empty[as]);
#pragma unroll
                    for (int j = 0; j < C::UPT; ++j) decode_store_unit<C::FMT>(in[j], dst, dt + j * C::DECODE_THREADS);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&d_full[ds]);
                    if (++as == C::SA) { as = 0; aph ^= 1u; }
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
