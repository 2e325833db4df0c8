// gemm_kernel.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M x N] = alpha * A[M x K] * B[N x K]^T      (both operands K-major)
//
// One CTA per SM walks a static list of work units (128 x BN output tiles,
// optionally split along K).  Roles:
//   warp 0      TMA producer of B (and, when A needs no decode, of A) into
//               the operand ring
//   warp 1      TMEM allocator and MMA issuer: one lane issues tcgen05.mma
//               (M = 128, N = BN, 32 bytes of K per instruction) into one of
//               two TMEM accumulators, so the epilogue of tile t overlaps the
//               main loop of tile t+1
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns the 32
//               TMEM lanes = tile rows of its warp-id quarter), scale by alpha,
//               convert, store to global memory
//   fused mode only:
//   warp 6      TMA producer of the raw (stored-format) A tiles into their own
//               ring.  A raw stage is 128 rows x 128 bytes (TF32: 256 bytes)
//               and so covers RK = 128 / (bytes per 64 values) k-blocks (two
//               for FP8, four for packed FP4): wide rows keep the TMA engine
//               moving full 128-byte lines.  The decode warps free a raw stage
//               as soon as they have read it, so raw A is prefetched
//               independently of the MMA.
//   warps 7-    decode warps (8, or 16 for the wide tiles of the one-byte and
//               wider formats): for each k-block (in rounds of DK), read its slice of the staged
//               raw tile, decode it to FP16 and write it, 128-byte swizzled,
//               into the A tile of the operand-ring stage that the MMA reads
//               directly; decoded weights never leave shared memory.  The
//               stage's full barrier completes only when both the B bytes have
//               landed and every decode warp has arrived, so the MMA issuer
//               waits once and commits once per k-block
//
// Shared-memory operand tiles use the canonical K-major SWIZZLE_128B layout:
// 128-byte rows (64 FP16 or 128 FP8 values of K), 8-row groups of 1024 bytes,
// the 16-byte chunk c of row r stored at chunk position c ^ (r & 7).  TMA
// writes that layout itself (the raw stages use it too); the decode warps
// write the decoded tiles in it explicitly.  Decode threads are assigned so
// that the 8 threads of each 16-byte shared-memory phase touch the same chunk
// of 8 consecutive rows: both the raw reads and the decoded writes are free
// of bank conflicts.
//
// The producer and MMA warps run their loops with the whole warp (so loop
// state and descriptors are warp-uniform) and let one elected lane issue the
// TMA / tcgen05 instructions.
//
// Every mbarrier wait is bounded (tb_ptx.cuh): on expiry the kernel sets the
// device error word, all roles leave their loops, asynchronous copies and
// MMAs already issued are drained, and the TMEM allocation is released before
// the CTA exits.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include "tb_host.h"
#include "tb_ptx.cuh"
#include "tb_decode.cuh"

namespace tb {

// Dynamic shared memory the GEMM configurations plan their rings in (of the
// 227 KB a CTA may use, leaving room for barriers and 1 KB alignment).
constexpr int kSmemBudget = 224 * 1024;

enum : int { kModeF16 = 0, kModeDecode = 1, kModeNative8 = 2, kModeInt8 = 3 };

// Stored-format ids (same values as tb_format in the C header).
enum : int { kF16 = 0, kE4M3 = 1, kE5M2 = 2, kE2M1 = 3, kE2M1U = 4, kBF16 = 5, kTF32 = 6, kE2M1HW = 7 };

// Bytes of one 64-value K slice of one row, per stored format.
__host__ __device__ constexpr int raw_row_bytes(int fmt) {
    return fmt == kE2M1 ? 32 : fmt == kBF16 ? 128 : fmt == kTF32 ? 256 : fmt == kF16 ? 128 : 64;
}
// k-blocks of 64 values per raw stage (one 128-byte TMA box per row; TF32 is
// 256 bytes per k-block and uses two boxes for one k-block).
__host__ __device__ constexpr int raw_kblocks(int fmt) { return fmt == kTF32 ? 1 : 128 / raw_row_bytes(fmt); }
// Bytes of one raw stage (128 rows).
__host__ __device__ constexpr int raw_stage_bytes(int fmt) { return fmt == kTF32 ? 2 * 16384 : 16384; }
// TMA box inner extent in elements of the tensor map (128 bytes).
__host__ __device__ constexpr int raw_box_elems(int fmt) {
    return fmt == kBF16 ? 64 : fmt == kTF32 ? 32 : 128;
}
// Tensor-map elements per k-block (packed FP4 maps bytes).
__host__ __device__ constexpr int raw_elems_per_kblock(int fmt) { return fmt == kE2M1 ? 32 : 64; }

__host__ __device__ constexpr int pow2_at_least(int x) {
    return x <= 32 ? 32 : x <= 64 ? 64 : x <= 128 ? 128 : x <= 256 ? 256 : 512;
}

// Compile-time configuration of one kernel instance.
//   S_  operand-ring stages: a B tile plus an A tile (the TMA-loaded A, or in
//       fused mode the decoded A the decode warps write)
//   SA_ raw-A ring stages (fused mode), each covering raw_kblocks(FMT) k-blocks
//   DK_ decode round: k-blocks decoded per synchronisation round (divides
//       raw_kblocks(FMT); at most S_ - 1)
template <int BN_, int MODE_, int FMT_, int S_, int SA_, int DK_>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int MODE = MODE_;
    static constexpr int FMT = FMT_;
    static constexpr bool kDecode = MODE == kModeDecode;
    // Both operands loaded raw by TMA, 128-value k-blocks (kind::f8f6f4, kind::i8).
    static constexpr bool kNativeLike = MODE == kModeNative8 || MODE == kModeInt8;
    static constexpr int S = S_;
    static constexpr int SA = kDecode ? SA_ : 0;
    // Decode warps: 16 for the wide tiles of the formats with at least 64 raw
    // bytes per k-block row (E4M3, E5M2, BF16, TF32: their decode, not the
    // MMA, bounds the fused kernel there); 8 otherwise.
    static constexpr int ND = kDecode ? ((BN >= 128 && raw_row_bytes(FMT) >= 64) ? 16 : 8) : 0;
    static constexpr int DECODE_WARP0 = 7;
    static constexpr int NUM_THREADS = kDecode ? (DECODE_WARP0 + ND) * 32 : 192;
    static constexpr int DECODE_THREADS = ND * 32;

    static constexpr int A_BYTES = BM * 128;  // one swizzled 128-row x 128-byte operand tile
    static constexpr int B_BYTES = BN * 128;
    static constexpr int RK = kDecode ? raw_kblocks(FMT) : 1;
    static constexpr int DK = kDecode ? DK_ : 1;
    static constexpr int RA_BYTES = kDecode ? raw_stage_bytes(FMT) : 0;
    // Narrow tiles: the raw-A producer also loads the stage's RK B tiles right
    // behind the raw A (B is small and then never waits behind far-ahead raw
    // prefetch in the TMA queue); the decode warps copy each B tile into the
    // operand stage next to its decoded A tile.
    static constexpr bool BRAW = kDecode && BN <= 64;
    static constexpr int RSTAGE_BYTES = RA_BYTES + (BRAW ? RK * BN * 128 : 0);
    static constexpr int FULL_COUNT = (BRAW ? 0 : 1) + ND;
    // K elements per k-block and the TMA inner-coordinate steps.
    static constexpr int KB_ELEMS = kNativeLike ? 128 : 64;
    static constexpr int B_X_STEP = KB_ELEMS;

    // Shared-memory layout (offsets from a 1024-byte aligned base).
    static constexpr int OFF_B = 0;                              // S x B tile
    static constexpr int OFF_A = OFF_B + S * B_BYTES;            // S x A tile (TMA-loaded or decoded)
    static constexpr int OFF_RA = OFF_A + S * A_BYTES;           // SA x raw A stage (fused mode)
    static constexpr int OFF_BAR = OFF_RA + SA * RSTAGE_BYTES;
    static constexpr int NUM_BARS = 2 * S + 2 * SA + 5;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to 1024-align the base

    // Independent accumulation chains: the four K=16 MMAs of a k-block go to
    // NACC accumulators in turn, summed by the epilogue.  Narrow tiles make
    // each MMA short, and MMAs into one accumulator run back to back at MMA
    // latency; separate chains overlap.
    // (kind::i8 accumulates integers exactly and keeps one chain.)
    static constexpr int NACC = MODE == kModeInt8 ? 1 : (BN <= 64 ? 4 : (BN <= 128 ? 2 : 1));
    static constexpr int TMEM_COLS = pow2_at_least(2 * NACC * BN);
    static constexpr int CW = BN < 32 ? BN : 32;  // epilogue column chunk

    // MMA: kind::f16 with FP16 operands, or kind::f8f6f4 (operand formats
    // OR'd in at run time from GemmArgs::idesc_ab), FP32 accumulation,
    // K-major operands.
    static constexpr uint32_t IDESC = MODE == kModeInt8 ? idesc_i8(BM, BN) : idesc_make(0u, 0u, BM, BN);
    // MMAs of a half tile (N = BN / 2; the launcher splits only BN = 256 tiles).
    static constexpr uint32_t IDESC_HALF =
        BN < 32 ? IDESC : (MODE == kModeInt8 ? idesc_i8(BM, BN / 2) : idesc_make(0u, 0u, BM, BN / 2));

    // Decode work per k-block: 16-byte raw units per row and in total, and
    // units per decode thread.
    static constexpr int U_ROW = kDecode ? raw_row_bytes(FMT) / 16 : 1;
    static constexpr int UNITS = 128 * U_ROW;
    static constexpr int UPT = UNITS / (ND > 0 ? ND * 32 : 256);

    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN");
    static_assert(B_BYTES % 1024 == 0 && RA_BYTES % 1024 == 0 && RSTAGE_BYTES % 1024 == 0, "stage alignment");
    static_assert(!BRAW || (B_BYTES / 16) % 32 == 0, "B copy split");
    static_assert(!kDecode || (UNITS % (DECODE_THREADS > 0 ? DECODE_THREADS : 1) == 0 && UPT >= 1), "decode split");
    static_assert(S >= 2 && (!kDecode || SA >= 2), "ring depth");
    static_assert(!kDecode || (RK % DK == 0 && DK <= S - 1), "decode round");
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct GemmArgs {
    int M, N, K;
    int tiles_m, tiles_n, splits;
    int kb_per_split, num_kb;  // kb_per_split is a multiple of the raw stage's k-blocks
    int num_units;
    float alpha;
    void* D;         // output (row stride ldd elements)
    long long ldd;
    int out_f16;     // 1: FP16 output, 0: FP32
    int vec_ok;      // 1: D rows allow 16-byte vector stores
    int n_fastest;   // fused pair kernel: tile order with N tiles varying fastest
    int out_i32;     // 1: D is INT32 (kind::i8), stored as accumulated, no alpha
    float* ws;       // split-K partials [splits][M][N] (FP32), when splits > 1
    uint32_t idesc_ab;  // native mode: A/B format fields of the instruction descriptor
    uint32_t tx_bytes;  // native mode: TMA bytes per operand stage (packed FP4 counts 64 per 128-value row)
    // Pair GEMM (k_gemm_pair): work units [0, pair_full) are whole 256 x 256
    // tiles; the tiles after them (the last, partial wave) run as two
    // 256 x 128 halves each.  tx_b_half: TMA bytes of 64 B rows.
    int pair_full;
    uint32_t tx_b_half;
    // One-CTA kernel (k_gemm): units [half_from, num_units) are the two
    // BN / 2-column halves of the tiles from half_from on (a partial last wave
    // split along N; == num_units when there are none).
    int half_from;
    // Fused pair kernel: after a tile's epilogue, copy its rows of D to the
    // same place in each of these buffers (other GPUs' copies of D, mapped
    // into this process).
    int n_peers;
    void* peer_D[kMaxPeers];
    // The accumulators hold D / alpha scaled by 2^-acc_shift (fused E4M3: the
    // decoded weights carry 2^-8, decode_e4m3_x4_scaled); the epilogue
    // multiplies them by 2^acc_shift, exactly, before alpha or the split-K
    // partials.
    int acc_shift;
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

// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-row swizzled tile.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// The decoded tiles only feed the tensor core, so E4M3 and BF16 take their
// branch-free paths (decode_e4m3_x4_scaled, whose 2^-8 the epilogue undoes,
// and decode_bf16_x2_fast): each gives every code the reference decoder's
// value, and only a NaN's FP16 payload differs from the reference's, which
// no product can show.  TF32 keeps its
// per-pair test: its fast path would saturate values at or above 2^16 that
// the reference turns into Inf.
// Decode one 16-byte raw unit holding K slice `col` (in 16-byte raw units) of
// tile row `row`, and store it into the swizzled FP16 tile at `dst`.
template <int FMT>
__device__ __forceinline__ void decode_store_unit(const uint4& in, uint32_t dst, int row, int col) {
    if constexpr (FMT == kE4M3 || FMT == kE5M2 || FMT == kE2M1U) {
        uint32_t o[8];  // 16 values -> FP16 chunks 2col, 2col+1
        if constexpr (FMT == kE4M3) {
            decode_e4m3_x4_scaled(in.x, o[0], o[1]); decode_e4m3_x4_scaled(in.y, o[2], o[3]);
            decode_e4m3_x4_scaled(in.z, o[4], o[5]); decode_e4m3_x4_scaled(in.w, o[6], o[7]);
        } else if constexpr (FMT == kE5M2) {
            decode_e5m2_x4(in.x, o[0], o[1]); decode_e5m2_x4(in.y, o[2], o[3]);
            decode_e5m2_x4(in.z, o[4], o[5]); decode_e5m2_x4(in.w, o[6], o[7]);
        } else {
            decode_e2m1_unpacked_x4(in.x, o[0], o[1]); decode_e2m1_unpacked_x4(in.y, o[2], o[3]);
            decode_e2m1_unpacked_x4(in.z, o[4], o[5]); decode_e2m1_unpacked_x4(in.w, o[6], o[7]);
        }
        sts128(dst + swz(row, 2 * col), o[0], o[1], o[2], o[3]);
        sts128(dst + swz(row, 2 * col + 1), o[4], o[5], o[6], o[7]);
    } else if constexpr (FMT == kE2M1) {
        uint32_t o[4];  // 32 values -> FP16 chunks 4col .. 4col+3
        decode_e2m1_packed_x8(in.x, o);
        sts128(dst + swz(row, 4 * col + 0), o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.y, o);
        sts128(dst + swz(row, 4 * col + 1), o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.z, o);
        sts128(dst + swz(row, 4 * col + 2), o[0], o[1], o[2], o[3]);
        decode_e2m1_packed_x8(in.w, o);
        sts128(dst + swz(row, 4 * col + 3), o[0], o[1], o[2], o[3]);
    } else if constexpr (FMT == kBF16) {
        // 8 values -> FP16 chunk col
        sts128(dst + swz(row, col), decode_bf16_x2_fast(in.x), decode_bf16_x2_fast(in.y), decode_bf16_x2_fast(in.z),
               decode_bf16_x2_fast(in.w));
    } else if constexpr (FMT == kTF32) {
        // 4 values -> half of FP16 chunk col/2
        sts64(dst + swz(row, col >> 1) + (col & 1) * 8, decode_tf32_x2(in.x, in.y), decode_tf32_x2(in.z, in.w));
    }
}

// Shared address of raw unit (row, col) of k-block slice `sub` in a raw stage.
// Each 128-byte box row holds (128 / raw_row_bytes) k-block slices; TF32 uses
// two boxes (columns 0-7 and 8-15 of its 16 units per row).
template <int FMT>
__device__ __forceinline__ uint32_t raw_unit_addr(uint32_t stage, int sub, int row, int col) {
    if constexpr (FMT == kTF32) {
        return stage + (col >> 3) * 16384 + swz(row, col & 7);
    } else {
        constexpr int U = raw_row_bytes(FMT) / 16;
        return stage + swz(row, sub * U + col);
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

// unit_coords for k_gemm, whose units from p.half_from on are halves of tiles:
// half = 0 for a whole tile, 1 or 2 for its first or second BN / 2 columns.
// Splitting a partial last wave along N keeps every output element one
// accumulation over its K range in the same order.
__device__ __forceinline__ void unit_coords_h(const GemmArgs& p, int u, int& tm, int& tn, int& sp, int& half) {
    half = 0;
    if (u >= p.half_from) {
        const int h = u - p.half_from;
        u = p.half_from + (h >> 1);
        half = 1 + (h & 1);
    }
    unit_coords(p, u, tm, tn, sp);
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
    if (p.out_i32) {
        uint32_t* dst = static_cast<uint32_t*>(p.D) + static_cast<size_t>(row) * p.ldd + col0;
        if (full && p.vec_ok) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) *reinterpret_cast<uint4*>(dst + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = v[j];
        }
        return;
    }
    const float sc = __int_as_float((127 + p.acc_shift) << 23);  // 2^acc_shift
    auto val = [&](int j) { return __uint_as_float(v[j]) * sc; };
    if (p.splits > 1) {
        float* dst = p.ws + (static_cast<size_t>(sp) * p.M + row) * static_cast<size_t>(p.N) + col0;
        if (full && (p.N & 3) == 0) {
#pragma unroll
            for (int j = 0; j < CW; j += 4)
                *reinterpret_cast<float4*>(dst + j) = make_float4(val(j), val(j + 1), val(j + 2), val(j + 3));
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = val(j);
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
                    const __half2 t = __floats2half2_rn(val(j + 2 * h) * a, val(j + 2 * h + 1) * a);
                    w[h] = *reinterpret_cast<const uint32_t*>(&t);
                }
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = __float2half_rn(val(j) * a);
        }
    } else {
        float* dst = static_cast<float*>(p.D) + static_cast<size_t>(row) * p.ldd + col0;
        if (full && p.vec_ok) {
#pragma unroll
            for (int j = 0; j < CW; j += 4) {
                *reinterpret_cast<float4*>(dst + j) =
                    make_float4(val(j) * a, val(j + 1) * a, val(j + 2) * a, val(j + 3) * a);
            }
        } else {
#pragma unroll
            for (int j = 0; j < CW; ++j)
                if (col0 + j < p.N) dst[j] = val(j) * a;
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
    // Operand ring: full[s] completes when the stage's TMA bytes have landed
    // and (fused mode) every decode warp has arrived after writing its part
    // of the decoded A tile; empty[s] when the MMAs reading the stage are done.
    uint64_t* b_full = bars;
    uint64_t* b_empty = b_full + C::S;
    uint64_t* a_full = b_empty + C::S;        // raw-A ring: TMA tx complete
    uint64_t* a_empty = a_full + C::SA;       // raw-A ring: decode warps done reading
    uint64_t* acc_full = a_empty + C::SA;     // accumulator ready for the epilogue
    uint64_t* acc_empty = acc_full + 2;       // accumulator drained by the epilogue
    uint64_t* fin_bar = acc_empty + 2;        // MMA drain on the abort path
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&b_full[s], C::FULL_COUNT);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < C::SA; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], C::ND);
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
        if (!C::BRAW) {
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            bool ok = true;
            const uint32_t kTx =
                C::kNativeLike ? p.tx_bytes : C::B_BYTES + (C::kDecode ? 0u : static_cast<uint32_t>(C::A_BYTES));
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                int tm, tn, sp, kb0, kb1, half;
                unit_coords_h(p, u, tm, tn, sp, half);
                unit_kblocks(p, sp, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&b_empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                    if (elect_one()) {
                        mbar_arrive_expect_tx(&b_full[s], kTx);
                        if constexpr (!C::kDecode)
                            tma_load_2d(smem + C::OFF_A + s * C::A_BYTES, &tmA, &b_full[s], kb * C::KB_ELEMS,
                                        tm * C::BM);
                        // (A half tile's box still has BN rows; its MMAs read the first BN / 2.)
                        tma_load_2d(smem + C::OFF_B + s * C::B_BYTES, &tmB, &b_full[s], kb * C::B_X_STEP,
                                    tn * C::BN + (half == 2 ? C::BN / 2 : 0));
                    }
                    __syncwarp();
                    ++issued;
                    if (++s == C::S) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok && lane == 0) drain_ring(b_full, C::S, issued);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (whole warp; one elected lane issues) ----------------
        // Descriptor low words of stage 0 (A and B); a stage advance adds the
        // tile size >> 4, a K=16 step (32 bytes) adds 2.
        {
            const uint32_t a_lo0 = sdesc_lo(sbase + C::OFF_A), b_lo0 = sdesc_lo(sbase + C::OFF_B);
            uint32_t a_lo = a_lo0, b_lo = b_lo0;
            int bs = 0;
            uint32_t bph = 0;
            int t = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++t) {
                int tm, tn, sp, kb0, kb1, half;
                unit_coords_h(p, u, tm, tn, sp, half);
                unit_kblocks(p, sp, kb0, kb1);
                const int acc = t & 1;
                const uint32_t aph = (t >> 1) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag))) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::NACC * C::BN);
                const uint32_t idesc = half ? C::IDESC_HALF : C::IDESC;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&b_full[bs], bph, abort_flag))) { ok = false; break; }
                    tc_fence_after();
                    if (elect_one()) {
                        const bool first = kb == kb0;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            // chain kk % NACC; its first MMA of the unit overwrites
                            const uint32_t accum = (!first || kk >= C::NACC) ? 1u : 0u;
                            const uint32_t d = d_tmem + static_cast<uint32_t>((kk % C::NACC) * C::BN);
                            const uint64_t ad = sdesc_make(a_lo + 2u * kk), bd = sdesc_make(b_lo + 2u * kk);
                            if constexpr (C::MODE == kModeNative8)
                                mma_f8f6f4_ss(d, ad, bd, idesc | p.idesc_ab, accum);
                            else if constexpr (C::MODE == kModeInt8)
                                mma_i8_ss(d, ad, bd, idesc, accum);
                            else mma_f16_ss(d, ad, bd, idesc, accum);
                        }
                        mma_commit(&b_empty[bs]);
                    }
                    __syncwarp();
                    if (++bs == C::S) {
                        bs = 0;
                        bph ^= 1u;
                        a_lo = a_lo0;
                        b_lo = b_lo0;
                    } else {
                        a_lo += C::A_BYTES >> 4;
                        b_lo += C::B_BYTES >> 4;
                    }
                }
                if (!ok) break;
                if (elect_one()) mma_commit(&acc_full[acc]);
                __syncwarp();
            }
            if ((!ok || *abort_flag) && lane == 0) {
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
            int tm, tn, sp, half;
            unit_coords_h(p, u, tm, tn, sp, half);
            const int acc = t & 1;
            const uint32_t aph = (t >> 1) & 1;
            const bool ok = mbar_wait(&acc_full[acc], aph, abort_flag);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            tc_fence_after();
            const int row = tm * C::BM + quarter * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * C::NACC * C::BN);
            const int ncols = half ? C::BN / 2 : C::BN;
            const int col0 = tn * C::BN + (half == 2 ? C::BN / 2 : 0);
#pragma unroll 1
            for (int c = 0; c < ncols; c += C::CW) {
                uint32_t v[C::CW];
                tmem_ld_chunk<C::CW>(t_row + c, v);
                if constexpr (C::NACC > 1) {
                    // Sum the accumulation chains in order 0, 1, ...
#pragma unroll
                    for (int ch = 1; ch < C::NACC; ++ch) {
                        uint32_t w[C::CW];
                        tmem_ld_chunk<C::CW>(t_row + ch * C::BN + c, w);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < C::CW; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
                    }
                }
                tmem_wait_ld();
                store_row_chunk<C::CW>(p, sp, row, col0 + c, v);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
        }
    } else if constexpr (C::kDecode) {
        if (warp == 6) {
            // ---------------- TMA producer: raw A (one stage = RK k-blocks) ----------------
            {
                int s = 0;
                uint32_t ph = 0;
                long long issued = 0;
                bool ok = true;
                for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                    int tm, tn, sp, kb0, kb1, half;
                    unit_coords_h(p, u, tm, tn, sp, half);
                    unit_kblocks(p, sp, kb0, kb1);
                    for (int kb = kb0; kb < kb1; kb += C::RK) {
                        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&a_empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                        const int nk = min(C::RK, kb1 - kb);  // k-blocks of this stage in the unit
                        if (elect_one()) {
                            mbar_arrive_expect_tx(&a_full[s], C::RA_BYTES + (C::BRAW ? nk * C::B_BYTES : 0));
                            uint8_t* dst = smem + C::OFF_RA + s * C::RSTAGE_BYTES;
                            const int x = kb * raw_elems_per_kblock(C::FMT);
                            tma_load_2d(dst, &tmA, &a_full[s], x, tm * C::BM);
                            if constexpr (C::FMT == kTF32)
                                tma_load_2d(dst + 16384, &tmA, &a_full[s], x + raw_box_elems(C::FMT), tm * C::BM);
                            if constexpr (C::BRAW) {
                                for (int j = 0; j < nk; ++j)
                                    tma_load_2d(dst + C::RA_BYTES + j * C::B_BYTES, &tmB, &a_full[s],
                                                (kb + j) * C::B_X_STEP, tn * C::BN);
                            }
                        }
                        __syncwarp();
                        ++issued;
                        if (++s == C::SA) { s = 0; ph ^= 1u; }
                    }
                }
                if (!ok && lane == 0) drain_ring(a_full, C::SA, issued);
            }
        } else {
            // ---------------- decode warps ----------------
            // Work is done in rounds of DK k-blocks (one raw stage or part of
            // one): one wait set, one proxy fence and one arrive set per round.
            // Unit q of a k-block slice: row = 8*(q / (8*U_ROW)) + q % 8,
            // col = (q / 8) % U_ROW, so each 8-thread shared-memory phase
            // covers one chunk of 8 consecutive rows.
            const int dt = threadIdx.x - C::DECODE_WARP0 * 32;
            int as = 0, ds = 0;
            uint32_t aph = 0, dph = 0;  // raw ring; operand ring (same order as the B producer)
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
                int tm, tn, sp, kb0, kb1, half;
                unit_coords_h(p, u, tm, tn, sp, half);
                unit_kblocks(p, sp, kb0, kb1);
                for (int kb = kb0; kb < kb1; kb += C::DK) {
                    const int cnt = min(C::DK, kb1 - kb);
                    const int sub0 = (kb - kb0) % C::RK;
                    int slot[C::DK];
                    uint32_t sph[C::DK];
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        slot[d] = ds + d;
                        sph[d] = dph;
                        if (slot[d] >= C::S) { slot[d] -= C::S; sph[d] ^= 1u; }
                    }
                    bool w_ok = true;
                    if (sub0 == 0) w_ok = mbar_wait(&a_full[as], aph, abort_flag);
#pragma unroll
                    for (int d = 0; d < C::DK; ++d)
                        if (d < cnt) w_ok = w_ok && mbar_wait(&b_empty[slot[d]], sph[d] ^ 1u, abort_flag);
                    if (!__all_sync(0xFFFFFFFFu, w_ok)) { ok = false; break; }
                    const uint32_t raw = sbase + C::OFF_RA + as * C::RSTAGE_BYTES;
                    uint4 in[C::DK][C::UPT];
                    constexpr int BCOPY = C::BRAW ? C::B_BYTES / 16 / C::DECODE_THREADS : 0;
                    constexpr int BCOPY_THREADS = C::BRAW ? C::B_BYTES / 16 / (BCOPY > 0 ? BCOPY : 1) : 0;
                    uint4 bcp[C::DK][BCOPY > 0 ? BCOPY : 1];
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        if (d < cnt) {
#pragma unroll
                            for (int j = 0; j < C::UPT; ++j) {
                                const int q = dt + j * C::DECODE_THREADS;
                                const int row = ((q / (8 * C::U_ROW)) << 3) + (q & 7);
                                const int col = (q >> 3) % C::U_ROW;
                                in[d][j] = lds128(raw_unit_addr<C::FMT>(raw, sub0 + d, row, col));
                            }
                            if constexpr (C::BRAW) {
                                // B tile of this k-block, staged with the raw A
#pragma unroll
                                for (int j = 0; j < (BCOPY > 0 ? BCOPY : 1); ++j) {
                                    const int v = dt + j * C::DECODE_THREADS;
                                    if (BCOPY > 0 || dt < C::B_BYTES / 16)
                                        bcp[d][j] = lds128(raw + C::RA_BYTES + (sub0 + d) * C::B_BYTES + v * 16);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        if (d < cnt) {
                            const uint32_t dst = sbase + C::OFF_A + slot[d] * C::A_BYTES;
#pragma unroll
                            for (int j = 0; j < C::UPT; ++j) {
                                const int q = dt + j * C::DECODE_THREADS;
                                const int row = ((q / (8 * C::U_ROW)) << 3) + (q & 7);
                                const int col = (q >> 3) % C::U_ROW;
                                decode_store_unit<C::FMT>(in[d][j], dst, row, col);
                            }
                            if constexpr (C::BRAW) {
                                const uint32_t bdst = sbase + C::OFF_B + slot[d] * C::B_BYTES;
#pragma unroll
                                for (int j = 0; j < (BCOPY > 0 ? BCOPY : 1); ++j) {
                                    const int v = dt + j * C::DECODE_THREADS;
                                    if (BCOPY > 0 || dt < C::B_BYTES / 16)
                                        sts128(bdst + v * 16, bcp[d][j].x, bcp[d][j].y, bcp[d][j].z, bcp[d][j].w);
                                }
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
#pragma unroll
                        for (int d = 0; d < C::DK; ++d)
                            if (d < cnt) mbar_arrive(&b_full[slot[d]]);
                    }
                    if (sub0 + cnt == C::RK || kb + cnt == kb1) {
                        // Last slices of this raw stage read by this warp: release it.
                        // Only after the loaded words have been consumed: the
                        // arrive does not order shared-memory reads still in
                        // flight against the next TMA write into the stage
                        // (an early release let refills overwrite live data).
                        if (lane == 0) mbar_arrive(&a_empty[as]);
                        if (++as == C::SA) { as = 0; aph ^= 1u; }
                    }
                    ds += cnt;
                    if (ds >= C::S) { ds -= C::S; dph ^= 1u; }
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
