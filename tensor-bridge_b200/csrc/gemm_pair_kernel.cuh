// gemm_pair_kernel.cuh -- GEMM on pairs of SMs (tcgen05 cta_group::2) for the
// operand-loading modes: FP16 x FP16 (kind::f16), FP8/FP4 x FP8/FP4
// (kind::f8f6f4) and INT8 x INT8 (kind::i8).
//
//   D[M x N] = alpha * A[M x K] * B[N x K]^T      (INT8: exact INT32 D)
//
// A cluster of two CTAs owns a 256 x 256 output tile (or, for the tiles of a
// partial last wave, a 256 x 128 half of one; see pair_unit).  Each CTA stages its own
// 128 rows of A and its own 128 rows of B (half of the tile's N) in its shared
// memory; one elected thread of the leader CTA (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, which reads both CTAs' halves and
// writes each CTA's 128 x 256 accumulator into that CTA's tensor memory.  Per
// CTA and k-block the tensor cores read 32 KB of operands instead of the 48 KB
// of a one-CTA 128 x 256 tile, and each CTA's TMA writes half the B.
//
// Roles per CTA (192 threads):
//   warp 0     TMA producer: A and B halves into an S-stage ring; the loads of
//              both CTAs count their bytes on the leader's full barrier, which
//              the leader's producer arms with the bytes of both.
//   warp 1     TMEM allocation for the pair (cta_group::2, 512 columns: two
//              256-column accumulators); in the leader, the MMA issuer.  Its
//              commits arrive on the barrier in both CTAs (multicast): a
//              stage's empty barrier, a finished accumulator's full barrier.
//   warps 2-5  epilogue: its own 128 rows from its own TMEM; each warp then
//              arrives on the leader's accumulator-empty barrier (8 arrivals).
// Every mbarrier wait is bounded; the cluster barriers at start (barriers
// initialised before any peer access) and end (no CTA leaves while its shared
// memory or TMEM may still be used by the pair) are reached by every thread.
#pragma once

#include "gemm_kernel.cuh"

namespace tb {

// After an abort: give TMA loads this thread issued time to land before the
// CTA's shared memory is released (about a millisecond).
__device__ __forceinline__ void settle_pair_loads() {
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 1000000ull) {
    }
}

template <int MODE_, int S_>
struct PairCfg {
    static constexpr int MODE = MODE_;  // kModeF16, kModeNative8 or kModeInt8
    static constexpr int BM = 256;      // rows per pair tile (128 per CTA)
    static constexpr int BN = 256;      // columns per pair tile (B rows: 128 per CTA)
    static constexpr int S = S_;
    static constexpr int KB_ELEMS = MODE == kModeF16 ? 64 : 128;
    static constexpr int A_BYTES = 128 * 128;  // one CTA's 128 rows x 128 bytes
    static constexpr int B_BYTES = 128 * 128;  // one CTA's half of B
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int OFF_BAR = S * STAGE_BYTES;
    static constexpr int NUM_BARS = 2 * S + 5;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
    static constexpr int NUM_THREADS = 192;
    static constexpr int TMEM_COLS = 512;
    static constexpr int KIND = MODE == kModeF16 ? 0 : MODE == kModeNative8 ? 1 : 2;
    static constexpr uint32_t IDESC = MODE == kModeInt8 ? idesc_i8(BM, BN) : idesc_make(0u, 0u, BM, BN);
    // Half tiles (256 x 128) of the last wave.
    static constexpr uint32_t IDESC_HALF =
        MODE == kModeInt8 ? idesc_i8(BM, BN / 2) : idesc_make(0u, 0u, BM, BN / 2);
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// Work unit u -> tile row, first column and width.  The tiles that would form
// a partial last wave are split into two 256 x 128 halves: the last wave then
// takes half a tile's time (4096^2: 222 whole tiles and 68 halves on 74
// clusters, 3.5 tile times instead of 4).  The split is along N only, so every
// output element is still one accumulation over all of K in the same order.
__device__ __forceinline__ void pair_unit(const GemmArgs& p, int u, int tiles_m, int& tm, int& col0, bool& half) {
    int tile, h = 0;
    half = u >= p.pair_full;
    if (half) {
        tile = p.pair_full + ((u - p.pair_full) >> 1);
        h = (u - p.pair_full) & 1;
    } else {
        tile = u;
    }
    tm = tile % tiles_m;
    col0 = (tile / tiles_m) * 256 + h * 128;
}

template <class C>
__global__ void __launch_bounds__(C::NUM_THREADS, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sbase = smem_addr(smem);

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;             // leader: both CTAs' stage bytes landed
    uint64_t* empty = full + C::S;     // both CTAs: the pair's MMAs are done with the stage
    uint64_t* acc_full = empty + C::S; // both CTAs: accumulator ready
    uint64_t* acc_empty = acc_full + 2;// leader: both CTAs' epilogues drained it
    uint64_t* fin_bar = acc_empty + 2; // leader: MMA drain on the abort path
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 8);
        }
        mbar_init(fin_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_mbarrier_init_cluster();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    const int tiles_m = (p.M + C::BM - 1) / C::BM;
    const int tiles_n = (p.N + C::BN - 1) / C::BN;
    const int units = p.pair_full + 2 * (tiles_m * tiles_n - p.pair_full);
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int u = cid; ok && u < units; u += ncl) {
            int tm, col0;
            bool half;
            pair_unit(p, u, tiles_m, tm, col0, half);
            // This CTA's B rows: 128 of a whole tile, 64 of a half (64-row boxes).
            const int brows = half ? 64 : 128;
            const uint32_t tx = half ? p.tx_bytes - p.tx_b_half : p.tx_bytes;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                if (elect_one()) {
                    if (leader) mbar_arrive_expect_tx(&full[s], 2u * tx);
                    const uint32_t fb = leader_bar(&full[s]);
                    uint8_t* st = smem + s * C::STAGE_BYTES;
                    tma_load_2d_pair(st, &tmA, fb, kb * C::KB_ELEMS, tm * C::BM + static_cast<int>(rank) * 128);
                    const int b0 = col0 + static_cast<int>(rank) * brows;
                    tma_load_2d_pair(st + C::A_BYTES, &tmB, fb, kb * C::KB_ELEMS, b0);
                    if (!half) tma_load_2d_pair(st + C::A_BYTES + 8192, &tmB, fb, kb * C::KB_ELEMS, b0 + 64);
                }
                __syncwarp();
                if (++s == C::S) { s = 0; ph ^= 1u; }
            }
        }
        if (!ok && lane == 0) settle_pair_loads();
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader only) ----------------
        if (leader) {
            int s = 0;
            uint32_t ph = 0;
            int t = 0;
            bool ok = true;
            for (int u = cid; ok && u < units; u += ncl, ++t) {
                const uint32_t idesc = (u >= p.pair_full ? C::IDESC_HALF : C::IDESC) | p.idesc_ab;
                const int acc = t & 1;
                const uint32_t aph = (t >> 1) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag))) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t a_lo = sdesc_lo(sbase + s * C::STAGE_BYTES);
                        const uint32_t b_lo = sdesc_lo(sbase + s * C::STAGE_BYTES + C::A_BYTES);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
                            mma_pair<C::KIND>(d_tmem, sdesc_make(a_lo + 2u * kk), sdesc_make(b_lo + 2u * kk), idesc,
                                              accum);
                        }
                        mma_commit_pair(&empty[s], 0x3);
                    }
                    __syncwarp();
                    if (++s == C::S) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                if (elect_one()) mma_commit_pair(&acc_full[acc], 0x3);
                __syncwarp();
            }
            if ((!ok || *abort_flag) && lane == 0) {
                mma_commit_pair(fin_bar, 0x1);
                mbar_wait_drain(fin_bar, 0u);
            }
        }
    } else {
        // ---------------- epilogue (both CTAs) ----------------
        const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
        int t = 0;
        for (int u = cid; u < units; u += ncl, ++t) {
            int tm, col0;
            bool half;
            pair_unit(p, u, tiles_m, tm, col0, half);
            const int ncols = half ? C::BN / 2 : C::BN;
            const int acc = t & 1;
            const uint32_t aph = (t >> 1) & 1;
            const bool ok = mbar_wait(&acc_full[acc], aph, abort_flag);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            tc_fence_after();
            const int row = tm * C::BM + static_cast<int>(rank) * 128 + quarter * 32 + lane;
            const uint32_t t_row =
                tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * C::BN);
#pragma unroll 1
            for (int c = 0; c < ncols; c += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(t_row + c, v);
                tmem_wait_ld();
                store_row_chunk<32>(p, 0, row, col0 + c, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(&acc_empty[acc], 0u);
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace tb
