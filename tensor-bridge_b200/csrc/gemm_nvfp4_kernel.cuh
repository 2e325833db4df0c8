// gemm_nvfp4_kernel.cuh -- block-scaled FP4 GEMM (the NVFP4 layout) on pairs of
// SMs with tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X.
//
//   D[M x N] = alpha * (A .* SA)[M x K] * ((B .* SB)[N x K])^T
//
// A and B hold E2M1 codes packed two per byte, first value in the LOW nibble
// (the tensor core's order), K-major; SA [M x K/16] and SB [N x K/16] hold
// one UE4M3 scale byte per 16 consecutive values of a row.  The tensor core
// multiplies every 16-value block by its scale itself, so FP4 runs at the FP4
// tensor rate with no decode.  alpha carries the per-tensor FP32 scales.
//
// A cluster of two CTAs owns a 256 x 256 output tile, as in
// gemm_pair_kernel.cuh: each CTA stages its own 128 rows of A and 128 rows of
// B (128 bytes = 256 values of K per k-block, 128-byte swizzle); the leader
// issues four K = 64 MMAs per k-block.  Scale factors live in tensor memory.
// Each SM of the pair computes its 128 rows against all 256 columns, so each
// CTA needs the scales of its own 128 A rows and of all 256 B rows of the
// tile.  With every stage the producer also brings in those scale bytes (two
// TMA boxes, 16 bytes x 128 and 16 bytes x 256 rows) on a barrier of its own
// CTA; four SF warps then copy them from shared to tensor memory with
// tcgen05.st into the stage's scale slot and signal the leader's sf_full
// barrier: the leader's SF warps arrive locally (one of them arming the
// barrier for the other CTA's bytes), the other CTA's SF warps each send a
// 16-byte DSMEM bulk copy whose completion counts on it.  A cluster-scope
// release arrival per warp and k-block (the first version) stalled the SF
// warps on the memory barrier it implies (ncu: membar 7 per issue, tensor
// pipe 24% active at 4096^3).  A stage and its scale slot are refilled only after the pair's
// MMAs of their previous use have completed (the empty barrier the producer
// waits on), so the SF warps need no wait of their own for the slot.
//
// Roles per CTA (320 threads):
//   warp 0     TMA producer of the A, B and scale tiles
//   warp 1     TMEM allocation (pair, 512 columns); in the leader, the MMA issuer
//   warps 2-5  epilogue: this CTA's 128 rows x 256 columns of the accumulator
//   warps 6-9  SF warps
// TMEM: columns [0, 256) the accumulator (one: the epilogue of a tile runs
// while the producer and SF warps fill the next tile's stages), then S scale
// slots of 48 columns: scales of A at +0 (4 columns per MMA), of B at +16 (8
// columns per MMA).
//
// Scale-factor layout in tensor memory (what kind::mxf4nvf4 reads): the
// scales of one MMA (K = 64: four 16-value blocks a row) for rows 32 j + l sit
// in column j of lane l, one byte per block in K order, and every lane
// quarter holds the same words (the tensor core's four sub-partitions each
// read their own quarter): 4 columns for 128 rows of A, 8 for 256 rows of B.
#pragma once

#include "gemm_pair_kernel.cuh"

namespace tb {

// Instruction descriptor of kind::mxf4nvf4 (dense, K-major): A and B E2M1
// (format code 1), scale factors UE4M3 (bit 23 clear), scale-factor data IDs
// 0 (bits 4-5 and 29-30), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_nvfp4(int m, int n) {
    return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

template <int S_>
struct Nvfp4Cfg {
    static constexpr int BM = 256;  // pair tile rows (128 per CTA)
    static constexpr int BN = 256;  // pair tile columns (B rows: 128 per CTA)
    static constexpr int S = S_;
    static constexpr int KB_VALUES = 256;       // values of K per k-block (128 bytes a row)
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = 128 * 128;
    static constexpr int SFA_BYTES = 128 * 16;  // this CTA's A rows, 16 scale bytes each
    static constexpr int SFB_BYTES = 256 * 16;  // the tile's 256 B rows
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
    static constexpr int AB_BYTES = A_BYTES + B_BYTES;
    static constexpr int SF_BYTES = SFA_BYTES + SFB_BYTES;
    static constexpr int OFF_BAR = S * STAGE_BYTES;
    static constexpr int NUM_BARS = 4 * S + 3;
    static constexpr int OFF_SIG = OFF_BAR + ((NUM_BARS * 8 + 16 + 127) / 128) * 128;  // 4 x 16 B signal sources / sinks
    static constexpr int SMEM_BYTES = OFF_SIG + 64;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
    static constexpr int SF_WARP0 = 6;
    static constexpr int NUM_THREADS = (SF_WARP0 + 4) * 32;
    static constexpr int TMEM_COLS = 512;
    static constexpr int SF_COL0 = 256;
    static constexpr int SF_SLOT = 48;
    static constexpr int SFB_COL = 16;
    static constexpr uint32_t IDESC = idesc_nvfp4(BM, BN);
    static_assert(SF_COL0 + S * SF_SLOT <= TMEM_COLS, "TMEM budget");
    static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// D (+)= A * B^T with block scales from TMEM, pair MMA (issued by the leader).
__device__ __forceinline__ void mma_pair_nvfp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::
            "r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
        : "memory");
}

// Wait with cluster-scope acquire: the arrivals come from both CTAs of the pair.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait_cluster(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_cluster(a, parity)) return true;
        if ((i & 63u) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                atomicOr(&g_tb_device_error, kErrTimeout);
                *abort = 1;
                return false;
            }
        }
    }
}

template <class C>
__global__ void __launch_bounds__(C::NUM_THREADS, 1)
    k_gemm_nvfp4(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB, const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sbase = smem_addr(smem);

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;               // leader: both CTAs' A and B bytes landed
    uint64_t* sf_full = full + C::S;     // leader: both CTAs' scale slots written (8 warp arrivals)
    uint64_t* empty = sf_full + C::S;    // both CTAs: the pair's MMAs are done with the stage and slot
    uint64_t* sf_land = empty + C::S;    // each CTA: its scale bytes of the stage landed
    uint64_t* acc_full = sf_land + C::S; // both CTAs: accumulator ready
    uint64_t* acc_empty = acc_full + 1;  // leader: both CTAs' epilogues drained it (8 warp arrivals)
    uint64_t* fin_bar = acc_empty + 1;   // leader: MMA drain on the abort path
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&sf_full[s], 4);
            mbar_init(&empty[s], 1);
            mbar_init(&sf_land[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 8);
        mbar_init(fin_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_mbarrier_init_cluster();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmSA);
        tma_prefetch_desc(&tmSB);
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

    const int tiles_m = p.tiles_m;
    const int units = p.num_units;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int u = cid; ok && u < units; u += ncl) {
            const int tm = u % tiles_m, tn = u / tiles_m;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                if (elect_one()) {
                    uint8_t* st = smem + s * C::STAGE_BYTES;
                    // Scale bytes first (this CTA's A rows and all of the tile's
                    // B rows, on its own barrier): one SM's TMA requests land in
                    // order, so the SF warps' copy to tensor memory then runs
                    // while the stage's A and B are still arriving.
                    mbar_arrive_expect_tx(&sf_land[s], C::SF_BYTES);
                    tma_load_2d(st + C::AB_BYTES, &tmSA, &sf_land[s], kb * 16, tm * C::BM + static_cast<int>(rank) * 128);
                    tma_load_2d(st + C::AB_BYTES + C::SFA_BYTES, &tmSB, &sf_land[s], kb * 16, tn * C::BN);
                    if (leader) mbar_arrive_expect_tx(&full[s], 2u * C::AB_BYTES);
                    const uint32_t fb = leader_bar(&full[s]);
                    tma_load_2d_pair(st, &tmA, fb, kb * 128, tm * C::BM + static_cast<int>(rank) * 128);
                    tma_load_2d_pair(st + C::A_BYTES, &tmB, fb, kb * 128, tn * C::BN + static_cast<int>(rank) * 128);
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
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_cluster(acc_empty, (t & 1) ^ 1u, abort_flag))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sf_full[s], ph, abort_flag))) { ok = false; break; }
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t a_lo = sdesc_lo(sbase + s * C::STAGE_BYTES);
                        const uint32_t b_lo = sdesc_lo(sbase + s * C::STAGE_BYTES + C::A_BYTES);
                        const uint32_t slot = tmem_base + static_cast<uint32_t>(C::SF_COL0 + s * C::SF_SLOT);
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const uint32_t accum = (kb > 0 || c > 0) ? 1u : 0u;
                            mma_pair_nvfp4(tmem_base, sdesc_make(a_lo + 2u * c), sdesc_make(b_lo + 2u * c), C::IDESC,
                                           slot + 4u * c, slot + C::SFB_COL + 8u * c, accum);
                        }
                        mma_commit_pair(&empty[s], 0x3);
                    }
                    __syncwarp();
                    if (++s == C::S) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                if (elect_one()) mma_commit_pair(acc_full, 0x3);
                __syncwarp();
            }
            if ((!ok || *abort_flag) && lane == 0) {
                mma_commit_pair(fin_bar, 0x1);
                mbar_wait_drain(fin_bar, 0u);
            }
        }
    } else if (warp < C::SF_WARP0) {
        // ---------------- epilogue (both CTAs) ----------------
        const int quarter = warp & 3;
        int t = 0;
        for (int u = cid; u < units; u += ncl, ++t) {
            const int tm = u % tiles_m, tn = u / tiles_m;
            const bool ok = mbar_wait(acc_full, t & 1, abort_flag);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            tc_fence_after();
            const int row = tm * C::BM + static_cast<int>(rank) * 128 + quarter * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
            if (p.out_f16 && p.vec_ok && tn * C::BN + C::BN <= p.N) {
                // FP16 out, a whole aligned tile row: it fits in registers as
                // FP16 pairs, so the accumulator is released before the global
                // stores, which then overlap the next tile's MMAs.
                uint32_t h[C::BN / 2];
#pragma unroll
                for (int c = 0; c < C::BN; c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(t_row + c, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const __half2 x = __floats2half2_rn(__uint_as_float(v[j]) * p.alpha,
                                                            __uint_as_float(v[j + 1]) * p.alpha);
                        h[(c + j) >> 1] = *reinterpret_cast<const uint32_t*>(&x);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc_empty, 0u);
                if (row < p.M) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.D) + static_cast<size_t>(row) * p.ldd +
                                                          tn * C::BN);
#pragma unroll
                    for (int j = 0; j < C::BN / 8; ++j) dst[j] = make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < C::BN; c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(t_row + c, v);
                    tmem_wait_ld();
                    store_row_chunk<32>(p, 0, row, tn * C::BN + c, v);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc_empty, 0u);
            }
        }
    } else {
        // ---------------- SF warps: scale bytes, shared -> tensor memory ----------------
        // Every warp writes the same words into its own lane quarter.
        const int q = warp & 3;
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int u = cid; ok && u < units; u += ncl) {
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&sf_land[s], ph, abort_flag))) { ok = false; break; }
                // 16 scale bytes per row (four MMAs x four 16-value blocks), rows 16 bytes apart.
                const uint32_t sa = sbase + static_cast<uint32_t>(s * C::STAGE_BYTES + C::AB_BYTES);
                const uint32_t sb = sa + C::SFA_BYTES;
                uint32_t va[16], vb[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4 x = lds128(sa + static_cast<uint32_t>((j * 32 + lane) * 16));
                    va[0 + j] = x.x; va[4 + j] = x.y; va[8 + j] = x.z; va[12 + j] = x.w;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 y = lds128(sb + static_cast<uint32_t>((j * 32 + lane) * 16));
                    vb[0 + j] = y.x; vb[8 + j] = y.y; vb[16 + j] = y.z; vb[24 + j] = y.w;
                }
                const uint32_t slot = t_lane + static_cast<uint32_t>(C::SF_COL0 + s * C::SF_SLOT);
                tmem_st_32x32b_x16(slot, va);
                tmem_st_32x32b_x32(slot + C::SFB_COL, vb);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (leader) {
                        if (q == 0) mbar_arrive_expect_tx(&sf_full[s], 4u * 16u);  // the other CTA's four signals
                        else mbar_arrive(&sf_full[s]);
                    } else {
                        uint8_t* sig = smem + C::OFF_SIG + q * 16;
                        bulk_copy_to_cluster(cluster_addr(sig, 0u), sig, 16u, leader_bar(&sf_full[s]));
                    }
                }
                if (++s == C::S) { s = 0; ph ^= 1u; }
            }
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
