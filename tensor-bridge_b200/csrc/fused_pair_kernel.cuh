// fused_pair_kernel.cuh -- fused decode + GEMM on pairs of SMs (tcgen05
// cta_group::2) for wide tiles.
//
//   D[M x N] = alpha * decode(A)[M x K] * B[N x K]^T
//
// A cluster of two CTAs owns a 256 x 512 output tile.  Each CTA decodes its
// own 128 rows of the stored-format A into FP16 in its shared memory and
// stages its own 128 rows of B per 256-column half there by TMA; one elected
// thread of the leader CTA (rank 0) issues tcgen05.mma.cta_group::2 with
// M = 256, N = 256 per half, which reads both CTAs' A and B tiles and writes
// each CTA's 128 x 256 accumulator per half into that CTA's tensor memory.
// Each decoded A tile thus feeds 512 output columns: half the decode per
// output element of the one-CTA 128 x 256 fused tile, which the decode bounds
// for the one-byte and wider formats.  (A 256 x 256 pair tile, same decode
// per output as the one-CTA tile, measured slower than it: the pair waits for
// the slower CTA's decode at every step.)
//
// Roles per CTA:
//   warp 0      TMA producer of this CTA's B rows into the operand ring; the
//               bytes count on the leader's full barrier (cta_group::2 TMA),
//               which the leader's producer arms with the bytes of both
//   warp 1      TMEM allocation for the pair (512 columns: the two halves'
//               256-column accumulators); in the leader, the MMA issuer.  Its
//               commits arrive in both CTAs (multicast): a stage's empty
//               barrier, a finished tile's accumulator-full barrier.  The
//               next tile's first MMAs into a half wait until the epilogue
//               has drained that half, so the drain of the second half
//               overlaps the first half's MMAs
//   warps 2-5   epilogue: this CTA's 128 rows from its own TMEM; after each
//               half each warp arrives on the leader's accumulator-empty
//               barrier of that half.  With peer buffers (the sharded GEMM)
//               each warp then copies its 32 finished rows from D into every
//               other GPU's D over NVLink, while the next tile's MMAs run
//   warp 6      TMA producer of this CTA's raw A rows into the raw ring
//   warps 7-    decode warps (as in the one-CTA fused kernel): for each
//               k-block, read the raw slice, decode to FP16, write the
//               128-byte swizzled A tile of the operand stage, make the writes
//               visible to the tensor core (proxy fence) and signal the
//               leader's full barrier: an arrival in the leader, a 16-byte
//               bulk copy whose bytes count on it from the second CTA
// The leader's full barrier of a stage thus completes when both CTAs' B bytes
// have landed and every decode warp of both CTAs has signalled.  Every wait
// is bounded; cluster barriers at start (barriers initialised before any peer
// access) and end (no CTA leaves while the pair may still read its shared
// memory or TMEM) are reached by every thread, also after an abort.
#pragma once

#include "gemm_kernel.cuh"
#include "gemm_pair_kernel.cuh"

namespace tb {

//   S_  operand-ring stages (this CTA's decoded A tile and its B rows of
//       both halves)
//   SA_ raw-A ring stages, each raw_kblocks(FMT) k-blocks of this CTA's rows
//   DK_ decode round in k-blocks (divides raw_kblocks(FMT), at most S_ - 1)
template <int FMT_, int S_, int SA_, int DK_>
struct FusedPairCfg {
    static constexpr int FMT = FMT_;
    static constexpr int NH = 2;         // 256-column halves, one accumulator each
    static constexpr int BM = 256;       // pair tile rows (128 decoded per CTA)
    static constexpr int BN = 256 * NH;  // pair tile columns (128 B rows per CTA and half)
    static constexpr int S = S_;
    static constexpr int SA = SA_;
    static constexpr int DK = DK_;
    static constexpr int RK = raw_kblocks(FMT);
    static constexpr int ND = raw_row_bytes(FMT) >= 64 ? 16 : 8;
    static constexpr int DECODE_WARP0 = 7;
    static constexpr int NUM_THREADS = (DECODE_WARP0 + ND) * 32;
    static constexpr int DECODE_THREADS = ND * 32;
    static constexpr int A_BYTES = 128 * 128;
    static constexpr int B_BYTES = NH * 128 * 128;  // this CTA's B rows of all halves
    static constexpr int RA_BYTES = raw_stage_bytes(FMT);
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + S * A_BYTES;
    static constexpr int OFF_RA = OFF_B + S * B_BYTES;
    static constexpr int OFF_BAR = OFF_RA + SA * RA_BYTES;
    static constexpr int NUM_BARS = 2 * S + 2 * SA + 4;
    // 16 bytes per decode warp: the second CTA's decode warps signal the
    // leader's full barrier with a 16-byte bulk copy into this area.
    static constexpr int OFF_SIG = (OFF_BAR + NUM_BARS * 8 + 16 + 15) / 16 * 16;
    static constexpr int SMEM_BYTES = OFF_SIG + ND * 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
    // Leader's full barrier: its producer's arrival and one arrival per
    // leader decode warp; bytes: both CTAs' B halves and one signal copy per
    // decode warp of the second CTA.
    static constexpr int FULL_COUNT = 1 + ND;
    static constexpr uint32_t FULL_TX = 2u * B_BYTES + ND * 16u;
    static constexpr int TMEM_COLS = 512;
    static constexpr uint32_t IDESC = idesc_make(0u, 0u, BM, 256);  // each MMA: M = 256, N = 256
    static constexpr int U_ROW = raw_row_bytes(FMT) / 16;
    static constexpr int UNITS = 128 * U_ROW;
    static constexpr int UPT = UNITS / DECODE_THREADS;
    static_assert(UNITS % DECODE_THREADS == 0 && UPT >= 1, "decode split");
    static_assert(S >= 2 && SA >= 2 && RK % DK == 0 && DK <= S - 1, "rings");
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// The launcher's rings for the fused 256 x 512 SM-pair tiles:
// four operand stages of 48 KB (this CTA's decoded A tile and 256 B rows; TF32
// three, for two 32 KB raw stages) and the rest of shared memory for the raw
// ring.
template <int FMT>
struct PickFusedPair {
    static constexpr int S = FMT == kTF32 ? 3 : 4;
    static constexpr int SA0 = (kSmemBudget - S * 3 * 128 * 128) / raw_stage_bytes(FMT);
    static constexpr int SA = SA0 > 8 ? 8 : SA0;
    static constexpr int DK = raw_kblocks(FMT) < 2 ? raw_kblocks(FMT) : 2;
    using Cfg = FusedPairCfg<FMT, S, SA, DK>;
};

// Pair tile u -> (tile row, tile column).  The operand that every wave of
// clusters reads whole stays in L2 across waves: with M tiles varying fastest
// a wave covers all rows of A and a few B columns, so A should be the smaller
// operand; otherwise N tiles vary fastest (GemmArgs::n_fastest).
__device__ __forceinline__ void pair_tile(const GemmArgs& p, int u, int tiles_m, int tiles_n, int& tm, int& tn) {
    if (p.n_fastest) {
        tm = u / tiles_n;
        tn = u % tiles_n;
    } else {
        tm = u % tiles_m;
        tn = u / tiles_m;
    }
}

// Copies rows [row0, row0 + 32) of the pair tile at column col0 from D to the
// same place in every peer buffer (GemmArgs::peer_D).  Consecutive lanes take
// consecutive 16-byte chunks of a row, so a warp's loads and stores cover 512
// contiguous bytes; each lane keeps PUSH_ITEMS chunks in flight.  The loads
// hit L2 (the epilogue has just written the rows); the stores cross NVLink.
// The rows were stored by this warp's lanes: the caller's __syncwarp orders
// those stores before these loads.  Peer buffers have D's alignment (16 bytes
// or more), so vec_ok holds for them too.
template <int BN>
__device__ __forceinline__ void push_rows_to_peers(const GemmArgs& p, int row0, int col0, int lane) {
    const int nrows = min(32, p.M - row0);
    const int ncols = min(BN, p.N - col0);
    if (nrows <= 0 || ncols <= 0) return;
    const size_t esz = p.out_f16 ? 2 : 4;
    const size_t ld_bytes = static_cast<size_t>(p.ldd) * esz;
    const size_t base = static_cast<size_t>(row0) * ld_bytes + static_cast<size_t>(col0) * esz;
    const char* src = static_cast<const char*>(p.D);
    const int n16 = p.vec_ok ? static_cast<int>((static_cast<size_t>(ncols) * esz) >> 4) : 0;
    const int items = nrows * n16;
    constexpr int PUSH_ITEMS = 4;  // (the epilogue warps share the decode warps' register budget)
    for (int q0 = 0; q0 < items; q0 += 32 * PUSH_ITEMS) {
        uint4 v[PUSH_ITEMS];
        size_t off[PUSH_ITEMS];
#pragma unroll
        for (int j = 0; j < PUSH_ITEMS; ++j) {
            const int q = q0 + j * 32 + lane;
            if (q < items) {
                const int r = q / n16;
                off[j] = base + static_cast<size_t>(r) * ld_bytes + static_cast<size_t>(q - r * n16) * 16u;
                v[j] = __ldcg(reinterpret_cast<const uint4*>(src + off[j]));
            }
        }
#pragma unroll
        for (int i = 0; i < kMaxPeers; ++i) {
            if (i >= p.n_peers) break;
            char* dst = static_cast<char*>(p.peer_D[i]);
#pragma unroll
            for (int j = 0; j < PUSH_ITEMS; ++j)
                if (q0 + j * 32 + lane < items) *reinterpret_cast<uint4*>(dst + off[j]) = v[j];
        }
    }
    // Columns past the 16-byte chunks (a ragged last tile, or no vector
    // access at all), one element at a time.
    const int c0 = static_cast<int>((static_cast<size_t>(n16) * 16u) / esz);
    const int tc = ncols - c0;
    for (int q = lane; tc > 0 && q < nrows * tc; q += 32) {
        const int r = q / tc;
        const size_t o = base + static_cast<size_t>(r) * ld_bytes + static_cast<size_t>(c0 + q - r * tc) * esz;
        if (esz == 2) {
            const unsigned short x = __ldcg(reinterpret_cast<const unsigned short*>(src + o));
#pragma unroll
            for (int i = 0; i < kMaxPeers; ++i) {
                if (i >= p.n_peers) break;
                *reinterpret_cast<unsigned short*>(static_cast<char*>(p.peer_D[i]) + o) = x;
            }
        } else {
            const unsigned int x = __ldcg(reinterpret_cast<const unsigned int*>(src + o));
#pragma unroll
            for (int i = 0; i < kMaxPeers; ++i) {
                if (i >= p.n_peers) break;
                *reinterpret_cast<unsigned int*>(static_cast<char*>(p.peer_D[i]) + o) = x;
            }
        }
    }
}

// PEERS: the instance that copies finished tiles to GemmArgs::peer_D (the
// sharded GEMM); the plain instance carries none of that code.
template <class C, bool PEERS = false>
__global__ void __launch_bounds__(C::NUM_THREADS, 1)
    k_fused_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sbase = smem_addr(smem);

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = bars;               // leader: both CTAs' B bytes and decode warps
    uint64_t* empty = full + C::S;       // both CTAs: the pair's MMAs are done with the stage
    uint64_t* a_full = empty + C::S;     // raw ring: TMA bytes landed
    uint64_t* a_empty = a_full + C::SA;  // raw ring: this CTA's decode warps done reading
    uint64_t* acc_full = a_empty + C::SA;  // both CTAs: the tile's accumulators are complete
    uint64_t* acc_empty = acc_full + 1;    // leader, per half: both CTAs' epilogues drained it
    uint64_t* fin_bar = acc_empty + C::NH;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::S; ++s) {
            mbar_init(&full[s], C::FULL_COUNT);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < C::SA; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], C::ND);
        }
        mbar_init(acc_full, 1);
        for (int h = 0; h < C::NH; ++h) mbar_init(&acc_empty[h], 8);
        mbar_init(fin_bar, 1);
        *abort_flag = 0;
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
    const int units = tiles_m * tiles_n;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    const int my_row0 = static_cast<int>(rank) * 128;

    if (warp == 0) {
        // ---------------- TMA producer: this CTA's B half ----------------
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int u = cid; ok && u < units; u += ncl) {
            int tm, tn;
            pair_tile(p, u, tiles_m, tiles_n, tm, tn);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                if (elect_one()) {
                    if (leader) mbar_arrive_expect_tx(&full[s], C::FULL_TX);
#pragma unroll
                    for (int h = 0; h < C::NH; ++h)
                        tma_load_2d_pair(smem + C::OFF_B + s * C::B_BYTES + h * 16384, &tmB, leader_bar(&full[s]),
                                         kb * 64, tn * C::BN + h * 256 + my_row0);
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
                // Half h's accumulator is free once the previous tile's half h
                // is drained (waited for right before its first MMA).
                const uint32_t aph = t & 1;
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, abort_flag))) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_lo = sdesc_lo(sbase + C::OFF_A + s * C::A_BYTES);
#pragma unroll
                    for (int h = 0; h < C::NH; ++h) {
                        if (kb == 0) {
                            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[h], aph ^ 1u, abort_flag))) { ok = false; break; }
                            tc_fence_after();
                        }
                        if (elect_one()) {
                            const uint32_t b_lo = sdesc_lo(sbase + C::OFF_B + s * C::B_BYTES + h * 16384);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
                                mma_pair<0>(tmem_base + static_cast<uint32_t>(h * 256), sdesc_make(a_lo + 2u * kk),
                                            sdesc_make(b_lo + 2u * kk), C::IDESC, accum);
                            }
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (elect_one()) mma_commit_pair(&empty[s], 0x3);
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
    } else if (warp < 6) {
        // ---------------- epilogue (both CTAs) ----------------
        const int quarter = warp & 3;
        int t = 0;
        for (int u = cid; u < units; u += ncl, ++t) {
            int tm, tn;
            pair_tile(p, u, tiles_m, tiles_n, tm, tn);
            const bool ok = mbar_wait(acc_full, t & 1, abort_flag);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            tc_fence_after();
            const int row = tm * C::BM + my_row0 + quarter * 32 + lane;
#pragma unroll 1
            for (int h = 0; h < C::NH; ++h) {
                const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       static_cast<uint32_t>(h * 256);
#pragma unroll 1
                for (int c = 0; c < 256; c += 32) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(t_row + c, v);
                    tmem_wait_ld();
                    store_row_chunk<32>(p, 0, row, tn * C::BN + h * 256 + c, v);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(&acc_empty[h], 0u);
            }
            // Sharded output: copy the tile's rows to the other GPUs while the
            // MMAs of the next tile, which no longer need this accumulator, run.
            if constexpr (PEERS)
                push_rows_to_peers<C::BN>(p, tm * C::BM + my_row0 + quarter * 32, tn * C::BN, lane);
        }
        // The peers read their D after the host's closing barrier: make this
        // warp's stores to them visible system-wide before the grid ends.
        if constexpr (PEERS) __threadfence_system();
    } else if (warp == 6) {
        // ---------------- TMA producer: this CTA's raw A rows ----------------
        int s = 0;
        uint32_t ph = 0;
        long long issued = 0;
        bool ok = true;
        for (int u = cid; ok && u < units; u += ncl) {
            int tm, tn;
            pair_tile(p, u, tiles_m, tiles_n, tm, tn);
            for (int kb = 0; kb < p.num_kb; kb += C::RK) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&a_empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                if (elect_one()) {
                    mbar_arrive_expect_tx(&a_full[s], C::RA_BYTES);
                    uint8_t* dst = smem + C::OFF_RA + s * C::RA_BYTES;
                    const int x = kb * raw_elems_per_kblock(C::FMT);
                    tma_load_2d(dst, &tmA, &a_full[s], x, tm * C::BM + my_row0);
                    if constexpr (C::FMT == kTF32)
                        tma_load_2d(dst + 16384, &tmA, &a_full[s], x + raw_box_elems(C::FMT), tm * C::BM + my_row0);
                }
                __syncwarp();
                ++issued;
                if (++s == C::SA) { s = 0; ph ^= 1u; }
            }
        }
        if (!ok && lane == 0) drain_ring(a_full, C::SA, issued);
    } else {
        // ---------------- decode warps ----------------
        // Same unit assignment as the one-CTA fused kernel: unit q of a
        // k-block slice is row 8*(q / (8*U_ROW)) + q % 8, raw column
        // (q / 8) % U_ROW, so every 8-thread shared-memory phase covers one
        // chunk of 8 consecutive rows.
        const int dt = threadIdx.x - C::DECODE_WARP0 * 32;
        int as = 0, ds = 0;
        uint32_t aph = 0, dph = 0;
        bool ok = true;
        for (int u = cid; ok && u < units; u += ncl) {
            for (int kb = 0; kb < p.num_kb; kb += C::DK) {
                const int cnt = min(C::DK, p.num_kb - kb);
                const int sub0 = kb % C::RK;
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
                    if (d < cnt) w_ok = w_ok && mbar_wait(&empty[slot[d]], sph[d] ^ 1u, abort_flag);
                if (!__all_sync(0xFFFFFFFFu, w_ok)) { ok = false; break; }
                const uint32_t raw = sbase + C::OFF_RA + as * C::RA_BYTES;
                uint4 in[C::DK][C::UPT];
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
                    }
                }
                // Decoded words visible to the tensor cores (async proxy), then
                // the leader's full barrier of each slot: a local arrival in the
                // leader; from the second CTA a 16-byte signal copy through the
                // async proxy, ordered after the proxy fence (a cluster-scope
                // release arrival stalls the warp for about a microsecond).
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        if (d < cnt) {
                            if (leader) {
                                mbar_arrive(&full[slot[d]]);
                            } else {
                                uint8_t* sig = smem + C::OFF_SIG + (warp - C::DECODE_WARP0) * 16;
                                bulk_copy_to_cluster(cluster_addr(sig, 0u), sig, 16u, leader_bar(&full[slot[d]]));
                            }
                        }
                    }
                }
                if (sub0 + cnt == C::RK || kb + cnt == p.num_kb) {
                    // Last slices of this raw stage: release it once the loaded
                    // words have been consumed (above).
                    if (lane == 0) mbar_arrive(&a_empty[as]);
                    if (++as == C::SA) { as = 0; aph ^= 1u; }
                }
                ds += cnt;
                if (ds >= C::S) { ds -= C::S; dph ^= 1u; }
            }
        }
        // Abort: signal copies may still be in flight towards the leader.
        if (!ok && !leader && lane == 0) settle_pair_loads();
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
