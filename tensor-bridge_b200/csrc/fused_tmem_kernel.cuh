// fused_tmem_kernel.cuh -- fused decode + GEMM for narrow tiles (BN <= 128),
// with the decoded weights written to tensor memory instead of shared memory.
//
//   D[M x N] = alpha * decode(A)[M x K] * B[N x K]^T
//
// Narrow tiles are the weight-streaming regime (few tokens): every weight
// byte is used for only BN output columns, so the kernel has to turn stored
// weights into MMA operands at HBM speed.  The decode warps store the FP16 A
// tile straight into a TMEM stage with tcgen05.st and the MMA reads A from
// TMEM (tcgen05.mma ... [a_tmem], b_desc), so shared memory carries only the
// raw weights and the small B tiles.
//
// Everything is organised in rounds of four k-blocks (256 values of K): per
// round the MMA issuer waits once (rdy) and commits once (fre).  On sm_100a an
// mbarrier wait or arrive costs on the order of 150 cycles of latency even
// when it does not block, while an M = 128, N = 16, K = 16 MMA with A in
// tensor memory occupies the tensor pipe for about 9 cycles, so the schedule
// is set by how many barrier operations sit on each role's path per round.
// The decode warps form NG groups of eight (two per TMEM lane quarter, each
// decoding two of the round's four k-blocks); group g decodes whole rounds
// r = g, g + NG, ... and does its own waits (the
// round's TMEM slot freed, its raw stages landed) and arrivals (raw stages
// consumed, round in TMEM), so NG rounds are decoded at once and a round's
// barrier latency is paid once per group, not once per round on a shared
// path.
//
// Roles (one persistent CTA per SM, same work units as gemm_kernel.cuh):
//   warp 0      TMA producer of the raw A ring.  A raw stage holds RSK
//               k-blocks of 128 rows in NBOX 128-byte-wide boxes (32 KB; the
//               packed-FP4 stage is one 16 KB box of four k-blocks); a round
//               spans SPR = 4 / RSK stages.
//   warp 1      TMEM allocator (all 512 columns) and MMA issuer
//   warps 2-5   epilogue (as in gemm_kernel.cuh)
//   warps 6-    decode warps.  A warp may only touch the 32 TMEM lanes of
//               its warp-id quarter q = warp % 4, so thread i owns tile row
//               32 q + i.  Group mode: NG = NRND groups of eight warps;
//               warp i = (warp - 6) % 8 of group g = (warp - 6) / 8 decodes
//               k-blocks 2 (i / 4) and 2 (i / 4) + 1 of its rounds (the
//               decode is issue-bound: the second warp per quarter hides
//               latency the first cannot).
//               Per-warp mode (TF32, whose 128 KB rounds leave a raw ring of
//               one round): sixteen warps, slice j = (warp - 6) / 4 decodes
//               k-block j of every round and waits and arrives itself.
//   last warp   TMA producer of the B tiles into their own ring of NBR round
//               slots (one tile per k-block), as far ahead of the MMAs as the
//               ring allows: B is the same for every CTA and usually in L2,
//               but one SM's TMA requests are served in order, so a B copy
//               waits behind the raw stages in flight (1.5-3.7 us a round
//               trip over a 14336 x 16 x 4096 launch) and its issue is paced
//               by them; the MMAs of a round often wait for its B tiles
// TMEM columns: [0, 2 BN) two accumulators, then from column max(128, 2 BN)
// NRND round slots (3 for BN <= 32; 2 for BN = 64, where the B tiles are
// larger, and for BN = 128, where TMEM holds no more) of four A stages of 32
// columns (64 FP16 values of K per lane).
//
// Barriers, all waits bounded:
//   raw_full / raw_empty  per raw slot: TMA bytes / the arrivals of the
//                         decode warps that read the stage.
//   rdy[r % NRND]         round r is in TMEM: the decode warps' arrivals (their
//                         tcgen05.st has completed).
//   fre[r % NRND]         round r's MMAs have completed (one commit): its TMEM
//                         stages may be overwritten.
//   b_full / b_empty      per B round slot: TMA bytes / the commit of the
//                         round's MMAs.
//   acc_full / acc_empty  as in gemm_kernel.cuh.
// A parity wait passes on a stale phase if the barrier is two phases behind
// the one waited for.  The MMA issuer, the producers and the per-warp decode
// warps walk every round in order, so they cannot be.  A decode group walks
// only its own rounds; it waits for its round's TMEM slot first (fre of round
// r - NRND, which its own previous wait, for round r - NG, kept from being two
// phases behind because NG <= NRND) and for the raw stages after that: the
// MMAs of round r - NRND imply that every earlier round was decoded, so the
// previous fill of each of its raw slots (round r - SR / SPR, with
// SR / SPR >= NRND) has landed.  tests/test_ring_protocol.py models both
// modes under random schedules and shows the failures these conditions rule
// out.
#pragma once

#include "gemm_kernel.cuh"

namespace tb {

template <int BN_, int FMT_, int SR_, int NRND_, int NBR_>
struct TmemCfg {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int FMT = FMT_;
    static constexpr int DK = 4;                          // k-blocks per round
    static constexpr int ROW_BYTES = raw_row_bytes(FMT);  // raw bytes of one k-block row
    static constexpr int RSK = ROW_BYTES <= 64 ? 4 : ROW_BYTES == 128 ? 2 : 1;  // k-blocks per raw stage
    static constexpr int SPR = DK / RSK;                  // raw stages per round
    static constexpr int NBOX = RSK * ROW_BYTES / 128;    // 128-byte boxes per stage
    static constexpr int STAGE_BYTES = NBOX * 16384;
    static constexpr int SR = SR_;                        // raw ring slots
    // Raw stages the producer keeps in flight: a CTA that asks for its whole
    // ring at once gets all stages at about the same time, late, because HBM
    // serves the requests of all CTAs interleaved; a bounded number in flight
    // lands in order and the first round arrives early.  Measured best: 64 KB
    // (four stages) for the 16 KB stages of packed FP4, whose ring holds up to
    // ten; all but one stage of the ring for the 32 KB stages (three of four
    // for one-byte weights at 16 columns).
    // The stage waited for must not have been refilled yet: INFLIGHT < SR.
    static constexpr int INFLIGHT_CAP = STAGE_BYTES <= 16384 ? 65536 / STAGE_BYTES : SR - 1;
    static constexpr int INFLIGHT = SR - 1 < INFLIGHT_CAP ? SR - 1 : INFLIGHT_CAP;
    static constexpr int NRND = NRND_;                    // round slots (TMEM A stages, B tiles)
    static constexpr int B_BYTES = BN * 128;              // one k-block of B
    static constexpr int NBR = NBR_;                      // B ring slots (rounds)
    // Group mode when the raw ring holds at least NRND rounds (every format
    // but TF32); NG = NRND groups of GW = 8 decode warps.
    static constexpr bool GROUPS = SR / SPR >= NRND;
    static constexpr int NG = GROUPS ? NRND : 0;
    static constexpr int GW = 8;
    static constexpr int ND = GROUPS ? GW * NG : 16;      // decode warps
    static constexpr int DECODE_WARP0 = 6;
    static constexpr int B_WARP = DECODE_WARP0 + ND;
    static constexpr int NUM_THREADS = (B_WARP + 1) * 32;
    static constexpr uint32_t NB_SETUP = 1;  // set-up named barrier: warp 0 arrives, the others wait

    static constexpr int A_COL0 = 2 * BN > 128 ? 2 * BN : 128;
    static constexpr int TMEM_COLS = 512;
    static constexpr int CW = BN < 32 ? BN : 32;

    // Decode of one k-block row slice: 16-byte raw units per row, processed
    // in H parts of UPH units / WPH output words (32-bit TMEM columns).
    static constexpr int U_ROW = ROW_BYTES / 16;
    static constexpr int H = U_ROW > 8 ? 2 : 1;
    static constexpr int UPH = U_ROW / H;
    static constexpr int WPU = 32 / U_ROW;
    static constexpr int WPH = 32 / H;

    static constexpr int OFF_R = 0;
    static constexpr int OFF_B = OFF_R + SR * STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_B + NBR * DK * B_BYTES;
    static constexpr int NUM_BARS = 2 * SR + 2 * NRND + 2 * NBR + 5;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;

    static constexpr uint32_t IDESC = idesc_make(0u, 0u, BM, BN);

    static_assert(BN == 16 || BN == 32 || BN == 64 || BN == 128, "narrow tiles only");
    static_assert(RSK * SPR == DK && NBOX >= 1 && RSK * ROW_BYTES == NBOX * 128, "raw stage geometry");
    static_assert(WPH == 32 || WPH == 16, "TMEM store width");
    static_assert(2 * BN <= A_COL0 && A_COL0 + NRND * DK * 32 <= TMEM_COLS && NRND >= 2, "TMEM budget");
    static_assert(SR % SPR == 0 && SR >= SPR, "each raw slot holds one stage position of a round");
    static_assert(!GROUPS || (NG <= NRND && SR / SPR >= NRND), "group mode parity conditions");
    static_assert(NUM_THREADS <= 1024, "block size");
    static_assert(B_BYTES % 1024 == 0, "B tile alignment");
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// The launcher's choice of rings for a narrow tile of BN columns.  The B
// ring gets about 64 KB (two to eight rounds), less if the raw ring would
// otherwise hold fewer than NRND rounds (the decode groups' condition); the
// raw ring the rest, up to twelve stages.
template <int BN, int FMT>
struct PickTmem {
    static constexpr int NRND = BN <= 32 ? 3 : 2;  // round slots of TMEM A stages
    static constexpr int ROW = raw_row_bytes(FMT);
    static constexpr int RSK = ROW <= 64 ? 4 : ROW == 128 ? 2 : 1;
    static constexpr int SPR = 4 / RSK;
    static constexpr int STAGE = RSK * ROW * 128;
    static constexpr int BROUND = 4 * BN * 128;
    static constexpr int AVAIL = kSmemBudget - 1024;
    static constexpr int NBR_T0 = 65536 / BROUND;
    static constexpr int NBR_T = NBR_T0 > 8 ? 8 : (NBR_T0 < 2 ? 2 : NBR_T0);
    static constexpr int NBR_G = (AVAIL - NRND * SPR * STAGE) / BROUND;  // most B rounds group mode allows
    static constexpr int NBR = NBR_G >= 2 && NBR_G < NBR_T ? NBR_G : NBR_T;
    static constexpr int SR0 = (AVAIL - NBR * BROUND) / STAGE;
    static constexpr int SR1 = SR0 > 12 ? 12 : SR0;
    static constexpr int SR = SR1 / SPR * SPR;
    using Cfg = TmemCfg<BN, FMT, SR, NRND, NBR>;
};

// Shared-memory address of 16-byte raw unit `col` of k-block `sub` (position
// within the stage), tile row `row`: byte `sub * ROW_BYTES + 16 col` of the
// row, in box (byte / 128) of the stage, 128-byte swizzled.
template <class C>
__device__ __forceinline__ uint32_t tmem_raw_addr(uint32_t stage, int sub, int row, int col) {
    const int off = sub * C::ROW_BYTES + col * 16;
    return stage + (off >> 7) * 16384 + swz(row, (off & 127) >> 4);
}

// After an abort: give TMA loads this thread issued time to land before the
// CTA's shared memory is released (at most about a millisecond).
__device__ __forceinline__ void settle_inflight_loads() {
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < 1000000ull) {
    }
}

// Decode one 16-byte raw unit into WPU words of FP16 pairs (lower K first).
// `scalar` (warp-uniform) selects the per-code path for TF32 units holding
// values at or above 2^16.  E4M3 and BF16 need none: their branch-free paths
// give every code its reference value (a NaN only another FP16 payload).
template <int FMT>
__device__ __forceinline__ void decode_unit_words(const uint4& in, uint32_t* o, bool scalar) {
    if constexpr (FMT == kE4M3) {
        decode_e4m3_x4_scaled(in.x, o[0], o[1]); decode_e4m3_x4_scaled(in.y, o[2], o[3]);
        decode_e4m3_x4_scaled(in.z, o[4], o[5]); decode_e4m3_x4_scaled(in.w, o[6], o[7]);
    } else if constexpr (FMT == kE5M2) {
        decode_e5m2_x4(in.x, o[0], o[1]); decode_e5m2_x4(in.y, o[2], o[3]);
        decode_e5m2_x4(in.z, o[4], o[5]); decode_e5m2_x4(in.w, o[6], o[7]);
    } else if constexpr (FMT == kE2M1U) {
        decode_e2m1_unpacked_x4(in.x, o[0], o[1]); decode_e2m1_unpacked_x4(in.y, o[2], o[3]);
        decode_e2m1_unpacked_x4(in.z, o[4], o[5]); decode_e2m1_unpacked_x4(in.w, o[6], o[7]);
    } else if constexpr (FMT == kE2M1) {
        uint32_t t[4];
        decode_e2m1_packed_x8(in.x, t); o[0] = t[0]; o[1] = t[1]; o[2] = t[2]; o[3] = t[3];
        decode_e2m1_packed_x8(in.y, t); o[4] = t[0]; o[5] = t[1]; o[6] = t[2]; o[7] = t[3];
        decode_e2m1_packed_x8(in.z, t); o[8] = t[0]; o[9] = t[1]; o[10] = t[2]; o[11] = t[3];
        decode_e2m1_packed_x8(in.w, t); o[12] = t[0]; o[13] = t[1]; o[14] = t[2]; o[15] = t[3];
    } else if constexpr (FMT == kBF16) {
        o[0] = decode_bf16_x2_fast(in.x); o[1] = decode_bf16_x2_fast(in.y);
        o[2] = decode_bf16_x2_fast(in.z); o[3] = decode_bf16_x2_fast(in.w);
    } else if constexpr (FMT == kTF32) {
        if (scalar) {
            o[0] = decode_tf32_x2_scalar(in.x, in.y);
            o[1] = decode_tf32_x2_scalar(in.z, in.w);
        } else {
            o[0] = decode_tf32_x2_fast(in.x, in.y);
            o[1] = decode_tf32_x2_fast(in.z, in.w);
        }
    }
}

// Nonzero if a TF32 unit holds a value the fast path does not reproduce.
template <int FMT>
__device__ __forceinline__ uint32_t unit_special_mask(const uint4& in) {
    if constexpr (FMT == kTF32)
        return max(tf32_max_mag(in.x, in.y), tf32_max_mag(in.z, in.w)) >= kTf32ScalarFrom ? 1u : 0u;
    else
        return 0u;
}

// One work unit of the narrow kernel: tile (tm, tn), split sp, k-blocks
// [kb0, kb1).
struct NUnit {
    int tm, tn, sp, kb0, kb1;
};

// This CTA's work units (persistent: blockIdx.x, + gridDim.x, ...), in the
// same order for every role.
struct NCursor {
    int u;
};

__device__ __forceinline__ void ncur_init(const GemmArgs&, NCursor& c) { c.u = blockIdx.x; }

__device__ __forceinline__ bool ncur_next(const GemmArgs& p, NCursor& c, NUnit& x) {
    if (c.u >= p.num_units) return false;
    unit_coords(p, c.u, x.tm, x.tn, x.sp);
    unit_kblocks(p, x.sp, x.kb0, x.kb1);
    c.u += gridDim.x;
    return true;
}

// Decode k-block `sub` of the raw stage at `raw` for tile row `row` (this
// thread's TMEM lane) and store its 64 FP16 values into TMEM columns
// [ta, ta + 32).  The stores are asynchronous (tcgen05.wait::st).
template <class C>
__device__ __forceinline__ void decode_kblock(uint32_t raw, int sub, int row, uint32_t ta) {
#pragma unroll
    for (int h = 0; h < C::H; ++h) {
        uint4 in[C::UPH];
#pragma unroll
        for (int x = 0; x < C::UPH; ++x) in[x] = lds128(tmem_raw_addr<C>(raw, sub, row, h * C::UPH + x));
        bool scalar = false;
        if constexpr (C::FMT == kTF32) {
            uint32_t m = 0;
#pragma unroll
            for (int x = 0; x < C::UPH; ++x) m |= unit_special_mask<C::FMT>(in[x]);
            scalar = __any_sync(0xFFFFFFFFu, m != 0u);
        }
        uint32_t o[C::WPH];
#pragma unroll
        for (int x = 0; x < C::UPH; ++x) decode_unit_words<C::FMT>(in[x], o + x * C::WPU, scalar);
        if constexpr (C::WPH == 32) tmem_st_32x32b_x32(ta, *reinterpret_cast<const uint32_t(*)[32]>(o));
        else tmem_st_32x32b_x16(ta + h * 16, *reinterpret_cast<const uint32_t(*)[16]>(o));
    }
}

template <class C>
__global__ void __launch_bounds__(C::NUM_THREADS, 1)
    k_fused_tmem(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_addr(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const uint32_t sbase = smem_addr(smem);

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + C::SR;
    uint64_t* rdy = raw_empty + C::SR;
    uint64_t* fre = rdy + C::NRND;
    uint64_t* b_full = fre + C::NRND;
    uint64_t* b_empty = b_full + C::NBR;
    uint64_t* acc_full = b_empty + C::NBR;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* fin_bar = acc_empty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::SR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], C::GROUPS ? C::GW : 4 * C::RSK);
        }
        for (int s = 0; s < C::NRND; ++s) {
            mbar_init(&rdy[s], C::GROUPS ? C::GW : C::ND);
            mbar_init(&fre[s], 1);
        }
        for (int s = 0; s < C::NBR; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 128);
        }
        mbar_init(fin_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        // The next narrow GEMM in the stream may start now: its weight stream
        // then overlaps this kernel's tail (launched with programmatic stream
        // serialisation; see the dependency waits below).
        grid_dep_launch_dependents();
    }
    if (warp == 0 && lane == 0) tma_prefetch_desc(&tmA);
    if (warp == C::B_WARP && lane == 0) tma_prefetch_desc(&tmB);
    if (warp == 1) {
        tmem_alloc(tmem_holder, C::TMEM_COLS);
        tmem_relinquish();
    }
    // Set-up barrier: the raw-A producer (warp 0, whose thread 0 initialised
    // the mbarriers) only arrives and starts streaming at once; the other
    // warps also need the TMEM allocation and wait for everyone.
    uint32_t tmem_base = 0;
    if (warp == 0) {
        __syncwarp();
        named_bar_arrive(C::NB_SETUP, C::NUM_THREADS);
    } else {
        tc_fence_before();
        named_bar_sync(C::NB_SETUP, C::NUM_THREADS);
        tc_fence_after();
        tmem_base = *tmem_holder;
    }

    if (warp == 0) {
        // ---------------- TMA producer: raw A stages ----------------
        // Weights in the one-byte and packed formats are streamed before the
        // previous kernel has completed (when it let this one start early, as
        // this kernel does): no kernel that triggers early writes them (this
        // library's quantizer does not trigger, so a GEMM after it waits).
        // BF16 and TF32 words could be an earlier GEMM's FP16 / FP32 output:
        // wait for it first.
        if constexpr (C::FMT == kBF16 || C::FMT == kTF32) grid_dep_wait();
        // Each weight byte is read once: evict-first in L2, which keeps the
        // activations (read by every CTA) resident.
        const uint64_t wpol = l2_policy_evict_first();
        uint32_t st = 0;  // CTA-wide stage number
        bool ok = true;
        NCursor cur;
        ncur_init(p, cur);
        NUnit x;
        while (ok && ncur_next(p, cur, x)) {
            const int tm = x.tm, kb0 = x.kb0, kb1 = x.kb1;
            for (int kb = kb0; ok && kb < kb1; kb += C::DK) {
#pragma unroll 1
                for (int pos = 0; pos < C::SPR; ++pos, ++st) {
                    const uint32_t rs = st % C::SR, fill = st / C::SR;
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&raw_empty[rs], (fill & 1u) ^ 1u, abort_flag))) {
                        ok = false;
                        break;
                    }
                    if (C::INFLIGHT > 0 && st >= static_cast<uint32_t>(C::INFLIGHT)) {
                        // This warp issued every earlier stage and waits for each
                        // of them in order, so the parity cannot be stale.
                        const uint32_t old = st - C::INFLIGHT;
                        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&raw_full[old % C::SR], (old / C::SR) & 1u, abort_flag))) {
                            ok = false;
                            break;
                        }
                    }
                    if (elect_one()) {
                        mbar_arrive_expect_tx(&raw_full[rs], C::STAGE_BYTES);
                        uint8_t* dst = smem + C::OFF_R + rs * C::STAGE_BYTES;
                        const int x0 = (kb + pos * C::RSK) * raw_elems_per_kblock(C::FMT);
#pragma unroll
                        for (int b = 0; b < C::NBOX; ++b)
                            tma_load_2d_hint(dst + b * 16384, &tmA, &raw_full[rs], x0 + b * raw_box_elems(C::FMT),
                                             tm * C::BM, wpol);
                    }
                    __syncwarp();
                }
            }
        }
        if (!ok && lane == 0) settle_inflight_loads();
    } else if (warp == C::B_WARP) {
        // ---------------- TMA producer: the four B tiles of each round ----------------
        // B (activations) may be the previous kernel's output: wait for it.
        grid_dep_wait();
        uint32_t r = 0;
        bool ok = true;
        NCursor cur;
        ncur_init(p, cur);
        NUnit x;
        while (ok && ncur_next(p, cur, x)) {
            const int tn = x.tn, kb0 = x.kb0, kb1 = x.kb1;
            for (int kb = kb0; kb < kb1; kb += C::DK, ++r) {
                const int cnt = min(C::DK, kb1 - kb);
                const uint32_t bs = r % C::NBR, buse = r / C::NBR;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&b_empty[bs], (buse & 1u) ^ 1u, abort_flag))) { ok = false; break; }
                if (elect_one()) {
                    mbar_arrive_expect_tx(&b_full[bs], static_cast<uint32_t>(cnt * C::B_BYTES));
                    uint8_t* dst = smem + C::OFF_B + bs * (C::DK * C::B_BYTES);
                    for (int d = 0; d < cnt; ++d)
                        tma_load_2d(dst + d * C::B_BYTES, &tmB, &b_full[bs], (kb + d) * 64, tn * C::BN);
                }
                __syncwarp();
            }
        }
        if (!ok && lane == 0) settle_inflight_loads();
    } else if (warp == 1) {
        // ---------------- MMA issuer: A from TMEM, B from shared memory ----------------
        uint32_t r = 0;
        int t = 0;
        bool ok = true;
        NCursor cur;
        ncur_init(p, cur);
        NUnit x;
        for (; ok && ncur_next(p, cur, x); ++t) {
            const int kb0 = x.kb0, kb1 = x.kb1;
            const int acc = t & 1;
            const uint32_t aph = (t >> 1) & 1;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag))) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
            for (int kb = kb0; kb < kb1; kb += C::DK, ++r) {
                const int cnt = min(C::DK, kb1 - kb);
                const uint32_t slot = r % C::NRND, use = r / C::NRND;
                const uint32_t bs = r % C::NBR, buse = r / C::NBR;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&b_full[bs], buse & 1u, abort_flag))) { ok = false; break; }
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&rdy[slot], use & 1u, abort_flag))) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t b_lo = sdesc_lo(sbase + C::OFF_B + bs * (C::DK * C::B_BYTES));
                    const uint32_t a_t = tmem_base + static_cast<uint32_t>(C::A_COL0 + slot * C::DK * 32);
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        if (d < cnt) {
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint32_t accum = (kb + d == kb0 && kk == 0) ? 0u : 1u;
                                mma_f16_ts(d_tmem, a_t + static_cast<uint32_t>(d * 32 + 8 * kk),
                                           sdesc_make(b_lo + static_cast<uint32_t>((d * C::B_BYTES) >> 4) + 2u * kk),
                                           C::IDESC, accum);
                            }
                        }
                    }
                    mma_commit(&fre[slot]);
                    mma_commit(&b_empty[bs]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (elect_one()) mma_commit(&acc_full[acc]);
            __syncwarp();
        }
        if ((!ok || *abort_flag) && lane == 0) {
            mma_commit(fin_bar);
            mbar_wait_drain(fin_bar, 0u);
        }
    } else if (warp < 6) {
        // ---------------- epilogue ----------------
        // D (or the split-K partials) may still be read or written by the
        // previous kernel: wait for it to complete before the first store.
        grid_dep_wait();
        const int quarter = warp & 3;
        int t = 0;
        NCursor cur;
        ncur_init(p, cur);
        NUnit x;
        for (; ncur_next(p, cur, x); ++t) {
            const int acc = t & 1;
            const uint32_t aph = (t >> 1) & 1;
            const bool ok = mbar_wait(&acc_full[acc], aph, abort_flag);
            if (!__all_sync(0xFFFFFFFFu, ok)) break;
            tc_fence_after();
            const int trow = quarter * 32 + lane;
            const int row = x.tm * C::BM + trow;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * C::BN);
#pragma unroll 1
            for (int c = 0; c < C::BN; c += C::CW) {
                uint32_t v[C::CW];
                tmem_ld_chunk<C::CW>(t_row + c, v);
                tmem_wait_ld();
                store_row_chunk<C::CW>(p, x.sp, row, x.tn * C::BN + c, v);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
        }
    } else if (warp < C::B_WARP) {
        // ---------------- decode warps: raw stages -> FP16 words -> TMEM ----------------
        const int q = warp & 3;                          // TMEM lane quarter
        const int row = q * 32 + lane;                   // tile row owned by this thread
        const uint32_t t_quarter = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(C::A_COL0);
        uint32_t r = 0;
        if constexpr (C::GROUPS) {
            // Group g decodes rounds g, g + NG, ...; this warp k-blocks d0 and d0 + 1 of each.
            const uint32_t g = static_cast<uint32_t>((warp - C::DECODE_WARP0) / C::GW);
            const int d0 = 2 * (((warp - C::DECODE_WARP0) % C::GW) >> 2);
            bool ok = true;
            NCursor cur;
            ncur_init(p, cur);
            NUnit x;
            while (ok && ncur_next(p, cur, x)) {
                const int kb0 = x.kb0, kb1 = x.kb1;
                for (int kb = kb0; kb < kb1; kb += C::DK, ++r) {
                    if (r % C::NG != g) continue;
                    const int cnt = min(C::DK, kb1 - kb);  // the short last round of a unit
                    const uint32_t slot = r % C::NRND, use = r / C::NRND;
                    // The round's TMEM slot first, then its raw stages (see the parity note above).
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&fre[slot], (use & 1u) ^ 1u, abort_flag))) { ok = false; break; }
#pragma unroll 1
                    for (int pos = 0; ok && pos < C::SPR; ++pos) {
                        const uint32_t st = r * C::SPR + pos;
                        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&raw_full[st % C::SR], (st / C::SR) & 1u, abort_flag));
                    }
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t t_slot = t_quarter + slot * (C::DK * 32);
#pragma unroll 1
                    for (int d = d0; d < d0 + 2 && d < cnt; ++d) {
                        const uint32_t st = r * C::SPR + d / C::RSK;
                        decode_kblock<C>(sbase + C::OFF_R + (st % C::SR) * C::STAGE_BYTES, d % C::RSK, row,
                                         t_slot + static_cast<uint32_t>(d * 32));
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
#pragma unroll 1
                        for (int pos = 0; pos < C::SPR; ++pos) mbar_arrive(&raw_empty[(r * C::SPR + pos) % C::SR]);
                        mbar_arrive(&rdy[slot]);
                    }
                }
            }
        } else {
            // Per-warp mode: slice j decodes k-block j of every round.
            const int j = (warp - C::DECODE_WARP0) >> 2;
            const int pos = j / C::RSK, sub = j % C::RSK;   // raw stage of the round, k-block within it
            const uint32_t t_lane = t_quarter + static_cast<uint32_t>(j * 32);
            bool ok = true;
            NCursor cur;
            ncur_init(p, cur);
            NUnit x;
            while (ok && ncur_next(p, cur, x)) {
                const int kb0 = x.kb0, kb1 = x.kb1;
                for (int kb = kb0; kb < kb1; kb += C::DK, ++r) {
                    const bool mine = j < kb1 - kb;  // the short last round of a unit
                    const uint32_t st = r * C::SPR + pos;
                    const uint32_t rs = st % C::SR, fill = st / C::SR;
                    const uint32_t slot = r % C::NRND, use = r / C::NRND;
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&raw_full[rs], fill & 1u, abort_flag))) { ok = false; break; }
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&fre[slot], (use & 1u) ^ 1u, abort_flag))) { ok = false; break; }
                    tc_fence_after();
                    if (mine)
                        decode_kblock<C>(sbase + C::OFF_R + rs * C::STAGE_BYTES, sub, row,
                                         t_lane + static_cast<uint32_t>(slot * C::DK * 32));
                    // The raw words are consumed (decoded above): release the stage.
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[rs]);
                    if (mine) tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&rdy[slot]);
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

}  // namespace tb
