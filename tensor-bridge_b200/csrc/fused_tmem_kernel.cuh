// fused_tmem_kernel.cuh -- fused decode + GEMM for narrow tiles (BN <= 64),
// with the decoded weights written to tensor memory instead of shared memory.
//
//   D[M x N] = alpha * decode(A)[M x K] * B[N x K]^T
//
// Narrow tiles are the weight-streaming regime (few tokens): every weight
// byte is used for only BN output columns, so the kernel has to turn stored
// weights into MMA operands at HBM speed.  Two things decide that here: the
// decode warps' instruction throughput, and keeping the decode, the MMAs and
// the raw loads overlapped.  The decode warps store the FP16 A tile straight
// into a TMEM stage with tcgen05.st and the MMA reads A from TMEM
// (tcgen05.mma ... [a_tmem], b_desc), so shared memory carries only the raw
// weights and the small B tiles.
//
// Roles (one persistent CTA per SM, same work units as gemm_kernel.cuh):
//   warp 0      TMA producer of the raw A ring: one stage = one raw A box (RK
//               k-blocks of 128 rows)
//   warp 1      TMEM allocator (all 512 columns) and MMA issuer
//   warps 2-5   epilogue (as in gemm_kernel.cuh)
//   warps 6-21  16 decode warps.  A warp may only touch the 32 TMEM lanes of
//               its warp-id quarter q = warp % 4, so thread i owns tile row
//               32 q + i.  Slice j = (warp - 6) / 4 of a quarter decodes the
//               k-blocks whose CTA-wide index is j mod 4, whole rows of 64
//               values, so four k-blocks are decoded at once.
//   warp 22     TMA producer of the B ring: one B tile per k-block
// TMEM columns: [0, ACC_COLS) two accumulators (NACC chains of BN columns
// each), then TS A stages of 32 columns (64 FP16 values of K per lane).
//
// The raw A ring is released by the decode warps alone, as soon as they have
// decoded their k-block of a stage, so weight loads stream independently of
// the MMAs; B has its own ring that only the MMA consumes.  Each full barrier
// is waited on only by the role whose arrivals free its slot, so no waiter can
// see a slot refilled twice.  Barriers: raw_full (TMA bytes); raw_empty
// (one arrival from each of the 16 decode warps, which all walk every stage);
// b_full (TMA bytes) / b_empty (MMA commit); t_full (4 arrivals from the owner
// slice once tcgen05.st has completed) / t_empty (MMA commit); acc_full /
// acc_empty as in gemm_kernel.cuh.  Every wait is bounded.
#pragma once

#include "gemm_kernel.cuh"

namespace tb {

template <int BN_, int FMT_, int SR_, int SB_>
struct TmemCfg {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int FMT = FMT_;
    static constexpr int SR = SR_;   // raw ring stages
    static constexpr int SB = SB_;   // B ring slots (one k-block's B tile each)
    static constexpr int NSLICE = 4; // decode warps per TMEM lane quarter
    static constexpr int ND = 4 * NSLICE;
    static constexpr int RK = raw_kblocks(FMT);
    static constexpr int RA_BYTES = raw_stage_bytes(FMT);
    static constexpr int B_BYTES = BN * 128;
    static constexpr int RSTAGE_BYTES = RA_BYTES;
    static constexpr int DECODE_WARP0 = 6;
    static constexpr int B_WARP = DECODE_WARP0 + ND;  // TMA producer of the B ring
    static constexpr int NUM_THREADS = (B_WARP + 1) * 32;
    static constexpr int DK = 4;     // k-blocks per MMA wait round

    static constexpr int NACC = BN <= 16 ? 4 : 2;
    static constexpr int ACC_COLS = 2 * NACC * BN;
    static constexpr int TS = (512 - ACC_COLS) / 32 > 12 ? 12 : (512 - ACC_COLS) / 32;  // TMEM A stages
    static constexpr int A_COL0 = ACC_COLS;
    static constexpr int TMEM_COLS = 512;
    static constexpr int CW = BN < 32 ? BN : 32;

    // Decode of one k-block row slice: 16-byte raw units per row, processed
    // in H parts of UPH units / WPH output words (32-bit TMEM columns).
    static constexpr int U_ROW = raw_row_bytes(FMT) / 16;
    static constexpr int H = U_ROW > 8 ? 2 : 1;
    static constexpr int UPH = U_ROW / H;
    static constexpr int WPU = 32 / U_ROW;
    static constexpr int WPH = 32 / H;

    static constexpr int OFF_R = 0;
    static constexpr int OFF_B = OFF_R + SR * RSTAGE_BYTES;
    static constexpr int OFF_BAR = OFF_B + SB * B_BYTES;
    static constexpr int NUM_BARS = 2 * SR + 2 * SB + 2 * TS + 5;
    static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16;
    static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;

    static constexpr uint32_t IDESC = idesc_make(0u, 0u, BM, BN);

    static_assert(BN == 16 || BN == 32 || BN == 64, "narrow tiles only");
    static_assert(RK <= NSLICE, "one k-block per slice per raw stage");
    static_assert(WPH == 32 || WPH == 16, "TMEM store width");
    static_assert(A_COL0 + TS * 32 <= TMEM_COLS && TS >= NSLICE + DK, "TMEM budget");
    static_assert(TS % NSLICE == 0, "each TMEM stage keeps one owner slice");
    static_assert(SR >= DK && SB >= DK, "ring depths");
    static_assert(RA_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "stage alignment");
    static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// Decode one 16-byte raw unit into WPU words of FP16 pairs (lower K first).
// `scalar` selects the reference-rule path for E4M3 / BF16 / TF32 special codes.
template <int FMT>
__device__ __forceinline__ void decode_unit_words(const uint4& in, uint32_t* o, bool scalar) {
    if constexpr (FMT == kE4M3) {
        if (scalar) {
            decode_e4m3_x4_scalar(in.x, o[0], o[1]); decode_e4m3_x4_scalar(in.y, o[2], o[3]);
            decode_e4m3_x4_scalar(in.z, o[4], o[5]); decode_e4m3_x4_scalar(in.w, o[6], o[7]);
        } else {
            decode_e4m3_x4_fast(in.x, o[0], o[1]); decode_e4m3_x4_fast(in.y, o[2], o[3]);
            decode_e4m3_x4_fast(in.z, o[4], o[5]); decode_e4m3_x4_fast(in.w, o[6], o[7]);
        }
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
        if (scalar) {
            o[0] = decode_bf16_x2_scalar(in.x); o[1] = decode_bf16_x2_scalar(in.y);
            o[2] = decode_bf16_x2_scalar(in.z); o[3] = decode_bf16_x2_scalar(in.w);
        } else {
            o[0] = decode_bf16_x2_fast(in.x); o[1] = decode_bf16_x2_fast(in.y);
            o[2] = decode_bf16_x2_fast(in.z); o[3] = decode_bf16_x2_fast(in.w);
        }
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

// Nonzero if a unit holds a code the fast path does not reproduce (E4M3,
// BF16, TF32).
template <int FMT>
__device__ __forceinline__ uint32_t unit_special_mask(const uint4& in) {
    if constexpr (FMT == kE4M3)
        return e4m3_special_mask(in.x) | e4m3_special_mask(in.y) | e4m3_special_mask(in.z) | e4m3_special_mask(in.w);
    else if constexpr (FMT == kBF16)
        return bf16_nan_lanes(in.x) | bf16_nan_lanes(in.y) | bf16_nan_lanes(in.z) | bf16_nan_lanes(in.w);
    else if constexpr (FMT == kTF32)
        return max(tf32_max_mag(in.x, in.y), tf32_max_mag(in.z, in.w)) >= kTf32ScalarFrom ? 1u : 0u;
    else
        return 0u;
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
    uint64_t* b_full = raw_empty + C::SR;
    uint64_t* b_empty = b_full + C::SB;
    uint64_t* t_full = b_empty + C::SB;
    uint64_t* t_empty = t_full + C::TS;
    uint64_t* acc_full = t_empty + C::TS;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* fin_bar = acc_empty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(fin_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::SR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], C::ND);
        }
        for (int s = 0; s < C::SB; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < C::TS; ++s) {
            mbar_init(&t_full[s], 4);
            mbar_init(&t_empty[s], 1);
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
    }
    if (warp == C::B_WARP && lane == 0) tma_prefetch_desc(&tmB);
    if (warp == 1) {
        tmem_alloc(tmem_holder, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // ---------------- TMA producer: raw A box + the stage's B tiles ----------------
        int s = 0;
        uint32_t ph = 0;
        long long issued = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            int tm, tn, sp, kb0, kb1;
            unit_coords(p, u, tm, tn, sp);
            unit_kblocks(p, sp, kb0, kb1);
            for (int kb = kb0; kb < kb1; kb += C::RK) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&raw_empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                const int nk = min(C::RK, kb1 - kb);
                if (elect_one()) {
                    mbar_arrive_expect_tx(&raw_full[s], C::RA_BYTES);
                    uint8_t* dst = smem + C::OFF_R + s * C::RSTAGE_BYTES;
                    const int x = kb * raw_elems_per_kblock(C::FMT);
                    tma_load_2d(dst, &tmA, &raw_full[s], x, tm * C::BM);
                    if constexpr (C::FMT == kTF32)
                        tma_load_2d(dst + 16384, &tmA, &raw_full[s], x + raw_box_elems(C::FMT), tm * C::BM);
                }
                __syncwarp();
                ++issued;
                if (++s == C::SR) { s = 0; ph ^= 1u; }
            }
        }
        if (!ok && lane == 0) drain_ring(raw_full, C::SR, issued);
    } else if (warp == 1) {
        // ---------------- MMA issuer: A from TMEM, B from the B ring ----------------
        int bs = 0, ts = 0;
        uint32_t bph = 0, tph = 0;
        int t = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++t) {
            int tm, tn, sp, kb0, kb1;
            unit_coords(p, u, tm, tn, sp);
            unit_kblocks(p, sp, kb0, kb1);
            const int acc = t & 1;
            const uint32_t aph = (t >> 1) & 1;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[acc], aph ^ 1u, abort_flag))) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::NACC * C::BN);
            for (int kb = kb0; kb < kb1; kb += C::DK) {
                const int cnt = min(C::DK, kb1 - kb);
                int tsd[C::DK], bsd[C::DK];
                bool w_ok = true;
                {
                    int bb = bs, tt = ts;
                    uint32_t bp = bph, tp = tph;
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        if (d < cnt) {
                            w_ok = w_ok && mbar_wait(&b_full[bb], bp, abort_flag);  // B tile landed
                            w_ok = w_ok && mbar_wait(&t_full[tt], tp, abort_flag);  // A decoded
                            tsd[d] = tt; bsd[d] = bb;
                            if (++tt == C::TS) { tt = 0; tp ^= 1u; }
                            if (++bb == C::SB) { bb = 0; bp ^= 1u; }
                        }
                    }
                    bs = bb; ts = tt; bph = bp; tph = tp;
                }
                if (!__all_sync(0xFFFFFFFFu, w_ok)) { ok = false; break; }
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (int d = 0; d < C::DK; ++d) {
                        if (d < cnt) {
                            const bool first = kb + d == kb0;
                            const uint32_t b_lo = sdesc_lo(sbase + C::OFF_B + bsd[d] * C::B_BYTES);
                            const uint32_t a_t = tmem_base + static_cast<uint32_t>(C::A_COL0 + tsd[d] * 32);
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk) {
                                const uint32_t accum = (!first || kk >= C::NACC) ? 1u : 0u;
                                const uint32_t dd = d_tmem + static_cast<uint32_t>((kk % C::NACC) * C::BN);
                                mma_f16_ts(dd, a_t + 8u * kk, sdesc_make(b_lo + 2u * kk), C::IDESC, accum);
                            }
                            mma_commit(&t_empty[tsd[d]]);
                            mma_commit(&b_empty[bsd[d]]);
                        }
                    }
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
    } else if (warp == C::B_WARP) {
        // ---------------- TMA producer: one B tile per k-block ----------------
        int s = 0;
        uint32_t ph = 0;
        long long issued = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            int tm, tn, sp, kb0, kb1;
            unit_coords(p, u, tm, tn, sp);
            unit_kblocks(p, sp, kb0, kb1);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&b_empty[s], ph ^ 1u, abort_flag))) { ok = false; break; }
                if (elect_one()) {
                    mbar_arrive_expect_tx(&b_full[s], C::B_BYTES);
                    tma_load_2d(smem + C::OFF_B + s * C::B_BYTES, &tmB, &b_full[s], kb * 64, tn * C::BN);
                }
                __syncwarp();
                ++issued;
                if (++s == C::SB) { s = 0; ph ^= 1u; }
            }
        }
        if (!ok && lane == 0) drain_ring(b_full, C::SB, issued);
    } else if (warp < 6) {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3;
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
                                   static_cast<uint32_t>(acc * C::NACC * C::BN);
#pragma unroll 1
            for (int c = 0; c < C::BN; c += C::CW) {
                uint32_t v[C::CW];
                tmem_ld_chunk<C::CW>(t_row + c, v);
#pragma unroll
                for (int ch = 1; ch < C::NACC; ++ch) {
                    uint32_t w[C::CW];
                    tmem_ld_chunk<C::CW>(t_row + ch * C::BN + c, w);
                    tmem_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < C::CW; ++jj)
                        v[jj] = __float_as_uint(__uint_as_float(v[jj]) + __uint_as_float(w[jj]));
                }
                tmem_wait_ld();
                store_row_chunk<C::CW>(p, sp, row, tn * C::BN + c, v);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
        }
    } else {
        // ---------------- decode warps: one k-block row slice -> FP16 words -> TMEM ----------------
        // Every decode warp walks every raw stage in order: it waits for the
        // stage, decodes the k-block of the stage that it owns (if any) and
        // arrives on the stage's empty barrier, so no slot can be refilled
        // before all sixteen warps have passed it.  The owner slice of a
        // k-block is its CTA-wide index t mod 4; TS is a multiple of 4, so each
        // TMEM stage is always written by the same four warps, which see every
        // phase of its empty barrier in order.
        const int q = warp & 3;                          // TMEM lane quarter
        const int j = (warp - C::DECODE_WARP0) >> 2;     // slice: owns k-blocks with t % 4 == j
        const int row = q * 32 + lane;                   // tile row owned by this thread
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(C::A_COL0);
        int rs = 0, ts = 0;              // raw slot of the next stage, TMEM stage of the next k-block
        uint32_t rph = 0, tph = 0;
        int t = 0;                       // CTA-wide k-block index
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
            int tm, tn, sp, kb0, kb1;
            unit_coords(p, u, tm, tn, sp);
            unit_kblocks(p, sp, kb0, kb1);
            for (int kb = kb0; kb < kb1; kb += C::RK) {
                const int nk = min(C::RK, kb1 - kb);
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(&raw_full[rs], rph, abort_flag))) { ok = false; break; }
                // This warp's k-block in the stage: sub with (t + sub) % 4 == j (RK <= 4).
                const int sub = (j - t) & 3;
                if (sub < nk) {
                    int tk = ts + sub;
                    uint32_t tpk = tph;
                    if (tk >= C::TS) { tk -= C::TS; tpk ^= 1u; }
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(&t_empty[tk], tpk ^ 1u, abort_flag))) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t raw = sbase + C::OFF_R + rs * C::RSTAGE_BYTES;
                    const uint32_t ta = t_lane + static_cast<uint32_t>(tk * 32);
#pragma unroll
                    for (int h = 0; h < C::H; ++h) {
                        uint4 in[C::UPH];
#pragma unroll
                        for (int x = 0; x < C::UPH; ++x)
                            in[x] = lds128(raw_unit_addr<C::FMT>(raw, sub, row, h * C::UPH + x));
                        bool scalar = false;
                        if constexpr (C::FMT == kE4M3 || C::FMT == kBF16 || C::FMT == kTF32) {
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
                    // The raw words are consumed (decoded above): release the stage.
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[rs]);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&t_full[tk]);
                } else {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[rs]);
                }
                t += nk;
                ts += nk;
                if (ts >= C::TS) { ts -= C::TS; tph ^= 1u; }
                if (++rs == C::SR) { rs = 0; rph ^= 1u; }
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
