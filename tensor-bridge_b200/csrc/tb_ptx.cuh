// tb_ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers with bounded
// waits, TMA tile loads, tcgen05 (TMEM alloc, MMA, commit, loads) and the
// shared-memory descriptor / instruction descriptor encodings used by the GEMMs.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace tb {

// Error codes written to the device error word.
enum : int { kErrTimeout = 1 };

// Device error word.  Set with atomicOr when a bounded wait expires; read by
// tb_device_error().  Without relocatable device code every translation unit
// has its own copy; only gemm.cu launches kernels that wait, and gemm.cu
// hosts the reader (device_error_read / device_error_clear).
static __device__ int g_tb_device_error = 0;

// Upper bound of any single mbarrier wait (ns).  Pipeline waits in these
// kernels last microseconds; two seconds means something is broken.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier -----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Arrive `count` times at once.
__device__ __forceinline__ void mbar_arrive_count(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait until the phase with the given parity has completed.  Bounded: gives up
// after kWaitLimitNs or as soon as *abort is set by another role, sets the
// device error word and *abort, and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(a, parity)) return true;
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

// Bounded wait that ignores the abort flag, used on the abort path to let
// asynchronous work that was already issued finish (at most 100 ms).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(a, parity)) {
        if (globaltimer() - t0 > 100000000ull) return;
    }
}

// One lane of the (converged) warp returns true.  Lets a whole warp run an
// issue loop with warp-uniform values (kept in the uniform datapath) while a
// single thread issues the TMA / tcgen05 instructions.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---- clusters of two CTAs (tcgen05 cta_group::2) --------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// All threads of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Make mbarrier initialisation visible to the other CTA of the cluster.
__device__ __forceinline__ void fence_mbarrier_init_cluster() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Shared::cluster address of the mbarrier at `bar`'s offset in cluster CTA 0.
__device__ __forceinline__ uint32_t leader_bar(const uint64_t* bar) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(smem_addr(bar)));
    return remote;
}

// TMA 2D tile load into this CTA's shared memory whose completion is counted
// on the mbarrier at `bar_cluster` (a shared::cluster address; cta_group::2
// lets it be the pair's leader's barrier).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}

// Arrive on the mbarrier at the same offset in cluster CTA `rank`.
__device__ __forceinline__ void mbar_arrive_cluster(const uint64_t* bar, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(bar)), "r"(rank));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

// Shared::cluster address of `p` (this CTA's shared memory) in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(p)), "r"(rank));
    return remote;
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from
// this CTA's shared memory to shared memory of a CTA of the cluster; its
// completion is counted (complete_tx) on the mbarrier at `bar_cluster` there.
// Issued through the async proxy: a cheap way to signal another CTA's
// barrier after a proxy fence, without a cluster-scope release.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                                     uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst_cluster),
        "r"(smem_addr(src)), "r"(bytes), "r"(bar_cluster)
        : "memory");
}

// TMEM allocation shared by the two CTAs: one warp with the same warp index
// in each CTA executes it.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Pair MMAs (issued by the leader CTA): M = 256 rows, 128 from each CTA's A
// tile, N from both CTAs' B halves, D in each CTA's TMEM for its rows.
template <int KIND>  // 0: kind::f16, 1: kind::f8f6f4, 2: kind::i8
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    if constexpr (KIND == 0)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else if constexpr (KIND == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
}

// Arrive on the mbarrier at `bar`'s offset in the CTAs of `cta_mask` once all
// pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void mma_commit_pair(const uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_addr(bar)),
        "h"(cta_mask)
        : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------------

// Wait until the grids this one depends on (the previous kernel in the
// stream, when this one was launched with programmatic stream serialisation)
// have completed and their memory operations are visible.  Returns at once
// otherwise.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Let the next kernel in the stream (if launched with programmatic stream
// serialisation) be scheduled before this grid completes.
__device__ __forceinline__ void grid_dep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- named (hardware) CTA barriers ---------------------------------------------------

// Wait at named barrier `id` until `count` threads (a multiple of 32, whole
// warps) have arrived or waited on it.  Unlike an mbarrier wait this cannot
// time out: every participant must reach it the same number of times.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Arrive at named barrier `id` without waiting.
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- proxy fences ---------------------------------------------------------------

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tcgen05.mma operands, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA -------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of the box at (x = inner coordinate, y = outer coordinate)
// into shared memory, completing `bytes` on the mbarrier.  Caller guarantees
// x * element_size is a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// L2 policy that marks lines evict-first (data read once, e.g. streamed weights).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// tma_load_2d with an L2 cache-policy hint.
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// ---- tcgen05 ---------------------------------------------------------------------

// Allocate `ncols` TMEM columns (power of two >= 32); whole warp executes.
// The TMEM base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (FP16/BF16 inputs).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Same for kind::f8f6f4 (FP8 / FP6 / FP4 inputs, per-tensor scaling only).
__device__ __forceinline__ void mma_f8f6f4_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8: signed 8-bit operands, S32
// accumulation (exact), K = 32 per instruction.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16: the A operand is read from
// tensor memory (M = 128 rows in the 128 lanes, K = 16 values in 8 columns
// starting at a_tmem, two FP16 values per 32-bit column, lower K in the low
// half).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Store 16 consecutive 32-bit TMEM columns of this warp's 32 lanes: thread t
// writes lane (base lane + t), columns [col, col + 16).  Asynchronous; see
// tmem_wait_st.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// 32-column variant.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// 4-column variant.
__device__ __forceinline__ void tmem_st_32x32b_x4(uint32_t taddr, const uint32_t (&v)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3])
                 : "memory");
}

// 8-column variant.
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(v[0]),
        "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}

// Wait until this thread's tcgen05.st stores have completed.
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05 MMAs of this
// thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// Load 32 consecutive 32-bit TMEM columns of this warp's 32 lanes:
// thread t receives lane (base lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

// 16-column variant of the above (tiles narrower than 32 columns).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- descriptors -------------------------------------------------------------------

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte-swizzle canonical layout: rows of 128 bytes, groups of 8 rows
// 1024 bytes apart (stride byte offset), 16-byte chunks XOR-swizzled by the
// row index within the group.  The tile base must be 1024-byte aligned; a
// start address inside the first 128 bytes selects a K offset within the
// swizzle atom.  Bit layout (sm_100 UMMA descriptor): [0,14) start >> 4,
// [16,30) leading byte offset >> 4 (unused for swizzled K-major, set to 1),
// [32,46) stride byte offset >> 4, [46,48) version = 1, [61,64) layout = 2
// (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t smem_byte_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// The same descriptor split into its two 32-bit words: the low word holds the
// start address (>> 4) and the leading byte offset, so advancing the start by
// b bytes adds b >> 4 to it (shared addresses stay below 2^18, so the 14-bit
// field does not carry); the high word is the same for every K-major
// SWIZZLE_128B tile.
__host__ __device__ constexpr uint32_t sdesc_lo(uint32_t smem_byte_addr) {
    return ((smem_byte_addr >> 4) & 0x3FFFu) | (1u << 16);
}
constexpr uint32_t kSdescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint64_t sdesc_make(uint32_t lo) {
    return (static_cast<uint64_t>(kSdescHi) << 32) | lo;
}

// Instruction descriptor (kind::f16 / kind::f8f6f4, dense): D format F32,
// both operands K-major, shape M x N.  a_fmt/b_fmt: for kind::f16 0 = F16,
// 1 = BF16; for kind::f8f6f4 0 = E4M3, 1 = E5M2, 5 = E2M1.
// Instruction descriptor for kind::i8: D format S32 (2), both operands
// signed 8-bit (1), K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__host__ __device__ constexpr uint32_t idesc_make(uint32_t a_fmt, uint32_t b_fmt, int m, int n) {
    return (1u << 4)                                  // D = F32
           | (a_fmt << 7) | (b_fmt << 10)             // operand formats
           | (0u << 15) | (0u << 16)                  // K-major A and B
           | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

}  // namespace tb
