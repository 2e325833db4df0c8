// sharded.cu -- column-sharded (output-feature-sharded) weight GEMM with an
// NCCL all-gather of the output row blocks, overlapped block by block.
//
// Overlap needs SMs for both at once: the fused GEMM is persistent and its
// CTAs take about 225 KB of shared memory, so an all-gather kernel cannot
// share an SM with it.  The communicator is therefore created with at most
// kCommCtas CTAs per collective (ncclCommInitRankConfig, maxCTAs) and the
// sharded GEMM runs on the other SMs; the all-gather of block group c then
// proceeds beside the GEMM of block c + 1 instead of after it.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing a copy that
// is already loaded in the process), so the library itself does not link
// NCCL and loads on machines without it.
#include <dlfcn.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <cuda_runtime.h>
#include <nccl.h>
#include "tensor_bridge_b200.h"
#include "tb_host.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, []() {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        auto sym = [h](const char* n) { return dlsym(h, n); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_init_rank_config =
            reinterpret_cast<decltype(api.comm_init_rank_config)>(sym("ncclCommInitRankConfig"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
        api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(sym("ncclCommUserRank"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_count &&
                 api.comm_user_rank && api.all_gather;
    });
    return api;
}

// CTAs an NCCL collective of this library's communicators may use, and so the
// SMs the sharded GEMM leaves free for it.
constexpr int kCommCtas = 16;

tb_status nccl_fail(ncclResult_t r, const char* what) {
    const NcclApi& n = nccl();
    fprintf(stderr, "tensor_bridge_b200: %s failed: %s\n", what, n.error_string ? n.error_string(r) : "?");
    return TB_ERR_NCCL;
}

}  // namespace

extern "C" {

tb_status tb_nccl_unique_id(uint8_t id_out[128]) {
    const NcclApi& n = nccl();
    if (!n.ok) return TB_ERR_NCCL;
    if (!id_out) return TB_ERR_INVALID_ARGUMENT;
    ncclUniqueId id;
    ncclResult_t r = n.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(id) == 128, "ncclUniqueId size");
    std::memcpy(id_out, &id, sizeof id);
    return TB_OK;
}

tb_status tb_nccl_comm_init(void** comm_out, int world, int rank, const uint8_t id[128]) {
    const NcclApi& n = nccl();
    if (!n.ok) return TB_ERR_NCCL;
    if (!comm_out || !id || world <= 0 || rank < 0 || rank >= world) return TB_ERR_INVALID_ARGUMENT;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclComm_t c = nullptr;
    ncclResult_t r;
    if (n.comm_init_rank_config) {
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.maxCTAs = kCommCtas;
        r = n.comm_init_rank_config(&c, world, uid, rank, &cfg);
    } else {
        r = n.comm_init_rank(&c, world, uid, rank);
    }
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm_out = c;
    return TB_OK;
}

tb_status tb_nccl_comm_destroy(void* comm) {
    const NcclApi& n = nccl();
    if (!n.ok) return TB_ERR_NCCL;
    if (!comm) return TB_OK;
    ncclResult_t r = n.comm_destroy(static_cast<ncclComm_t>(comm));
    return r == ncclSuccess ? TB_OK : nccl_fail(r, "ncclCommDestroy");
}

tb_status tb_gemm_sharded_fused(tb_format a_fmt, const void* A_shard, const uint16_t* B, void* D, int M, int N, int K,
                                tb_out_type out, float alpha, void* comm, int chunks, tb_stream_t stream,
                                tb_stream_t comm_stream) {
    const NcclApi& n = nccl();
    if (!n.ok) return TB_ERR_NCCL;
    if (!comm || chunks <= 0 || !A_shard || !B || !D) return TB_ERR_INVALID_ARGUMENT;
    int world = 0, rank = 0;
    ncclResult_t nr = n.comm_count(static_cast<ncclComm_t>(comm), &world);
    if (nr != ncclSuccess) return nccl_fail(nr, "ncclCommCount");
    nr = n.comm_user_rank(static_cast<ncclComm_t>(comm), &rank);
    if (nr != ncclSuccess) return nccl_fail(nr, "ncclCommUserRank");
    if (M <= 0 || M % (world * chunks * 128) != 0) return TB_ERR_SHAPE;
    const int Mc = M / (world * chunks);
    const size_t elem = out == TB_OUT_F16 ? 2 : 4;
    const size_t block_elems = static_cast<size_t>(Mc) * N;
    const size_t a_block_bytes = tb::stored_bytes(a_fmt, static_cast<size_t>(Mc) * K);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TB_ERR_CUDA;
    const int sms = tb::device_info(dev).sms;

    cudaEvent_t done[64];
    if (chunks > 64) return TB_ERR_INVALID_ARGUMENT;
    for (int c = 0; c < chunks; ++c) {
        if (cudaEventCreateWithFlags(&done[c], cudaEventDisableTiming) != cudaSuccess) {
            for (int j = 0; j < c; ++j) cudaEventDestroy(done[j]);
            return TB_ERR_CUDA;
        }
    }
    tb_status st = TB_OK;
    for (int c = 0; c < chunks && st == TB_OK; ++c) {
        const size_t g0 = static_cast<size_t>(c * world + rank) * Mc;  // global first row of this block
        char* dblk = static_cast<char*>(D) + g0 * N * elem;
        const void* ablk = static_cast<const char*>(A_shard) + c * a_block_bytes;
        st = tb::gemm_fused_capped(a_fmt, ablk, B, dblk, Mc, N, K, out, alpha, sms - kCommCtas, stream);
        if (st != TB_OK) break;
        if (cudaEventRecord(done[c], stream) != cudaSuccess || cudaStreamWaitEvent(comm_stream, done[c], 0) != cudaSuccess) {
            st = TB_ERR_CUDA;
            break;
        }
        char* group = static_cast<char*>(D) + static_cast<size_t>(c) * world * block_elems * elem;
        nr = n.all_gather(dblk, group, block_elems, out == TB_OUT_F16 ? ncclFloat16 : ncclFloat32,
                          static_cast<ncclComm_t>(comm), comm_stream);
        if (nr != ncclSuccess) st = nccl_fail(nr, "ncclAllGather");
    }
    if (st == TB_OK) {
        // Make `stream` wait for the last all-gather so that one stream orders the result.
        if (cudaEventRecord(done[0], comm_stream) != cudaSuccess || cudaStreamWaitEvent(stream, done[0], 0) != cudaSuccess)
            st = TB_ERR_CUDA;
    }
    for (int c = 0; c < chunks; ++c) cudaEventDestroy(done[c]);
    return st;
}

}  // extern "C"
