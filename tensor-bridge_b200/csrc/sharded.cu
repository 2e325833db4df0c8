// sharded.cu -- column-sharded (output-feature-sharded) weight GEMM whose
// output row blocks reach every rank either by an NCCL all-gather per block
// group (tb_gemm_sharded_fused) or by the fused kernel's own epilogue, which
// stores each finished tile into the peers' copies of D through CUDA IPC
// mappings (tb_gemm_sharded_fused_p2p).  The second needs no SMs beyond the
// GEMM's: an NCCL kernel cannot share an SM with the persistent fused kernel
// (~225 KB of shared memory per CTA), so the all-gathers mostly run after the
// block GEMMs, while the epilogue's stores overlap the next tile's MMAs.
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
#include <vector>
#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>
#include "tensor_bridge_b200.h"
#include "tb_host.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
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
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
        api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(sym("ncclCommUserRank"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_count &&
                 api.comm_user_rank && api.all_gather && api.all_reduce;
    });
    return api;
}

tb_status nccl_fail(ncclResult_t r, const char* what) {
    const NcclApi& n = nccl();
    fprintf(stderr, "tensor_bridge_b200: %s failed: %s\n", what, n.error_string ? n.error_string(r) : "?");
    return TB_ERR_NCCL;
}

tb_status cuda_fail(cudaError_t e, const char* what) {
    return tb::set_last_error(TB_ERR_CUDA, what, cudaGetErrorString(e));
}

// ---- peer buffers (CUDA IPC) -----------------------------------------------------

constexpr int kMaxRanks = tb::kMaxPeers + 1;

// What each rank tells the others about its buffer at registration.
struct PeerRecord {
    cudaIpcMemHandle_t handle;  // of the allocation holding the buffer
    uint64_t offset;            // buffer start - allocation base
    uint64_t bytes;             // 0: this rank could not export its buffer
    uint64_t addr;              // buffer address in its owner (alignment check)
    uint8_t pad[40];
};
static_assert(sizeof(PeerRecord) == 128, "peer record size");

struct PeerBuffer {
    ncclComm_t comm;
    int world, rank;
    char* local;
    size_t bytes;
    char* peer[kMaxRanks];    // rank r's buffer as mapped here (local for r == rank)
    void* opened[kMaxRanks];  // allocation bases opened by IPC, closed at release
    int* word;                // device word the barrier all-reduces
};

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
    static AddressRangeFn fn = []() -> AddressRangeFn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<AddressRangeFn>(p);
    }();
    return fn;
}

// Every rank reaches this point of `stream` before any passes it: a one-word
// max all-reduce (the word stays 0).
tb_status barrier(const PeerBuffer& pb, cudaStream_t stream) {
    const ncclResult_t r = nccl().all_reduce(pb.word, pb.word, 1, ncclInt32, ncclMax, pb.comm, stream);
    return r == ncclSuccess ? TB_OK : nccl_fail(r, "ncclAllReduce (barrier)");
}

// Sum of `v` over all ranks (host value; synchronises `stream`).
tb_status all_sum(const PeerBuffer& pb, int v, cudaStream_t stream, int* out) {
    cudaError_t e = cudaMemcpyAsync(pb.word + 1, &v, sizeof v, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync");
    const ncclResult_t r = nccl().all_reduce(pb.word + 1, pb.word + 1, 1, ncclInt32, ncclSum, pb.comm, stream);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    e = cudaMemcpyAsync(out, pb.word + 1, sizeof *out, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaStreamSynchronize");
}

void close_peers(PeerBuffer* pb) {
    for (int r = 0; r < pb->world; ++r)
        if (pb->opened[r]) cudaIpcCloseMemHandle(pb->opened[r]);
    if (pb->word) cudaFree(pb->word);
    delete pb;
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
    ncclResult_t r = n.comm_init_rank(&c, world, uid, rank);
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
        st = tb_gemm_fused(a_fmt, ablk, B, dblk, Mc, N, K, out, alpha, nullptr, 0, stream);
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

tb_status tb_peer_buffer_register(void* comm, void* buf, size_t bytes, tb_stream_t stream, void** peer_buffer_out) {
    const NcclApi& n = nccl();
    if (!n.ok) return TB_ERR_NCCL;
    if (!comm || !peer_buffer_out) return tb::set_last_error(TB_ERR_INVALID_ARGUMENT, "null argument", "");
    *peer_buffer_out = nullptr;
    int world = 0, rank = 0;
    ncclResult_t nr = n.comm_count(static_cast<ncclComm_t>(comm), &world);
    if (nr != ncclSuccess) return nccl_fail(nr, "ncclCommCount");
    nr = n.comm_user_rank(static_cast<ncclComm_t>(comm), &rank);
    if (nr != ncclSuccess) return nccl_fail(nr, "ncclCommUserRank");
    // Every rank knows world, so this rejection is the same on all of them.
    if (world > kMaxRanks) return tb::set_last_error(TB_ERR_INVALID_ARGUMENT, "peer buffers span at most 8 ranks", "");

    PeerBuffer* pb = new PeerBuffer{};
    pb->comm = static_cast<ncclComm_t>(comm);
    pb->world = world;
    pb->rank = rank;
    pb->local = static_cast<char*>(buf);
    pb->bytes = bytes;
    // Word 0: the barrier's; word 1: all_sum's; then world records + this rank's.
    char* dev = nullptr;
    const size_t rec_off = 256;
    cudaError_t e = cudaMalloc(&dev, rec_off + (world + 1) * sizeof(PeerRecord));
    if (e != cudaSuccess) {
        delete pb;
        return cuda_fail(e, "cudaMalloc");
    }
    pb->word = reinterpret_cast<int*>(dev);
    e = cudaMemsetAsync(dev, 0, rec_off, stream);
    if (e != cudaSuccess) {
        close_peers(pb);
        return cuda_fail(e, "cudaMemsetAsync");
    }

    // This rank's record; a buffer that cannot be exported is reported to
    // the others (bytes = 0) instead of failing alone.
    PeerRecord mine{};
    AddressRangeFn range = address_range_fn();
    CUdeviceptr base = 0;
    size_t alloc_bytes = 0;
    if (buf && bytes > 0 && range &&
        range(&base, &alloc_bytes, reinterpret_cast<CUdeviceptr>(buf)) == CUDA_SUCCESS &&
        reinterpret_cast<uintptr_t>(buf) + bytes <= base + alloc_bytes &&
        cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void*>(base)) == cudaSuccess) {
        mine.offset = reinterpret_cast<uintptr_t>(buf) - base;
        mine.bytes = bytes;
        mine.addr = reinterpret_cast<uintptr_t>(buf);
    }
    cudaGetLastError();  // a failed export above is reported through the record
    std::vector<PeerRecord> recs(world);
    char* drecs = dev + rec_off;
    e = cudaMemcpyAsync(drecs + world * sizeof(PeerRecord), &mine, sizeof mine, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) {
        close_peers(pb);
        return cuda_fail(e, "cudaMemcpyAsync");
    }
    nr = n.all_gather(drecs + world * sizeof(PeerRecord), drecs, sizeof(PeerRecord), ncclUint8, pb->comm, stream);
    if (nr != ncclSuccess) {
        close_peers(pb);
        return nccl_fail(nr, "ncclAllGather (peer records)");
    }
    e = cudaMemcpyAsync(recs.data(), drecs, world * sizeof(PeerRecord), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        close_peers(pb);
        return cuda_fail(e, "peer record exchange");
    }
    for (int r = 0; r < world; ++r) {
        if (recs[r].bytes == 0 || recs[r].bytes != bytes || (recs[r].addr & 15u) != 0) {
            close_peers(pb);
            return tb::set_last_error(TB_ERR_INVALID_ARGUMENT, "peer buffer registration",
                                      "every rank needs a 16-byte aligned cudaMalloc buffer of the same size");
        }
    }
    int failed = 0;
    for (int r = 0; r < world; ++r) {
        if (r == rank) {
            pb->peer[r] = pb->local;
            continue;
        }
        void* opened = nullptr;
        if (cudaIpcOpenMemHandle(&opened, recs[r].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            failed = 1;
            continue;
        }
        pb->opened[r] = opened;
        pb->peer[r] = static_cast<char*>(opened) + recs[r].offset;
    }
    // Agree on the outcome, so that no rank goes on with a partial mapping.
    int failures = 0;
    const tb_status st = all_sum(*pb, failed, stream, &failures);
    if (st != TB_OK || failures != 0) {
        close_peers(pb);
        return st != TB_OK ? st
                           : tb::set_last_error(TB_ERR_CUDA, "cudaIpcOpenMemHandle failed on a rank",
                                                "peer buffers need one process per GPU with peer access");
    }
    *peer_buffer_out = pb;
    return TB_OK;
}

tb_status tb_peer_buffer_release(void* peer_buffer, tb_stream_t stream) {
    if (!peer_buffer) return TB_OK;
    if (!nccl().ok) return TB_ERR_NCCL;
    PeerBuffer* pb = static_cast<PeerBuffer*>(peer_buffer);
    tb_status st = barrier(*pb, stream);
    if (st == TB_OK) {
        const cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) st = cuda_fail(e, "cudaStreamSynchronize");
    }
    close_peers(pb);
    return st;
}

tb_status tb_gemm_sharded_fused_p2p(tb_format a_fmt, const void* A_shard, const uint16_t* B, void* peer_buffer,
                                    int M, int N, int K, tb_out_type out, float alpha, int chunks,
                                    tb_stream_t stream) {
    const NcclApi& n = nccl();
    if (!n.ok) return TB_ERR_NCCL;
    if (!peer_buffer || chunks <= 0 || !A_shard || !B)
        return tb::set_last_error(TB_ERR_INVALID_ARGUMENT, "null argument or chunks <= 0", "");
    const PeerBuffer& pb = *static_cast<const PeerBuffer*>(peer_buffer);
    const int world = pb.world, rank = pb.rank;
    if (M <= 0 || N <= 0 || M % (world * chunks * 128) != 0)
        return tb::set_last_error(TB_ERR_SHAPE, "M must be a positive multiple of world * chunks * 128", "");
    if (out != TB_OUT_F16 && out != TB_OUT_F32) return tb::set_last_error(TB_ERR_INVALID_ARGUMENT, "bad output type", "");
    const int Mc = M / (world * chunks);
    const size_t elem = out == TB_OUT_F16 ? 2 : 4;
    if (static_cast<size_t>(M) * N * elem > pb.bytes)
        return tb::set_last_error(TB_ERR_INVALID_ARGUMENT, "D [M x N] does not fit the registered buffer", "");
    const size_t a_block_bytes = tb::stored_bytes(a_fmt, static_cast<size_t>(Mc) * K);

    tb_status st = barrier(pb, stream);
    for (int c = 0; c < chunks && st == TB_OK; ++c) {
        const size_t off = static_cast<size_t>(c * world + rank) * Mc * N * elem;  // this block's place in D
        // Peers in the order rank + 1, rank + 2, ...: at any moment the ranks'
        // epilogues store to different GPUs rather than all to the same one.
        void* peers[tb::kMaxPeers];
        int np = 0;
        for (int i = 1; i < world; ++i) peers[np++] = pb.peer[(rank + i) % world] + off;
        const void* ablk = static_cast<const char*>(A_shard) + c * a_block_bytes;
        st = tb::gemm_fused_to_peers(a_fmt, ablk, B, pb.local + off, Mc, N, K, out, alpha, np, peers, stream);
    }
    // Every rank runs the closing barrier, also after a failed launch, so
    // that the ranks' collectives on `comm` stay matched.
    const tb_status st2 = barrier(pb, stream);
    return st != TB_OK ? st : st2;
}

}  // extern "C"
