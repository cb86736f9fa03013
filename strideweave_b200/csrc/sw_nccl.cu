// sw_nccl.cu - the collectives of a sharded contraction behind the C ABI, for
// hosts that drive the carrier without torch.distributed: a communicator per
// rank from a 128-byte id that rank 0 creates and the host distributes, and
// Float32 reduce-scatter / all-gather on a stream.
//
// NCCL is loaded at first use (dlopen of libnccl.so.2, which resolves to a
// copy the process already loaded when there is one), so the library itself
// has no link-time dependency on it; every entry point reports a missing
// NCCL as SW_ERR_UNSUPPORTED.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "sw_common.cuh"

namespace sw {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                   cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.reduce_scatter && api.all_gather &&
                 api.comm_destroy && api.error_string;
    });
    return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
    return fail(SW_ERR_CUDA, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

#define SW_NCCL_READY(what)                                                                   \
    do {                                                                                      \
        if (!::sw::nccl().ok) return ::sw::fail(SW_ERR_UNSUPPORTED, "%s: libnccl.so.2 is not available", what); \
    } while (0)

}  // namespace
}  // namespace sw

extern "C" int sw_nccl_get_unique_id(uint8_t* id) {
    using namespace sw;
    if (!id) return fail(SW_ERR_INVALID, "sw_nccl_get_unique_id: null output");
    SW_NCCL_READY("sw_nccl_get_unique_id");
    ncclUniqueId u;
    const ncclResult_t r = nccl().get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(u.internal) == SW_NCCL_ID_BYTES, "NCCL id size");
    for (int i = 0; i < SW_NCCL_ID_BYTES; ++i) id[i] = uint8_t(u.internal[i]);
    return ok();
}

extern "C" int sw_nccl_comm_init(void** comm, int world, int rank, const uint8_t* id) {
    using namespace sw;
    if (!comm || !id) return fail(SW_ERR_INVALID, "sw_nccl_comm_init: null argument");
    if (world < 1 || rank < 0 || rank >= world) return fail(SW_ERR_INVALID, "sw_nccl_comm_init: bad rank / world");
    SW_NCCL_READY("sw_nccl_comm_init");
    ncclUniqueId u;
    for (int i = 0; i < SW_NCCL_ID_BYTES; ++i) u.internal[i] = char(id[i]);
    ncclComm_t c = nullptr;
    const ncclResult_t r = nccl().comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    *comm = (void*)c;
    return ok();
}

extern "C" int sw_nccl_reduce_scatter_f32(const float* send, float* recv, int64_t recv_count, void* comm,
                                          void* stream) {
    using namespace sw;
    if (!comm || recv_count < 0) return fail(SW_ERR_INVALID, "sw_nccl_reduce_scatter_f32: bad argument");
    if (recv_count == 0) return ok();
    if (!send || !recv) return fail(SW_ERR_INVALID, "sw_nccl_reduce_scatter_f32: null buffer");
    SW_NCCL_READY("sw_nccl_reduce_scatter_f32");
    const ncclResult_t r = nccl().reduce_scatter(send, recv, size_t(recv_count), ncclFloat32, ncclSum,
                                                 (ncclComm_t)comm, (cudaStream_t)stream);
    if (r != ncclSuccess) return nccl_fail(r, "ncclReduceScatter");
    return ok();
}

extern "C" int sw_nccl_all_gather_f32(const float* send, float* recv, int64_t send_count, void* comm,
                                      void* stream) {
    using namespace sw;
    if (!comm || send_count < 0) return fail(SW_ERR_INVALID, "sw_nccl_all_gather_f32: bad argument");
    if (send_count == 0) return ok();
    if (!send || !recv) return fail(SW_ERR_INVALID, "sw_nccl_all_gather_f32: null buffer");
    SW_NCCL_READY("sw_nccl_all_gather_f32");
    const ncclResult_t r = nccl().all_gather(send, recv, size_t(send_count), ncclFloat32, (ncclComm_t)comm,
                                             (cudaStream_t)stream);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    return ok();
}

extern "C" int sw_nccl_comm_destroy(void* comm) {
    using namespace sw;
    if (!comm) return ok();
    SW_NCCL_READY("sw_nccl_comm_destroy");
    const ncclResult_t r = nccl().comm_destroy((ncclComm_t)comm);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
    return ok();
}
