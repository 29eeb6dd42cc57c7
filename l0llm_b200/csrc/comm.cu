// Tensor-parallel communicator: NCCL over NVLink / NVSwitch, one process per GPU.
//
// NCCL is opened at run time (dlopen "libnccl.so.2") the first time a communicator is made, so the
// library has no link-time NCCL dependency and shares whichever libnccl the process already loaded
// (torch bundles one). Collectives go on the device stream like kernels; inside a command list they
// are recorded and captured into the CUDA graph with the kernels around them.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "runtime.h"

struct l0b_comm {
    ncclComm_t comm = nullptr;
    int nranks = 1;
    int rank = 0;
    l0b_device* dev = nullptr;
};

namespace l0b {

namespace {

struct NcclApi {
    void* handle = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_nccl_mu;

l0b_status nccl_load() {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.handle) return L0B_OK;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail(L0B_ERR_NCCL, "NCCL is not available: %s", dlerror());
    NcclApi a;
    a.handle = h;
    a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!a.get_unique_id || !a.comm_init_rank || !a.comm_destroy || !a.all_reduce || !a.all_gather || !a.error_string)
        return fail(L0B_ERR_NCCL, "libnccl.so.2 lacks an expected entry point");
    g_nccl = a;
    return L0B_OK;
}

ncclDataType_t nccl_type(int dtype) {
    switch (dtype) {
        case L0B_F16: return ncclFloat16;
        case L0B_BF16: return ncclBfloat16;
        case L0B_I32: return ncclInt32;
        case kDtypeU64: return ncclUint64;
        default: return ncclFloat32;
    }
}

}  // namespace

l0b_status collective_issue(int kind, const CollArgs& a, cudaStream_t stream) {
    L0B_REQUIRE(g_nccl.handle, L0B_ERR_NCCL, "NCCL is not loaded");
    ncclResult_t r;
    if (kind == REC_ALLREDUCE)
        r = g_nccl.all_reduce(a.send, a.recv, a.count, nccl_type(a.dtype), a.op == COLL_MAX ? ncclMax : ncclSum,
                              static_cast<ncclComm_t>(a.comm), stream);
    else
        r = g_nccl.all_gather(a.send, a.recv, a.count, nccl_type(a.dtype), static_cast<ncclComm_t>(a.comm), stream);
    if (r != ncclSuccess) return fail(L0B_ERR_NCCL, "NCCL collective failed: %s", g_nccl.error_string(r));
    return L0B_OK;
}

l0b_status comm_allreduce(l0b_comm* c, void* buf, size_t count, int dtype, int op) {
    CollArgs a{buf, buf, count, dtype, op, c->comm};
    return c->dev->collective(REC_ALLREDUCE, a);
}

l0b_status comm_allgather(l0b_comm* c, const void* send, void* recv, size_t count, int dtype) {
    CollArgs a{send, recv, count, dtype, COLL_SUM, c->comm};
    return c->dev->collective(REC_ALLGATHER, a);
}

int comm_size(const l0b_comm* c) { return c ? c->nranks : 1; }
int comm_rank(const l0b_comm* c) { return c ? c->rank : 0; }

}  // namespace l0b

using namespace l0b;

L0B_API l0b_status l0b_comm_unique_id(uint8_t* id, int32_t bytes) {
    L0B_REQUIRE(id && bytes >= static_cast<int32_t>(sizeof(ncclUniqueId)), L0B_ERR_ARGUMENT,
                "the unique id needs %zu bytes", sizeof(ncclUniqueId));
    L0B_TRY(nccl_load());
    ncclUniqueId u;
    ncclResult_t r = g_nccl.get_unique_id(&u);
    if (r != ncclSuccess) return fail(L0B_ERR_NCCL, "ncclGetUniqueId failed: %s", g_nccl.error_string(r));
    std::memcpy(id, &u, sizeof(u));
    return L0B_OK;
}

L0B_API l0b_status l0b_comm_create(l0b_device* dev, const uint8_t* id, int32_t bytes, int32_t nranks, int32_t rank,
                                   l0b_comm** out) {
    L0B_REQUIRE(dev && id && out, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(bytes >= static_cast<int32_t>(sizeof(ncclUniqueId)), L0B_ERR_ARGUMENT, "short unique id");
    L0B_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, L0B_ERR_OUT_OF_RANGE, "rank %d of %d", rank, nranks);
    *out = nullptr;
    L0B_TRY(nccl_load());
    L0B_CHECK_CUDA(cudaSetDevice(dev->index));
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    l0b_comm* c = new l0b_comm();
    c->nranks = nranks;
    c->rank = rank;
    c->dev = dev;
    ncclResult_t r = g_nccl.comm_init_rank(&c->comm, nranks, u, rank);
    if (r != ncclSuccess) {
        delete c;
        return fail(L0B_ERR_NCCL, "ncclCommInitRank failed: %s", g_nccl.error_string(r));
    }
    // One small all-reduce and all-gather outside any stream capture, waited for: NCCL sets up its
    // connections on first use, which must not happen inside the capture of a command list.
    void* scratch = nullptr;
    cudaError_t e = cudaMalloc(&scratch, 64 * sizeof(float) * (nranks + 1));
    if (e == cudaSuccess) {
        float* f = static_cast<float*>(scratch);
        cudaMemsetAsync(f, 0, 64 * sizeof(float) * (nranks + 1), dev->stream);
        r = g_nccl.all_reduce(f, f, 64, ncclFloat32, ncclSum, c->comm, dev->stream);
        if (r == ncclSuccess) r = g_nccl.all_gather(f, f + 64, 64, ncclFloat32, c->comm, dev->stream);
        if (r == ncclSuccess) r = g_nccl.all_reduce(f, f, 32, ncclUint64, ncclMax, c->comm, dev->stream);
        e = cudaStreamSynchronize(dev->stream);
        cudaFree(scratch);
    }
    if (e != cudaSuccess || r != ncclSuccess) {
        g_nccl.comm_destroy(c->comm);
        delete c;
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "communicator warm-up failed: %s", cudaGetErrorString(e));
        return fail(L0B_ERR_NCCL, "communicator warm-up failed: %s", g_nccl.error_string(r));
    }
    *out = c;
    return L0B_OK;
}

L0B_API l0b_status l0b_comm_free(l0b_comm* c) {
    if (!c) return L0B_OK;
    if (c->comm && g_nccl.handle) {
        cudaSetDevice(c->dev->index);
        // Captured collectives keep the communicator busy: release the device's graphs first.
        c->dev->drop_graphs();
        g_nccl.comm_destroy(c->comm);
    }
    delete c;
    return L0B_OK;
}

L0B_API l0b_status l0b_comm_allreduce(l0b_comm* c, l0b_buffer* buf, int64_t count) {
    L0B_REQUIRE(c && buf, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(count >= 0 && count <= buf->count, L0B_ERR_OUT_OF_RANGE, "count %lld of %lld", (long long)count,
                (long long)buf->count);
    L0B_REQUIRE(buf->dev == c->dev, L0B_ERR_ARGUMENT, "the buffer lives on another device");
    L0B_CHECK_CUDA(cudaSetDevice(c->dev->index));
    return comm_allreduce(c, buf->ptr, static_cast<size_t>(count), buf->dtype, COLL_SUM);
}
