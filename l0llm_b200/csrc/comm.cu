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
#include <vector>

#include "common.cuh"
#include "gemv.cuh"
#include "runtime.h"

// Peer all-reduce (small collectives of the decode step): every rank owns a mailbox in its HBM, mapped
// into every other rank's address space by CUDA IPC. A mailbox holds three regions:
// 1. the u64 max all-reduce (the vocab-split argmax keys):
//   data  [2 parities][kMaxRanks][slot_floats]   partials written by the ranks (peer stores over NVLink)
//   flags [2 parities][kMaxRanks][kPeerCtas]     epoch of the partial a rank's CTA has published here
//   epoch [kPeerCtas]                            this rank's own count of all-reduces, per CTA
// 2. the peer-sum region of the row-split GEMV epilogue (layout in gemv.cuh);
// 3. the tagged f32 sum all-reduce (kLLBytes, below).
constexpr int kMaxRanks = 8;
constexpr int kPeerCtas = 32;
constexpr int kPeerChunkBytes = 8192;  // bytes per chunk; chunk j is always handled by CTA j % kPeerCtas
constexpr size_t kPeerSlotFloats = size_t(1) << 19;  // 2 MB per partial: 64 rows of 8192

struct l0b_comm {
    ncclComm_t comm = nullptr;
    int nranks = 1;
    int rank = 0;
    l0b_device* dev = nullptr;
    char* mbox = nullptr;                  // own mailbox
    char* peer_mbox[kMaxRanks] = {};       // every rank's mailbox in this process's address space
    bool peer = false;                     // peer all-reduce available
    l0b::PeerSum* peer_sum = nullptr;      // device copy of the peer-sum mailboxes (GEMV all-reduce epilogue)
    size_t ll_off = 0;                     // tagged f32 all-reduce region in every mailbox
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
bool g_peer_disabled = false;  // l0b_comm_set_peer_allreduce(0): every collective on NCCL
bool g_peer_sum = true;        // l0b_comm_set_fused_allreduce: row-split GEMVs sum over peers in their epilogue

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

// ---------------------------------------------------------------------------------------------
// One-shot all-reduce over peer memory. The buffer is cut into chunks of kPeerChunkBytes and chunk j
// always belongs to CTA j % kPeerCtas, whatever the count and type (the grid is min(kPeerCtas, chunks)
// CTAs). CTA c of every rank writes its chunks into its slot of every rank's mailbox (parity = the CTA's
// epoch & 1), makes the stores visible system-wide, publishes the epoch in each rank's flag for
// (itself, c), waits -- bounded -- until every rank's flag for c in its own mailbox holds the epoch, and
// sums the slots in rank order, so every rank gets the same bits. Every mailbox byte is only ever
// handled by the same CTA index, whose epoch advances by one per call that reaches it: a rank can start
// CTA c's next call only after finishing its current one, which needs every rank's partial of it, and a
// peer publishes that only after its own previous call (stream order), so the two parities cover the
// rank that is one call ahead. All ranks make the same sequence of calls with the same counts, so their
// per-CTA epochs agree.
// ---------------------------------------------------------------------------------------------
struct PeerArgs {
    void* buf;
    long long count;
    char* mbox[kMaxRanks];
    int nranks, rank;
    int* error;
    size_t ll_off;  // offset of the tagged f32 region in every mailbox
};

// Tagged f32 region (the f32 sums): data [2 parities][kMaxRanks][kLLSlotElems] 64-bit words (epoch << 32 |
// f32 bits), then one epoch per CTA index. A value and its tag travel in one 64-bit store, so a reader
// that sees the call's tag has the value: no fence, no separate flag.
constexpr long long kLLSlotElems = 1LL << 17;
constexpr int kLLChunk = 1024;  // elements per chunk; chunk j always belongs to CTA j % kPeerCtas
constexpr size_t kLLBytes = 2ull * kMaxRanks * kLLSlotElems * 8 + kPeerCtas * sizeof(unsigned);

__device__ __forceinline__ unsigned peer_ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void peer_st_release(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <typename T, bool MAX>
__global__ void __launch_bounds__(512) peer_allreduce_kernel(const PeerArgs a) {
    pdl_wait();
    const int c = blockIdx.x, n = a.nranks;
    constexpr long long CH = kPeerChunkBytes / sizeof(T);        // elements per chunk
    const long long stride = static_cast<long long>(gridDim.x) * CH;  // gridDim.x == kPeerCtas past 32 chunks
    char* mine = a.mbox[a.rank];
    const size_t data_bytes = 2ull * kMaxRanks * kPeerSlotFloats * sizeof(float);
    unsigned* epoch_p = reinterpret_cast<unsigned*>(mine + data_bytes + 2ull * kMaxRanks * kPeerCtas * sizeof(unsigned)) + c;
    __shared__ unsigned ep_s;
    if (threadIdx.x == 0) ep_s = *epoch_p + 1;
    __syncthreads();
    const unsigned ep = ep_s;
    const int par = ep & 1;
    T* buf = static_cast<T*>(a.buf);
    auto slot = [&](char* mb, int src) {
        return reinterpret_cast<T*>(mb + (static_cast<size_t>(par) * kMaxRanks + src) * kPeerSlotFloats * sizeof(float));
    };
    auto flag = [&](char* mb, int src) {
        return reinterpret_cast<unsigned*>(mb + data_bytes) + (static_cast<size_t>(par) * kMaxRanks + src) * kPeerCtas + c;
    };
    // 1. This rank's slice into its slot of every rank's mailbox.
    for (long long lo = c * CH; lo < a.count; lo += stride) {
        const long long hi = min(a.count, lo + CH);
        for (int r = 0; r < n; ++r) {
            T* dst = slot(a.mbox[r], a.rank);
            for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = buf[i];
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < n) peer_st_release(flag(a.mbox[threadIdx.x], a.rank), ep);
    // 2. Every rank's slice has arrived here (bounded wait: ~2 s, then the device error flag).
    if (threadIdx.x < n) {
        const unsigned* f = flag(mine, threadIdx.x);
        const long long t0 = clock64();
        while (peer_ld_acquire(f) != ep) {
            if (clock64() - t0 > 4000000000LL) {
                if (a.error) atomicExch(a.error, 1);
                break;
            }
        }
    }
    __syncthreads();
    // 3. Sum in rank order (identical on every rank). The slots were written by other GPUs: read them at
    // L2 (ld.cg), past any line this SM's L1 kept from the same parity two calls ago.
    for (long long lo = c * CH; lo < a.count; lo += stride) {
        const long long hi = min(a.count, lo + CH);
        for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            T v = __ldcg(slot(mine, 0) + i);
            for (int r = 1; r < n; ++r) {
                const T w = __ldcg(slot(mine, r) + i);
                if constexpr (MAX) v = w > v ? w : v;
                else v += w;
            }
            buf[i] = v;
        }
    }
    if (threadIdx.x == 0) *epoch_p = ep;
}

// f32 sum over peer memory with tagged values: CTA c owns chunks c, c + grid, ... of kLLChunk elements;
// each thread sends its elements to every rank tagged with the CTA's epoch, then reads every rank's
// copy of them from its own mailbox as they arrive (bounded wait, then the error flag) and sums them in
// rank order -- the same bits on every rank. Parities and per-CTA epochs as in peer_allreduce_kernel.
__global__ void __launch_bounds__(512) peer_allreduce_ll_kernel(const PeerArgs a) {
    pdl_wait();
    const int c = blockIdx.x, n = a.nranks;
    const long long stride = static_cast<long long>(gridDim.x) * kLLChunk;
    char* mine = a.mbox[a.rank] + a.ll_off;
    unsigned* epoch_p = reinterpret_cast<unsigned*>(mine + 2ull * kMaxRanks * kLLSlotElems * 8) + c;
    const unsigned ep = *reinterpret_cast<volatile unsigned*>(epoch_p) + 1;
    const int par = ep & 1;
    float* buf = static_cast<float*>(a.buf);
    auto slot = [&](char* region, int src) {
        return reinterpret_cast<unsigned long long*>(region) + (static_cast<long long>(par) * kMaxRanks + src) * kLLSlotElems;
    };
    for (long long lo = c * static_cast<long long>(kLLChunk); lo < a.count; lo += stride) {
        const long long hi = min(a.count, lo + kLLChunk);
        for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const unsigned long long w = (static_cast<unsigned long long>(ep) << 32) | __float_as_uint(buf[i]);
            for (int r = 0; r < n; ++r) {
                unsigned long long* dst = slot(a.mbox[r] + a.ll_off, a.rank) + i;
                asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
            }
        }
    }
    const long long t0 = clock64();
    bool late = false;
    for (long long lo = c * static_cast<long long>(kLLChunk); lo < a.count; lo += stride) {
        const long long hi = min(a.count, lo + kLLChunk);
        for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            float v = 0.f;
            for (int r = 0; r < n; ++r) {
                const unsigned long long* q = slot(mine, r) + i;
                unsigned long long w;
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(q) : "memory");
                while (static_cast<unsigned>(w >> 32) != ep && !late) {
                    if (clock64() - t0 > 4000000000LL) {
                        late = true;
                        if (a.error) atomicExch(a.error, 1);
                    }
                    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(q) : "memory");
                }
                const float x = __uint_as_float(static_cast<unsigned>(w));
                v = r == 0 ? x : v + x;
            }
            buf[i] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *epoch_p = ep;
}

l0b_status comm_allreduce(l0b_comm* c, void* buf, size_t count, int dtype, int op) {
    if (c->peer && dtype == L0B_F32 && op == COLL_SUM && static_cast<long long>(count) <= kLLSlotElems) {
        PeerArgs a{};
        a.buf = buf;
        a.count = static_cast<long long>(count);
        for (int r = 0; r < c->nranks; ++r) a.mbox[r] = c->peer_mbox[r];
        a.nranks = c->nranks;
        a.rank = c->rank;
        a.error = c->dev->error_flag;
        a.ll_off = c->ll_off;
        long long ctas = (static_cast<long long>(count) + kLLChunk - 1) / kLLChunk;
        if (ctas > kPeerCtas) ctas = kPeerCtas;
        if (ctas < 1) ctas = 1;
        return c->dev->launch(peer_allreduce_ll_kernel, dim3(static_cast<unsigned>(ctas)), dim3(512), 0, a);
    }
    const size_t esize = dtype == kDtypeU64 ? 8 : 4;
    const bool fits = count * esize <= kPeerSlotFloats * sizeof(float);
    if (c->peer && fits && ((dtype == L0B_F32 && op == COLL_SUM) || (dtype == kDtypeU64 && op == COLL_MAX))) {
        PeerArgs a{};
        a.buf = buf;
        a.count = static_cast<long long>(count);
        for (int r = 0; r < c->nranks; ++r) a.mbox[r] = c->peer_mbox[r];
        a.nranks = c->nranks;
        a.rank = c->rank;
        a.error = c->dev->error_flag;
        const long long ch = kPeerChunkBytes / static_cast<long long>(esize);
        long long ctas = (static_cast<long long>(count) + ch - 1) / ch;
        if (ctas > kPeerCtas) ctas = kPeerCtas;
        if (ctas < 1) ctas = 1;
        if (dtype == kDtypeU64)
            return c->dev->launch(peer_allreduce_kernel<unsigned long long, true>, dim3(static_cast<unsigned>(ctas)),
                                  dim3(512), 0, a);
        return c->dev->launch(peer_allreduce_kernel<float, false>, dim3(static_cast<unsigned>(ctas)), dim3(512), 0, a);
    }
    CollArgs a{buf, buf, count, dtype, op, c->comm};
    return c->dev->collective(REC_ALLREDUCE, a);
}

// Maps every rank's mailbox into this process: the mailbox handles are all-gathered over NCCL (outside
// any capture) and opened with peer access. Returns without enabling the peer path when IPC is refused
// (the NCCL collectives then serve every call).
l0b_status peer_setup(l0b_comm* c) {
    if (c->nranks < 2 || c->nranks > kMaxRanks || g_peer_disabled) return L0B_OK;
    static_assert(kMaxPeerRanks == kMaxRanks, "one rank limit for both mailboxes");
    // One allocation: the u64 all-reduce region, the GEMV epilogue's peer-sum region (from psum_off) and the
    // tagged f32 all-reduce region (from ll_off).
    const size_t ar_bytes = 2ull * kMaxRanks * kPeerSlotFloats * sizeof(float) +
                            2ull * kMaxRanks * kPeerCtas * sizeof(unsigned) + kPeerCtas * sizeof(unsigned);
    const size_t psum_off = (ar_bytes + 255) & ~static_cast<size_t>(255);
    const size_t ll_off = (psum_off + kPeerSumBytes + 255) & ~static_cast<size_t>(255);
    const size_t mbox_bytes = ll_off + kLLBytes;
    c->ll_off = ll_off;
    if (cudaMalloc(&c->mbox, mbox_bytes) != cudaSuccess) {
        cudaGetLastError();
        c->mbox = nullptr;
        return L0B_OK;
    }
    cudaMemsetAsync(c->mbox, 0, mbox_bytes, c->dev->stream);
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, c->mbox) != cudaSuccess) {
        cudaGetLastError();
        return L0B_OK;
    }
    char* xfer = nullptr;
    L0B_CHECK_CUDA(cudaMalloc(&xfer, sizeof(h) * (c->nranks + 1)));
    L0B_CHECK_CUDA(cudaMemcpyAsync(xfer, &h, sizeof(h), cudaMemcpyHostToDevice, c->dev->stream));
    ncclResult_t r = g_nccl.all_gather(xfer, xfer + sizeof(h), sizeof(h), ncclUint8, c->comm, c->dev->stream);
    std::vector<cudaIpcMemHandle_t> all(c->nranks);
    cudaError_t e = cudaSuccess;
    if (r == ncclSuccess)
        e = cudaMemcpyAsync(all.data(), xfer + sizeof(h), sizeof(h) * c->nranks, cudaMemcpyDeviceToHost, c->dev->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->dev->stream);
    cudaFree(xfer);
    if (r != ncclSuccess) return fail(L0B_ERR_NCCL, "mailbox handle exchange failed: %s", g_nccl.error_string(r));
    L0B_CHECK_CUDA(e);
    bool ok = true;
    for (int q = 0; q < c->nranks; ++q) {
        if (q == c->rank) {
            c->peer_mbox[q] = c->mbox;
            continue;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            break;
        }
        c->peer_mbox[q] = static_cast<char*>(p);
    }
    // Every rank must take the same path: agree on it (a max over ranks of "failed").
    int* flag = nullptr;
    L0B_CHECK_CUDA(cudaMalloc(&flag, sizeof(int)));
    const int bad = ok ? 0 : 1;
    L0B_CHECK_CUDA(cudaMemcpyAsync(flag, &bad, sizeof(int), cudaMemcpyHostToDevice, c->dev->stream));
    r = g_nccl.all_reduce(flag, flag, 1, ncclInt32, ncclMax, c->comm, c->dev->stream);
    int any_bad = 1;
    if (r == ncclSuccess) e = cudaMemcpyAsync(&any_bad, flag, sizeof(int), cudaMemcpyDeviceToHost, c->dev->stream);
    if (r == ncclSuccess && e == cudaSuccess) e = cudaStreamSynchronize(c->dev->stream);
    cudaFree(flag);
    if (r != ncclSuccess) return fail(L0B_ERR_NCCL, "peer setup agreement failed: %s", g_nccl.error_string(r));
    L0B_CHECK_CUDA(e);
    c->peer = any_bad == 0;
    if (c->peer) {
        PeerSum h{};
        for (int q = 0; q < c->nranks; ++q) h.mbox[q] = c->peer_mbox[q] + psum_off;
        h.nranks = c->nranks;
        h.rank = c->rank;
        h.error = c->dev->error_flag;
        L0B_CHECK_CUDA(cudaMalloc(&c->peer_sum, sizeof(PeerSum)));
        L0B_CHECK_CUDA(cudaMemcpyAsync(c->peer_sum, &h, sizeof(h), cudaMemcpyHostToDevice, c->dev->stream));
        L0B_CHECK_CUDA(cudaStreamSynchronize(c->dev->stream));
    }
    return L0B_OK;
}

const PeerSum* comm_peer_sum(const l0b_comm* c) { return c && c->peer && g_peer_sum ? c->peer_sum : nullptr; }

void peer_release(l0b_comm* c) {
    for (int q = 0; q < c->nranks && q < kMaxRanks; ++q)
        if (q != c->rank && c->peer_mbox[q]) cudaIpcCloseMemHandle(c->peer_mbox[q]);
    if (c->mbox) cudaFree(c->mbox);
    if (c->peer_sum) cudaFree(c->peer_sum);
    c->mbox = nullptr;
    c->peer_sum = nullptr;
    c->peer = false;
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
    l0b_status ps = peer_setup(c);
    if (ps != L0B_OK) {
        peer_release(c);
        g_nccl.comm_destroy(c->comm);
        delete c;
        return ps;
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
        cudaStreamSynchronize(c->dev->stream);
        peer_release(c);
        g_nccl.comm_destroy(c->comm);
    }
    delete c;
    return L0B_OK;
}

L0B_API l0b_status l0b_comm_set_peer_allreduce(int32_t enable) {
    g_peer_disabled = enable == 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_comm_set_fused_allreduce(int32_t enable) {
    g_peer_sum = enable != 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_comm_uses_peer_allreduce(l0b_comm* c, int32_t* enabled) {
    L0B_REQUIRE(c && enabled, L0B_ERR_ARGUMENT, "null argument");
    *enabled = c->peer ? 1 : 0;
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
