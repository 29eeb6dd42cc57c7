// Internal runtime of libl0b200: device and buffer handles, error state, and the launch recorder.
//
// Every kernel goes through Device::launch(). Outside a recording it is launched at once on the
// device's stream. Inside a recording (ComputeDevice.BeginRecording .. EndRecording,
// L/LlmModel.cs:415-442) it is appended to a command list; EndRecording turns the list into a CUDA
// graph and launches it once. Lists are cached: a list equal to a cached one relaunches the cached
// executable graph, a list that differs only in kernel arguments patches the changed kernel nodes,
// anything else is captured anew. The fused decode step keeps every per-token value (position,
// token id) in device memory, so its list is identical from token to token and costs one graph
// launch.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>
#include <memory>

#include "../../include/l0b200.h"

namespace l0b {

// ---------------------------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------------------------

struct Error {
    l0b_status status;
    std::string message;
};

// Sets the thread-local last error and returns the status.
l0b_status fail(l0b_status status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

#define L0B_CHECK_CUDA(call)                                                                       \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) {                                                                   \
            return ::l0b::fail(e_ == cudaErrorMemoryAllocation ? L0B_ERR_OUT_OF_MEMORY : L0B_ERR_CUDA, \
                               "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__,   \
                               __LINE__);                                                          \
        }                                                                                          \
    } while (0)

#define L0B_TRY(expr)                                                                              \
    do {                                                                                           \
        l0b_status s_ = (expr);                                                                    \
        if (s_ != L0B_OK) return s_;                                                               \
    } while (0)

#define L0B_REQUIRE(cond, status, ...)                                                             \
    do {                                                                                           \
        if (!(cond)) return ::l0b::fail(status, __VA_ARGS__);                                      \
    } while (0)

size_t dtype_size(l0b_dtype t);
const char* dtype_name(l0b_dtype t);

// Copy ordered on `s` (the device's non-blocking stream) and waited for. A plain cudaMemcpy runs on the
// legacy stream, which does not order against non-blocking streams, and from pageable memory it may
// return before its DMA lands, so a kernel queued on `s` right after it could read stale bytes.
inline cudaError_t copy_sync(cudaStream_t s, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind) {
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, s);
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(s);
}

// ---------------------------------------------------------------------------------------------
// Launch records
// ---------------------------------------------------------------------------------------------

constexpr int kMaxArgBytes = 768;
constexpr int kMaxArgs = 24;

// A command-list entry is a kernel launch or a collective on the device stream (tensor parallelism).
enum RecordKind : uint8_t { REC_KERNEL = 0, REC_ALLREDUCE = 1, REC_ALLGATHER = 2 };
enum CollOp : int { COLL_SUM = 0, COLL_MAX = 1 };
constexpr int kDtypeU64 = 100;  // collective element type for 64-bit argmax keys (internal)
struct CollArgs {
    const void* send;
    void* recv;
    size_t count;
    int dtype;
    int op;
    void* comm;  // ncclComm_t
};
// Issues a collective on `stream` (comm.cu; NCCL is loaded when the first communicator is made).
l0b_status collective_issue(int kind, const CollArgs& a, cudaStream_t stream);

struct LaunchRecord {
    const void* func = nullptr;
    dim3 grid, block;
    uint32_t smem = 0;
    uint8_t pdl = 0;
    uint8_t cluster_y = 0;  // > 1: thread-block clusters of (1, cluster_y, 1)
    uint8_t kind = REC_KERNEL;
    uint8_t nargs = 0;
    uint16_t blob_size = 0;
    uint16_t offsets[kMaxArgs];
    alignas(16) uint8_t blob[kMaxArgBytes];

    bool same_shape(const LaunchRecord& o) const {
        return func == o.func && grid.x == o.grid.x && grid.y == o.grid.y && grid.z == o.grid.z &&
               block.x == o.block.x && block.y == o.block.y && block.z == o.block.z && smem == o.smem &&
               pdl == o.pdl && cluster_y == o.cluster_y && kind == o.kind && nargs == o.nargs &&
               blob_size == o.blob_size && std::memcmp(offsets, o.offsets, nargs * sizeof(uint16_t)) == 0 &&
               (kind == REC_KERNEL || same_args(o));  // a captured collective cannot be patched
    }
    bool same_args(const LaunchRecord& o) const { return std::memcmp(blob, o.blob, blob_size) == 0; }

    template <typename T>
    void push(const T& v) {
        static_assert(std::is_trivially_copyable<T>::value, "kernel args must be trivially copyable");
        size_t align = alignof(T) < 16 ? alignof(T) : 16;
        size_t off = (blob_size + align - 1) & ~(align - 1);
        offsets[nargs++] = static_cast<uint16_t>(off);
        std::memcpy(blob + off, &v, sizeof(T));
        blob_size = static_cast<uint16_t>(off + sizeof(T));
    }
    void arg_pointers(void** out) {
        for (int i = 0; i < nargs; ++i) out[i] = blob + offsets[i];
    }
};

struct CachedGraph {
    std::vector<LaunchRecord> log;
    std::vector<cudaGraphNode_t> nodes;  // kernel node per record, in launch order
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    uint64_t last_use = 0;
};

// ---------------------------------------------------------------------------------------------
// Device
// ---------------------------------------------------------------------------------------------

struct DeviceScratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};

}  // namespace l0b

struct l0b_device {
    int index = 0;
    int sm_count = 148;
    int cc_major = 10;
    size_t smem_optin = 227 * 1024;
    cudaStream_t stream = nullptr;
    bool pdl = true;
    bool recording = false;
    std::vector<l0b::LaunchRecord> log;
    size_t log_used = 0;
    std::vector<std::unique_ptr<l0b::CachedGraph>> graphs;
    uint64_t use_clock = 0;
    int64_t graphs_built = 0, graphs_reused = 0, graphs_updated = 0;
    // Scratch for op-level kernels that need temporary device memory, one slot per purpose so two ops
    // of one command list never share it: 0 = split-KV partials, 1 = 16-bit activation copies.
    l0b::DeviceScratch scratch;
    l0b::DeviceScratch scratch16;
    // Zeroed counters for last-block-done reductions; each user resets what it used.
    unsigned* counters = nullptr;
    size_t counter_count = 0;
    // Set by kernels whose bounded waits gave up (read and cleared by l0b_device_error_status).
    int* error_flag = nullptr;

    ~l0b_device();

    l0b_status ensure_scratch(size_t bytes, void** out, int slot = 0);
    l0b_status ensure_counters(size_t count, unsigned** out);

    // Appends (recording) or launches (immediate) one kernel.
    l0b_status submit(l0b::LaunchRecord& rec);

    template <typename... KArgs, typename... Args>
    l0b_status launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
        return launch_cluster(kernel, grid, block, smem, 0, static_cast<Args&&>(args)...);
    }

    // As launch(), in thread-block clusters of (1, cluster_y, 1) CTAs when cluster_y > 1.
    template <typename... KArgs, typename... Args>
    l0b_status launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_y,
                              Args&&... args) {
        static_assert(sizeof...(KArgs) == sizeof...(Args), "argument count mismatch");
        if (grid.x == 0 || grid.y == 0 || grid.z == 0) return L0B_OK;
        l0b::LaunchRecord* rec;
        l0b::LaunchRecord local;
        if (recording) {
            if (log_used == log.size()) log.emplace_back();
            rec = &log[log_used];
        } else {
            rec = &local;
        }
        rec->func = reinterpret_cast<const void*>(kernel);
        rec->grid = grid;
        rec->block = block;
        rec->smem = static_cast<uint32_t>(smem);
        rec->pdl = pdl ? 1 : 0;
        rec->cluster_y = static_cast<uint8_t>(cluster_y > 1 ? cluster_y : 0);
        rec->kind = l0b::REC_KERNEL;
        rec->nargs = 0;
        rec->blob_size = 0;
        (rec->push(static_cast<KArgs>(args)), ...);
        return submit(*rec);
    }

    // Appends (recording) or issues (immediate) one collective.
    l0b_status collective(int kind, const l0b::CollArgs& a);

    // Destroys every cached command-list graph (after the stream drains); lists are captured anew
    // when next recorded. Graphs holding collectives must go before their communicator.
    void drop_graphs();

    l0b_status end_recording();
    void abort_recording();
    l0b_status build_graph(l0b::CachedGraph& g);
};

struct l0b_buffer {
    l0b_device* dev = nullptr;
    l0b_dtype dtype = L0B_F32;
    int64_t count = 0;
    void* ptr = nullptr;
    bool owns = true;  // false for a view into another buffer's memory
    size_t bytes() const { return static_cast<size_t>(count) * l0b::dtype_size(dtype); }
};

struct l0b_comm;

namespace l0b {
// Tensor-parallel collectives on the communicator's device stream (recorded like kernels).
l0b_status comm_allreduce(l0b_comm* c, void* buf, size_t count, int dtype, int op);
l0b_status comm_allgather(l0b_comm* c, const void* send, void* recv, size_t count, int dtype);
int comm_size(const l0b_comm* c);
int comm_rank(const l0b_comm* c);
// Process-wide counter of kernels launched (immediate + graph kernel nodes).
void add_launches(int64_t n);
// Checks that the current device is an sm_100-class GPU. Cached.
bool device_available();
}  // namespace l0b
