// Device, buffer and command-list (CUDA graph) runtime of libl0b200. See runtime.h.
#include "runtime.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <new>

namespace l0b {

namespace {
thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};
}  // namespace

l0b_status fail(l0b_status status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

void clear_error() { g_last_error.clear(); }

void add_launches(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

size_t dtype_size(l0b_dtype t) {
    switch (t) {
        case L0B_F32: return 4;
        case L0B_F16: return 2;
        case L0B_BF16: return 2;
        case L0B_I8: return 1;
        case L0B_I32: return 4;
        case L0B_U8: return 1;
    }
    return 0;
}

const char* dtype_name(l0b_dtype t) {
    switch (t) {
        case L0B_F32: return "f32";
        case L0B_F16: return "f16";
        case L0B_BF16: return "bf16";
        case L0B_I8: return "i8";
        case L0B_I32: return "i32";
        case L0B_U8: return "u8";
    }
    return "?";
}

bool device_available() {
    static int cached = -1;
    if (cached >= 0) return cached == 1;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        cached = 0;
        return false;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, 0) != cudaSuccess) {
        cudaGetLastError();
        cached = 0;
        return false;
    }
    cached = p.major >= 10 ? 1 : 0;
    return cached == 1;
}

}  // namespace l0b

using namespace l0b;

// ---------------------------------------------------------------------------------------------
// l0b_device
// ---------------------------------------------------------------------------------------------

l0b_device::~l0b_device() {
    cudaSetDevice(index);
    if (stream) cudaStreamSynchronize(stream);
    for (auto& g : graphs) {
        if (g->exec) cudaGraphExecDestroy(g->exec);
        if (g->graph) cudaGraphDestroy(g->graph);
    }
    graphs.clear();
    if (scratch.ptr) cudaFree(scratch.ptr);
    if (scratch16.ptr) cudaFree(scratch16.ptr);
    if (counters) cudaFree(counters);
    if (error_flag) cudaFree(error_flag);
    if (stream) cudaStreamDestroy(stream);
}

l0b_status l0b_device::ensure_scratch(size_t bytes, void** out, int slot) {
    DeviceScratch& sc = slot == 0 ? scratch : scratch16;
    if (bytes > sc.bytes) {
        // Growing the scratch moves it: cached command lists that captured the old address no longer
        // match any new list (the address is a kernel argument), so they simply stop being reused.
        L0B_REQUIRE(!recording, L0B_ERR_INVALID_OPERATION,
                    "op scratch must grow to %zu bytes while a command list is being recorded; run the op "
                    "once outside a recording first",
                    bytes);
        if (sc.ptr) {
            L0B_CHECK_CUDA(cudaStreamSynchronize(stream));
            L0B_CHECK_CUDA(cudaFree(sc.ptr));
            sc.ptr = nullptr;
            sc.bytes = 0;
        }
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        L0B_CHECK_CUDA(cudaMalloc(&sc.ptr, want));
        sc.bytes = want;
    }
    *out = sc.ptr;
    return L0B_OK;
}

l0b_status l0b_device::ensure_counters(size_t count, unsigned** out) {
    if (count > counter_count) {
        L0B_REQUIRE(!recording, L0B_ERR_INVALID_OPERATION,
                    "op counters must grow while a command list is being recorded");
        if (counters) {
            L0B_CHECK_CUDA(cudaStreamSynchronize(stream));
            L0B_CHECK_CUDA(cudaFree(counters));
            counters = nullptr;
        }
        size_t want = count < 4096 ? 4096 : count;
        L0B_CHECK_CUDA(cudaMalloc(&counters, want * sizeof(unsigned)));
        L0B_CHECK_CUDA(cudaMemsetAsync(counters, 0, want * sizeof(unsigned), stream));
        counter_count = want;
    }
    *out = counters;
    return L0B_OK;
}

static cudaLaunchConfig_t make_config(const LaunchRecord& rec, cudaStream_t stream, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = rec.grid;
    cfg.blockDim = rec.block;
    cfg.dynamicSmemBytes = rec.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 0;
    if (rec.pdl) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
        ++cfg.numAttrs;
    }
    if (rec.cluster_y > 1) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = 1;
        attr[cfg.numAttrs].val.clusterDim.y = rec.cluster_y;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        ++cfg.numAttrs;
    }
    return cfg;
}

l0b_status l0b_device::submit(LaunchRecord& rec) {
    if (recording) {
        ++log_used;
        return L0B_OK;
    }
    void* args[kMaxArgs];
    rec.arg_pointers(args);
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = make_config(rec, stream, attr);
    L0B_CHECK_CUDA(cudaLaunchKernelExC(&cfg, rec.func, args));
    add_launches(1);
    return L0B_OK;
}

l0b_status l0b_device::collective(int kind, const CollArgs& a) {
    LaunchRecord* rec;
    LaunchRecord local;
    if (recording) {
        if (log_used == log.size()) log.emplace_back();
        rec = &log[log_used];
    } else {
        rec = &local;
    }
    rec->func = nullptr;
    rec->grid = dim3(0, 0, 0);
    rec->block = dim3(0, 0, 0);
    rec->smem = 0;
    rec->pdl = 0;
    rec->cluster_y = 0;
    rec->kind = static_cast<uint8_t>(kind);
    rec->nargs = 0;
    rec->blob_size = 0;
    rec->push(a);
    if (recording) {
        ++log_used;
        return L0B_OK;
    }
    return collective_issue(kind, a, stream);
}

l0b_status l0b_device::build_graph(CachedGraph& g) {
    if (g.exec) {
        cudaGraphExecDestroy(g.exec);
        g.exec = nullptr;
    }
    if (g.graph) {
        cudaGraphDestroy(g.graph);
        g.graph = nullptr;
    }
    g.nodes.clear();
    L0B_CHECK_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    for (auto& rec : g.log) {
        if (rec.kind != REC_KERNEL) {
            CollArgs a;
            std::memcpy(&a, rec.blob + rec.offsets[0], sizeof(a));
            l0b_status st = collective_issue(rec.kind, a, stream);
            if (st != L0B_OK) {
                cudaGraph_t junk = nullptr;
                cudaStreamEndCapture(stream, &junk);
                if (junk) cudaGraphDestroy(junk);
                return st;
            }
            g.nodes.push_back(nullptr);  // never patched: collectives only match with equal arguments
            continue;
        }
        void* args[kMaxArgs];
        rec.arg_pointers(args);
        cudaLaunchAttribute attr[2];
        cudaLaunchConfig_t cfg = make_config(rec, stream, attr);
        cudaError_t e = cudaLaunchKernelExC(&cfg, rec.func, args);
        if (e != cudaSuccess) {
            cudaGraph_t junk = nullptr;
            cudaStreamEndCapture(stream, &junk);
            if (junk) cudaGraphDestroy(junk);
            return fail(L0B_ERR_CUDA, "capturing a command list failed: %s", cudaGetErrorString(e));
        }
        cudaStreamCaptureStatus st;
        const cudaGraphNode_t* deps = nullptr;
        size_t ndeps = 0;
        e = cudaStreamGetCaptureInfo(stream, &st, nullptr, nullptr, &deps, &ndeps);
        if (e != cudaSuccess || ndeps != 1) {
            cudaGraph_t junk = nullptr;
            cudaStreamEndCapture(stream, &junk);
            if (junk) cudaGraphDestroy(junk);
            return fail(L0B_ERR_CUDA, "capture bookkeeping failed (%s, %zu deps)", cudaGetErrorString(e), ndeps);
        }
        g.nodes.push_back(deps[0]);
    }
    L0B_CHECK_CUDA(cudaStreamEndCapture(stream, &g.graph));
    L0B_CHECK_CUDA(cudaGraphInstantiateWithFlags(&g.exec, g.graph, 0));
    ++graphs_built;
    return L0B_OK;
}

l0b_status l0b_device::end_recording() {
    recording = false;
    size_t n = log_used;
    log_used = 0;
    if (n == 0) return L0B_OK;
    ++use_clock;
    // 1. An identical cached list: relaunch it.
    CachedGraph* shape_match = nullptr;
    for (auto& gp : graphs) {
        CachedGraph& g = *gp;
        if (g.log.size() != n) continue;
        bool shape = true, args = true;
        for (size_t i = 0; i < n && shape; ++i) {
            if (!g.log[i].same_shape(log[i])) shape = false;
            else if (args && !g.log[i].same_args(log[i])) args = false;
        }
        if (!shape) continue;
        if (args) {
            g.last_use = use_clock;
            L0B_CHECK_CUDA(cudaGraphLaunch(g.exec, stream));
            add_launches(static_cast<int64_t>(n));
            ++graphs_reused;
            return L0B_OK;
        }
        if (!shape_match) shape_match = &g;
    }
    // 2. Same kernels and launch shapes, other arguments: patch the changed kernel nodes.
    if (shape_match) {
        CachedGraph& g = *shape_match;
        bool ok = true;
        for (size_t i = 0; i < n; ++i) {
            if (g.log[i].same_args(log[i])) continue;
            void* args[kMaxArgs];
            log[i].arg_pointers(args);
            cudaKernelNodeParams p = {};
            p.func = const_cast<void*>(log[i].func);
            p.gridDim = log[i].grid;
            p.blockDim = log[i].block;
            p.sharedMemBytes = log[i].smem;
            p.kernelParams = args;
            if (cudaGraphExecKernelNodeSetParams(g.exec, g.nodes[i], &p) != cudaSuccess) {
                cudaGetLastError();
                ok = false;
                break;
            }
            g.log[i] = log[i];
        }
        if (ok) {
            g.last_use = use_clock;
            L0B_CHECK_CUDA(cudaGraphLaunch(g.exec, stream));
            add_launches(static_cast<int64_t>(n));
            ++graphs_updated;
            return L0B_OK;
        }
    }
    // 3. Capture a new list; keep at most 8, evicting the least recently used.
    std::unique_ptr<CachedGraph> fresh(new CachedGraph());
    fresh->log.assign(log.begin(), log.begin() + n);
    L0B_TRY(build_graph(*fresh));
    fresh->last_use = use_clock;
    L0B_CHECK_CUDA(cudaGraphLaunch(fresh->exec, stream));
    add_launches(static_cast<int64_t>(n));
    if (graphs.size() >= 8) {
        size_t victim = 0;
        for (size_t i = 1; i < graphs.size(); ++i)
            if (graphs[i]->last_use < graphs[victim]->last_use) victim = i;
        L0B_CHECK_CUDA(cudaStreamSynchronize(stream));
        if (graphs[victim]->exec) cudaGraphExecDestroy(graphs[victim]->exec);
        if (graphs[victim]->graph) cudaGraphDestroy(graphs[victim]->graph);
        graphs.erase(graphs.begin() + victim);
    }
    graphs.push_back(std::move(fresh));
    return L0B_OK;
}

void l0b_device::drop_graphs() {
    cudaStreamSynchronize(stream);
    for (auto& g : graphs) {
        if (g->exec) cudaGraphExecDestroy(g->exec);
        if (g->graph) cudaGraphDestroy(g->graph);
    }
    graphs.clear();
}

void l0b_device::abort_recording() {
    recording = false;
    log_used = 0;
}

// ---------------------------------------------------------------------------------------------
// C ABI: errors, runtime, device, buffers
// ---------------------------------------------------------------------------------------------

#define L0B_GUARD_BEGIN try {
#define L0B_GUARD_END                                                                              \
    }                                                                                              \
    catch (const std::bad_alloc&) {                                                                \
        return fail(L0B_ERR_OUT_OF_MEMORY, "host allocation failed");                              \
    }                                                                                              \
    catch (const std::exception& e) {                                                              \
        return fail(L0B_ERR_INVALID_OPERATION, "%s", e.what());                                    \
    }

extern "C" {

L0B_API const char* l0b_last_error(void) { return g_last_error.c_str(); }

L0B_API int32_t l0b_version(void) { return (1 << 16) | 0; }

L0B_API int64_t l0b_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

L0B_API l0b_status l0b_runtime_is_available(int32_t* available) {
    L0B_REQUIRE(available, L0B_ERR_ARGUMENT, "available is null");
    *available = device_available() ? 1 : 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_count(int32_t* count) {
    L0B_REQUIRE(count, L0B_ERR_ARGUMENT, "count is null");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    int usable = 0;
    for (int i = 0; i < n; ++i) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, i) == cudaSuccess && p.major >= 10) ++usable;
    }
    *count = usable;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_info(int32_t index, char* name, int32_t name_len, int32_t* sm_count,
                                   int64_t* total_bytes) {
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, index);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(L0B_ERR_NO_DEVICE, "no CUDA device %d: %s", index, cudaGetErrorString(e));
    }
    if (name && name_len > 0) {
        snprintf(name, static_cast<size_t>(name_len), "%s", p.name);
    }
    if (sm_count) *sm_count = p.multiProcessorCount;
    if (total_bytes) *total_bytes = static_cast<int64_t>(p.totalGlobalMem);
    return L0B_OK;
}

L0B_API l0b_status l0b_device_create(int32_t index, l0b_device** out) {
    L0B_GUARD_BEGIN
    L0B_REQUIRE(out, L0B_ERR_ARGUMENT, "out is null");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(L0B_ERR_NO_DEVICE, "no CUDA device is available");
    }
    L0B_REQUIRE(index >= 0 && index < n, L0B_ERR_OUT_OF_RANGE, "device index %d out of range [0, %d)", index, n);
    cudaDeviceProp p;
    L0B_CHECK_CUDA(cudaGetDeviceProperties(&p, index));
    L0B_REQUIRE(p.major >= 10, L0B_ERR_NO_DEVICE,
                "device %d (%s, sm_%d%d) is not an sm_100 GPU; this library is built for sm_100a only", index,
                p.name, p.major, p.minor);
    L0B_CHECK_CUDA(cudaSetDevice(index));
    std::unique_ptr<l0b_device> d(new l0b_device());
    d->index = index;
    d->sm_count = p.multiProcessorCount;
    d->cc_major = p.major;
    d->smem_optin = p.sharedMemPerBlockOptin;
    L0B_CHECK_CUDA(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    L0B_CHECK_CUDA(cudaMalloc(&d->error_flag, sizeof(int)));
    L0B_CHECK_CUDA(cudaMemsetAsync(d->error_flag, 0, sizeof(int), d->stream));
    L0B_CHECK_CUDA(cudaStreamSynchronize(d->stream));
    d->log.reserve(512);
    *out = d.release();
    return L0B_OK;
    L0B_GUARD_END
}

L0B_API l0b_status l0b_device_free(l0b_device* dev) {
    delete dev;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_begin_recording(l0b_device* dev) {
    L0B_REQUIRE(dev, L0B_ERR_ARGUMENT, "device is null");
    L0B_REQUIRE(!dev->recording, L0B_ERR_INVALID_OPERATION, "the device is already recording");
    dev->recording = true;
    dev->log_used = 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_end_recording(l0b_device* dev) {
    L0B_GUARD_BEGIN
    L0B_REQUIRE(dev, L0B_ERR_ARGUMENT, "device is null");
    L0B_REQUIRE(dev->recording, L0B_ERR_INVALID_OPERATION, "the device is not recording");
    L0B_CHECK_CUDA(cudaSetDevice(dev->index));
    L0B_TRY(dev->end_recording());
    L0B_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
    return L0B_OK;
    L0B_GUARD_END
}

L0B_API l0b_status l0b_device_abort_recording(l0b_device* dev) {
    L0B_REQUIRE(dev, L0B_ERR_ARGUMENT, "device is null");
    dev->abort_recording();
    return L0B_OK;
}

L0B_API l0b_status l0b_device_is_recording(l0b_device* dev, int32_t* recording) {
    L0B_REQUIRE(dev && recording, L0B_ERR_ARGUMENT, "null argument");
    *recording = dev->recording ? 1 : 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_synchronize(l0b_device* dev) {
    L0B_REQUIRE(dev, L0B_ERR_ARGUMENT, "device is null");
    L0B_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
    return L0B_OK;
}

L0B_API l0b_status l0b_device_stream(l0b_device* dev, void** stream) {
    L0B_REQUIRE(dev && stream, L0B_ERR_ARGUMENT, "null argument");
    *stream = dev->stream;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_graph_stats(l0b_device* dev, int64_t* built, int64_t* reused, int64_t* updated) {
    L0B_REQUIRE(dev, L0B_ERR_ARGUMENT, "device is null");
    if (built) *built = dev->graphs_built;
    if (reused) *reused = dev->graphs_reused;
    if (updated) *updated = dev->graphs_updated;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_error_status(l0b_device* dev, int32_t* code) {
    L0B_REQUIRE(dev && code, L0B_ERR_ARGUMENT, "null argument");
    int v = 0;
    L0B_CHECK_CUDA(cudaMemcpyAsync(&v, dev->error_flag, sizeof(int), cudaMemcpyDeviceToHost, dev->stream));
    L0B_CHECK_CUDA(cudaMemsetAsync(dev->error_flag, 0, sizeof(int), dev->stream));
    L0B_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
    *code = v;
    return L0B_OK;
}

L0B_API l0b_status l0b_device_set_pdl(l0b_device* dev, int32_t enabled) {
    L0B_REQUIRE(dev, L0B_ERR_ARGUMENT, "device is null");
    dev->pdl = enabled != 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_alloc(l0b_device* dev, l0b_dtype dtype, int64_t count, l0b_buffer** out) {
    L0B_GUARD_BEGIN
    L0B_REQUIRE(dev && out, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(count >= 0, L0B_ERR_OUT_OF_RANGE, "count %lld is negative", (long long)count);
    L0B_REQUIRE(dtype_size(dtype) != 0, L0B_ERR_ARGUMENT, "unknown dtype %d", (int)dtype);
    *out = nullptr;
    std::unique_ptr<l0b_buffer> b(new l0b_buffer());
    b->dev = dev;
    b->dtype = dtype;
    b->count = count;
    size_t bytes = b->bytes();
    L0B_CHECK_CUDA(cudaSetDevice(dev->index));
    // Round allocations up to 256 bytes so vectorised kernels may read whole 16-byte words at the end.
    size_t alloc = (bytes + 255) & ~size_t(255);
    if (alloc == 0) alloc = 256;
    L0B_CHECK_CUDA(cudaMalloc(&b->ptr, alloc));
    L0B_CHECK_CUDA(cudaMemsetAsync(b->ptr, 0, alloc, dev->stream));
    *out = b.release();
    return L0B_OK;
    L0B_GUARD_END
}

L0B_API l0b_status l0b_buffer_alloc_from(l0b_device* dev, l0b_dtype dtype, int64_t count, const void* host,
                                         l0b_buffer** out) {
    L0B_TRY(l0b_buffer_alloc(dev, dtype, count, out));
    if (count > 0) {
        L0B_REQUIRE(host, L0B_ERR_ARGUMENT, "host data is null");
        l0b_status s = l0b_buffer_write(*out, 0, host, count);
        if (s != L0B_OK) {
            l0b_buffer_free(*out);
            *out = nullptr;
            return s;
        }
    }
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_view(l0b_buffer* base, int64_t offset, int64_t count, l0b_buffer** out) {
    L0B_REQUIRE(base && out, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(offset >= 0 && count >= 0 && offset + count <= base->count, L0B_ERR_OUT_OF_RANGE,
                "view [%lld, %lld) outside a %lld-element buffer", (long long)offset, (long long)(offset + count),
                (long long)base->count);
    l0b_buffer* v = new l0b_buffer();
    v->dev = base->dev;
    v->dtype = base->dtype;
    v->count = count;
    v->ptr = static_cast<char*>(base->ptr) + offset * dtype_size(base->dtype);
    v->owns = false;
    *out = v;
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_free(l0b_buffer* buf) {
    if (!buf) return L0B_OK;
    if (buf->ptr && buf->owns) {
        cudaSetDevice(buf->dev->index);
        // The buffer may still be read by queued work.
        cudaStreamSynchronize(buf->dev->stream);
        cudaFree(buf->ptr);
    }
    delete buf;
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_write(l0b_buffer* buf, int64_t offset, const void* host, int64_t count) {
    L0B_REQUIRE(buf, L0B_ERR_ARGUMENT, "buffer is null");
    L0B_REQUIRE(offset >= 0 && count >= 0 && offset + count <= buf->count, L0B_ERR_OUT_OF_RANGE,
                "write of [%lld, %lld) outside a buffer of %lld elements", (long long)offset,
                (long long)(offset + count), (long long)buf->count);
    if (count == 0) return L0B_OK;
    L0B_REQUIRE(host, L0B_ERR_ARGUMENT, "host pointer is null");
    size_t es = dtype_size(buf->dtype);
    L0B_CHECK_CUDA(cudaSetDevice(buf->dev->index));
    // Stream-ordered: lands after work already queued and, while recording, before the command list.
    L0B_CHECK_CUDA(cudaMemcpyAsync(static_cast<char*>(buf->ptr) + offset * es, host, count * es,
                                   cudaMemcpyHostToDevice, buf->dev->stream));
    // The host array may be reused as soon as we return (C# arrays, numpy temporaries).
    L0B_CHECK_CUDA(cudaStreamSynchronize(buf->dev->stream));
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_read(l0b_buffer* buf, int64_t offset, void* host, int64_t count) {
    L0B_REQUIRE(buf, L0B_ERR_ARGUMENT, "buffer is null");
    L0B_REQUIRE(offset >= 0 && count >= 0 && offset + count <= buf->count, L0B_ERR_OUT_OF_RANGE,
                "read of [%lld, %lld) outside a buffer of %lld elements", (long long)offset,
                (long long)(offset + count), (long long)buf->count);
    L0B_REQUIRE(!buf->dev->recording, L0B_ERR_INVALID_OPERATION,
                "buffers cannot be read while the device is recording a command list");
    if (count == 0) return L0B_OK;
    L0B_REQUIRE(host, L0B_ERR_ARGUMENT, "host pointer is null");
    size_t es = dtype_size(buf->dtype);
    L0B_CHECK_CUDA(cudaSetDevice(buf->dev->index));
    L0B_CHECK_CUDA(cudaMemcpyAsync(host, static_cast<const char*>(buf->ptr) + offset * es, count * es,
                                   cudaMemcpyDeviceToHost, buf->dev->stream));
    L0B_CHECK_CUDA(cudaStreamSynchronize(buf->dev->stream));
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_copy(l0b_buffer* dst, int64_t dst_offset, l0b_buffer* src, int64_t src_offset,
                                   int64_t count) {
    L0B_REQUIRE(dst && src, L0B_ERR_ARGUMENT, "buffer is null");
    L0B_REQUIRE(dst->dtype == src->dtype, L0B_ERR_ARGUMENT, "copy between %s and %s buffers",
                dtype_name(src->dtype), dtype_name(dst->dtype));
    L0B_REQUIRE(count >= 0 && dst_offset >= 0 && src_offset >= 0 && dst_offset + count <= dst->count &&
                    src_offset + count <= src->count,
                L0B_ERR_OUT_OF_RANGE, "copy range outside the buffers");
    L0B_REQUIRE(!dst->dev->recording, L0B_ERR_INVALID_OPERATION, "buffer copies are not recorded");
    if (count == 0) return L0B_OK;
    size_t es = dtype_size(dst->dtype);
    L0B_CHECK_CUDA(cudaMemcpyAsync(static_cast<char*>(dst->ptr) + dst_offset * es,
                                   static_cast<const char*>(src->ptr) + src_offset * es, count * es,
                                   cudaMemcpyDeviceToDevice, dst->dev->stream));
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_zero(l0b_buffer* buf) {
    L0B_REQUIRE(buf, L0B_ERR_ARGUMENT, "buffer is null");
    L0B_REQUIRE(!buf->dev->recording, L0B_ERR_INVALID_OPERATION, "buffer fills are not recorded");
    if (buf->count == 0) return L0B_OK;
    L0B_CHECK_CUDA(cudaMemsetAsync(buf->ptr, 0, buf->bytes(), buf->dev->stream));
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_count(l0b_buffer* buf, int64_t* count) {
    L0B_REQUIRE(buf && count, L0B_ERR_ARGUMENT, "null argument");
    *count = buf->count;
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_dtype(l0b_buffer* buf, l0b_dtype* dtype) {
    L0B_REQUIRE(buf && dtype, L0B_ERR_ARGUMENT, "null argument");
    *dtype = buf->dtype;
    return L0B_OK;
}

L0B_API l0b_status l0b_buffer_device_ptr(l0b_buffer* buf, void** ptr) {
    L0B_REQUIRE(buf && ptr, L0B_ERR_ARGUMENT, "null argument");
    *ptr = buf->ptr;
    return L0B_OK;
}

}  // extern "C"
