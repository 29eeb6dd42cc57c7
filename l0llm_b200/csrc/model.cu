// C++ mirror of the reference decoder host: LlmModel (L/LlmModel.cs), LlmDecoderLayer
// (L/LlmDecoderLayer.cs), LlmMatrix (L/LlmMatrix.cs), LlmKvCache (L/LlmKvCache.cs) and the weight
// loading rules of LlmLayerWeights (L/LlmLayerWeights.cs:110-212).
//
// Two ways to run a layer:
//  - fused (default): 5 kernels per layer at decode --
//      QKV GEMV (+input RMSNorm prologue, +bias epilogue) -> attention (+RoPE on q and the new k,
//      KV-cache store, split-KV softmax, merge) -> o_proj GEMV (+residual add) ->
//      gate/up GEMV (+post-attention RMSNorm prologue, SiLU(gate)*up epilogue) -> down GEMV (+residual).
//    Every per-token value (token id, position) lives in device memory, so a decode step records the
//    same command list every time and replays one cached CUDA graph.
//  - reference sequence (set_fused(0)): the op-by-op sequence of LlmDecoderLayer.Forward/ForwardBatch
//    (RMSNorm, projections, BiasAdd, QK-norm, RoPE, KvCacheStore, Attention, o_proj, RMSNorm+residual,
//    gate/up, SwiGLU, down, Add), used to check the fused kernels and for per-stage inspection.
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "model.h"
#include "ops.cuh"
#include "suite.h"

using namespace l0b;

struct l0b_model {
    l0b_device* dev = nullptr;
    l0b_suite* suite = nullptr;
    l0b_model_config cfg = {};
    int max_seq = 0;
    int precision = L0B_PRECISION_AUTO;
    int wdtype = L0B_F16;
    int group = 0;
    int batch_cap = 1;  // sequences in the KV caches
    int cap = 1;        // activation rows (max(prefill chunk, batch))
    // Dimensions (per tensor-parallel rank).
    int h = 0, inter = 0, nh = 0, nkv = 0, hd = 0, qdim = 0, kvdim = 0, qkv_w = 0, vocab = 0, rot = 0;
    float attn_scale = 1.f;  // rope cos/sin factor (YaRN)
    float softmax_scale = 1.f;
    int cache_dtype = L0B_F32;
    // Weights.
    float* inv_freq = nullptr;
    float* embed = nullptr;  // f32 [vocab, h] (the reference keeps the embedding table in f32)
    float* final_norm = nullptr;
    ModelMatrix lm_head;
    std::vector<ModelLayer> layers;
    // Activations [cap, width] f32.
    float *hidden = nullptr, *normed = nullptr, *qkv = nullptr, *qb = nullptr, *kb = nullptr, *vb = nullptr;
    float *attn = nullptr, *attn_proj = nullptr, *gate = nullptr, *up = nullptr, *act = nullptr, *down = nullptr;
    float* logits = nullptr;  // [batch_cap, vocab]
    float* head_in = nullptr; // [h] last prompt row (reference sequence: Copy.Execute)
    // Tensor-core GEMM for projections of >= tc_rows activation rows (16-bit weights, or int8 with one
    // scale per row; 0 = off): the rows are split into [hi | lo] 16-bit halves in x16 with a per-row
    // scale in rscale.
    int tc_rows = 0;
    void* x16 = nullptr;      // paired hi / lo rows, [2 * cap + 256, max K] 16-bit
    float* rscale = nullptr;  // [cap]
    float* tc_part = nullptr; // split-K partial tiles (tc_gemm_part_floats)
    unsigned* tc_counters = nullptr;  // [kTcCounters], zero at rest
    long long* ks_acc = nullptr;      // k-split GEMV row sums [ks_acc_count], zero at rest
    int ks_acc_count = 0;
    // Device-side step state: io = [tok(batch_cap) | pos(batch_cap)] written in one copy.
    int* io = nullptr;
    int* tok = nullptr;
    int* pos = nullptr;
    int* prompt_tok = nullptr;  // [cap]
    int* prompt_pos = nullptr;  // [cap]
    int* sampled = nullptr;     // [batch_cap]
    int* out_tokens = nullptr;  // [max_seq * batch_cap]
    int* step_idx = nullptr;
    unsigned long long* keys = nullptr;  // [batch_cap]
    // Device sampling of sequence 0 (LlmSampler.Sample): the context bitmap for the repetition penalty,
    // key scratch, the context ids of the last l0b_model_sample_logits call, and the active parameters
    // while a sampled decode records its steps.
    uint32_t* seen = nullptr;     // [ceil(vocab_full / 32)]
    uint32_t* skeys = nullptr;    // [vocab_full]
    int* ctx_ids = nullptr;       // [max_seq + 1]
    bool sampling = false;
    float s_temperature = 0.f, s_top_p = 1.f, s_penalty = 1.f;
    int s_top_k = 0;
    unsigned long long s_seed = 0;
    int prefill_seq = 0;           // cache row (sequence) the prefill path writes
    // Tensor parallelism: q/k/v, gate/up and lm_head column-split, o/down row-split (partial sums
    // all-reduced before the residual add), attention head-split, embedding replicated.
    l0b_comm* comm = nullptr;
    int tp = 1, tp_rank = 0;
    int vocab_full = 0;            // tokens in the (replicated) embedding; vocab is this rank's lm_head shard
    float* logits_all = nullptr;   // [tp, batch_cap, vocab / tp] gathered logits
    std::vector<int> seq_pos;      // host mirror of each sequence's next position
    // Host state.
    int* host_io = nullptr;       // pinned [2 * batch_cap]
    float* host_logits = nullptr; // pinned [batch_cap * vocab]
    bool fused = true;
    bool recording = true;
    // Qwen3.5 hybrid (Gated DeltaNet layers, gated attention): one GPU, one sequence, reference op sequence.
    bool hybrid = false;
    int lin_hk = 0, lin_hv = 0, lin_dk = 0, lin_dv = 0, lin_kconv = 0, lin_cd = 0, lin_vd = 0;
    float *lq = nullptr, *lz = nullptr, *lb = nullptr, *la = nullptr, *lc = nullptr, *lo = nullptr;
    float* gb = nullptr;  // attention output gate rows [cap, qdim]
    int position = 0;
    l0b_probe_fn probe = nullptr;
    void* probe_user = nullptr;
    std::vector<float> probe_host;
    std::vector<void*> allocations;

    ~l0b_model() {
        if (dev) {
            cudaSetDevice(dev->index);
            cudaStreamSynchronize(dev->stream);
        }
        for (void* p : allocations) cudaFree(p);
        if (host_io) cudaFreeHost(host_io);
        if (host_logits) cudaFreeHost(host_logits);
    }

    template <typename T>
    l0b_status alloc(T** out, size_t count) {
        void* p = nullptr;
        const size_t bytes = count * sizeof(T) < 256 ? 256 : ((count * sizeof(T) + 255) & ~size_t(255));
        L0B_CHECK_CUDA(cudaMalloc(&p, bytes));
        L0B_CHECK_CUDA(cudaMemsetAsync(p, 0, bytes, dev->stream));
        allocations.push_back(p);
        *out = static_cast<T*>(p);
        return L0B_OK;
    }
    // Int8 per-row-scaled projections with few 16-row tiles (under 8 per SM: q/k/v, o_proj, down) go in
    // the blocked layout, whose units of contiguous k blocks the one-row bulk GEMV streams as whole copies.
    // any_size: block whatever the tile count. Large matrices (gate/up of a whole model, the LM head) are
    // otherwise row-major for the whole-tile bulk GEMV; blocked [gate; up] (TP shards) takes the k-split
    // GEMV at batch 1, which pairs each gate tile with its up tile, and the tcgen05 GEMM above it. (A
    // blocked config-2 gate/up on the k-split GEMV measured the same step time as the bulk GEMV.)
    l0b_status alloc_matrix(ModelMatrix& m, int n, int k, bool may_block = true, bool any_size = false) {
        m.n = n;
        m.k = k;
        m.dtype = wdtype;
        m.group = wdtype == L0B_I8 ? (group > 0 ? group : k) : 0;
        m.kb = (may_block && weight_blocking() && wdtype == L0B_I8 && m.group >= k && k % kWeightBlock == 0 &&
                n % 16 == 0 && (any_size || n / 16 < 8 * dev->sm_count))
                   ? kWeightBlock
                   : 0;
        if (wdtype == L0B_I8) {
            L0B_REQUIRE(k % m.group == 0, L0B_ERR_UNSUPPORTED, "int8 scale group %d does not divide K %d", m.group, k);
            int8_t* w;
            L0B_TRY(alloc(&w, static_cast<size_t>(n) * k));
            m.w = w;
            L0B_TRY(alloc(&m.scales, static_cast<size_t>(n) * (k / m.group)));
        } else {
            char* w;
            L0B_TRY(alloc(&w, static_cast<size_t>(n) * k * dtype_size(static_cast<l0b_dtype>(wdtype))));
            m.w = w;
        }
        return L0B_OK;
    }
};

namespace {

// ---------------------------------------------------------------------------------------------
// Seeded synthetic weights, generated on the device. Integer hashing and exactly rounded float
// operations only, so a CPU restatement reproduces every value bit for bit.
// ---------------------------------------------------------------------------------------------

__host__ __device__ inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

enum SynthMode { SYN_NORMAL = 0, SYN_CONST = 1, SYN_I8 = 2, SYN_UNIFORM = 3 };

// Element i of the destination maps to index (row0 + i / row_len) * full_len + col0 + i % row_len of the
// full HuggingFace tensor, so a tensor-parallel shard holds exactly the values of the full tensor.
// int8 destinations in the blocked layout (blk_kb > 0): element i goes to row blk_row0 + i / row_len,
// column i % row_len of a blocked matrix with blk_k columns.
__global__ void synth_kernel(void* dst, int dtype, long long count, uint64_t stream, int mode, float a, float b,
                             long long row_len, long long full_len, long long row0, long long col0, long long blk_k,
                             int blk_kb, long long blk_row0) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / row_len;
        const long long idx = (row0 + r) * full_len + col0 + (i - r * row_len);
        const uint64_t bits = splitmix64(stream + static_cast<uint64_t>(idx) * 0xD1B54A32D192ED03ULL);
        if (mode == SYN_I8) {
            const long long di = blk_kb > 0 ? blocked_index(blk_row0 + r, i - r * row_len, blk_k, blk_kb) : i;
            static_cast<int8_t*>(dst)[di] = static_cast<int8_t>(static_cast<int>(bits % 255ULL) - 127);
            continue;
        }
        float v;
        if (mode == SYN_NORMAL) {
            const uint32_t s = static_cast<uint32_t>(bits & 0xFFFF) + static_cast<uint32_t>((bits >> 16) & 0xFFFF) +
                               static_cast<uint32_t>((bits >> 32) & 0xFFFF) + static_cast<uint32_t>(bits >> 48);
            const float u = __fmul_rn(static_cast<float>(s), 1.0f / 65536.0f);
            v = __fmul_rn(__fmul_rn(__fsub_rn(u, 2.0f), 1.7320508f), a);
        } else if (mode == SYN_UNIFORM) {
            const float u = __fmul_rn(static_cast<float>(bits >> 40), 1.0f / 16777216.0f);
            v = __fadd_rn(a, __fmul_rn(u, __fsub_rn(b, a)));
        } else {
            v = a;
        }
        store_from_float(dst, dtype, i, v);
    }
}

// Columns [col0, col0 + cols) of `rows` row-major int8 rows (row stride src_ld) into rows
// [dst_row0, dst_row0 + rows) of an int8 matrix in the blocked layout (K columns, kb per block).
__global__ void scatter_blocked_kernel(const int8_t* src, long long src_ld, long long col0, long long rows, long long cols,
                                       int8_t* dst, long long K, int kb, long long dst_row0) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < rows * cols;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / cols, c = i - r * cols;
        dst[blocked_index(dst_row0 + r, c, K, kb)] = src[r * src_ld + col0 + c];
    }
}

// Converts (or offsets) an f32 staging tensor into the destination dtype.
__global__ void convert_kernel(const float* src, void* dst, int dtype, long long count, long long row_len,
                               long long full_len, long long col0, float offset) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = i / row_len;
        const float v = src[r * full_len + col0 + (i - r * row_len)] + offset;
        store_from_float(dst, dtype, i, v);
    }
}

// First kernel of a fused step: token rows of the embedding table into the residual stream, and the
// argmax keys cleared for the head.
__global__ void step_begin_kernel(const int* tok, const float* embed, float* hidden, int h, int rows, int vocab,
                                  unsigned long long* keys, int key_rows) {
    pdl_wait();
    if (blockIdx.x == 0 && threadIdx.x < key_rows) keys[threadIdx.x] = 0ull;
    const long long total = static_cast<long long>(rows) * h;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long t = e / h;
        const int id = tok[t];
        hidden[e] = (id >= 0 && id < vocab) ? embed[static_cast<long long>(id) * h + (e - t * h)] : 0.f;
    }
}

// Last kernel of a step: greedy token from the argmax key, fed back as the next input token; the
// position advances by `advance`; the token is appended to the device token log.
__global__ void step_finish_kernel(const unsigned long long* keys, int* sampled, int* tok, int* pos, int* out_tokens,
                                   int* step_idx, int rows, int advance) {
    pdl_wait();
    const int b = threadIdx.x;
    const int step = *step_idx;
    if (b < rows) {
        const int t = argmax_key_index(keys[b]);
        sampled[b] = t;
        tok[b] = t;
        pos[b] += advance;
        if (out_tokens) out_tokens[static_cast<long long>(step) * rows + b] = t;
    }
    __syncthreads();
    if (b == 0) *step_idx = step + 1;
}

inline int grid_for(long long n, int sm) {
    long long g = (n + 255) / 256;
    if (g > sm * 8LL) g = sm * 8LL;
    return g < 1 ? 1 : static_cast<int>(g);
}

uint64_t tensor_stream(uint64_t seed, uint64_t id) { return splitmix64(seed ^ (id * 0x9E3779B97F4A7C15ULL)); }

// Tensor ids of the synthetic generator (also used by the CPU oracle).
enum TensorKind {
    T_IN_NORM = 0, T_POST_NORM, T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_QB, T_KB, T_VB, T_QN, T_KN,
    T_SCALE = 16  // + projection kind: int8 scales of that projection
};
uint64_t layer_tensor_id(int layer, int kind) { return 1000ULL + static_cast<uint64_t>(layer) * 64 + kind; }
constexpr uint64_t kIdEmbed = 1, kIdFinalNorm = 2, kIdLmHead = 3, kIdLmHeadScale = 4;

}  // namespace

// Launch helpers bound to a model -------------------------------------------------------------

namespace {

struct Synth {
    l0b_model* m;
    uint64_t seed;
    float std;
    float lo, hi;
    l0b_status fill(void* dst, int dtype, long long count, uint64_t id, int mode, float a, float b,
                    long long row_len = 0, long long full_len = 0, long long row0 = 0, long long col0 = 0,
                    long long blk_k = 0, int blk_kb = 0, long long blk_row0 = 0) {
        if (count == 0) return L0B_OK;
        if (row_len <= 0) row_len = count;
        if (full_len <= 0) full_len = row_len;
        synth_kernel<<<grid_for(count, m->dev->sm_count), 256, 0, m->dev->stream>>>(
            dst, dtype, count, tensor_stream(seed, id), mode, a, b, row_len, full_len, row0, col0, blk_k, blk_kb,
            blk_row0);
        L0B_CHECK_CUDA(cudaGetLastError());
        return L0B_OK;
    }
    // A projection shard: rows [row0, row0 + rows) x cols [col0, col0 + cols) of an HF [full_n, full_k]
    // tensor, written at row `dst_row` of the stacked matrix.
    l0b_status matrix(ModelMatrix& mat, int dst_row, uint64_t id, uint64_t scale_id, int rows, int cols, int full_k,
                      int row0, int col0) {
        const long long count = static_cast<long long>(rows) * cols;
        if (mat.dtype == L0B_I8) {
            if (mat.kb > 0) {
                L0B_TRY(fill(mat.w, L0B_I8, count, id, SYN_I8, 0.f, 0.f, cols, full_k, row0, col0, mat.k, mat.kb,
                             dst_row));
            } else {
                int8_t* q = static_cast<int8_t*>(mat.w) + static_cast<long long>(dst_row) * mat.k;
                L0B_TRY(fill(q, L0B_I8, count, id, SYN_I8, 0.f, 0.f, cols, full_k, row0, col0));
            }
            // Scales: one per (row, group) of the full tensor; a column shard takes its groups. With one
            // scale per output row (group = this shard's K) every column shard takes the row's only scale.
            const bool per_row = mat.group >= mat.k;
            const int gpr_full = per_row ? 1 : full_k / mat.group;
            const int gpr = per_row ? 1 : cols / mat.group;
            __half* s = mat.scales + static_cast<long long>(dst_row) * gpr;
            return fill(s, L0B_F16, static_cast<long long>(rows) * gpr, scale_id, SYN_UNIFORM, lo, hi, gpr, gpr_full,
                        row0, per_row ? 0 : col0 / mat.group);
        }
        char* w = static_cast<char*>(mat.w) +
                  static_cast<long long>(dst_row) * mat.k * dtype_size(static_cast<l0b_dtype>(mat.dtype));
        return fill(w, mat.dtype, count, id, SYN_NORMAL, std, 0.f, cols, full_k, row0, col0);
    }
};

}  // namespace

// ---------------------------------------------------------------------------------------------
// Step recording
// ---------------------------------------------------------------------------------------------

namespace {

// Cache row of the sequence being prefilled (caches are [batch_cap, max_seq, kv_dim]).
void* seq_cache(l0b_model* m, void* cache) {
    const size_t off = static_cast<size_t>(m->prefill_seq) * m->max_seq * m->kvdim * dtype_size(static_cast<l0b_dtype>(m->cache_dtype));
    return static_cast<char*>(cache) + off;
}

// Cluster size of the decode attention for `rows` sequences in this step.
int cluster_splits(l0b_model* m, int rows) {
    return attention_cluster_splits(m->max_seq, rows * m->nkv * ((m->nh / m->nkv + 7) / 8), m->dev->sm_count);
}

GemvParams linear_params(const ModelMatrix& w, int m_rows, const void* x, long long x_ld) {
    GemvParams p = {};
    p.w = w.w;
    p.scales = w.scales;
    p.group = w.group;
    p.N = w.n;
    p.K = w.k;
    p.M = m_rows;
    p.x = x;
    p.x_dtype = L0B_F32;
    p.x_ld = x_ld;
    p.epi = EPI_STORE;
    p.out_dtype = L0B_F32;
    p.nseg = 1;
    p.prefetch = 1;
    p.kb = w.kb;
    return p;
}

// The model's split-K scratch (shared with the tensor-core GEMM: kernels on the stream run in order and
// every user leaves the counters at zero).
GemvParams model_linear_params(const l0b_model* m, const ModelMatrix& w, int m_rows, const void* x, long long x_ld) {
    GemvParams p = linear_params(w, m_rows, x, x_ld);
    p.part = m->tc_part;
    p.counters = m->tc_counters;
    p.counter_count = m->tc_counters ? kTcCounters : 0;
    p.acc = m->ks_acc;
    p.acc_count = m->ks_acc_count;
    return p;
}

// Projections over many rows (prefill chunks) run on the tcgen05 GEMM, which reads the weights once; the
// f32 activations go in as hi + lo 16-bit halves so the products keep about the precision of the
// f32-activation GEMV. int8 weights qualify with one scale per row (exact f16 integers times the row
// scale in the epilogue, as on the GEMV); group-wise int8 and everything else runs on the GEMV.
bool tc_takes(const l0b_model* m, const ModelMatrix& w, const GemvParams& p) {
    if (!m->x16 || m->tc_rows <= 0 || p.M < m->tc_rows) return false;
    if (w.dtype != L0B_F16 && w.dtype != L0B_BF16 && !(w.dtype == L0B_I8 && w.group >= w.k)) return false;
    if (p.nseg != 1 || p.x_dtype != L0B_F32 || p.out_dtype != L0B_F32) return false;
    if (p.epi != EPI_STORE && p.epi != EPI_ACCUM && p.epi != EPI_SWIGLU && p.epi != EPI_ARGMAX) return false;
    const int cols = p.epi == EPI_SWIGLU ? w.n / 2 : w.n;
    if (p.seg[0].row_end != cols) return false;
    return tc_gemm_supported(w.dtype, p.M, w.n, w.k, p.epi);
}

l0b_status gemv(l0b_model* m, const ModelMatrix& w, const GemvParams& p) {
    if (!tc_takes(m, w, p)) return gemv_nk_launch(m->dev, w.dtype, p);
    const TcPlan plan = tc_gemm_plan(p.M, w.n, w.k, p.epi, true, w.dtype, m->dev->sm_count);
    L0B_TRY(cast_rows_split_launch(m->dev, static_cast<const float*>(p.x), p.x_ld, p.norm_w, p.eps, m->x16,
                                   m->rscale, w.dtype, p.M, w.k, plan));
    TcGemmArgs a;
    a.part = m->tc_part;
    a.part_floats = tc_gemm_part_floats(m->dev->sm_count);
    a.counters = m->tc_counters;
    a.counter_count = kTcCounters;
    a.M = p.M;
    a.N = w.n;
    a.K = w.k;
    a.x16 = m->x16;
    a.w = w.w;
    a.wdtype = w.dtype;
    a.epi = p.epi;
    a.out = static_cast<float*>(p.seg[0].out);
    a.ld = p.seg[0].ld;
    a.bias = p.seg[0].bias;
    a.split = 1;
    a.rscale = m->rscale;
    a.wscale = w.dtype == L0B_I8 ? w.scales : nullptr;
    a.kb = w.kb;
    a.argmax = p.argmax;
    a.argmax_base = p.argmax_base;
    return tc_gemm_launch(m->dev, a);
}

// Probe (LlmDecoderLayer.Emit, L/LlmDecoderLayer.cs:427): hand a host copy of row 0 of a stage buffer to
// the callback. Only reached when the step runs unrecorded.
l0b_status emit(l0b_model* m, int li, const char* stage, const float* dptr, long long count) {
    if (!m->probe) return L0B_OK;
    m->probe_host.resize(static_cast<size_t>(count));
    L0B_CHECK_CUDA(cudaStreamSynchronize(m->dev->stream));
    L0B_CHECK_CUDA(copy_sync(m->dev->stream, m->probe_host.data(), dptr, count * sizeof(float), cudaMemcpyDeviceToHost));
    m->probe(m->probe_user, li, stage, m->probe_host.data(), count);
    return L0B_OK;
}

// A row-split projection under TP, folded into the residual stream. Where the register-streamed
// tensor-core GEMV takes it (decode rows of 16-bit or row-major int8 weights) and the communicator has
// peer mailboxes, one kernel does both: each CTA sends its tiles' partials to every rank and adds every
// rank's partials of the same tiles to `hidden` in rank order. Otherwise (the tcgen05 GEMM's rows, the
// k-split GEMV's blocked int8) one in-place all-reduce after the GEMV: rank 0 accumulates its partial
// into `hidden`, the other ranks store theirs there, so the sum over ranks is hidden + the partials on
// every rank. Both give ((hidden + p0) + p1) + ... in fp32 over the same partials, the same bits.
l0b_status project_into_residual(l0b_model* m, const ModelMatrix& w, GemvParams p, int rows) {
    if (const PeerSum* ps = comm_peer_sum(m->comm)) {
        GemvParams q = p;
        q.epi = EPI_PEER_SUM;
        q.out_dtype = L0B_F32;
        q.seg[0] = {m->hidden, nullptr, m->h, m->h};
        q.peer = ps;
        GemvParams t = q;
        t.epi = EPI_ACCUM;  // what the pair would run: the tcgen05 GEMM or the k-split GEMV stay in the pair
        if (!tc_takes(m, w, t) && !gemv_takes_ksplit(w.dtype, t, m->dev->sm_count) &&
            gemv_peer_sum_applies(w.dtype, q))
            return gemv_nk_launch(m->dev, w.dtype, q);
    }
    p.epi = m->tp_rank == 0 ? EPI_ACCUM : EPI_STORE;
    p.out_dtype = L0B_F32;
    p.seg[0] = {m->hidden, nullptr, m->h, m->h};
    L0B_TRY(gemv(m, w, p));
    return comm_allreduce(m->comm, m->hidden, static_cast<size_t>(rows) * m->h, L0B_F32, COLL_SUM);
}

// Fused decoder layer for `rows` tokens. decode: each row is its own sequence (cache row b, position
// pos[b]); prefill: the rows are consecutive positions of sequence 0 starting at pos0.
l0b_status record_layer_fused(l0b_model* m, int li, int rows, bool decode, int pos0) {
    ModelLayer& L = m->layers[li];
    const l0b_model_config& c = m->cfg;
    // L2 prefetch plan of the one-row decode step (l0b_set_l2_prefetch): the latency-bound k-split GEMVs
    // pull the weights of the projections after them into L2 (weights only: a row-major int8 matrix's
    // bytes, without its scales).
    const long long pf_gate_up = decode && rows == 1 && !m->comm ? 1048576LL * gemv_l2_prefetch_mb() : 0;
    auto w_bytes = [](const ModelMatrix& w) {
        return static_cast<long long>(w.n) * w.k * dtype_size(static_cast<l0b_dtype>(w.dtype));
    };
    // 1. QKV projection with the input RMSNorm prologue and the bias epilogue.
    GemvParams p = model_linear_params(m, L.qkv, rows, m->hidden, m->h);
    p.norm_w = L.in_norm;
    p.eps = c.rms_norm_eps;
    p.seg[0] = {m->qkv, L.qkv_bias, m->qkv_w, m->qkv_w};
    if (pf_gate_up > 0) {
        p.l2pf[0] = L.o.w;
        p.l2pf_bytes[0] = w_bytes(L.o);
    }
    L0B_TRY(gemv(m, L.qkv, p));
    // QK-norm (Qwen3): each query and key head RMS-normalised in place before RoPE.
    if (c.qk_norm)
        L0B_TRY(k_head_norm(m->dev, m->qkv, m->qkv_w, m->nh, m->nkv, m->hd, L.q_norm, L.k_norm, c.rms_norm_eps, rows));
    // 2. Attention.
    AttnParams a = {};
    a.q = m->qkv;
    a.q_bstride = m->qkv_w;
    a.inv_freq = m->inv_freq;
    a.rot = m->rot;
    a.attn_scale = m->attn_scale;
    a.kc = L.kc;
    a.vc = L.vc;
    a.cache_dtype = m->cache_dtype;
    a.kv_dim = m->kvdim;
    a.out = m->attn;
    a.out_bstride = m->qdim;
    a.nh = m->nh;
    a.nkv = m->nkv;
    a.hd = m->hd;
    a.scale = m->softmax_scale;
    if (decode) {
        a.rope = 1;
        a.store_new = 1;
        a.k_new = m->qkv + m->qdim;
        a.v_new = m->qkv + m->qdim + m->kvdim;
        a.new_bstride = m->qkv_w;
        a.cache_bstride = static_cast<long long>(m->max_seq) * m->kvdim;
        a.positions = m->pos;
        a.chunk = 32;
        L0B_TRY(attention_cluster_launch(m->dev, a, rows, cluster_splits(m, rows)));
    } else {
        // Prefill: rotate and store the whole chunk first (queries attend to each other's keys).
        L0B_TRY(k_rope(m->dev, m->qkv, m->qkv + m->qdim, m->prompt_pos, m->inv_freq, m->hd, m->nh, m->nkv,
                       m->attn_scale, m->rot, rows, m->qkv_w, m->qkv_w));
        void* kc = seq_cache(m, L.kc);
        void* vc = seq_cache(m, L.vc);
        L0B_TRY(k_kv_store(m->dev, m->qkv + m->qdim, m->qkv + m->qdim + m->kvdim, kc, vc, m->cache_dtype, pos0,
                           m->kvdim, rows, m->qkv_w));
        a.kc = kc;
        a.vc = vc;
        a.rope = 0;
        a.store_new = 0;
        a.cache_bstride = 0;
        a.positions = m->prompt_pos;
        a.chunk = (pos0 + rows + 31) / 32 * 32;
        a.max_splits = 1;
        L0B_TRY(attention_launch(m->dev, a, rows));
    }
    // 3. o_proj, added into the residual stream (under TP: this rank's partial, summed over ranks).
    p = model_linear_params(m, L.o, rows, m->attn, m->qdim);
    if (m->comm) {
        L0B_TRY(project_into_residual(m, L.o, p, rows));
    } else {
        if (pf_gate_up > 0) {
            // The first rows of the gate half and of the up half ([gate; up] is stacked row-major).
            const long long half = w_bytes(L.gate_up) / 2;
            const long long each = std::min(pf_gate_up / 2, half);
            p.l2pf[0] = L.gate_up.w;
            p.l2pf_bytes[0] = each;
            p.l2pf[1] = static_cast<const char*>(L.gate_up.w) + half;
            p.l2pf_bytes[1] = each;
        }
        p.epi = EPI_ACCUM;
        p.seg[0] = {m->hidden, nullptr, m->h, m->h};
        L0B_TRY(gemv(m, L.o, p));
    }
    // 4. gate/up with the post-attention RMSNorm prologue and the SwiGLU epilogue.
    p = model_linear_params(m, L.gate_up, rows, m->hidden, m->h);
    p.norm_w = L.post_norm;
    p.eps = c.rms_norm_eps;
    p.epi = EPI_SWIGLU;
    p.seg[0] = {m->act, nullptr, m->inter, m->inter};
    L0B_TRY(gemv(m, L.gate_up, p));
    // 5. down, added into the residual stream.
    p = model_linear_params(m, L.down, rows, m->act, m->inter);
    if (m->comm) return project_into_residual(m, L.down, p, rows);
    if (pf_gate_up > 0 && li + 1 < c.num_layers) {
        p.l2pf[0] = m->layers[li + 1].qkv.w;
        p.l2pf_bytes[0] = w_bytes(m->layers[li + 1].qkv);
    }
    p.epi = EPI_ACCUM;
    p.seg[0] = {m->hidden, nullptr, m->h, m->h};
    return gemv(m, L.down, p);
}

l0b_status record_layer_tail(l0b_model* m, int li, int rows);

// LlmDecoderLayer.MixLinear (L/LlmDecoderLayer.cs:381-397) for `rows` consecutive tokens of the sequence at
// pos0, pos0 + 1, ...: the four in-projections in one launch ([qkv; z; b; a] stacked, ProjectShared), the
// causal conv + SiLU over the conv window, the gated delta rule over the recurrent state (both reset when
// the rows start at position 0), out_proj into attn_proj.
l0b_status record_mix_linear(l0b_model* m, ModelLayer& L, int rows, int pos0) {
    const l0b_model_config& c = m->cfg;
    l0b_device* d = m->dev;
    const int cd = m->lin_cd, vd = m->lin_vd, hv = m->lin_hv;
    GemvParams p = model_linear_params(m, L.lin_in, rows, m->normed, m->h);
    p.nseg = 4;
    p.seg[0] = {m->lq, nullptr, cd, cd};
    p.seg[1] = {m->lz, nullptr, cd + vd, vd};
    p.seg[2] = {m->lb, nullptr, cd + vd + hv, hv};
    p.seg[3] = {m->la, nullptr, cd + vd + 2 * hv, hv};
    L0B_TRY(gemv(m, L.lin_in, p));
    if (pos0 == 0) {  // LlmLinearState.Reset at position 0
        L0B_TRY(k_fill_u32(d, reinterpret_cast<uint32_t*>(L.conv_state), 0u, cd * (m->lin_kconv - 1)));
        L0B_TRY(k_fill_u32(d, reinterpret_cast<uint32_t*>(L.rec_state), 0u, hv * m->lin_dk * m->lin_dv));
    }
    L0B_TRY(k_causal_conv(d, m->lq, L.conv_state, L.conv_w, m->lc, cd, m->lin_kconv, rows));
    L0B_TRY(k_gated_delta(m->suite, d, m->lc, m->lz, m->lb, m->la, L.a_log, L.dt_bias, L.lin_norm, L.rec_state, m->lo,
                          m->lin_hk, hv, m->lin_dk, m->lin_dv, rows, c.rms_norm_eps));
    p = model_linear_params(m, L.lin_out, rows, m->lo, vd);
    p.seg[0] = {m->attn_proj, nullptr, m->h, m->h};
    return gemv(m, L.lin_out, p);
}

// The reference op sequence of LlmDecoderLayer.Forward / ForwardBatch (L/LlmDecoderLayer.cs:129-378).
l0b_status record_layer_reference(l0b_model* m, int li, int rows, bool decode, int pos0) {
    ModelLayer& L = m->layers[li];
    const l0b_model_config& c = m->cfg;
    l0b_device* d = m->dev;
    L0B_TRY(k_rmsnorm(d, m->hidden, nullptr, L.in_norm, m->normed, c.rms_norm_eps, m->h, rows, 0));
    L0B_TRY(emit(m, li, "input_norm", m->normed, m->h));
    if (L.linear) {
        L0B_TRY(record_mix_linear(m, L, rows, pos0));
        return record_layer_tail(m, li, rows);
    }
    GemvParams p = model_linear_params(m, L.qkv, rows, m->normed, m->h);
    p.nseg = 3;
    p.seg[0] = {m->qb, nullptr, m->qdim, m->qdim};
    p.seg[1] = {m->kb, nullptr, m->qdim + m->kvdim, m->kvdim};
    p.seg[2] = {m->vb, nullptr, m->qkv_w, m->kvdim};
    if (c.attention_output_gate) {  // Qwen3.5: the gate rows stacked after v
        p.nseg = 4;
        p.seg[3] = {m->gb, nullptr, m->qkv_w + m->qdim, m->qdim};
    }
    L0B_TRY(gemv(m, L.qkv, p));
    if (L.qkv_bias) {
        L0B_TRY(k_bias_add(d, m->qb, L.qkv_bias, m->qdim, rows));
        L0B_TRY(k_bias_add(d, m->kb, L.qkv_bias + m->qdim, m->kvdim, rows));
        L0B_TRY(k_bias_add(d, m->vb, L.qkv_bias + m->qdim + m->kvdim, m->kvdim, rows));
    }
    if (c.qk_norm) {
        L0B_TRY(k_rmsnorm(d, m->qb, nullptr, L.q_norm, m->qb, c.rms_norm_eps, m->hd, rows * m->nh, 0));
        L0B_TRY(k_rmsnorm(d, m->kb, nullptr, L.k_norm, m->kb, c.rms_norm_eps, m->hd, rows * m->nkv, 0));
    }
    L0B_TRY(emit(m, li, "q", m->qb, m->qdim));
    L0B_TRY(emit(m, li, "k", m->kb, m->kvdim));
    L0B_TRY(emit(m, li, "v", m->vb, m->kvdim));
    const int* positions = decode ? m->pos : m->prompt_pos;
    L0B_TRY(k_rope(d, m->qb, m->kb, positions, m->inv_freq, m->hd, m->nh, m->nkv, m->attn_scale, m->rot, rows));
    // Decode on this path is single-sequence (row 0); prefill writes the sequence being ingested.
    void* kc = decode ? L.kc : seq_cache(m, L.kc);
    void* vc = decode ? L.vc : seq_cache(m, L.vc);
    L0B_TRY(k_kv_store(d, m->kb, m->vb, kc, vc, m->cache_dtype, pos0, m->kvdim, rows));
    AttnParams a = {};
    a.q = m->qb;
    a.q_bstride = m->qdim;
    a.kc = kc;
    a.vc = vc;
    a.cache_dtype = m->cache_dtype;
    a.kv_dim = m->kvdim;
    a.out = m->attn;
    a.out_bstride = m->qdim;
    a.nh = m->nh;
    a.nkv = m->nkv;
    a.hd = m->hd;
    a.scale = m->softmax_scale;
    a.pos_base = pos0;
    a.pos_step = 1;
    if (decode) {
        a.chunk = 32;
        L0B_TRY(attention_cluster_launch(d, a, rows, cluster_splits(m, rows)));
    } else {
        a.chunk = (pos0 + rows + 31) / 32 * 32;
        a.max_splits = 1;
        L0B_TRY(attention_launch(d, a, rows));
    }
    // MixFull's optional sigmoid output gate before o_proj (L/LlmDecoderLayer.cs:328-331,372-375).
    if (c.attention_output_gate) L0B_TRY(k_sigmoid_gate(d, m->attn, m->gb, static_cast<long long>(rows) * m->qdim));
    p = model_linear_params(m, L.o, rows, m->attn, m->qdim);
    p.seg[0] = {m->attn_proj, nullptr, m->h, m->h};
    L0B_TRY(gemv(m, L.o, p));
    if (m->comm) L0B_TRY(comm_allreduce(m->comm, m->attn_proj, static_cast<size_t>(rows) * m->h, L0B_F32, COLL_SUM));
    return record_layer_tail(m, li, rows);
}

// Forward steps 3-5 after the token mixer's output is in attn_proj: residual + post-attention RMSNorm,
// gate/up + SwiGLU, down, residual add (L/LlmDecoderLayer.cs:178-195).
l0b_status record_layer_tail(l0b_model* m, int li, int rows) {
    ModelLayer& L = m->layers[li];
    const l0b_model_config& c = m->cfg;
    l0b_device* d = m->dev;
    GemvParams p;
    L0B_TRY(emit(m, li, "attn_out", m->attn_proj, m->h));
    L0B_TRY(k_rmsnorm(d, m->hidden, m->attn_proj, L.post_norm, m->normed, c.rms_norm_eps, m->h, rows, 1));
    L0B_TRY(emit(m, li, "post_norm", m->normed, m->h));
    p = model_linear_params(m, L.gate_up, rows, m->normed, m->h);
    p.nseg = 2;
    p.seg[0] = {m->gate, nullptr, m->inter, m->inter};
    p.seg[1] = {m->up, nullptr, 2 * m->inter, m->inter};
    L0B_TRY(gemv(m, L.gate_up, p));
    L0B_TRY(k_swiglu(d, m->gate, m->up, static_cast<long long>(rows) * m->inter));
    p = model_linear_params(m, L.down, rows, m->gate, m->inter);
    p.seg[0] = {m->down, nullptr, m->h, m->h};
    L0B_TRY(gemv(m, L.down, p));
    if (m->comm) L0B_TRY(comm_allreduce(m->comm, m->down, static_cast<size_t>(rows) * m->h, L0B_F32, COLL_SUM));
    L0B_TRY(emit(m, li, "mlp_out", m->down, m->h));
    L0B_TRY(k_add(d, m->hidden, m->down, static_cast<long long>(rows) * m->h));
    return emit(m, li, "output", m->hidden, m->h);
}

// Final norm, LM head and greedy argmax for `rows` rows starting at hidden row `row0`; the greedy token,
// position and argmax key of row r go to sequence slot seq0 + r.
l0b_status record_head(l0b_model* m, int row0, int rows, int advance, int seq0 = 0) {
    const l0b_model_config& c = m->cfg;
    l0b_device* d = m->dev;
    if (m->fused && !m->probe) {
        GemvParams p = model_linear_params(m, m->lm_head, rows, m->hidden + static_cast<long long>(row0) * m->h, m->h);
        p.norm_w = m->final_norm;
        p.eps = c.rms_norm_eps;
        p.epi = EPI_ARGMAX;
        p.argmax = m->keys + seq0;
        p.argmax_base = m->tp_rank * m->vocab;
        p.seg[0] = {m->logits, nullptr, m->vocab, m->vocab};
        L0B_TRY(gemv(m, m->lm_head, p));
    } else {
        // L/LlmModel.cs:365-399: Copy the last row, RMSNorm, lm_head, Sampling (argmax).
        const float* src = m->hidden;
        if (row0 > 0) {
            L0B_TRY(k_copy(d, m->hidden, m->head_in, static_cast<long long>(row0) * m->h,
                           static_cast<long long>(rows) * m->h));
            src = m->head_in;
        }
        L0B_TRY(k_rmsnorm(d, const_cast<float*>(src), nullptr, m->final_norm, m->normed, c.rms_norm_eps, m->h, rows, 0));
        GemvParams p = model_linear_params(m, m->lm_head, rows, m->normed, m->h);
        p.epi = EPI_ARGMAX;
        p.argmax = m->keys + seq0;
        p.argmax_base = m->tp_rank * m->vocab;
        p.seg[0] = {m->logits, nullptr, m->vocab, m->vocab};
        L0B_TRY(gemv(m, m->lm_head, p));
    }
    // Under TP each rank holds the argmax of its vocab shard (global indices): the largest key wins.
    if (m->comm) L0B_TRY(comm_allreduce(m->comm, m->keys + seq0, rows, kDtypeU64, COLL_MAX));
    // A sampled decode replaces the greedy key with the drawn token's (position of the new token:
    // the input position + 1), and records the token in the context bitmap.
    if (m->sampling && seq0 == 0 && rows == 1)
        L0B_TRY(sample_step(d, m->logits, m->vocab_full, m->seen, m->s_temperature, m->s_top_p, m->s_top_k,
                            m->s_penalty, m->skeys, 0.0, m->s_seed, m->pos, 1, nullptr, m->keys, m->seen));
    return d->launch(step_finish_kernel, dim3(1), dim3(rows < 32 ? 32 : ((rows + 31) / 32) * 32), 0, m->keys + seq0,
                     m->sampled + seq0, m->tok + seq0, m->pos + seq0, seq0 ? nullptr : m->out_tokens, m->step_idx,
                     rows, advance);
}

// One decode step for `rows` sequences whose token ids and positions are already in tok/pos.
l0b_status record_decode_step(l0b_model* m, int rows) {
    l0b_device* d = m->dev;
    L0B_TRY(d->launch(step_begin_kernel, dim3(grid_for(static_cast<long long>(rows) * m->h, d->sm_count)), dim3(256),
                      0, m->tok, m->embed, m->hidden, m->h, rows, m->vocab_full, m->keys, rows));
    for (int li = 0; li < static_cast<int>(m->layers.size()); ++li) {
        if (m->fused && !m->probe) L0B_TRY(record_layer_fused(m, li, rows, true, 0));
        else {
            // The reference sequence reads the position as an argument (KvCacheStore pos0, Attention seqLen).
            L0B_TRY(record_layer_reference(m, li, rows, true, m->position));
        }
    }
    return record_head(m, 0, rows, 1);
}

// One prefill chunk of `count` tokens at positions [pos0, pos0 + count); prompt_tok / prompt_pos hold them.
l0b_status record_prefill_chunk(l0b_model* m, int count, int pos0, bool head) {
    l0b_device* d = m->dev;
    L0B_TRY(d->launch(step_begin_kernel, dim3(grid_for(static_cast<long long>(count) * m->h, d->sm_count)),
                      dim3(256), 0, m->prompt_tok, m->embed, m->hidden, m->h, count, m->vocab_full,
                      m->keys + m->prefill_seq, 1));
    for (int li = 0; li < static_cast<int>(m->layers.size()); ++li) {
        if (m->fused && !m->probe) L0B_TRY(record_layer_fused(m, li, count, false, pos0));
        else L0B_TRY(record_layer_reference(m, li, count, false, pos0));
    }
    if (head) L0B_TRY(record_head(m, count - 1, 1, 0, m->prefill_seq));
    return L0B_OK;
}

// Runs `body` as one command list (or immediately when recording is off) and waits.
template <typename Body>
l0b_status run_recorded(l0b_model* m, Body body, bool wait = true) {
    l0b_device* d = m->dev;
    L0B_CHECK_CUDA(cudaSetDevice(d->index));
    if (m->recording && !m->probe) {
        L0B_REQUIRE(!d->recording, L0B_ERR_INVALID_OPERATION, "the device is already recording");
        d->recording = true;
        d->log_used = 0;
        l0b_status s = body();
        if (s != L0B_OK) {
            d->abort_recording();
            return s;
        }
        L0B_TRY(d->end_recording());
    } else {
        L0B_TRY(body());
    }
    if (wait) L0B_CHECK_CUDA(cudaStreamSynchronize(d->stream));
    return L0B_OK;
}

// Tokens and positions of sequences 0..rows-1 to the device. Only those rows are copied: the other
// sequences keep their device-side token and position (a batched device decode continues from them).
l0b_status write_io(l0b_model* m, int rows, const int* tokens, const int* positions) {
    for (int b = 0; b < rows; ++b) {
        m->host_io[b] = tokens[b];
        m->host_io[m->batch_cap + b] = positions[b];
    }
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->tok, m->host_io, sizeof(int) * rows, cudaMemcpyHostToDevice, m->dev->stream));
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->pos, m->host_io + m->batch_cap, sizeof(int) * rows, cudaMemcpyHostToDevice,
                                   m->dev->stream));
    return L0B_OK;
}

// Sequence 0's length: the single-sequence calls keep it in `position`, the batched ones in seq_pos[0].
// Every change goes through here so the two never drift apart.
void set_position0(l0b_model* m, int position) {
    m->position = position;
    m->seq_pos[0] = position;
}

l0b_status read_logits(l0b_model* m, float* out, int rows) {
    if (!out) return L0B_OK;
    const size_t bytes = static_cast<size_t>(rows) * m->vocab * sizeof(float);
    if (m->comm) {
        // Every rank joins the gather (each holds a vocab shard); rows come back as [rank][row][shard].
        L0B_TRY(comm_allgather(m->comm, m->logits, m->logits_all, static_cast<size_t>(rows) * m->vocab, L0B_F32));
        L0B_CHECK_CUDA(cudaMemcpyAsync(m->host_logits, m->logits_all, bytes * m->tp, cudaMemcpyDeviceToHost,
                                       m->dev->stream));
        L0B_CHECK_CUDA(cudaStreamSynchronize(m->dev->stream));
        const size_t full = static_cast<size_t>(m->vocab) * m->tp;
        for (int r = 0; r < m->tp; ++r)
            for (int b = 0; b < rows; ++b)
                std::memcpy(out + b * full + static_cast<size_t>(r) * m->vocab,
                            m->host_logits + (static_cast<size_t>(r) * rows + b) * m->vocab, m->vocab * sizeof(float));
        return L0B_OK;
    }
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->host_logits, m->logits, bytes, cudaMemcpyDeviceToHost, m->dev->stream));
    L0B_CHECK_CUDA(cudaStreamSynchronize(m->dev->stream));
    std::memcpy(out, m->host_logits, bytes);
    return L0B_OK;
}

// LlmModel.Step (L/LlmModel.cs:402-444): one token at `position`.
l0b_status step(l0b_model* m, int token, int position) {
    L0B_REQUIRE(token >= 0 && token < m->vocab_full, L0B_ERR_OUT_OF_RANGE, "Vocabulary has %d tokens (got %d).", m->vocab_full,
                token);
    L0B_REQUIRE(position >= 0 && position < m->max_seq, L0B_ERR_OUT_OF_RANGE, "Cache holds %d positions.", m->max_seq);
    L0B_TRY(write_io(m, 1, &token, &position));
    const int saved = m->position;
    m->position = position;  // the reference sequence passes it as an argument
    l0b_status s = run_recorded(m, [&] { return record_decode_step(m, 1); });
    m->position = saved;
    return s;
}

// LlmModel.IngestPrompt (L/LlmModel.cs:320-333): chunks of kPrefillRows tokens (the reference chunks by
// LlmGemvKernel.MaxRows; here a chunk is one tensor-core GEMM per projection, which reads each weight
// once per chunk, so larger chunks stream the weights fewer times); a 1-token chunk is a Step.
// `seq` selects the cache row (sequence) for a batched model; sequences other than 0 always take the
// chunk path, whose head writes that sequence's greedy token and next position.
l0b_status ingest_prompt(l0b_model* m, const int32_t* ids, int count, int seq = 0) {
    const int chunk = kPrefillRows < m->cap ? kPrefillRows : m->cap;
    m->prefill_seq = seq;
    for (int start = 0; start < count; start += chunk) {
        const int n = count - start < chunk ? count - start : chunk;
        const bool last = start + n == count;
        for (int i = 0; i < n; ++i)
            L0B_REQUIRE(ids[start + i] >= 0 && ids[start + i] < m->vocab_full, L0B_ERR_OUT_OF_RANGE,
                        "Vocabulary has %d tokens (got %d).", m->vocab_full, ids[start + i]);
        if (n == 1 && seq == 0) {
            L0B_TRY(step(m, ids[start], start));
            continue;
        }
        std::vector<int> pos(n);
        for (int i = 0; i < n; ++i) pos[i] = start + i;
        L0B_CHECK_CUDA(cudaMemcpyAsync(m->prompt_tok, ids + start, sizeof(int) * n, cudaMemcpyHostToDevice,
                                       m->dev->stream));
        L0B_CHECK_CUDA(cudaMemcpyAsync(m->prompt_pos, pos.data(), sizeof(int) * n, cudaMemcpyHostToDevice,
                                       m->dev->stream));
        // The next decode step continues from the end of the prompt.
        if (last) {
            // Only this sequence's slot: the others keep their device-side token and position.
            m->host_io[seq] = ids[start + n - 1];
            m->host_io[m->batch_cap + seq] = start + n;
            L0B_CHECK_CUDA(cudaMemcpyAsync(m->tok + seq, &m->host_io[seq], sizeof(int), cudaMemcpyHostToDevice,
                                           m->dev->stream));
            L0B_CHECK_CUDA(cudaMemcpyAsync(m->pos + seq, &m->host_io[m->batch_cap + seq], sizeof(int),
                                           cudaMemcpyHostToDevice, m->dev->stream));
        }
        l0b_status st = run_recorded(m, [&] { return record_prefill_chunk(m, n, start, last); });
        if (st != L0B_OK) {
            m->prefill_seq = 0;
            return st;
        }
    }
    m->prefill_seq = 0;
    m->seq_pos[seq] = count;
    return L0B_OK;
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// Weight loading
// ---------------------------------------------------------------------------------------------

namespace {

// Where an HF tensor goes. Column-split tensors (q/k/v/gate/up, lm_head) keep rows [r0, r0 + rows);
// row-split tensors (o, down) keep columns [c0, c0 + cols) of every row.
struct Target {
    ModelMatrix* mat = nullptr;
    int dst_row = 0;
    float* vec = nullptr;   // f32 vector destination
    int length = 0;         // vector length (local)
    int full_rows = 0, full_cols = 0;
    int row0 = 0, rows = 0, col0 = 0, cols = 0;
    float offset = 0.f;
    uint64_t id = 0, scale_id = 0;
    bool embed = false;
    bool query_gate = false;  // Qwen3.5 q_proj: split into query rows and gate rows on load
};

bool parse_layer(const std::string& name, const std::string& prefix, int* layer, std::string* rest) {
    if (name.compare(0, prefix.size(), prefix) != 0) return false;
    size_t p = prefix.size();
    size_t dot = name.find('.', p);
    if (dot == std::string::npos) return false;
    *layer = std::atoi(name.substr(p, dot - p).c_str());
    *rest = name.substr(dot + 1);
    return true;
}

// Where checkpoint tensor `name` goes for rank c.tp_rank of c.tp_size: pure arithmetic on the config
// (l0b_model_shard_plan exports it). Column-split projections (q/k/v, gate/up, lm_head) keep whole output
// rows [row0, row0 + rows) -- q/k/v whole heads, so each rank's query heads keep their KV head -- placed
// at dst_row of the stacked local matrix; row-split ones (o_proj, down) keep input columns
// [col0, col0 + cols) of every row; the q/k/v biases follow their projection's rows; norms and the
// embedding table are replicated. *tkind: the TensorKind of a layer tensor (ids of the synthetic
// generator), -1 otherwise.
l0b_status shard_plan(const l0b_model_config& c, const std::string& name, l0b_shard_plan* sp, int* tkind) {
    const int tp = c.tp_size > 1 ? c.tp_size : 1, rank = c.tp_size > 1 ? c.tp_rank : 0;
    const int H = c.hidden_size, I = c.intermediate_size;
    const int QD = c.num_attention_heads * c.head_dim, KD = c.num_key_value_heads * c.head_dim;
    const int qd = QD / tp, kd = KD / tp, inter = I / tp, vocab = c.vocab_size / tp;
    *sp = l0b_shard_plan{};
    *tkind = -1;
    sp->layer = -1;
    auto matrix = [&](int slot, int full_rows, int full_cols) {
        sp->kind = L0B_SHARD_MATRIX;
        sp->slot = slot;
        sp->full_rows = full_rows;
        sp->full_cols = full_cols;
        sp->rows = full_rows;
        sp->cols = full_cols;
    };
    auto col_split = [&](int slot, int dst_row, int full_rows, int kind) {
        matrix(slot, full_rows, H);
        sp->rows = full_rows / tp;
        sp->row0 = rank * sp->rows;
        sp->dst_row = dst_row;
        *tkind = kind;
    };
    auto row_split = [&](int slot, int full_cols, int kind) {
        matrix(slot, H, full_cols);
        sp->cols = full_cols / tp;
        sp->col0 = rank * sp->cols;
        *tkind = kind;
    };
    auto vec = [&](int slot, int full, int local, int src_off, int dst_off, int kind) {
        sp->kind = L0B_SHARD_VECTOR;
        sp->slot = slot;
        sp->full_rows = 1;
        sp->full_cols = full;
        sp->rows = 1;
        sp->cols = local;
        sp->col0 = src_off;
        sp->dst_row = dst_off;
        *tkind = kind;
    };
    if (name == "model.embed_tokens.weight") {
        matrix(0, c.vocab_size, H);
        sp->kind = L0B_SHARD_EMBEDDING;
        return L0B_OK;
    }
    if (name == "model.norm.weight") {
        vec(L0B_SLOT_FINAL_NORM, H, H, 0, 0, -1);
        return L0B_OK;
    }
    if (name == "lm_head.weight") {
        matrix(L0B_SLOT_LM_HEAD, c.vocab_size, H);
        sp->rows = vocab;
        sp->row0 = rank * vocab;
        return L0B_OK;
    }
    int li;
    std::string rest;
    if (!parse_layer(name, "model.layers.", &li, &rest) || li < 0 || li >= c.num_layers)
        return fail(L0B_ERR_INVALID_DATA, "unknown tensor '%s'", name.c_str());
    sp->layer = li;
    const bool linear = li < 64 && ((c.linear_layer_mask >> li) & 1ULL);
    if (linear) {
        // A Gated DeltaNet layer (LlmLayerWeights.Load, L/LlmLayerWeights.cs:146-163): its in-projections
        // stacked [qkv; z; b; a] in one matrix, out_proj, conv taps [conv_dim, k], A_log, dt_bias, norm.
        const int hv = c.linear_num_value_heads, dv = c.linear_value_head_dim;
        const int cd = 2 * c.linear_num_key_heads * c.linear_key_head_dim + hv * dv, vd = hv * dv;
        if (rest == "input_layernorm.weight") vec(L0B_SLOT_IN_NORM, H, H, 0, 0, T_IN_NORM);
        else if (rest == "post_attention_layernorm.weight") vec(L0B_SLOT_POST_NORM, H, H, 0, 0, T_POST_NORM);
        else if (rest == "mlp.gate_proj.weight") col_split(L0B_SLOT_GATE_UP, 0, I, T_GATE);
        else if (rest == "mlp.up_proj.weight") col_split(L0B_SLOT_GATE_UP, inter, I, T_UP);
        else if (rest == "mlp.down_proj.weight") row_split(L0B_SLOT_DOWN, I, T_DOWN);
        else if (rest == "linear_attn.in_proj_qkv.weight") col_split(L0B_SLOT_LIN_IN, 0, cd, -1);
        else if (rest == "linear_attn.in_proj_z.weight") col_split(L0B_SLOT_LIN_IN, cd, vd, -1);
        else if (rest == "linear_attn.in_proj_b.weight") col_split(L0B_SLOT_LIN_IN, cd + vd, hv, -1);
        else if (rest == "linear_attn.in_proj_a.weight") col_split(L0B_SLOT_LIN_IN, cd + vd + hv, hv, -1);
        else if (rest == "linear_attn.out_proj.weight") row_split(L0B_SLOT_LIN_OUT, vd, -1);
        else if (rest == "linear_attn.conv1d.weight") {
            const int n = cd * c.linear_conv_kernel;
            vec(L0B_SLOT_LIN_CONV, n, n, 0, 0, -1);
        } else if (rest == "linear_attn.A_log") vec(L0B_SLOT_LIN_A_LOG, hv, hv, 0, 0, -1);
        else if (rest == "linear_attn.dt_bias") vec(L0B_SLOT_LIN_DT_BIAS, hv, hv, 0, 0, -1);
        else if (rest == "linear_attn.norm.weight") vec(L0B_SLOT_LIN_NORM, dv, dv, 0, 0, -1);
        else return fail(L0B_ERR_INVALID_DATA, "unknown or unused tensor '%s'", name.c_str());
        return L0B_OK;
    }
    if (rest == "self_attn.q_proj.weight" && c.attention_output_gate) {
        // [query | gate] rows per head (SplitQueryAndGate): the query rows go to the top of [q; k; v; gate].
        matrix(L0B_SLOT_QKV, 2 * QD, H);
        sp->kind = L0B_SHARD_QUERY_GATE;
        sp->rows = QD;
        *tkind = T_Q;
        return L0B_OK;
    }
    if (rest == "input_layernorm.weight") vec(L0B_SLOT_IN_NORM, H, H, 0, 0, T_IN_NORM);
    else if (rest == "post_attention_layernorm.weight") vec(L0B_SLOT_POST_NORM, H, H, 0, 0, T_POST_NORM);
    else if (rest == "self_attn.q_proj.weight") col_split(L0B_SLOT_QKV, 0, QD, T_Q);
    else if (rest == "self_attn.k_proj.weight") col_split(L0B_SLOT_QKV, qd, KD, T_K);
    else if (rest == "self_attn.v_proj.weight") col_split(L0B_SLOT_QKV, qd + kd, KD, T_V);
    else if (rest == "self_attn.o_proj.weight") row_split(L0B_SLOT_O, QD, T_O);
    else if (rest == "mlp.gate_proj.weight") col_split(L0B_SLOT_GATE_UP, 0, I, T_GATE);
    else if (rest == "mlp.up_proj.weight") col_split(L0B_SLOT_GATE_UP, inter, I, T_UP);
    else if (rest == "mlp.down_proj.weight") row_split(L0B_SLOT_DOWN, I, T_DOWN);
    else if (rest == "self_attn.q_proj.bias" && c.attention_bias) vec(L0B_SLOT_QKV_BIAS, QD, qd, rank * qd, 0, T_QB);
    else if (rest == "self_attn.k_proj.bias" && c.attention_bias) vec(L0B_SLOT_QKV_BIAS, KD, kd, rank * kd, qd, T_KB);
    else if (rest == "self_attn.v_proj.bias" && c.attention_bias)
        vec(L0B_SLOT_QKV_BIAS, KD, kd, rank * kd, qd + kd, T_VB);
    else if (rest == "self_attn.q_norm.weight" && c.qk_norm) vec(L0B_SLOT_Q_NORM, c.head_dim, c.head_dim, 0, 0, T_QN);
    else if (rest == "self_attn.k_norm.weight" && c.qk_norm) vec(L0B_SLOT_K_NORM, c.head_dim, c.head_dim, 0, 0, T_KN);
    else return fail(L0B_ERR_INVALID_DATA, "unknown or unused tensor '%s'", name.c_str());
    return L0B_OK;
}

// The plan of `name` bound to this model's buffers.
l0b_status resolve(l0b_model* m, const std::string& name, Target* t) {
    l0b_shard_plan sp;
    int kind;
    L0B_TRY(shard_plan(m->cfg, name, &sp, &kind));
    t->full_rows = sp.full_rows;
    t->full_cols = sp.full_cols;
    if (sp.kind == L0B_SHARD_EMBEDDING) {
        t->embed = true;
        t->id = kIdEmbed;
        return L0B_OK;
    }
    if (sp.kind == L0B_SHARD_VECTOR) {
        float* dst = nullptr;
        if (sp.slot == L0B_SLOT_FINAL_NORM) {
            dst = m->final_norm;
            t->id = kIdFinalNorm;
        } else {
            ModelLayer& L = m->layers[sp.layer];
            switch (sp.slot) {
                case L0B_SLOT_IN_NORM: dst = L.in_norm; break;
                case L0B_SLOT_POST_NORM: dst = L.post_norm; break;
                case L0B_SLOT_QKV_BIAS: dst = L.qkv_bias; break;
                case L0B_SLOT_Q_NORM: dst = L.q_norm; break;
                case L0B_SLOT_K_NORM: dst = L.k_norm; break;
                case L0B_SLOT_LIN_CONV: dst = L.conv_w; break;
                case L0B_SLOT_LIN_A_LOG: dst = L.a_log; break;
                case L0B_SLOT_LIN_DT_BIAS: dst = L.dt_bias; break;
                case L0B_SLOT_LIN_NORM: dst = L.lin_norm; break;
                default: dst = nullptr;
            }
            if (kind >= 0) t->id = layer_tensor_id(sp.layer, kind);
        }
        // RmsNormOffset (Qwen3.5: 1) on the input, post-attention, final and q / k norms, not on the gated
        // norm of a linear layer (L/LlmLayerWeights.cs:127-129,162; L/LlmModel.cs:59).
        if (sp.slot == L0B_SLOT_IN_NORM || sp.slot == L0B_SLOT_POST_NORM || sp.slot == L0B_SLOT_FINAL_NORM ||
            sp.slot == L0B_SLOT_Q_NORM || sp.slot == L0B_SLOT_K_NORM)
            t->offset = m->cfg.rms_norm_offset;
        L0B_REQUIRE(dst, L0B_ERR_INVALID_DATA, "unknown or unused tensor '%s'", name.c_str());
        t->vec = dst + sp.dst_row;
        t->length = sp.cols;
        t->col0 = sp.col0;
        return L0B_OK;
    }
    if (sp.slot == L0B_SLOT_LM_HEAD) {
        t->mat = &m->lm_head;
        t->id = kIdLmHead;
        t->scale_id = kIdLmHeadScale;
    } else {
        ModelLayer& L = m->layers[sp.layer];
        t->mat = sp.slot == L0B_SLOT_QKV ? &L.qkv : sp.slot == L0B_SLOT_O ? &L.o
               : sp.slot == L0B_SLOT_GATE_UP ? &L.gate_up : sp.slot == L0B_SLOT_DOWN ? &L.down
               : sp.slot == L0B_SLOT_LIN_IN ? &L.lin_in : &L.lin_out;
        L0B_REQUIRE(t->mat->w, L0B_ERR_INVALID_DATA, "unknown or unused tensor '%s'", name.c_str());
        if (kind >= 0) {
            t->id = layer_tensor_id(sp.layer, kind);
            t->scale_id = layer_tensor_id(sp.layer, T_SCALE + kind);
        }
        t->query_gate = sp.kind == L0B_SHARD_QUERY_GATE;
    }
    t->dst_row = sp.dst_row;
    t->row0 = sp.row0;
    t->rows = sp.rows;
    t->col0 = sp.col0;
    t->cols = sp.cols;
    return L0B_OK;
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------

#define GUARD_BEGIN try {
#define GUARD_END                                                                                  \
    }                                                                                              \
    catch (const std::bad_alloc&) {                                                                \
        return fail(L0B_ERR_OUT_OF_MEMORY, "host allocation failed");                              \
    }                                                                                              \
    catch (const std::exception& e) {                                                              \
        return fail(L0B_ERR_INVALID_OPERATION, "%s", e.what());                                    \
    }

extern "C" {

L0B_API l0b_status l0b_model_shard_plan(const l0b_model_config* cfg, const char* name, l0b_shard_plan* out) {
    GUARD_BEGIN
    L0B_REQUIRE(cfg && name && out, L0B_ERR_ARGUMENT, "null argument");
    const int tp = cfg->tp_size > 1 ? cfg->tp_size : 1;
    L0B_REQUIRE(tp == 1 || (cfg->tp_rank >= 0 && cfg->tp_rank < tp), L0B_ERR_ARGUMENT, "tp_rank %d of %d",
                cfg->tp_rank, tp);
    L0B_REQUIRE(cfg->num_attention_heads > 0 && cfg->num_key_value_heads > 0 && cfg->head_dim > 0 &&
                    cfg->num_layers > 0 && cfg->hidden_size > 0,
                L0B_ERR_INVALID_DATA, "head counts, head_dim, layers and hidden size must be positive");
    L0B_REQUIRE(cfg->num_key_value_heads % tp == 0 && cfg->intermediate_size % tp == 0 && cfg->vocab_size % tp == 0,
                L0B_ERR_UNSUPPORTED, "kv heads, intermediate size and vocab must divide by tp_size %d", tp);
    L0B_REQUIRE(tp == 1 || (cfg->linear_layer_mask == 0 && cfg->attention_output_gate == 0), L0B_ERR_UNSUPPORTED,
                "Qwen3.5 hybrid models run on one GPU");
    int kind;
    return shard_plan(*cfg, name, out, &kind);
    GUARD_END
}

L0B_API l0b_status l0b_model_config_init(l0b_model_config* c) {
    L0B_REQUIRE(c, L0B_ERR_ARGUMENT, "config is null");
    std::memset(c, 0, sizeof(*c));
    c->max_position_embeddings = 2048;
    c->rms_norm_eps = 1e-6f;
    c->rope_theta = 10000.0;
    c->rope_type = L0B_ROPE_DEFAULT;
    c->rope_factor = 1.0;
    c->rope_low_freq_factor = 1.0;
    c->rope_high_freq_factor = 4.0;
    c->rope_beta_fast = 32.0;
    c->rope_beta_slow = 1.0;
    c->rope_truncate = 1;
    c->partial_rotary_factor = 1.0;
    c->kv_dtype = L0B_F32;
    c->q8_group = 32;
    c->tp_size = 1;
    c->tp_rank = 0;
    c->max_batch = 1;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_create(l0b_device* dev, l0b_suite* suite, const l0b_model_config* cfg, int32_t max_seq_len,
                                    l0b_precision precision, l0b_comm* comm, l0b_model** out) {
    GUARD_BEGIN
    L0B_REQUIRE(dev && suite && cfg && out, L0B_ERR_ARGUMENT, "null argument");
    *out = nullptr;
    const l0b_model_config& c = *cfg;
    // HfModelConfig.EnsureSupported (L/HfModelConfig.cs:211-257) for the fields this path reads.
    L0B_REQUIRE(c.num_attention_heads > 0 && c.num_key_value_heads > 0 && c.head_dim > 0 && c.num_layers > 0,
                L0B_ERR_INVALID_DATA, "Head counts, head_dim and layer count must be positive.");
    L0B_REQUIRE(c.num_attention_heads % c.num_key_value_heads == 0, L0B_ERR_INVALID_DATA,
                "num_attention_heads (%d) is not a multiple of num_key_value_heads (%d).", c.num_attention_heads,
                c.num_key_value_heads);
    L0B_REQUIRE(c.head_dim % 2 == 0, L0B_ERR_INVALID_DATA, "head_dim (%d) must be even for rotary embeddings.",
                c.head_dim);
    L0B_REQUIRE(c.hidden_size > 0 && c.intermediate_size > 0 && c.vocab_size > 0, L0B_ERR_INVALID_DATA,
                "hidden, intermediate and vocab sizes must be positive");
    L0B_REQUIRE(max_seq_len > 0, L0B_ERR_OUT_OF_RANGE, "maxSeqLen must be positive");
    L0B_REQUIRE(c.kv_dtype == L0B_F32 || c.kv_dtype == L0B_F16 || c.kv_dtype == L0B_BF16, L0B_ERR_ARGUMENT,
                "kv_dtype must be f32, f16 or bf16");
    const int tp = c.tp_size > 1 ? c.tp_size : 1;
    L0B_REQUIRE(tp == 1 || comm, L0B_ERR_ARGUMENT, "tensor parallelism needs a communicator");
    L0B_REQUIRE(tp == 1 || (comm_size(comm) == tp && comm_rank(comm) == c.tp_rank), L0B_ERR_ARGUMENT,
                "communicator is rank %d of %d, the config says %d of %d", comm_rank(comm), comm_size(comm),
                c.tp_rank, tp);
    L0B_REQUIRE(c.num_key_value_heads % tp == 0 && c.intermediate_size % tp == 0 && c.vocab_size % tp == 0,
                L0B_ERR_UNSUPPORTED, "kv heads, intermediate size and vocab must divide by tp_size %d", tp);
    L0B_REQUIRE(c.head_dim == 64 || c.head_dim == 128, L0B_ERR_UNSUPPORTED, "head_dim %d (64 or 128 are supported)",
                c.head_dim);
    L0B_REQUIRE((c.num_attention_heads / c.num_key_value_heads) <= 64, L0B_ERR_UNSUPPORTED, "GQA group too large");
    const bool hybrid = c.linear_layer_mask != 0 || c.attention_output_gate != 0;
    if (hybrid) {
        L0B_REQUIRE(tp == 1 && c.max_batch <= 1, L0B_ERR_UNSUPPORTED,
                    "Qwen3.5 hybrid models run on one GPU and one sequence");
        L0B_REQUIRE(c.num_layers <= 64, L0B_ERR_UNSUPPORTED, "linear_layer_mask covers 64 layers");
    }
    if (c.linear_layer_mask) {
        L0B_REQUIRE(c.linear_num_key_heads > 0 && c.linear_num_value_heads > 0 &&
                        c.linear_num_value_heads % c.linear_num_key_heads == 0,
                    L0B_ERR_INVALID_DATA, "linear value heads (%d) must be a multiple of key heads (%d)",
                    c.linear_num_value_heads, c.linear_num_key_heads);
        L0B_REQUIRE(c.linear_key_head_dim == 64 || c.linear_key_head_dim == 128, L0B_ERR_UNSUPPORTED,
                    "linear key head dim %d (64 or 128 are supported)", c.linear_key_head_dim);
        L0B_REQUIRE(c.linear_value_head_dim > 0 && c.linear_value_head_dim <= 256, L0B_ERR_UNSUPPORTED,
                    "linear value head dim %d (1..256)", c.linear_value_head_dim);
        L0B_REQUIRE(c.linear_conv_kernel >= 2 && c.linear_conv_kernel <= 8, L0B_ERR_UNSUPPORTED,
                    "linear conv kernel %d (2..8)", c.linear_conv_kernel);
    }

    std::unique_ptr<l0b_model> m(new l0b_model());
    m->dev = dev;
    m->suite = suite;
    m->cfg = c;
    m->max_seq = max_seq_len;
    m->precision = precision;
    switch (precision) {
        case L0B_PRECISION_AUTO:
        case L0B_PRECISION_INT8: m->wdtype = L0B_I8; break;
        case L0B_PRECISION_FLOAT32: m->wdtype = L0B_F32; break;
        case L0B_PRECISION_FLOAT16: m->wdtype = L0B_F16; break;
        case L0B_PRECISION_BFLOAT16: m->wdtype = L0B_BF16; break;
        default: return fail(L0B_ERR_ARGUMENT, "unknown precision %d", (int)precision);
    }
    m->group = c.q8_group;
    m->h = c.hidden_size;
    m->inter = c.intermediate_size / tp;
    m->nh = c.num_attention_heads / tp;
    m->nkv = c.num_key_value_heads / tp;
    m->hd = c.head_dim;
    m->qdim = m->nh * m->hd;
    m->kvdim = m->nkv * m->hd;
    m->qkv_w = m->qdim + 2 * m->kvdim;
    m->vocab = c.vocab_size / tp;
    m->vocab_full = c.vocab_size;
    m->cache_dtype = c.kv_dtype;
    m->softmax_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(c.head_dim)));
    m->fused = !hybrid;
    m->hybrid = hybrid;
    m->lin_hk = c.linear_num_key_heads;
    m->lin_hv = c.linear_num_value_heads;
    m->lin_dk = c.linear_key_head_dim;
    m->lin_dv = c.linear_value_head_dim;
    m->lin_kconv = c.linear_conv_kernel;
    m->lin_cd = 2 * m->lin_hk * m->lin_dk + m->lin_hv * m->lin_dv;
    m->lin_vd = m->lin_hv * m->lin_dv;
    m->tp = tp;
    m->tp_rank = tp > 1 ? c.tp_rank : 0;
    m->comm = tp > 1 ? comm : nullptr;
    m->batch_cap = c.max_batch < 1 ? 1 : c.max_batch;
    L0B_REQUIRE(m->batch_cap <= kMaxRows, L0B_ERR_OUT_OF_RANGE, "max_batch %d exceeds %d sequences", c.max_batch,
                kMaxRows);
    m->seq_pos.assign(m->batch_cap, 0);
    m->cap = kPrefillRows;
    L0B_CHECK_CUDA(cudaSetDevice(dev->index));

    std::vector<float> table;
    L0B_TRY(rope_frequencies(c, &table, &m->attn_scale));
    m->rot = static_cast<int>(table.size()) * 2;
    L0B_TRY(m->alloc(&m->inv_freq, table.size()));
    L0B_CHECK_CUDA(copy_sync(m->dev->stream, m->inv_freq, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice));

    // Weights.
    L0B_TRY(m->alloc(&m->embed, static_cast<size_t>(c.vocab_size) * m->h));
    L0B_TRY(m->alloc(&m->final_norm, m->h));
    L0B_TRY(m->alloc_matrix(m->lm_head, m->vocab, m->h, false));
    m->layers.resize(c.num_layers);
    const size_t cache_elems = static_cast<size_t>(m->batch_cap) * max_seq_len * m->kvdim;
    for (int li = 0; li < c.num_layers; ++li) {
        ModelLayer& L = m->layers[li];
        L.linear = li < 64 && ((c.linear_layer_mask >> li) & 1ULL);
        L0B_TRY(m->alloc(&L.in_norm, m->h));
        L0B_TRY(m->alloc(&L.post_norm, m->h));
        if (L.linear) {
            // Gated DeltaNet layer: no attention projections and no KV cache.
            L0B_TRY(m->alloc_matrix(L.lin_in, m->lin_cd + m->lin_vd + 2 * m->lin_hv, m->h));
            L0B_TRY(m->alloc_matrix(L.lin_out, m->h, m->lin_vd));
            L0B_TRY(m->alloc_matrix(L.gate_up, 2 * m->inter, m->h, (m->inter % 64) == 0));
            L0B_TRY(m->alloc_matrix(L.down, m->h, m->inter));
            L0B_TRY(m->alloc(&L.conv_w, static_cast<size_t>(m->lin_cd) * m->lin_kconv));
            L0B_TRY(m->alloc(&L.a_log, m->lin_hv));
            L0B_TRY(m->alloc(&L.dt_bias, m->lin_hv));
            L0B_TRY(m->alloc(&L.lin_norm, m->lin_dv));
            L0B_TRY(m->alloc(&L.conv_state, static_cast<size_t>(m->lin_cd) * (m->lin_kconv - 1)));
            L0B_TRY(m->alloc(&L.rec_state, static_cast<size_t>(m->lin_hv) * m->lin_dk * m->lin_dv));
            continue;
        }
        // [q; k; v] (+ the output gate rows of a Qwen3.5 full-attention layer).
        L0B_TRY(m->alloc_matrix(L.qkv, m->qkv_w + (c.attention_output_gate ? m->qdim : 0), m->h));
        L0B_TRY(m->alloc_matrix(L.o, m->h, m->qdim));
        L0B_TRY(m->alloc_matrix(L.gate_up, 2 * m->inter, m->h, (m->inter % 64) == 0));
        L0B_TRY(m->alloc_matrix(L.down, m->h, m->inter));
        if (c.attention_bias) L0B_TRY(m->alloc(&L.qkv_bias, m->qkv_w));
        if (c.qk_norm) {
            L0B_TRY(m->alloc(&L.q_norm, m->hd));
            L0B_TRY(m->alloc(&L.k_norm, m->hd));
        }
        char* kc;
        char* vc;
        L0B_TRY(m->alloc(&kc, cache_elems * dtype_size(static_cast<l0b_dtype>(m->cache_dtype))));
        L0B_TRY(m->alloc(&vc, cache_elems * dtype_size(static_cast<l0b_dtype>(m->cache_dtype))));
        L.kc = kc;
        L.vc = vc;
    }
    // Norms default to 1 (identity), as a freshly initialised HF model has them.
    {
        const float one = 1.f;
        std::vector<float> ones(std::max(m->h, m->hd), one);
        L0B_CHECK_CUDA(copy_sync(m->dev->stream, m->final_norm, ones.data(), m->h * sizeof(float), cudaMemcpyHostToDevice));
        for (auto& L : m->layers) {
            L0B_CHECK_CUDA(copy_sync(m->dev->stream, L.in_norm, ones.data(), m->h * sizeof(float), cudaMemcpyHostToDevice));
            L0B_CHECK_CUDA(copy_sync(m->dev->stream, L.post_norm, ones.data(), m->h * sizeof(float), cudaMemcpyHostToDevice));
            if (L.q_norm) {
                L0B_CHECK_CUDA(copy_sync(m->dev->stream, L.q_norm, ones.data(), m->hd * sizeof(float), cudaMemcpyHostToDevice));
                L0B_CHECK_CUDA(copy_sync(m->dev->stream, L.k_norm, ones.data(), m->hd * sizeof(float), cudaMemcpyHostToDevice));
            }
            if (L.lin_norm) {
                std::vector<float> ones_v(m->lin_dv, one);
                L0B_CHECK_CUDA(copy_sync(m->dev->stream, L.lin_norm, ones_v.data(), m->lin_dv * sizeof(float),
                                         cudaMemcpyHostToDevice));
            }
        }
    }
    // Activations.
    const size_t cap = static_cast<size_t>(m->cap);
    L0B_TRY(m->alloc(&m->hidden, cap * m->h));
    L0B_TRY(m->alloc(&m->normed, cap * m->h));
    L0B_TRY(m->alloc(&m->qkv, cap * m->qkv_w));
    L0B_TRY(m->alloc(&m->qb, cap * m->qdim));
    L0B_TRY(m->alloc(&m->kb, cap * m->kvdim));
    L0B_TRY(m->alloc(&m->vb, cap * m->kvdim));
    L0B_TRY(m->alloc(&m->attn, cap * m->qdim));
    L0B_TRY(m->alloc(&m->attn_proj, cap * m->h));
    if (hybrid) {
        L0B_TRY(m->alloc(&m->gb, cap * m->qdim));
        if (c.linear_layer_mask) {
            L0B_TRY(m->alloc(&m->lq, cap * m->lin_cd));
            L0B_TRY(m->alloc(&m->lc, cap * m->lin_cd));
            L0B_TRY(m->alloc(&m->lz, cap * m->lin_vd));
            L0B_TRY(m->alloc(&m->lo, cap * m->lin_vd));
            L0B_TRY(m->alloc(&m->lb, cap * m->lin_hv));
            L0B_TRY(m->alloc(&m->la, cap * m->lin_hv));
        }
    }
    L0B_TRY(m->alloc(&m->gate, cap * m->inter));
    L0B_TRY(m->alloc(&m->up, cap * m->inter));
    L0B_TRY(m->alloc(&m->act, cap * m->inter));
    L0B_TRY(m->alloc(&m->down, cap * m->h));
    L0B_TRY(m->alloc(&m->head_in, static_cast<size_t>(m->batch_cap) * m->h));
    if (m->wdtype == L0B_F16 || m->wdtype == L0B_BF16 || m->wdtype == L0B_I8) {
        int kmax = m->h > m->inter ? m->h : m->inter;
        if (m->qdim > kmax) kmax = m->qdim;
        if (m->lin_vd > kmax) kmax = m->lin_vd;  // Gated DeltaNet out_proj reads value-dim rows
        uint16_t* x16 = nullptr;
        L0B_TRY(m->alloc(&x16, (2 * cap + 256) * static_cast<size_t>(kmax)));
        m->x16 = x16;
        L0B_TRY(m->alloc(&m->rscale, cap));
        L0B_TRY(m->alloc(&m->tc_part, tc_gemm_part_floats(m->dev->sm_count)));
        L0B_TRY(m->alloc(&m->tc_counters, kTcCounters));
        m->ks_acc_count = std::max(std::max(m->qkv_w, m->h), 2 * m->inter);
        L0B_TRY(m->alloc(&m->ks_acc, static_cast<size_t>(m->ks_acc_count)));
        m->tc_rows = 8;
    }
    L0B_TRY(m->alloc(&m->logits, static_cast<size_t>(m->batch_cap) * m->vocab));
    L0B_TRY(m->alloc(&m->io, 2 * static_cast<size_t>(m->batch_cap)));
    m->tok = m->io;
    m->pos = m->io + m->batch_cap;
    L0B_TRY(m->alloc(&m->prompt_tok, cap));
    L0B_TRY(m->alloc(&m->prompt_pos, cap));
    L0B_TRY(m->alloc(&m->sampled, m->batch_cap));
    L0B_TRY(m->alloc(&m->out_tokens, static_cast<size_t>(max_seq_len + 1) * m->batch_cap));
    L0B_TRY(m->alloc(&m->step_idx, 1));
    L0B_TRY(m->alloc(&m->seen, sample_seen_words(m->vocab_full)));
    L0B_TRY(m->alloc(&m->skeys, sample_keys_words(m->vocab_full)));  // zeroed: the max word starts at 0
    L0B_TRY(m->alloc(&m->ctx_ids, static_cast<size_t>(max_seq_len) + 1));
    L0B_TRY(m->alloc(&m->keys, m->batch_cap));
    L0B_CHECK_CUDA(cudaMallocHost(&m->host_io, sizeof(int) * 2 * m->batch_cap));
    if (m->tp > 1) L0B_TRY(m->alloc(&m->logits_all, static_cast<size_t>(m->tp) * m->batch_cap * m->vocab));
    L0B_CHECK_CUDA(cudaMallocHost(&m->host_logits, sizeof(float) * m->batch_cap * m->vocab * m->tp));
    L0B_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
    *out = m.release();
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_model_free(l0b_model* model) {
    delete model;
    return L0B_OK;
}

}  // extern "C"

namespace {

// The load-time rules of LlmLayerWeights / LlmMatrix applied to one HF tensor already on the device as
// f32 (`staging`, the full tensor): norm offset, int8 quantization or 16-bit storage, the rank's shard.
l0b_status set_tensor_staged(l0b_model* m, const Target& t, const float* staging) {
    struct Free {
        float* p;
        ~Free() { cudaFree(p); }
    };
    cudaStream_t st = m->dev->stream;
    const int sm = m->dev->sm_count;
    const long long full = static_cast<long long>(t.full_rows) * t.full_cols;
    if (t.embed) {
        L0B_CHECK_CUDA(cudaMemcpyAsync(m->embed, staging, static_cast<size_t>(full) * sizeof(float),
                                       cudaMemcpyDeviceToDevice, st));
    } else if (t.vec) {
        convert_kernel<<<grid_for(t.length, sm), 256, 0, st>>>(staging, t.vec, L0B_F32, t.length, t.length, t.full_cols,
                                                                t.col0, t.offset);
    } else {
        ModelMatrix& mat = *t.mat;
        const long long count_local = static_cast<long long>(t.rows) * t.cols;
        const float* src = staging + static_cast<long long>(t.row0) * t.full_cols;
        if (mat.dtype == L0B_I8) {
            // Quantise the full rows (scales over the whole input width), then keep this rank's columns.
            float* rows_f = nullptr;
            L0B_CHECK_CUDA(cudaMalloc(&rows_f, static_cast<size_t>(t.rows) * t.full_cols * sizeof(float)));
            Free g2{rows_f};
            L0B_CHECK_CUDA(cudaMemcpyAsync(rows_f, src, static_cast<size_t>(t.rows) * t.full_cols * sizeof(float),
                                           cudaMemcpyDeviceToDevice, st));
            int8_t* q_full = nullptr;
            __half* s_full = nullptr;
            L0B_CHECK_CUDA(cudaMalloc(&q_full, static_cast<size_t>(t.rows) * t.full_cols));
            const int gfull = mat.group == mat.k ? t.full_cols : mat.group;
            L0B_CHECK_CUDA(cudaMalloc(&s_full, static_cast<size_t>(t.rows) * (t.full_cols / gfull) * sizeof(__half)));
            struct FreeV {
                void* p;
                ~FreeV() { cudaFree(p); }
            } g3{q_full}, g4{s_full};
            // Quantisation runs immediately (not recorded): load time.
            const bool was = m->dev->recording;
            m->dev->recording = false;
            l0b_status s = k_quantize(m->dev, rows_f, L0B_F32, t.rows, t.full_cols, gfull, q_full, s_full);
            m->dev->recording = was;
            L0B_TRY(s);
            if (mat.kb > 0) {
                const long long n = static_cast<long long>(t.rows) * t.cols;
                scatter_blocked_kernel<<<grid_for(n, sm), 256, 0, st>>>(q_full, t.full_cols, t.col0, t.rows, t.cols,
                                                                        static_cast<int8_t*>(mat.w), mat.k, mat.kb,
                                                                        t.dst_row);
                L0B_CHECK_CUDA(cudaGetLastError());
            } else {
                int8_t* qdst = static_cast<int8_t*>(mat.w) + static_cast<long long>(t.dst_row) * mat.k;
                L0B_CHECK_CUDA(cudaMemcpy2DAsync(qdst, mat.k, q_full + t.col0, t.full_cols, t.cols, t.rows,
                                                 cudaMemcpyDeviceToDevice, st));
            }
            if (gfull == t.full_cols) {
                L0B_REQUIRE(t.cols == t.full_cols || mat.group == mat.k, L0B_ERR_UNSUPPORTED, "scale layout");
                L0B_CHECK_CUDA(cudaMemcpyAsync(mat.scales + t.dst_row, s_full, static_cast<size_t>(t.rows) * sizeof(__half),
                                               cudaMemcpyDeviceToDevice, st));
            } else {
                const int gpr_full = t.full_cols / gfull, gpr = t.cols / gfull;
                L0B_CHECK_CUDA(cudaMemcpy2DAsync(mat.scales + static_cast<long long>(t.dst_row) * gpr,
                                                 gpr * sizeof(__half), s_full + t.col0 / gfull,
                                                 gpr_full * sizeof(__half), gpr * sizeof(__half), t.rows,
                                                 cudaMemcpyDeviceToDevice, st));
            }
            L0B_CHECK_CUDA(cudaStreamSynchronize(st));
        } else {
            char* dst = static_cast<char*>(mat.w) +
                        static_cast<long long>(t.dst_row) * mat.k * dtype_size(static_cast<l0b_dtype>(mat.dtype));
            convert_kernel<<<grid_for(count_local, sm), 256, 0, st>>>(src, dst, mat.dtype, count_local, t.cols,
                                                                       t.full_cols, t.col0, 0.f);
        }
    }
    L0B_CHECK_CUDA(cudaGetLastError());
    L0B_CHECK_CUDA(cudaStreamSynchronize(st));
    return L0B_OK;
}

// 16-bit HF tensor values (F16 or BF16 bits) widened to f32 on the device.
__global__ void widen16_kernel(const uint16_t* src, int dtype, float* dst, long long count) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint16_t b = src[i];
        dst[i] = dtype == L0B_BF16 ? __uint_as_float(static_cast<uint32_t>(b) << 16) : __half2float(__ushort_as_half(b));
    }
}

// LlmMatrix.FitsInHalf on the device: *bad = 1 when a value is not finite or exceeds 65000 in magnitude.
__global__ void half_range_kernel(const float* v, long long count, int* bad) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        if (!isfinite(v[i]) || fabsf(v[i]) > 65000.f) *bad = 1;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// SplitQueryAndGate (L/LlmLayerWeights.cs:282-297) on the host: [heads][2][hd][hidden] rows of a Qwen3.5
// q_proj become [query rows (heads * hd); gate rows (heads * hd)], elements of `elem` bytes.
std::vector<char> split_query_gate(const void* src, size_t elem, int heads, int hd, int hidden) {
    const size_t blk = static_cast<size_t>(hd) * hidden * elem;
    std::vector<char> out(2 * blk * heads);
    const char* s = static_cast<const char*>(src);
    for (int h = 0; h < heads; ++h) {
        std::memcpy(out.data() + h * blk, s + (2 * static_cast<size_t>(h)) * blk, blk);
        std::memcpy(out.data() + (heads + h) * blk, s + (2 * static_cast<size_t>(h) + 1) * blk, blk);
    }
    return out;
}

// A split q_proj in staging ([query; gate] rows): the query rows to the top of [q; k; v; gate], the gate rows
// after v.
l0b_status set_query_gate_staged(l0b_model* m, const Target& t, const float* staging) {
    Target q = t;
    q.row0 = 0;
    q.rows = m->qdim;
    q.dst_row = 0;
    L0B_TRY(set_tensor_staged(m, q, staging));
    Target g = t;
    g.row0 = m->qdim;
    g.rows = m->qdim;
    g.dst_row = m->qkv_w;
    return set_tensor_staged(m, g, staging);
}

}  // namespace

extern "C" {

L0B_API l0b_status l0b_model_set_tensor(l0b_model* m, const char* name, const float* data, int64_t count) {
    GUARD_BEGIN
    L0B_REQUIRE(m && name && data, L0B_ERR_ARGUMENT, "null argument");
    Target t;
    L0B_TRY(resolve(m, name, &t));
    const long long full = static_cast<long long>(t.full_rows) * t.full_cols;
    L0B_REQUIRE(count == full, L0B_ERR_INVALID_DATA, "Tensor '%s' has %lld values, expected %lld.", name,
                (long long)count, full);
    if (t.mat && t.mat->dtype == L0B_F16) {
        // LlmMatrix.FitsInHalf (L/LlmMatrix.cs:110-120): Float16 storage refuses values a half cannot hold.
        for (long long i = 0; i < full; ++i)
            L0B_REQUIRE(std::isfinite(data[i]) && std::fabs(data[i]) <= 65000.f, L0B_ERR_INVALID_DATA,
                        "Tensor '%s' has values outside the half-precision range.", name);
    }
    if (t.embed && m->cfg.tie_word_embeddings) {
        // Tied head: lm_head.weight is the embedding table (L/LlmModel.cs:62).
        L0B_TRY(l0b_model_set_tensor(m, "lm_head.weight", data, count));
    }
    L0B_CHECK_CUDA(cudaSetDevice(m->dev->index));
    float* staging = nullptr;
    L0B_CHECK_CUDA(cudaMalloc(&staging, static_cast<size_t>(full) * sizeof(float)));
    struct Free {
        float* p;
        ~Free() { cudaFree(p); }
    } guard{staging};
    if (t.query_gate) {
        const std::vector<char> split = split_query_gate(data, sizeof(float), m->nh, m->hd, m->h);
        L0B_CHECK_CUDA(copy_sync(m->dev->stream, staging, split.data(), static_cast<size_t>(full) * sizeof(float),
                                 cudaMemcpyHostToDevice));
        return set_query_gate_staged(m, t, staging);
    }
    L0B_CHECK_CUDA(copy_sync(m->dev->stream, staging, data, static_cast<size_t>(full) * sizeof(float), cudaMemcpyHostToDevice));
    return set_tensor_staged(m, t, staging);
    GUARD_END
}

// The raw checkpoint bytes of a 16-bit tensor (SafetensorsReader's F16 / BF16 payload) go to the device as
// they are -- half the bytes of the f32 upload -- and are widened, range-checked and converted or
// quantized there (the host-side conversion of L/SafetensorsReader.cs:262-277 and L/LlmMatrix.cs:95-105).
L0B_API l0b_status l0b_model_set_tensor_raw(l0b_model* m, const char* name, const void* data, int32_t dtype,
                                            int64_t count) {
    GUARD_BEGIN
    L0B_REQUIRE(m && name && data, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(dtype == L0B_F16 || dtype == L0B_BF16, L0B_ERR_UNSUPPORTED, "raw tensors are F16 or BF16 (dtype %d)",
                dtype);
    Target t;
    L0B_TRY(resolve(m, name, &t));
    const long long full = static_cast<long long>(t.full_rows) * t.full_cols;
    L0B_REQUIRE(count == full, L0B_ERR_INVALID_DATA, "Tensor '%s' has %lld values, expected %lld.", name,
                (long long)count, full);
    L0B_CHECK_CUDA(cudaSetDevice(m->dev->index));
    cudaStream_t st = m->dev->stream;
    const int sm = m->dev->sm_count;
    void* raw = nullptr;
    float* staging = nullptr;
    int* bad = nullptr;
    L0B_CHECK_CUDA(cudaMalloc(&raw, static_cast<size_t>(full) * 2));
    struct FreeV {
        void* p;
        ~FreeV() { cudaFree(p); }
    } g1{raw};
    L0B_CHECK_CUDA(cudaMalloc(&staging, static_cast<size_t>(full) * sizeof(float)));
    FreeV g2{staging};
    L0B_CHECK_CUDA(cudaMalloc(&bad, sizeof(int)));
    FreeV g3{bad};
    std::vector<char> split;
    if (t.query_gate) {
        split = split_query_gate(data, 2, m->nh, m->hd, m->h);
        data = split.data();
    }
    L0B_CHECK_CUDA(copy_sync(st, raw, data, static_cast<size_t>(full) * 2, cudaMemcpyHostToDevice));
    widen16_kernel<<<grid_for(full, sm), 256, 0, st>>>(static_cast<const uint16_t*>(raw), dtype, staging, full);
    L0B_CHECK_CUDA(cudaGetLastError());
    const bool f16_store = t.mat && t.mat->dtype == L0B_F16;
    const bool tied_f16 = t.embed && m->cfg.tie_word_embeddings && m->lm_head.dtype == L0B_F16;
    if (f16_store || tied_f16) {
        L0B_CHECK_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), st));
        half_range_kernel<<<grid_for(full, sm), 256, 0, st>>>(staging, full, bad);
        int h = 0;
        L0B_CHECK_CUDA(copy_sync(st, &h, bad, sizeof(int), cudaMemcpyDeviceToHost));
        L0B_REQUIRE(!h, L0B_ERR_INVALID_DATA, "Tensor '%s' has values outside the half-precision range.", name);
    }
    if (t.embed && m->cfg.tie_word_embeddings) {
        Target head;
        L0B_TRY(resolve(m, "lm_head.weight", &head));
        L0B_TRY(set_tensor_staged(m, head, staging));
    }
    if (t.query_gate) return set_query_gate_staged(m, t, staging);
    return set_tensor_staged(m, t, staging);
    GUARD_END
}

L0B_API l0b_status l0b_model_init_synthetic(l0b_model* m, uint64_t seed, float std, float scale_lo, float scale_hi) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(!m->hybrid, L0B_ERR_UNSUPPORTED, "synthetic weights cover the standard decoders, not Qwen3.5 hybrids");
    L0B_CHECK_CUDA(cudaSetDevice(m->dev->index));
    Synth s{m, seed, std, scale_lo, scale_hi};
    const l0b_model_config& c = m->cfg;
    const int tp = c.tp_size > 1 ? c.tp_size : 1, rank = c.tp_size > 1 ? c.tp_rank : 0;
    const int H = c.hidden_size, I = c.intermediate_size;
    const int QD = c.num_attention_heads * c.head_dim, KD = c.num_key_value_heads * c.head_dim;
    L0B_TRY(s.fill(m->embed, L0B_F32, static_cast<long long>(c.vocab_size) * H, kIdEmbed, SYN_NORMAL, std, 0.f));
    if (c.tie_word_embeddings) {
        // The LM head is the embedding table (L/LlmModel.cs:62); values are stored in the model precision.
        if (m->lm_head.dtype == L0B_I8) {
            const bool was = m->dev->recording;
            m->dev->recording = false;
            l0b_status st = k_quantize(m->dev, m->embed + static_cast<long long>(rank) * m->vocab * H, L0B_F32, m->vocab,
                                       H, m->lm_head.group, static_cast<int8_t*>(m->lm_head.w), m->lm_head.scales);
            m->dev->recording = was;
            L0B_TRY(st);
        } else {
            const long long n = static_cast<long long>(m->vocab) * H;
            convert_kernel<<<grid_for(n, m->dev->sm_count), 256, 0, m->dev->stream>>>(
                m->embed + static_cast<long long>(rank) * m->vocab * H, m->lm_head.w, m->lm_head.dtype, n, H, H, 0, 0.f);
        }
    } else {
        L0B_TRY(s.matrix(m->lm_head, 0, kIdLmHead, kIdLmHeadScale, m->vocab, H, H, rank * m->vocab, 0));
    }
    for (int li = 0; li < c.num_layers; ++li) {
        ModelLayer& L = m->layers[li];
        auto id = [&](int kind) { return layer_tensor_id(li, kind); };
        auto sid = [&](int kind) { return layer_tensor_id(li, T_SCALE + kind); };
        L0B_TRY(s.matrix(L.qkv, 0, id(T_Q), sid(T_Q), m->qdim, H, H, rank * m->qdim, 0));
        L0B_TRY(s.matrix(L.qkv, m->qdim, id(T_K), sid(T_K), m->kvdim, H, H, rank * m->kvdim, 0));
        L0B_TRY(s.matrix(L.qkv, m->qdim + m->kvdim, id(T_V), sid(T_V), m->kvdim, H, H, rank * m->kvdim, 0));
        L0B_TRY(s.matrix(L.o, 0, id(T_O), sid(T_O), H, m->qdim, QD, 0, rank * m->qdim));
        L0B_TRY(s.matrix(L.gate_up, 0, id(T_GATE), sid(T_GATE), m->inter, H, H, rank * m->inter, 0));
        L0B_TRY(s.matrix(L.gate_up, m->inter, id(T_UP), sid(T_UP), m->inter, H, H, rank * m->inter, 0));
        L0B_TRY(s.matrix(L.down, 0, id(T_DOWN), sid(T_DOWN), H, m->inter, I, 0, rank * m->inter));
        if (L.qkv_bias) {
            L0B_TRY(s.fill(L.qkv_bias, L0B_F32, m->qdim, id(T_QB), SYN_NORMAL, std, 0.f, m->qdim, QD, 0, rank * m->qdim));
            L0B_TRY(s.fill(L.qkv_bias + m->qdim, L0B_F32, m->kvdim, id(T_KB), SYN_NORMAL, std, 0.f, m->kvdim, KD, 0,
                           rank * m->kvdim));
            L0B_TRY(s.fill(L.qkv_bias + m->qdim + m->kvdim, L0B_F32, m->kvdim, id(T_VB), SYN_NORMAL, std, 0.f, m->kvdim,
                           KD, 0, rank * m->kvdim));
        }
        (void)tp;
    }
    L0B_CHECK_CUDA(cudaGetLastError());
    L0B_CHECK_CUDA(cudaStreamSynchronize(m->dev->stream));
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_model_prefill(l0b_model* m, const int32_t* ids, int32_t count, float* logits) {
    GUARD_BEGIN
    L0B_REQUIRE(m && ids, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(count > 0, L0B_ERR_ARGUMENT, "The prompt must contain at least one token.");
    L0B_REQUIRE(count <= m->max_seq, L0B_ERR_ARGUMENT, "Prompt of %d tokens exceeds the %d-token cache.", count,
                m->max_seq);
    set_position0(m, 0);
    L0B_TRY(ingest_prompt(m, ids, count));
    set_position0(m, count);
    return read_logits(m, logits, 1);
    GUARD_END
}

L0B_API l0b_status l0b_model_decode(l0b_model* m, int32_t token, float* logits) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(m->position < m->max_seq, L0B_ERR_INVALID_OPERATION, "The %d-token KV cache is full.", m->max_seq);
    L0B_TRY(step(m, token, m->position));
    set_position0(m, m->position + 1);
    return read_logits(m, logits, 1);
    GUARD_END
}

L0B_API l0b_status l0b_model_compute_logits(l0b_model* m, int32_t token, int32_t position, float* logits) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_TRY(step(m, token, position));
    return read_logits(m, logits, 1);
    GUARD_END
}

L0B_API l0b_status l0b_model_generate_greedy(l0b_model* m, const int32_t* ids, int32_t count, int32_t max_new,
                                             const int32_t* stop_ids, int32_t n_stop, int32_t* out,
                                             int32_t* out_count) {
    GUARD_BEGIN
    L0B_REQUIRE(m && ids && out_count, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(max_new >= 0, L0B_ERR_OUT_OF_RANGE, "maxNewTokens must be non-negative");
    L0B_REQUIRE(count > 0, L0B_ERR_ARGUMENT, "The prompt must contain at least one token.");
    L0B_REQUIRE(count + max_new <= m->max_seq, L0B_ERR_ARGUMENT,
                "Prompt of %d tokens plus %d new tokens exceeds the %d-token cache.", count, max_new, m->max_seq);
    *out_count = 0;
    if (max_new == 0) return L0B_OK;
    L0B_REQUIRE(out, L0B_ERR_ARGUMENT, "out is null");
    L0B_TRY(ingest_prompt(m, ids, count));
    int next = 0;
    L0B_CHECK_CUDA(copy_sync(m->dev->stream, &next, m->sampled, sizeof(int), cudaMemcpyDeviceToHost));
    int position = count;
    int n = 0;
    while (true) {
        out[n++] = next;
        bool stop = false;
        for (int i = 0; i < n_stop; ++i) stop = stop || stop_ids[i] == next;
        if (n >= max_new || stop) break;
        L0B_TRY(step(m, next, position));
        L0B_CHECK_CUDA(copy_sync(m->dev->stream, &next, m->sampled, sizeof(int), cudaMemcpyDeviceToHost));
        ++position;
    }
    *out_count = n;
    return L0B_OK;
    GUARD_END
}

// Samples the token after the last processed position from the last step's logits on the device (no
// logits readback), as LevelZeroLlmEngine.PickToken -> LlmSampler.Sample does on the host
// (src/HFLabs.ML.LLM.LevelZero/LevelZeroLlmEngine.cs:292-310), and makes it the next input token. The
// repetition context (prompt and generated ids) is given here once; later sampled decode steps add
// their tokens to it on the device.
L0B_API l0b_status l0b_model_sample_logits(l0b_model* m, float temperature, float top_p, int32_t top_k,
                                           float repetition_penalty, uint64_t seed, const int32_t* context,
                                           int32_t n_context, int32_t* token) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(m->tp == 1, L0B_ERR_UNSUPPORTED, "device sampling runs on single-GPU models");
    L0B_REQUIRE(m->position > 0, L0B_ERR_INVALID_OPERATION, "no logits yet: prefill or decode first");
    L0B_REQUIRE(n_context >= 0 && n_context <= m->max_seq + 1 && (n_context == 0 || context), L0B_ERR_OUT_OF_RANGE,
                "context of %d ids (at most %d)", n_context, m->max_seq + 1);
    L0B_TRY(sample_check(temperature, top_p, top_k, repetition_penalty, m->vocab_full));
    l0b_device* d = m->dev;
    L0B_CHECK_CUDA(cudaSetDevice(d->index));
    if (n_context > 0)
        L0B_CHECK_CUDA(cudaMemcpyAsync(m->ctx_ids, context, sizeof(int) * n_context, cudaMemcpyHostToDevice, d->stream));
    m->host_io[0] = m->position;
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->pos, &m->host_io[0], sizeof(int), cudaMemcpyHostToDevice, d->stream));
    L0B_TRY(seen_build(d, m->ctx_ids, n_context, m->vocab_full, m->seen));
    L0B_TRY(sample_step(d, m->logits, m->vocab_full, m->seen, temperature, top_p, top_k, repetition_penalty, m->skeys,
                        0.0, seed, m->pos, 0, m->sampled, nullptr, m->seen));
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->tok, m->sampled, sizeof(int), cudaMemcpyDeviceToDevice, d->stream));
    int t = 0;
    L0B_CHECK_CUDA(cudaMemcpyAsync(&m->host_io[0], m->sampled, sizeof(int), cudaMemcpyDeviceToHost, d->stream));
    L0B_CHECK_CUDA(cudaStreamSynchronize(d->stream));
    t = m->host_io[0];
    if (token) *token = t;
    return L0B_OK;
    GUARD_END
}

// Device-resident sampled decode of sequence 0: `steps` times, decode the pending token and sample the
// next from its logits with the given parameters (the draw of the token at position p is seeded by
// (seed, p)); the context bitmap of the last l0b_model_sample_logits call grows with every token.
L0B_API l0b_status l0b_model_decode_sample_device(l0b_model* m, int32_t steps, float temperature, float top_p,
                                                  int32_t top_k, float repetition_penalty, uint64_t seed,
                                                  int32_t* out) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(m->tp == 1, L0B_ERR_UNSUPPORTED, "device sampling runs on single-GPU models");
    L0B_TRY(sample_check(temperature, top_p, top_k, repetition_penalty, m->vocab_full));
    m->sampling = true;
    m->s_temperature = temperature;
    m->s_top_p = top_p;
    m->s_top_k = top_k;
    m->s_penalty = repetition_penalty;
    m->s_seed = seed;
    const l0b_status st = l0b_model_decode_greedy_device(m, steps, out);
    m->sampling = false;
    return st;
    GUARD_END
}

L0B_API l0b_status l0b_model_decode_greedy_device(l0b_model* m, int32_t steps, int32_t* out) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(steps >= 0, L0B_ERR_OUT_OF_RANGE, "steps must be non-negative");
    L0B_REQUIRE(m->fused, L0B_ERR_UNSUPPORTED, "device-resident decode needs the fused path");
    L0B_REQUIRE(m->position + steps <= m->max_seq, L0B_ERR_INVALID_OPERATION, "The %d-token KV cache is full.",
                m->max_seq);
    if (steps == 0) return L0B_OK;
    l0b_device* d = m->dev;
    L0B_CHECK_CUDA(cudaSetDevice(d->index));
    // tok already holds the last sampled token; pos = current position; the step index restarts.
    m->host_io[0] = m->position;
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->pos, &m->host_io[0], sizeof(int), cudaMemcpyHostToDevice, d->stream));
    L0B_CHECK_CUDA(cudaMemsetAsync(m->step_idx, 0, sizeof(int), d->stream));
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->tok, m->sampled, sizeof(int), cudaMemcpyDeviceToDevice, d->stream));
    for (int i = 0; i < steps; ++i) {
        d->recording = true;
        d->log_used = 0;
        l0b_status s = record_decode_step(m, 1);
        if (s != L0B_OK) {
            d->abort_recording();
            return s;
        }
        L0B_TRY(d->end_recording());
    }
    set_position0(m, m->position + steps);
    if (out) {
        L0B_CHECK_CUDA(cudaMemcpyAsync(out, m->out_tokens, sizeof(int) * steps, cudaMemcpyDeviceToHost, d->stream));
    }
    L0B_CHECK_CUDA(cudaStreamSynchronize(d->stream));
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_model_prefill_sequence(l0b_model* m, int32_t seq, const int32_t* ids, int32_t count,
                                              float* logits) {
    GUARD_BEGIN
    L0B_REQUIRE(m && ids, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(seq >= 0 && seq < m->batch_cap, L0B_ERR_OUT_OF_RANGE, "sequence %d outside the %d-sequence batch",
                seq, m->batch_cap);
    L0B_REQUIRE(count > 0, L0B_ERR_ARGUMENT, "The prompt must contain at least one token.");
    L0B_REQUIRE(count <= m->max_seq, L0B_ERR_ARGUMENT, "Prompt of %d tokens exceeds the %d-token cache.", count,
                m->max_seq);
    L0B_TRY(ingest_prompt(m, ids, count, seq));
    if (seq == 0) set_position0(m, count);
    return read_logits(m, logits, 1);
    GUARD_END
}

L0B_API l0b_status l0b_model_decode_batch(l0b_model* m, const int32_t* tokens, const int32_t* positions,
                                          int32_t count, float* logits) {
    GUARD_BEGIN
    L0B_REQUIRE(m && tokens && positions, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(count > 0 && count <= m->batch_cap, L0B_ERR_OUT_OF_RANGE, "%d sequences (batch capacity %d)", count,
                m->batch_cap);
    L0B_REQUIRE(m->fused && !m->probe, L0B_ERR_UNSUPPORTED, "batched decode needs the fused path");
    for (int b = 0; b < count; ++b) {
        L0B_REQUIRE(tokens[b] >= 0 && tokens[b] < m->vocab_full, L0B_ERR_OUT_OF_RANGE,
                    "Vocabulary has %d tokens (got %d).", m->vocab_full, tokens[b]);
        L0B_REQUIRE(positions[b] >= 0 && positions[b] < m->max_seq, L0B_ERR_OUT_OF_RANGE,
                    "Cache holds %d positions (got %d).", m->max_seq, positions[b]);
    }
    L0B_TRY(write_io(m, count, tokens, positions));
    L0B_TRY(run_recorded(m, [&] { return record_decode_step(m, count); }));
    for (int b = 0; b < count; ++b) m->seq_pos[b] = positions[b] + 1;
    set_position0(m, positions[0] + 1);
    return read_logits(m, logits, count);
    GUARD_END
}

L0B_API l0b_status l0b_model_decode_greedy_device_batch(l0b_model* m, int32_t steps, int32_t count, int32_t* out) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(steps >= 0, L0B_ERR_OUT_OF_RANGE, "steps must be non-negative");
    L0B_REQUIRE(count > 0 && count <= m->batch_cap, L0B_ERR_OUT_OF_RANGE, "%d sequences (batch capacity %d)", count,
                m->batch_cap);
    L0B_REQUIRE(m->fused, L0B_ERR_UNSUPPORTED, "device-resident decode needs the fused path");
    for (int b = 0; b < count; ++b)
        L0B_REQUIRE(m->seq_pos[b] + steps <= m->max_seq, L0B_ERR_INVALID_OPERATION,
                    "Sequence %d: the %d-token KV cache is full.", b, m->max_seq);
    if (steps == 0) return L0B_OK;
    l0b_device* d = m->dev;
    L0B_CHECK_CUDA(cudaSetDevice(d->index));
    // Each sequence's token and position are already on the device (its prefill head or last step).
    L0B_CHECK_CUDA(cudaMemsetAsync(m->step_idx, 0, sizeof(int), d->stream));
    for (int i = 0; i < steps; ++i) {
        d->recording = true;
        d->log_used = 0;
        l0b_status s = record_decode_step(m, count);
        if (s != L0B_OK) {
            d->abort_recording();
            return s;
        }
        L0B_TRY(d->end_recording());
    }
    for (int b = 0; b < count; ++b) m->seq_pos[b] += steps;
    set_position0(m, m->seq_pos[0]);
    if (out) {
        L0B_CHECK_CUDA(cudaMemcpyAsync(out, m->out_tokens, sizeof(int) * steps * count, cudaMemcpyDeviceToHost,
                                       d->stream));
    }
    L0B_CHECK_CUDA(cudaStreamSynchronize(d->stream));
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_model_sequence_position(l0b_model* m, int32_t seq, int32_t* position) {
    L0B_REQUIRE(m && position, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(seq >= 0 && seq < m->batch_cap, L0B_ERR_OUT_OF_RANGE, "sequence %d", seq);
    *position = m->seq_pos[seq];
    return L0B_OK;
}

// Device-side fork (the reference's CaptureState + RestoreState, src/HFLabs.ML.LLM.LevelZero/LlmModel.cs:
// 257-306, which round-trips the KV tail through host arrays): sequence dst becomes a copy of sequence
// src. Cache rows [base_position, length) of every layer are copied on the device (rows below
// base_position are taken to be equal already, the shared prompt), and so are the device token,
// position and last sampled token that the device-resident decode continues from.
L0B_API l0b_status l0b_model_fork_sequence(l0b_model* m, int32_t src, int32_t dst, int32_t base_position) {
    GUARD_BEGIN
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(src >= 0 && src < m->batch_cap && dst >= 0 && dst < m->batch_cap, L0B_ERR_OUT_OF_RANGE,
                "sequences %d -> %d outside the %d-sequence batch", src, dst, m->batch_cap);
    L0B_REQUIRE(src != dst, L0B_ERR_ARGUMENT, "a sequence cannot be forked onto itself");
    const int length = m->seq_pos[src];
    L0B_REQUIRE(base_position >= 0 && base_position <= length, L0B_ERR_OUT_OF_RANGE,
                "base position %d outside [0, %d]", base_position, length);
    l0b_device* d = m->dev;
    L0B_CHECK_CUDA(cudaSetDevice(d->index));
    const size_t row = static_cast<size_t>(m->kvdim) * dtype_size(static_cast<l0b_dtype>(m->cache_dtype));
    const size_t bytes = static_cast<size_t>(length - base_position) * row;
    if (bytes > 0) {
        for (ModelLayer& L : m->layers) {
            for (int which = 0; which < 2; ++which) {
                char* cache = static_cast<char*>(which ? L.vc : L.kc);
                const size_t s_off = (static_cast<size_t>(src) * m->max_seq + base_position) * row;
                const size_t d_off = (static_cast<size_t>(dst) * m->max_seq + base_position) * row;
                L0B_CHECK_CUDA(cudaMemcpyAsync(cache + d_off, cache + s_off, bytes, cudaMemcpyDeviceToDevice, d->stream));
            }
        }
    }
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->tok + dst, m->tok + src, sizeof(int), cudaMemcpyDeviceToDevice, d->stream));
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->pos + dst, m->pos + src, sizeof(int), cudaMemcpyDeviceToDevice, d->stream));
    L0B_CHECK_CUDA(cudaMemcpyAsync(m->sampled + dst, m->sampled + src, sizeof(int), cudaMemcpyDeviceToDevice, d->stream));
    m->seq_pos[dst] = length;
    if (dst == 0) set_position0(m, length);
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_model_position(l0b_model* m, int32_t* position) {
    L0B_REQUIRE(m && position, L0B_ERR_ARGUMENT, "null argument");
    *position = m->position;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_reset_sequence(l0b_model* m) {
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    set_position0(m, 0);
    return L0B_OK;
}

L0B_API l0b_status l0b_model_projection_bytes(l0b_model* m, int64_t* bytes) {
    L0B_REQUIRE(m && bytes, L0B_ERR_ARGUMENT, "null argument");
    int64_t b = static_cast<int64_t>(m->lm_head.bytes());
    for (auto& L : m->layers)
        b += L.qkv.bytes() + L.o.bytes() + L.gate_up.bytes() + L.down.bytes() + L.lin_in.bytes() + L.lin_out.bytes();
    *bytes = b;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_set_recording(l0b_model* m, int32_t enabled) {
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    m->recording = enabled != 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_set_fused(l0b_model* m, int32_t enabled) {
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(!(enabled && m->hybrid), L0B_ERR_UNSUPPORTED, "Qwen3.5 hybrid models run the reference op sequence");
    m->fused = enabled != 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_set_gemm_rows(l0b_model* m, int32_t min_rows) {
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    L0B_REQUIRE(min_rows >= 0, L0B_ERR_OUT_OF_RANGE, "min_rows %d", min_rows);
    m->tc_rows = m->x16 ? min_rows : 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_set_probe(l0b_model* m, l0b_probe_fn fn, void* user) {
    L0B_REQUIRE(m, L0B_ERR_ARGUMENT, "model is null");
    m->probe = fn;
    m->probe_user = user;
    return L0B_OK;
}

L0B_API l0b_status l0b_model_read_weight(l0b_model* m, int32_t layer, int32_t kind, void* out, int64_t bytes) {
    GUARD_BEGIN
    L0B_REQUIRE(m && out, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(layer >= -1 && layer < static_cast<int>(m->layers.size()), L0B_ERR_OUT_OF_RANGE, "layer %d", layer);
    L0B_REQUIRE(kind >= 0 && kind < 8, L0B_ERR_OUT_OF_RANGE, "kind %d", kind);
    const ModelMatrix* mats[4];
    if (layer < 0) {
        L0B_REQUIRE(kind % 4 == 0, L0B_ERR_ARGUMENT, "the LM head is kind 0 (weights) or 4 (scales)");
        mats[0] = &m->lm_head;
    } else {
        const ModelLayer& L = m->layers[layer];
        mats[0] = &L.qkv;
        mats[1] = &L.o;
        mats[2] = &L.gate_up;
        mats[3] = &L.down;
    }
    const ModelMatrix& mat = *mats[kind % 4];
    L0B_REQUIRE(mat.w, L0B_ERR_INVALID_OPERATION, "layer %d has no such matrix (a linear-attention layer)", layer);
    const void* src;
    size_t size;
    if (kind < 4) {
        src = mat.w;
        size = static_cast<size_t>(mat.n) * mat.k * dtype_size(static_cast<l0b_dtype>(mat.dtype));
    } else {
        L0B_REQUIRE(mat.dtype == L0B_I8, L0B_ERR_ARGUMENT, "the matrix has no int8 scales");
        src = mat.scales;
        size = static_cast<size_t>(mat.n) * (mat.k / mat.group) * sizeof(__half);
    }
    L0B_REQUIRE(static_cast<size_t>(bytes) == size, L0B_ERR_ARGUMENT, "storage is %zu bytes, %lld requested", size,
                (long long)bytes);
    L0B_CHECK_CUDA(cudaStreamSynchronize(m->dev->stream));
    if (kind < 4 && mat.kb > 0) {
        // Back to the [out, in] order.
        std::vector<int8_t> tmp(size);
        L0B_CHECK_CUDA(copy_sync(m->dev->stream, tmp.data(), src, size, cudaMemcpyDeviceToHost));
        int8_t* o = static_cast<int8_t*>(out);
        for (long long r = 0; r < mat.n; ++r)
            for (long long c = 0; c < mat.k; ++c) o[r * mat.k + c] = tmp[blocked_index(r, c, mat.k, mat.kb)];
        return L0B_OK;
    }
    L0B_CHECK_CUDA(copy_sync(m->dev->stream, out, src, size, cudaMemcpyDeviceToHost));
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_model_read_kv(l0b_model* m, int32_t layer, int32_t row0, int32_t rows, float* keys,
                                     float* values) {
    GUARD_BEGIN
    L0B_REQUIRE(m && keys && values, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(layer >= 0 && layer < static_cast<int>(m->layers.size()), L0B_ERR_OUT_OF_RANGE, "layer %d", layer);
    L0B_REQUIRE(row0 >= 0 && rows >= 0 && row0 + rows <= m->max_seq, L0B_ERR_OUT_OF_RANGE, "rows outside the cache");
    L0B_REQUIRE(!m->layers[layer].linear, L0B_ERR_INVALID_OPERATION, "layer %d is a linear-attention layer (no KV cache)",
                layer);
    if (rows == 0) return L0B_OK;
    const size_t n = static_cast<size_t>(rows) * m->kvdim;
    const size_t es = dtype_size(static_cast<l0b_dtype>(m->cache_dtype));
    std::vector<uint8_t> tmp(n * es);
    ModelLayer& L = m->layers[layer];
    L0B_CHECK_CUDA(cudaStreamSynchronize(m->dev->stream));
    for (int which = 0; which < 2; ++which) {
        const char* src = static_cast<const char*>(which ? L.vc : L.kc) + static_cast<size_t>(row0) * m->kvdim * es;
        L0B_CHECK_CUDA(copy_sync(m->dev->stream, tmp.data(), src, n * es, cudaMemcpyDeviceToHost));
        float* dst = which ? values : keys;
        for (size_t i = 0; i < n; ++i) {
            if (m->cache_dtype == L0B_F32) dst[i] = reinterpret_cast<const float*>(tmp.data())[i];
            else if (m->cache_dtype == L0B_F16) dst[i] = __half2float(reinterpret_cast<const __half*>(tmp.data())[i]);
            else {
                uint32_t bits = static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(tmp.data())[i]) << 16;
                std::memcpy(&dst[i], &bits, 4);
            }
        }
    }
    return L0B_OK;
    GUARD_END
}

}  // extern "C"
