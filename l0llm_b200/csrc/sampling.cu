// On-device token sampling: the reference's LlmSampler.Sample
// (src/HFLabs.ML.LLM.LevelZero/LlmAbstractions.cs:40-165) without the per-token logits readback.
//
// Steps, as the reference orders them: repetition penalty on every distinct context token (logit >= 0
// divided by the penalty, else multiplied), greedy argmax when T <= 0, logits / T, softmax in double,
// descending sort, top-k cut, top-p cut (the shortest prefix whose cumulative probability reaches p),
// then the inverse CDF of the kept mass at u * (kept mass), u the caller's uniform draw in [0, 1).
//
// GPU form. A grid-wide kernel writes each token's penalised, temperature-scaled logit as an
// order-preserving 32-bit key. One CTA of 1024 threads then
//   - finds the k-th largest key by a 4-pass radix select (8 bits per pass, shared-memory histograms)
//     and the maximum, and accumulates the softmax normaliser in double on the second pass;
//   - gathers the k candidates (every key above the k-th, and the lowest-index tokens equal to it) and
//     bitonic-sorts them by (key descending, index ascending);
//   - forms the probabilities in parallel and runs the cumulative sum sequentially in sorted order (the
//     same order and the same double arithmetic as the reference), which gives the top-p cut, the kept
//     mass and the sampled position in one pass.
// Ties in probability fall back to the lower token index; the reference's List.Sort is unstable, so
// its order among exact ties is unspecified. top_k must lie in [1, 1024] (the reference's default is
// 40); larger or disabled top-k is refused with L0B_ERR_UNSUPPORTED rather than sampled differently.
#include <cstdint>

#include "common.cuh"
#include "ops.cuh"
#include "suite.h"

namespace l0b {

namespace {

constexpr int kSelThreads = 1024;
constexpr int kMaxTopK = 1024;

constexpr int kNormBlocks = 148;  // blocks of the normaliser kernel (fixed: the partials sum in order)
constexpr int kMaxTies = 1024;

struct SampleArgs {
    const float* logits;
    int vocab;
    const uint32_t* seen;  // context bitmap for the repetition penalty, or null
    float temperature, top_p, penalty;
    int top_k;
    uint32_t* keys;        // [vocab] scratch
    uint32_t* kmax;        // [1] scratch: the largest key, zero at rest (the select kernel re-arms it)
    double* norm_part;     // [kNormBlocks] scratch: per-block partial softmax normalisers
    double u;              // uniform draw when use_seed == 0
    unsigned long long seed;
    const int* pos;        // use_seed: the draw is sample_uniform(seed, *pos + pos_offset)
    int pos_offset;
    int use_seed;
    int* out_token;                // may be null
    unsigned long long* out_key;   // argmax-style key of the chosen token (model step), may be null
    uint32_t* seen_update;         // bitmap that records the chosen token, may be null
    int* error;                    // set when more tied candidates than the select can hold
};

__device__ __forceinline__ uint32_t ord_u32(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ord_f32(uint32_t u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

__device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

// The draw of the token at position p for a seeded generation: 53 random bits in [0, 1).
__device__ __forceinline__ double sample_uniform(unsigned long long seed, int p) {
    const unsigned long long h = mix64(seed ^ (static_cast<unsigned long long>(p + 1) * 0x9E3779B97F4A7C15ULL));
    return static_cast<double>(h >> 11) * (1.0 / 9007199254740992.0);
}

// Keys (penalty, then / T, as float) and their maximum.
__global__ void __launch_bounds__(256) sample_keys_kernel(const SampleArgs a) {
    pdl_wait();
    uint32_t mx = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.vocab; i += gridDim.x * blockDim.x) {
        float l = a.logits[i];
        if (a.seen && ((a.seen[i >> 5] >> (i & 31)) & 1u)) l = l >= 0.0f ? l / a.penalty : l * a.penalty;
        if (a.temperature > 0.0f) l = l / a.temperature;
        const uint32_t u = ord_u32(l);
        a.keys[i] = u;
        mx = max(mx, u);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) atomicMax(a.kmax, mx);
}

__device__ double block_sum_f64(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = lane < (blockDim.x >> 5) ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

// Partial softmax normalisers: block b sums exp(double(key - max)) (the float difference, as the
// reference forms it) over its share of the vocabulary.
__global__ void __launch_bounds__(256) sample_norm_kernel(const SampleArgs a) {
    __shared__ double red[32];
    pdl_wait();
    const float mx = ord_f32(*a.kmax);
    double s = 0.0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.vocab; i += gridDim.x * blockDim.x)
        s += exp(static_cast<double>(ord_f32(a.keys[i]) - mx));
    s = block_sum_f64(s, red);
    if (threadIdx.x == 0) a.norm_part[blockIdx.x] = s;
}

// Histogram increment with lanes of equal bins merged (float keys share few top bytes).
__device__ __forceinline__ void hist_add(unsigned* hist, bool active, unsigned bin) {
    const unsigned act = __ballot_sync(0xffffffffu, active);
    if (!active) return;
    const unsigned peers = __match_any_sync(act, bin);
    if ((threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
}

__global__ void __launch_bounds__(kSelThreads) sample_select_kernel(const SampleArgs a) {
    __shared__ unsigned hist[256];
    __shared__ unsigned long long cand[kMaxTopK];
    __shared__ double prob[kMaxTopK];
    __shared__ int ties[kMaxTies];
    __shared__ unsigned sel_bucket, sel_remaining, gt_count, tie_count;
    __shared__ int pick;
    pdl_wait();
    const int tid = threadIdx.x;
    const bool greedy = a.temperature <= 0.0f;
    const int k = greedy ? 1 : ((a.top_k > 0 && a.top_k < a.vocab) ? a.top_k : a.vocab);
    const uint32_t max_key = *a.kmax;
    const float mx = ord_f32(max_key);
    if (tid == 0) {
        gt_count = 0;
        tie_count = 0;
    }
    // Radix select: after the 4 passes, `prefix` is the k-th largest key and `remaining` the number of
    // tokens equal to it that belong to the top k (the lowest-index ones).
    uint32_t prefix = 0, mask = 0;
    unsigned remaining = static_cast<unsigned>(k);
    const int trips = (a.vocab + kSelThreads - 1) / kSelThreads;  // uniform loop count for the warp votes
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int b = tid; b < 256; b += kSelThreads) hist[b] = 0;
        __syncthreads();
        for (int it = 0; it < trips; ++it) {
            const int i = it * kSelThreads + tid;
            const uint32_t u = i < a.vocab ? a.keys[i] : 0u;
            hist_add(hist, i < a.vocab && (u & mask) == prefix, (u >> shift) & 255u);
        }
        __syncthreads();
        if (tid == 0) {
            unsigned cum = 0;
            int b = 255;
            for (; b > 0; --b) {
                if (cum + hist[b] >= remaining) break;
                cum += hist[b];
            }
            sel_bucket = static_cast<unsigned>(b);
            sel_remaining = remaining - cum;
        }
        __syncthreads();
        prefix |= sel_bucket << shift;
        mask |= 255u << shift;
        remaining = sel_remaining;
        __syncthreads();
    }
    double total = 1.0;
    if (!greedy && tid == 0) {
        total = 0.0;
        for (int b = 0; b < kNormBlocks; ++b) total += a.norm_part[b];
    }
    // Gather: keys above the threshold in any order; ties at the threshold listed, then ranked by index.
    const unsigned above = static_cast<unsigned>(k) - remaining;
    for (int i = tid; i < a.vocab; i += kSelThreads) {
        const uint32_t u = a.keys[i];
        if (u > prefix) {
            const unsigned at = atomicAdd(&gt_count, 1u);
            if (at < above) cand[at] = (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
        } else if (u == prefix) {
            const unsigned at = atomicAdd(&tie_count, 1u);
            if (at < kMaxTies) ties[at] = i;
        }
    }
    __syncthreads();
    const unsigned nties = tie_count < kMaxTies ? tie_count : kMaxTies;
    if (tid == 0 && (gt_count != above || tie_count > kMaxTies) && a.error) atomicExch(a.error, 1);
    if (tid < static_cast<int>(nties)) {
        const int mine = ties[tid];
        unsigned rank = 0;
        for (unsigned j = 0; j < nties; ++j) rank += ties[j] < mine;
        if (rank < remaining)
            cand[above + rank] = (static_cast<unsigned long long>(prefix) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(mine));
    }
    // Bitonic sort of the k candidates, descending (padding sorts last).
    if (tid >= k) cand[tid] = 0ull;
    __syncthreads();
    for (int size = 2; size <= kSelThreads; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const int j = tid ^ stride;
            if (j > tid) {
                const bool desc = (tid & size) == 0;
                const unsigned long long x = cand[tid], y = cand[j];
                if (desc ? (x < y) : (x > y)) {
                    cand[tid] = y;
                    cand[j] = x;
                }
            }
            __syncthreads();
        }
    }
    __shared__ double total_s;
    if (tid == 0) total_s = total;
    __syncthreads();
    // Probabilities of the sorted candidates, then the cumulative sum in sorted order.
    if (tid < k && !greedy)
        prob[tid] = exp(static_cast<double>(ord_f32(static_cast<uint32_t>(cand[tid] >> 32)) - mx)) / total_s;
    __syncthreads();
    if (tid == 0) {
        int chosen = 0;
        if (!greedy) {
            const double u = a.use_seed ? sample_uniform(a.seed, *a.pos + a.pos_offset) : a.u;
            // Top-p: the shortest prefix whose cumulative probability reaches top_p.
            int keep = k;
            if (a.top_p > 0.0f && a.top_p < 1.0f) {
                double cum = 0.0;
                for (int t = 0; t < k; ++t) {
                    cum += prob[t];
                    if (cum >= static_cast<double>(a.top_p)) {
                        keep = t + 1;
                        break;
                    }
                }
            }
            double kept = 0.0;
            for (int t = 0; t < keep; ++t) kept += prob[t];
            chosen = keep - 1;
            if (kept <= 0.0) {
                chosen = 0;
            } else {
                const double r = u * kept;
                double cur = 0.0;
                for (int t = 0; t < keep; ++t) {
                    cur += prob[t];
                    if (r <= cur) {
                        chosen = t;
                        break;
                    }
                }
            }
        }
        pick = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(cand[chosen] & 0xFFFFFFFFull));
    }
    __syncthreads();
    if (tid == 0) {
        const int token = pick;
        if (a.out_token) *a.out_token = token;
        if (a.out_key) *a.out_key = (0xFFFFFFFFull << 32) | static_cast<uint32_t>(0x7FFFFFFF - token);
        if (a.seen_update) atomicOr(&a.seen_update[token >> 5], 1u << (token & 31));
        *a.kmax = 0u;  // re-armed for the next draw
    }
}

// Context bitmap for the repetition penalty: zero `words`, then set the bit of every id in [0, vocab).
__global__ void __launch_bounds__(1024) seen_build_kernel(const int* ids, int n, int vocab, uint32_t* bits, int words) {
    pdl_wait();
    for (int w = threadIdx.x; w < words; w += blockDim.x) bits[w] = 0u;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int t = ids[i];
        if (t >= 0 && t < vocab) atomicOr(&bits[t >> 5], 1u << (t & 31));
    }
}

__global__ void fill_u32_kernel(uint32_t* p, uint32_t v, int n) {
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

l0b_status sample_launch(l0b_device* d, const SampleArgs& a) {
    const int grid = (a.vocab + 255) / 256 < d->sm_count * 4 ? (a.vocab + 255) / 256 : d->sm_count * 4;
    L0B_TRY(d->launch(sample_keys_kernel, dim3(grid), dim3(256), 0, a));
    if (a.temperature > 0.0f) L0B_TRY(d->launch(sample_norm_kernel, dim3(kNormBlocks), dim3(256), 0, a));
    return d->launch(sample_select_kernel, dim3(1), dim3(kSelThreads), 0, a);
}

}  // namespace

l0b_status sample_check(float temperature, float top_p, int top_k, float penalty, int vocab) {
    L0B_REQUIRE(vocab > 0, L0B_ERR_ARGUMENT, "Logits array cannot be null or empty.");
    L0B_REQUIRE(penalty > 0.0f, L0B_ERR_ARGUMENT, "repetition penalty must be positive");
    (void)top_p;
    if (temperature > 0.0f) {
        const int k = (top_k > 0 && top_k < vocab) ? top_k : vocab;
        L0B_REQUIRE(k <= kMaxTopK, L0B_ERR_UNSUPPORTED,
                    "device sampling keeps at most %d candidates: top_k must lie in [1, %d] (got %d, vocab %d)",
                    kMaxTopK, kMaxTopK, top_k, vocab);
    }
    return L0B_OK;
}

l0b_status k_fill_u32(l0b_device* d, uint32_t* p, uint32_t v, int n) {
    return d->launch(fill_u32_kernel, dim3((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024), dim3(256), 0, p, v, n);
}

size_t sample_seen_words(int vocab) { return (static_cast<size_t>(vocab) + 31) / 32; }

size_t sample_keys_words(int vocab) {
    return ((static_cast<size_t>(vocab) + 1 + 1) & ~static_cast<size_t>(1)) + 2 * kNormBlocks;
}

l0b_status seen_build(l0b_device* d, const int* ids, int n, int vocab, uint32_t* bits) {
    const int words = static_cast<int>(sample_seen_words(vocab));
    return d->launch(seen_build_kernel, dim3(1), dim3(1024), 0, ids, n, vocab, bits, words);
}

l0b_status sample_step(l0b_device* d, const float* logits, int vocab, const uint32_t* seen, float temperature,
                       float top_p, int top_k, float penalty, uint32_t* keys, double u, unsigned long long seed,
                       const int* pos, int pos_offset, int* out_token, unsigned long long* out_key,
                       uint32_t* seen_update) {
    L0B_TRY(sample_check(temperature, top_p, top_k, penalty, vocab));
    SampleArgs a = {};
    a.logits = logits;
    a.vocab = vocab;
    a.seen = (penalty != 1.0f) ? seen : nullptr;
    a.temperature = temperature;
    a.top_p = top_p;
    a.penalty = penalty;
    a.top_k = top_k;
    a.keys = keys;
    // Scratch after the keys: the max word (zero at rest), then the double partials (8-byte aligned).
    a.kmax = keys + vocab;
    a.norm_part = reinterpret_cast<double*>(keys + ((static_cast<size_t>(vocab) + 1 + 1) & ~static_cast<size_t>(1)));
    a.u = u;
    a.seed = seed;
    a.pos = pos;
    a.pos_offset = pos_offset;
    a.use_seed = pos ? 1 : 0;
    a.out_token = out_token;
    a.out_key = out_key;
    a.seen_update = seen_update;
    a.error = d->error_flag;
    return sample_launch(d, a);
}

}  // namespace l0b
