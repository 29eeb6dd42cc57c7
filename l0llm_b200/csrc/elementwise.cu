// Small ops of the LlmKernelSuite surface: RMSNorm, BiasAdd, RoPE, KV-cache store, SwiGLU, Add,
// SigmoidGate, Embedding, Copy, Sampling, and the device int8 quantizer. These are launch-bound at
// decode; the fused decode path folds most of them into the GEMV and attention kernels.
#include "common.cuh"
#include "ops.cuh"

namespace l0b {

namespace {

__global__ void __launch_bounds__(256) rmsnorm_kernel(float* x, const float* res, const float* w, float* out,
                                                      float eps, int width, int add_res) {
    __shared__ float red[32];
    pdl_wait();
    const long long base = static_cast<long long>(blockIdx.x) * width;
    float ss = 0.f;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        float v = x[base + i];
        if (add_res) {
            v += res[base + i];
            x[base + i] = v;
        }
        ss += v * v;
    }
    ss = block_sum(ss, red);
    const float rstd = 1.0f / sqrtf(ss / static_cast<float>(width) + eps);
    for (int i = threadIdx.x; i < width; i += blockDim.x) out[base + i] = (x[base + i] * rstd) * w[i];
}

// QK-norm of the fused layer (LlmDecoderLayer, L/LlmDecoderLayer.cs:308-313): RMSNorm of every query and
// key head of the stacked q|k|v rows in place, CTA (row, head) -- the arithmetic of rmsnorm_kernel at 32
// threads (the same sums in the same order: head dims below 256, where that kernel runs 32 threads).
__global__ void __launch_bounds__(32) head_norm_kernel(float* qkv, long long ld, int nq, int hd, const float* wq,
                                                       const float* wk, float eps) {
    __shared__ float red[32];
    pdl_wait();
    const int h = blockIdx.y;
    const bool is_q = h < nq;
    float* x = qkv + static_cast<long long>(blockIdx.x) * ld + static_cast<long long>(h) * hd;
    const float* w = is_q ? wq : wk;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) ss += x[i] * x[i];
    ss = block_sum(ss, red);
    const float rstd = 1.0f / sqrtf(ss / static_cast<float>(hd) + eps);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) x[i] = (x[i] * rstd) * w[i];
}

__global__ void bias_add_kernel(float* x, const float* b, int width, long long total) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        x[i] += b[i % width];
}

// Rotates pairs (i, i + rot/2) of the first `rot` elements of every head of q and k.
__global__ void rope_kernel(float* q, float* k, const int* positions, const float* inv_freq, int hd, int nh,
                            int nkv, float attn_scale, int rot, int tokens, long long q_stride, long long k_stride) {
    pdl_wait();
    const int half = rot / 2;
    const long long per_token = static_cast<long long>(nh + nkv) * half;
    const long long total = per_token * tokens;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i / per_token);
        const long long r = i - t * per_token;
        const int head = static_cast<int>(r / half);
        const int j = static_cast<int>(r - static_cast<long long>(head) * half);
        float* v = head < nh ? q + t * q_stride + static_cast<long long>(head) * hd
                             : k + t * k_stride + static_cast<long long>(head - nh) * hd;
        const float ang = __fmul_rn(static_cast<float>(positions[t]), inv_freq[j]);
        float s, c;
        sincosf(ang, &s, &c);
        c = __fmul_rn(c, attn_scale);
        s = __fmul_rn(s, attn_scale);
        const float x1 = v[j], x2 = v[j + half];
        v[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        v[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
}

__global__ void kv_store_kernel(const float* k, const float* v, void* kc, void* vc, int cache_dtype, int pos0,
                                int kv_dim, int tokens, long long in_stride) {
    pdl_wait();
    const long long total = static_cast<long long>(tokens) * kv_dim;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long t = i / kv_dim, c = i - t * kv_dim;
        const long long dst = static_cast<long long>(pos0) * kv_dim + i;
        store_from_float(kc, cache_dtype, dst, k[t * in_stride + c]);
        store_from_float(vc, cache_dtype, dst, v[t * in_stride + c]);
    }
}

__global__ void swiglu_kernel(float* gate, const float* up, long long n) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        gate[i] = silu(gate[i]) * up[i];
}

__global__ void add_kernel(float* a, const float* b, long long n) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        a[i] += b[i];
}

__global__ void sigmoid_gate_kernel(float* x, const float* g, long long n) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        x[i] *= 1.0f / (1.0f + expf(-g[i]));
}

__global__ void embedding_kernel(const int* ids, const void* table, int table_dtype, float* out, int h,
                                 long long count, int vocab, int* error) {
    pdl_wait();
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < count;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long t = e / h;
        const int col = static_cast<int>(e - t * h);
        const int id = ids[t];
        if (id < 0 || id >= vocab) {
            if (error) *error = 1;
            out[e] = 0.f;
            continue;
        }
        out[e] = load_as_float(table, table_dtype, static_cast<long long>(id) * h + col);
    }
}

__global__ void copy_kernel(const float* src, float* dst, long long offset, long long n) {
    pdl_wait();
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        dst[i] = src[offset + i];
}

// Greedy argmax (temperature 0) or inverse-CDF sampling of softmax(logits / T) with one block.
__global__ void __launch_bounds__(1024) sampling_kernel(const float* logits, int* sampled, float temperature,
                                                        float random_val, int vocab) {
    __shared__ unsigned long long best_s;
    __shared__ float red[32];
    __shared__ float scan_s[1024];
    pdl_wait();
    if (threadIdx.x == 0) best_s = 0ull;
    __syncthreads();
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float v = logits[i];
        if (v == v) {  // NaN never wins
            const unsigned long long key = argmax_key(v, i);
            best = key > best ? key : best;
        }
    }
    atomicMax(&best_s, best);
    __syncthreads();
    const int arg = best_s ? argmax_key_index(best_s) : 0;
    if (temperature <= 0.f) {
        if (threadIdx.x == 0) *sampled = arg;
        return;
    }
    const float mx = logits[arg];
    const float inv_t = 1.0f / temperature;
    // Each thread owns a contiguous slice; slice sums are scanned, then the owner of the target scans.
    const int per = (vocab + blockDim.x - 1) / blockDim.x;
    const int lo = threadIdx.x * per, hi = min(vocab, lo + per);
    float local = 0.f;
    for (int i = lo; i < hi; ++i) local += expf((logits[i] - mx) * inv_t);
    scan_s[threadIdx.x] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float run = 0.f;
        for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
            const float v = scan_s[t];
            scan_s[t] = run;
            run += v;
        }
        red[0] = run;
    }
    __syncthreads();
    const float target = random_val * red[0];
    const float before = scan_s[threadIdx.x];
    // The chosen slice is the first whose inclusive prefix reaches the target; the slice holding the
    // last token also takes the target when rounding left every prefix short of it.
    const bool starts_before = threadIdx.x == 0 || before < target;
    const bool reaches = before + local >= target || hi == vocab;
    if (lo < hi && starts_before && reaches) {
        float run = before;
        int pick = hi - 1;
        for (int i = lo; i < hi; ++i) {
            run += expf((logits[i] - mx) * inv_t);
            if (run >= target) {
                pick = i;
                break;
            }
        }
        atomicMin(sampled, pick);
    }
}

__global__ void fill_int_kernel(int* p, int v) {
    pdl_wait();
    *p = v;
}

// Symmetric int8 quantisation of [N, K] weights, one warp per (row, group).
__global__ void quantize_kernel(const void* w, int w_dtype, int n, int k, int group, int8_t* q, __half* s) {
    pdl_wait();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int gpr = k / group;
    if (warp >= n * gpr) return;
    const int row = warp / gpr, g = warp - row * gpr;
    const long long base = static_cast<long long>(row) * k + static_cast<long long>(g) * group;
    float mx = 0.f;
    for (int i = lane; i < group; i += 32) mx = fmaxf(mx, fabsf(load_as_float(w, w_dtype, base + i)));
    mx = warp_max(mx);
    const __half sh = __float2half_rn(mx / 127.0f);
    const float sf = __half2float(sh);
    for (int i = lane; i < group; i += 32) {
        float r = 0.f;
        if (sf > 0.f) r = fminf(127.f, fmaxf(-127.f, rintf(load_as_float(w, w_dtype, base + i) / sf)));
        q[base + i] = static_cast<int8_t>(r);
    }
    if (lane == 0) s[static_cast<long long>(row) * gpr + g] = sh;
}

inline int grid_for(long long n, int threads, int sm_count) {
    long long g = (n + threads - 1) / threads;
    const long long cap = static_cast<long long>(sm_count) * 8;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return static_cast<int>(g);
}

}  // namespace

l0b_status k_rmsnorm(l0b_device* d, float* x, const float* res, const float* w, float* out, float eps, int width,
                     int rows, int add_res) {
    const int threads = width >= 1024 ? 256 : (width >= 256 ? 128 : 32);
    return d->launch(rmsnorm_kernel, dim3(rows), dim3(threads), 0, x, res, w, out, eps, width, add_res);
}

l0b_status k_head_norm(l0b_device* d, float* qkv, long long ld, int nq, int nk, int hd, const float* wq,
                       const float* wk, float eps, int rows) {
    return d->launch(head_norm_kernel, dim3(rows, nq + nk), dim3(32), 0, qkv, ld, nq, hd, wq, wk, eps);
}

l0b_status k_bias_add(l0b_device* d, float* x, const float* b, int width, int rows) {
    const long long total = static_cast<long long>(width) * rows;
    return d->launch(bias_add_kernel, dim3(grid_for(total, 256, d->sm_count)), dim3(256), 0, x, b, width, total);
}

l0b_status k_rope(l0b_device* d, float* q, float* k, const int* positions, const float* inv_freq, int hd, int nh,
                  int nkv, float attn_scale, int rot, int tokens, long long q_stride, long long k_stride) {
    const long long total = static_cast<long long>(nh + nkv) * (rot / 2) * tokens;
    if (q_stride <= 0) q_stride = static_cast<long long>(nh) * hd;
    if (k_stride <= 0) k_stride = static_cast<long long>(nkv) * hd;
    return d->launch(rope_kernel, dim3(grid_for(total, 256, d->sm_count)), dim3(256), 0, q, k, positions, inv_freq,
                     hd, nh, nkv, attn_scale, rot, tokens, q_stride, k_stride);
}

l0b_status k_kv_store(l0b_device* d, const float* k, const float* v, void* kc, void* vc, int cache_dtype, int pos0,
                      int kv_dim, int tokens, long long in_stride) {
    const long long total = static_cast<long long>(tokens) * kv_dim;
    if (in_stride <= 0) in_stride = kv_dim;
    return d->launch(kv_store_kernel, dim3(grid_for(total, 256, d->sm_count)), dim3(256), 0, k, v, kc, vc,
                     cache_dtype, pos0, kv_dim, tokens, in_stride);
}

l0b_status k_swiglu(l0b_device* d, float* gate, const float* up, long long n) {
    return d->launch(swiglu_kernel, dim3(grid_for(n, 256, d->sm_count)), dim3(256), 0, gate, up, n);
}

l0b_status k_add(l0b_device* d, float* a, const float* b, long long n) {
    return d->launch(add_kernel, dim3(grid_for(n, 256, d->sm_count)), dim3(256), 0, a, b, n);
}

l0b_status k_sigmoid_gate(l0b_device* d, float* x, const float* g, long long n) {
    return d->launch(sigmoid_gate_kernel, dim3(grid_for(n, 256, d->sm_count)), dim3(256), 0, x, g, n);
}

l0b_status k_embedding(l0b_device* d, const int* ids, const void* table, int table_dtype, float* out, int h,
                       long long count, int vocab, int* error) {
    return d->launch(embedding_kernel, dim3(grid_for(count, 256, d->sm_count)), dim3(256), 0, ids, table,
                     table_dtype, out, h, count, vocab, error);
}

l0b_status k_copy(l0b_device* d, const float* src, float* dst, long long offset, long long n) {
    return d->launch(copy_kernel, dim3(grid_for(n, 256, d->sm_count)), dim3(256), 0, src, dst, offset, n);
}

l0b_status k_sampling(l0b_device* d, const float* logits, int* sampled, float temperature, float random_val,
                      int vocab) {
    if (temperature > 0.f) L0B_TRY(d->launch(fill_int_kernel, dim3(1), dim3(1), 0, sampled, vocab - 1));
    return d->launch(sampling_kernel, dim3(1), dim3(1024), 0, logits, sampled, temperature, random_val, vocab);
}

l0b_status k_quantize(l0b_device* d, const void* w, int w_dtype, int n, int k, int group, int8_t* q, __half* s) {
    const long long warps = static_cast<long long>(n) * (k / group);
    const long long blocks = (warps * 32 + 255) / 256;
    return d->launch(quantize_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, w, w_dtype, n, k, group, q,
                     s);
}

}  // namespace l0b
