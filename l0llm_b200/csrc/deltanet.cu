// Gated DeltaNet (Qwen3.5 linear attention): causal depthwise conv + SiLU, and the gated delta-rule
// recurrence with the gated RMSNorm epilogue (L/LlmDecoderLayer.cs:381-397, ops CausalConv and GatedDelta).
//
// Recurrence: one CTA per value head, one thread per value column j. Thread j keeps column j of the
// head's state S [dk, dv] in registers for the whole call, so the state is read from HBM once and
// written once per call however many tokens it carries (decode: 1 token -> 2 x 64 KB per head, the
// HBM-bound step). Per token: S *= e^g; delta_j = beta (v_j - sum_i S[i,j] k_i); S[:, j] += k delta_j;
// o_j = sum_i S[i,j] q_i / sqrt(dk); then out_j = rmsnorm(o)_j * w_j * silu(z_j).
#include "common.cuh"
#include "ops.cuh"
#include "suite.h"

namespace l0b {

namespace {

__global__ void causal_conv_kernel(const float* x, float* state, const float* w, float* out, int conv_dim, int kernel,
                                   int tokens) {
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= conv_dim) return;
    const int hist = kernel - 1;
    float win[8];  // kernel <= 8
    float wc[8];
    for (int j = 0; j < hist; ++j) win[j] = state[static_cast<long long>(c) * hist + j];
    for (int j = 0; j < kernel; ++j) wc[j] = w[static_cast<long long>(c) * kernel + j];
    for (int t = 0; t < tokens; ++t) {
        const float xt = x[static_cast<long long>(t) * conv_dim + c];
        float acc = 0.f;
        for (int j = 0; j < hist; ++j) acc = fmaf(wc[j], win[j], acc);
        acc = fmaf(wc[hist], xt, acc);
        out[static_cast<long long>(t) * conv_dim + c] = silu(acc);
        for (int j = 0; j + 1 < hist; ++j) win[j] = win[j + 1];
        if (hist > 0) win[hist - 1] = xt;
    }
    for (int j = 0; j < hist; ++j) state[static_cast<long long>(c) * hist + j] = win[j];
}

// Many tokens, input and output apart: every (token, channel) output at once. Input at time tau < 0
// comes from the conv window (state holds times -hist .. -1); the window is rolled by the next kernel.
__global__ void causal_conv_tokens_kernel(const float* __restrict__ x, const float* __restrict__ state,
                                          const float* __restrict__ w, float* __restrict__ out, int conv_dim,
                                          int kernel, int tokens) {
    pdl_wait();
    const int hist = kernel - 1;
    const long long total = static_cast<long long>(tokens) * conv_dim;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(e / conv_dim), c = static_cast<int>(e - static_cast<long long>(t) * conv_dim);
        float acc = 0.f;
        for (int j = 0; j < kernel; ++j) {
            const int tau = t - hist + j;
            const float v = tau >= 0 ? x[static_cast<long long>(tau) * conv_dim + c]
                                     : state[static_cast<long long>(c) * hist + hist + tau];
            acc = fmaf(w[static_cast<long long>(c) * kernel + j], v, acc);
        }
        out[e] = silu(acc);
    }
}

// The conv window after `tokens` inputs: times tokens - hist .. tokens - 1, each channel read whole
// before it is written.
__global__ void causal_conv_window_kernel(const float* __restrict__ x, float* state, int conv_dim, int kernel,
                                          int tokens) {
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int hist = kernel - 1;
    if (c >= conv_dim || hist == 0) return;
    float nw[8];
    for (int j = 0; j < hist; ++j) {
        const int tau = tokens - hist + j;
        nw[j] = tau >= 0 ? x[static_cast<long long>(tau) * conv_dim + c] : state[static_cast<long long>(c) * hist + hist + tau];
    }
    for (int j = 0; j < hist; ++j) state[static_cast<long long>(c) * hist + j] = nw[j];
}

template <int DK>
__global__ void __launch_bounds__(256) gated_delta_kernel(const float* conv, const float* z, const float* b,
                                                          const float* a, const float* a_log, const float* dt_bias,
                                                          const float* norm_w, float* state, float* out, int hk, int hv,
                                                          int dv, int tokens, float eps) {
    __shared__ float qs[DK], ks[DK];
    __shared__ float red[32];
    pdl_wait();
    const int h = blockIdx.x;
    const int j = threadIdx.x;  // value column
    const int rep = hv / hk, kh = h / rep;
    const int conv_dim = 2 * hk * DK + hv * dv;
    float* S = state + static_cast<long long>(h) * DK * dv;
    float s[DK];
#pragma unroll
    for (int i = 0; i < DK; ++i) s[i] = j < dv ? S[static_cast<long long>(i) * dv + j] : 0.f;
    const float A = -expf(a_log[h]);
    const float bias = dt_bias[h];
    const float qscale = rsqrtf(static_cast<float>(DK));
    const float wj = j < dv ? norm_w[j] : 0.f;
    for (int t = 0; t < tokens; ++t) {
        const float* row = conv + static_cast<long long>(t) * conv_dim;
        // L2-normalise q and k of key head kh (eps 1e-6 inside the root, HF l2norm).
        float qv = 0.f, kv = 0.f;
        for (int i = j; i < DK; i += blockDim.x) {
            qv = row[kh * DK + i];
            kv = row[hk * DK + kh * DK + i];
            qs[i] = qv;
            ks[i] = kv;
        }
        __syncthreads();
        float pq = 0.f, pk = 0.f;
        for (int i = j; i < DK; i += blockDim.x) {
            pq += qs[i] * qs[i];
            pk += ks[i] * ks[i];
        }
        const float nq = block_sum(pq, red);
        __syncthreads();
        const float nk = block_sum(pk, red);
        const float iq = rsqrtf(nq + 1e-6f) * qscale, ik = rsqrtf(nk + 1e-6f);
        const float beta = 1.f / (1.f + expf(-b[static_cast<long long>(t) * hv + h]));
        const float xa = a[static_cast<long long>(t) * hv + h] + bias;
        const float softplus = xa > 20.f ? xa : log1pf(expf(xa));
        const float decay = expf(A * softplus);
        float o = 0.f;
        if (j < dv) {
            const float v = row[2 * hk * DK + h * dv + j];
            float mem = 0.f;
#pragma unroll
            for (int i = 0; i < DK; ++i) {
                s[i] *= decay;
                mem = fmaf(s[i], ks[i] * ik, mem);
            }
            const float delta = (v - mem) * beta;
#pragma unroll
            for (int i = 0; i < DK; ++i) {
                s[i] = fmaf(ks[i] * ik, delta, s[i]);
                o = fmaf(s[i], qs[i] * iq, o);
            }
        }
        __syncthreads();
        const float ss = block_sum(o * o, red);
        const float rstd = rsqrtf(ss / static_cast<float>(dv) + eps);
        if (j < dv) {
            const float zz = z[static_cast<long long>(t) * hv * dv + static_cast<long long>(h) * dv + j];
            out[static_cast<long long>(t) * hv * dv + static_cast<long long>(h) * dv + j] = (o * rstd) * wj * silu(zz);
        }
        __syncthreads();
    }
    if (j < dv) {
#pragma unroll
        for (int i = 0; i < DK; ++i) S[static_cast<long long>(i) * dv + j] = s[i];
    }
}

// Prefill form of the recurrence: the columns of a head's state are independent given the token's
// normalised q and k, beta and decay, so one warp owns 16 columns of one value head (grid: value head x
// column group) and walks the tokens with no block barrier. Lane l holds rows [(l / 16) DK/2, +DK/2) of
// column l % 16 in registers; the two halves of each dot product meet with one shuffle. The warp
// L2-normalises q and k itself (shuffles) and loads the next token while computing this one. It writes
// the raw output o; gated_norm_kernel applies the gated RMSNorm afterwards over all tokens at once.
template <int DK>
__global__ void __launch_bounds__(32) gated_delta_scan_kernel(const float* __restrict__ conv, const float* __restrict__ b,
                                                              const float* __restrict__ a, const float* __restrict__ a_log,
                                                              const float* __restrict__ dt_bias, float* state,
                                                              float* __restrict__ out, int hk, int hv, int dv, int tokens) {
    constexpr int PER = DK / 32;  // q/k elements each lane loads
    constexpr int HR = DK / 2;    // state rows per lane
    __shared__ float qs[2][DK], ks[2][DK];
    pdl_wait();
    const int h = blockIdx.x, lane = threadIdx.x;
    const int j = blockIdx.y * 16 + (lane & 15), r0 = (lane >> 4) * HR;
    const bool live = j < dv;
    const int rep = hv / hk, kh = h / rep;
    const int conv_dim = 2 * hk * DK + hv * dv;
    float* S = state + static_cast<long long>(h) * DK * dv;
    float s[HR];
#pragma unroll
    for (int i = 0; i < HR; ++i) s[i] = live ? S[static_cast<long long>(r0 + i) * dv + j] : 0.f;
    const float A = -expf(a_log[h]);
    const float bias = dt_bias[h];
    const float qscale = rsqrtf(static_cast<float>(DK));
    // Token t's inputs, loaded one token ahead.
    float qv[PER], kv[PER], vv = 0.f, bv = 0.f, av = 0.f;
    auto load = [&](int t) {
        const float* row = conv + static_cast<long long>(t) * conv_dim;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            qv[e] = row[kh * DK + lane + 32 * e];
            kv[e] = row[hk * DK + kh * DK + lane + 32 * e];
        }
        vv = live ? row[2 * hk * DK + h * dv + j] : 0.f;
        bv = b[static_cast<long long>(t) * hv + h];
        av = a[static_cast<long long>(t) * hv + h];
    };
    if (tokens > 0) load(0);
    for (int t = 0; t < tokens; ++t) {
        const int buf = t & 1;
        float pq = 0.f, pk = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            pq = fmaf(qv[e], qv[e], pq);
            pk = fmaf(kv[e], kv[e], pk);
        }
        pq = warp_sum(pq);
        pk = warp_sum(pk);
        const float iq = rsqrtf(pq + 1e-6f) * qscale, ik = rsqrtf(pk + 1e-6f);
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            qs[buf][lane + 32 * e] = qv[e] * iq;
            ks[buf][lane + 32 * e] = kv[e] * ik;
        }
        const float beta = 1.f / (1.f + expf(-bv));
        const float xa = av + bias;
        const float decay = expf(A * (xa > 20.f ? xa : log1pf(expf(xa))));
        const float v = vv;
        __syncwarp();
        if (t + 1 < tokens) load(t + 1);
        const float* kb = &ks[buf][r0];
        const float* qb = &qs[buf][r0];
        float m0 = 0.f, m1 = 0.f;
#pragma unroll
        for (int i = 0; i < HR; i += 2) {
            s[i] *= decay;
            s[i + 1] *= decay;
            m0 = fmaf(s[i], kb[i], m0);
            m1 = fmaf(s[i + 1], kb[i + 1], m1);
        }
        float mem = m0 + m1;
        mem += __shfl_xor_sync(0xffffffffu, mem, 16);
        const float delta = (v - mem) * beta;
        float o0 = 0.f, o1 = 0.f;
#pragma unroll
        for (int i = 0; i < HR; i += 2) {
            s[i] = fmaf(kb[i], delta, s[i]);
            s[i + 1] = fmaf(kb[i + 1], delta, s[i + 1]);
            o0 = fmaf(s[i], qb[i], o0);
            o1 = fmaf(s[i + 1], qb[i + 1], o1);
        }
        float o = o0 + o1;
        o += __shfl_xor_sync(0xffffffffu, o, 16);
        if (live && lane < 16) out[static_cast<long long>(t) * hv * dv + static_cast<long long>(h) * dv + j] = o;
    }
    if (live) {
#pragma unroll
        for (int i = 0; i < HR; ++i) S[static_cast<long long>(r0 + i) * dv + j] = s[i];
    }
}

// out[t, h, :] = rmsnorm(o) * w * silu(z), in place over the raw outputs of every (token, value head).
__global__ void __launch_bounds__(256) gated_norm_kernel(float* out, const float* __restrict__ z,
                                                         const float* __restrict__ norm_w, int dv, float eps) {
    __shared__ float red[32];
    pdl_wait();
    const long long base = static_cast<long long>(blockIdx.x) * dv;
    const int j = threadIdx.x;
    const float o = j < dv ? out[base + j] : 0.f;
    const float ss = block_sum(o * o, red);
    const float rstd = rsqrtf(ss / static_cast<float>(dv) + eps);
    if (j < dv) out[base + j] = (o * rstd) * norm_w[j] * silu(z[base + j]);
}

}  // namespace

l0b_status k_causal_conv(l0b_device* d, const float* x, float* state, const float* w, float* out, int conv_dim,
                         int kernel, int tokens) {
    if (tokens >= 16 && x != out) {
        // Prefill: token-parallel outputs, then the window roll.
        const long long total = static_cast<long long>(tokens) * conv_dim;
        long long blocks = (total + 255) / 256;
        if (blocks > d->sm_count * 16LL) blocks = d->sm_count * 16LL;
        L0B_TRY(d->launch(causal_conv_tokens_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, x,
                          static_cast<const float*>(state), w, out, conv_dim, kernel, tokens));
        return d->launch(causal_conv_window_kernel, dim3((conv_dim + 127) / 128), dim3(128), 0, x, state, conv_dim,
                         kernel, tokens);
    }
    return d->launch(causal_conv_kernel, dim3((conv_dim + 127) / 128), dim3(128), 0, x, state, w, out, conv_dim, kernel,
                     tokens);
}

l0b_status k_gated_delta(l0b_device* d, const float* conv, const float* z, const float* b, const float* a,
                         const float* a_log, const float* dt_bias, const float* norm_w, float* state, float* out, int hk,
                         int hv, int dk, int dv, int tokens, float eps) {
    const int threads = ((dv + 31) / 32) * 32;
    if (tokens >= 16 && (dk == 128 || dk == 64)) {
        // Prefill: the warp-level scan, then the gated norm over all tokens.
        const dim3 grid(hv, (dv + 15) / 16);
        if (dk == 128)
            L0B_TRY(d->launch(gated_delta_scan_kernel<128>, grid, dim3(32), 0, conv, b, a, a_log, dt_bias, state, out,
                              hk, hv, dv, tokens));
        else
            L0B_TRY(d->launch(gated_delta_scan_kernel<64>, grid, dim3(32), 0, conv, b, a, a_log, dt_bias, state, out,
                              hk, hv, dv, tokens));
        return d->launch(gated_norm_kernel, dim3(tokens * hv), dim3(threads), 0, out, z, norm_w, dv, eps);
    }
    if (dk == 128)
        return d->launch(gated_delta_kernel<128>, dim3(hv), dim3(threads), 0, conv, z, b, a, a_log, dt_bias, norm_w,
                         state, out, hk, hv, dv, tokens, eps);
    if (dk == 64)
        return d->launch(gated_delta_kernel<64>, dim3(hv), dim3(threads), 0, conv, z, b, a, a_log, dt_bias, norm_w,
                         state, out, hk, hv, dv, tokens, eps);
    return fail(L0B_ERR_UNSUPPORTED, "gated delta key head dim %d (64 or 128 are supported)", dk);
}

}  // namespace l0b

using namespace l0b;

namespace {

l0b_status need_f32(l0b_buffer* b, const char* name, long long count) {
    L0B_REQUIRE(b, L0B_ERR_ARGUMENT, "%s is null", name);
    L0B_REQUIRE(b->dtype == L0B_F32, L0B_ERR_ARGUMENT, "%s must be an f32 buffer", name);
    L0B_REQUIRE(b->count >= count, L0B_ERR_ARGUMENT, "%s holds %lld elements, need %lld", name, (long long)b->count,
                count);
    return L0B_OK;
}

float* P(l0b_buffer* b) { return static_cast<float*>(b->ptr); }

}  // namespace

extern "C" {

L0B_API l0b_status l0b_causal_conv_execute(l0b_suite* s, l0b_device* d, l0b_buffer* qkv, l0b_buffer* conv_state,
                                           l0b_buffer* conv_w, l0b_buffer* out, int32_t conv_dim, int32_t kernel,
                                           int32_t tokens) {
    L0B_REQUIRE(s && d && s->dev == d, L0B_ERR_ARGUMENT, "suite/device mismatch");
    L0B_REQUIRE(conv_dim > 0 && kernel >= 1 && kernel <= 8 && tokens > 0, L0B_ERR_OUT_OF_RANGE,
                "convDim %d kernel %d tokens %d (kernel 1..8)", conv_dim, kernel, tokens);
    const long long n = static_cast<long long>(tokens) * conv_dim;
    L0B_TRY(need_f32(qkv, "qkv", n));
    L0B_TRY(need_f32(out, "out", n));
    L0B_TRY(need_f32(conv_state, "convState", static_cast<long long>(conv_dim) * (kernel - 1)));
    L0B_TRY(need_f32(conv_w, "convW", static_cast<long long>(conv_dim) * kernel));
    return k_causal_conv(d, P(qkv), P(conv_state), P(conv_w), P(out), conv_dim, kernel, tokens);
}

L0B_API l0b_status l0b_gated_delta_execute_grouped(l0b_suite* s, l0b_device* d, l0b_buffer* conv, l0b_buffer* z,
                                                   l0b_buffer* b, l0b_buffer* a, l0b_buffer* a_log, l0b_buffer* dt_bias,
                                                   l0b_buffer* norm_w, l0b_buffer* state, l0b_buffer* out,
                                                   int32_t n_k_heads, int32_t n_v_heads, int32_t key_dim,
                                                   int32_t value_dim, int32_t tokens, float eps) {
    L0B_REQUIRE(s && d && s->dev == d, L0B_ERR_ARGUMENT, "suite/device mismatch");
    L0B_REQUIRE(n_k_heads > 0 && n_v_heads > 0 && n_v_heads % n_k_heads == 0, L0B_ERR_ARGUMENT,
                "value heads %d must be a multiple of key heads %d", n_v_heads, n_k_heads);
    L0B_REQUIRE(value_dim > 0 && value_dim <= 256 && tokens > 0, L0B_ERR_OUT_OF_RANGE, "value dim %d tokens %d",
                value_dim, tokens);
    const long long conv_dim = 2LL * n_k_heads * key_dim + static_cast<long long>(n_v_heads) * value_dim;
    const long long vd = static_cast<long long>(n_v_heads) * value_dim;
    L0B_TRY(need_f32(conv, "conv", tokens * conv_dim));
    L0B_TRY(need_f32(z, "z", tokens * vd));
    L0B_TRY(need_f32(b, "b", static_cast<long long>(tokens) * n_v_heads));
    L0B_TRY(need_f32(a, "a", static_cast<long long>(tokens) * n_v_heads));
    L0B_TRY(need_f32(a_log, "A_log", n_v_heads));
    L0B_TRY(need_f32(dt_bias, "dt_bias", n_v_heads));
    L0B_TRY(need_f32(norm_w, "normW", value_dim));
    L0B_TRY(need_f32(state, "S", static_cast<long long>(n_v_heads) * key_dim * value_dim));
    L0B_TRY(need_f32(out, "out", tokens * vd));
    return k_gated_delta(d, P(conv), P(z), P(b), P(a), P(a_log), P(dt_bias), P(norm_w), P(state), P(out), n_k_heads,
                         n_v_heads, key_dim, value_dim, tokens, eps);
}

L0B_API l0b_status l0b_gated_delta_execute(l0b_suite* s, l0b_device* d, l0b_buffer* conv, l0b_buffer* z, l0b_buffer* b,
                                           l0b_buffer* a, l0b_buffer* a_log, l0b_buffer* dt_bias, l0b_buffer* norm_w,
                                           l0b_buffer* state, l0b_buffer* out, int32_t n_v_heads, int32_t key_dim,
                                           int32_t value_dim, int32_t tokens, float eps) {
    return l0b_gated_delta_execute_grouped(s, d, conv, z, b, a, a_log, dt_bias, norm_w, state, out, n_v_heads,
                                           n_v_heads, key_dim, value_dim, tokens, eps);
}

}  // extern "C"
