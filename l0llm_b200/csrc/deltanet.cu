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

}  // namespace

l0b_status k_causal_conv(l0b_device* d, const float* x, float* state, const float* w, float* out, int conv_dim,
                         int kernel, int tokens) {
    return d->launch(causal_conv_kernel, dim3((conv_dim + 127) / 128), dim3(128), 0, x, state, w, out, conv_dim, kernel,
                     tokens);
}

l0b_status k_gated_delta(l0b_device* d, const float* conv, const float* z, const float* b, const float* a,
                         const float* a_log, const float* dt_bias, const float* norm_w, float* state, float* out, int hk,
                         int hv, int dk, int dv, int tokens, float eps) {
    const int threads = ((dv + 31) / 32) * 32;
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
