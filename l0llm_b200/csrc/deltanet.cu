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

bool g_gdn_chunked = true;  // chunked prefill of the recurrence (l0b_set_gated_delta_chunked)

namespace {

// blockIdx.y selects a sequence of a batch: its rows of x / out start seq_x floats apart and its conv
// window seq_state floats apart (0 for one sequence).
__global__ void causal_conv_kernel(const float* x, float* state, const float* w, float* out, int conv_dim, int kernel,
                                   int tokens, long long seq_x, long long seq_state) {
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= conv_dim) return;
    x += blockIdx.y * seq_x;
    out += blockIdx.y * seq_x;
    state += blockIdx.y * seq_state;
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

// blockIdx.y selects a sequence of a batch (one token each): its conv / z / out / b / a rows and its state
// lie seq (its index) rows and seq * hv * DK * dv floats further on.
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
    {
        const long long sq = blockIdx.y;
        conv += sq * conv_dim;
        z += sq * hv * dv;
        out += sq * hv * dv;
        b += sq * hv;
        a += sq * hv;
        state += sq * hv * static_cast<long long>(DK) * dv;
    }
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

// ---------------------------------------------------------------------------------------------
// Chunked prefill of the recurrence (the WY form of the gated delta rule, chunks of kGdnChunk tokens).
//
// Within a chunk, with G_i the running sum of the log-decays g (so e^(G_i - G_j) <= 1 for j <= i),
// beta_i the write strength, q (scaled by 1/sqrt(dk)) and k L2-normalised, and S0 the state entering
// the chunk, the per-token recurrence S_i = e^(g_i) S_(i-1) + k_i d_i^T,
// d_i = beta_i (v_i - (e^(g_i) S_(i-1))^T k_i), unrolls to
//     (I + A) D = beta*V - (beta e^G K) S0,   A_ij = beta_i e^(G_i - G_j) k_i.k_j  (j < i)
// so D = U - W S0 with U = (I + A)^-1 beta*V and W = (I + A)^-1 beta e^G K (forward substitution), and
//     O = (e^G Q) S0 + P D,                    P_ij = e^(G_i - G_j) q_i.k_j       (j <= i)
//     S_end = e^(G_last) S0 + K'^T D,          K'_j = e^(G_last - G_j) k_j.
// gdn_chunk_prep_kernel builds U, W, e^G Q, K', P and e^(G_last) for every (value head, chunk) at once
// (none depends on the state); gdn_chunk_scan_kernel then walks the chunks of a head in order for a
// group of state columns (the columns of S are independent given those), holding its columns of S in
// shared memory, and writes the raw outputs o that gated_norm_kernel turns into
// rmsnorm(o) * w * silu(z). fp32 throughout.
// ---------------------------------------------------------------------------------------------
constexpr int kGdnChunk = 64;
constexpr int kGdnCols = 32;  // state columns per scan CTA

// Floats of one (value head, chunk) record: U [C, dv], W [C, DK], e^G Q [C, DK], K' [C, DK], P [C, C],
// e^(G_last) (padded to 4).
__host__ __device__ inline long long gdn_record_floats(int dk, int dv) {
    return static_cast<long long>(kGdnChunk) * (dv + 3 * dk) + kGdnChunk * kGdnChunk + 4;
}

template <int DK>
__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(const float* __restrict__ conv, const float* __restrict__ b,
                                                             const float* __restrict__ a, const float* __restrict__ a_log,
                                                             const float* __restrict__ dt_bias, float* __restrict__ rec,
                                                             int hk, int hv, int dv, int tokens) {
    constexpr int C = kGdnChunk, LD = DK + 1, LA = C + 4;
    extern __shared__ float gsm[];
    float* qs = gsm;                 // [C][LD] normalised, scaled q
    float* ks = qs + C * LD;         // [C][LD] normalised k
    float* As = ks + C * LD;         // [C][LA] (rows 16-byte aligned for 4-wide reads)
    __shared__ float G[C], beta[C];
    pdl_wait();
    const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nchunks = gridDim.x;
    const int t0 = c * C, L = min(C, tokens - t0);
    const int rep = hv / hk, kh = h / rep;
    const long long conv_dim = 2LL * hk * DK + static_cast<long long>(hv) * dv;
    float* R = rec + (static_cast<long long>(h) * nchunks + c) * gdn_record_floats(DK, dv);
    float* U = R;
    float* W = U + C * dv;
    float* Qg = W + C * DK;
    float* Kp = Qg + C * DK;
    float* P = Kp + C * DK;
    float* gl = P + C * C;
    // q and k rows, L2-normalised (eps 1e-6 inside the root); rows past the chunk are zero.
    const float qscale = rsqrtf(static_cast<float>(DK));
    for (int i = warp; i < C; i += 8) {
        float qv[DK / 32], kv[DK / 32], pq = 0.f, pk = 0.f;
        const float* row = conv + static_cast<long long>(t0 + i) * conv_dim;
#pragma unroll
        for (int e = 0; e < DK / 32; ++e) {
            qv[e] = i < L ? row[kh * DK + lane + 32 * e] : 0.f;
            kv[e] = i < L ? row[hk * DK + kh * DK + lane + 32 * e] : 0.f;
            pq = fmaf(qv[e], qv[e], pq);
            pk = fmaf(kv[e], kv[e], pk);
        }
        pq = warp_sum(pq);
        pk = warp_sum(pk);
        const float iq = rsqrtf(pq + 1e-6f) * qscale, ik = rsqrtf(pk + 1e-6f);
#pragma unroll
        for (int e = 0; e < DK / 32; ++e) {
            qs[i * LD + lane + 32 * e] = qv[e] * iq;
            ks[i * LD + lane + 32 * e] = kv[e] * ik;
        }
    }
    if (tid < C) {
        const int i = tid;
        float bt = 0.f, gt = 0.f;
        if (i < L) {
            bt = 1.f / (1.f + expf(-b[static_cast<long long>(t0 + i) * hv + h]));
            const float xa = a[static_cast<long long>(t0 + i) * hv + h] + dt_bias[h];
            gt = -expf(a_log[h]) * (xa > 20.f ? xa : log1pf(expf(xa)));
        }
        beta[i] = bt;
        G[i] = gt;
    }
    __syncthreads();
    if (tid == 0) {
        float run = 0.f;
        for (int i = 0; i < C; ++i) {
            run += G[i];
            G[i] = run;
        }
    }
    __syncthreads();
    // A (strictly lower, times beta_i) and P (lower with the diagonal): thread = (row i, columns
    // j = jr + 4 jj), so the four lanes of a row read four consecutive key rows (distinct banks).
    {
        const int i = tid >> 2, jr = tid & 3;
        float kk[16], qk[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) kk[jj] = qk[jj] = 0.f;
        for (int d = 0; d < DK; ++d) {
            const float ki = ks[i * LD + d], qi = qs[i * LD + d];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                const float kj = ks[(jr + 4 * jj) * LD + d];
                kk[jj] = fmaf(ki, kj, kk[jj]);
                qk[jj] = fmaf(qi, kj, qk[jj]);
            }
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
            const int j = jr + 4 * jj;
            const bool in = i < L && j < L;
            const float dec = (in && j <= i) ? expf(G[i] - G[j]) : 0.f;
            As[i * LA + j] = (j < i) ? beta[i] * dec * kk[jj] : 0.f;
            P[i * C + j] = dec * qk[jj];
        }
    }
    __syncthreads();
    // Forward substitution for the columns of [U | W]: X_i = rhs_i - sum_(j < i) A_ij X_j.
    if (tid < dv + DK) {
        const bool is_u = tid < dv;
        const int col = is_u ? tid : tid - dv;
        const float* vrow = conv + static_cast<long long>(t0) * conv_dim + 2LL * hk * DK + static_cast<long long>(h) * dv + col;
        float x[C];
#pragma unroll
        for (int i = 0; i < C; ++i) {
            float rhs = 0.f;
            if (i < L) rhs = is_u ? beta[i] * vrow[static_cast<long long>(i) * conv_dim] : beta[i] * expf(G[i]) * ks[i * LD + col];
            // Two chains (even and odd j) and 4-wide reads of row i of A.
            float r1 = 0.f;
#pragma unroll
            for (int j = 0; j < (i & ~3); j += 4) {
                const float4 av = *reinterpret_cast<const float4*>(&As[i * LA + j]);
                rhs = fmaf(-av.x, x[j], rhs);
                r1 = fmaf(-av.y, x[j + 1], r1);
                rhs = fmaf(-av.z, x[j + 2], rhs);
                r1 = fmaf(-av.w, x[j + 3], r1);
            }
#pragma unroll
            for (int j = i & ~3; j < i; ++j) rhs = fmaf(-As[i * LA + j], x[j], rhs);
            x[i] = rhs + r1;
        }
        float* dst = is_u ? U + col : W + col;
        const int ld = is_u ? dv : DK;
#pragma unroll
        for (int i = 0; i < C; ++i) dst[i * ld] = x[i];
    }
    // e^G q and the decayed keys K'.
    const float glast = L > 0 ? G[L - 1] : 0.f;
    for (int e = tid; e < C * DK; e += 256) {
        const int i = e / DK, d = e - i * DK;
        const bool in = i < L;
        Qg[e] = in ? expf(G[i]) * qs[i * LD + d] : 0.f;
        Kp[e] = in ? expf(glast - G[i]) * ks[i * LD + d] : 0.f;
    }
    if (tid == 0) {
        gl[0] = expf(glast);
        gl[1] = gl[2] = gl[3] = 0.f;
    }
}

__device__ __forceinline__ void cp_async16(float* smem_dst, const float* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                 "l"(gmem_src)
                 : "memory");
}

template <int DK>
__global__ void __launch_bounds__(256) gdn_chunk_scan_kernel(const float* __restrict__ rec, float* state,
                                                             float* __restrict__ out, int hv, int dv, int tokens) {
    constexpr int C = kGdnChunk, NC = kGdnCols, LW = DK + 4;
    extern __shared__ float ssm[];
    float* Ws = ssm;              // [C][LW]
    float* Qs = Ws + C * LW;      // [C][LW]
    float* Ks = Qs + C * LW;      // [C][DK]
    float* Ps = Ks + C * DK;      // [C][C]
    float* Us = Ps + C * C;       // [C][NC]
    float* Ds = Us + C * NC;      // [C][NC]
    float* Ss = Ds + C * NC;      // [DK][NC]
    pdl_wait();
    const int h = blockIdx.x, col0 = blockIdx.y * NC, tid = threadIdx.x;
    const int nchunks = (tokens + C - 1) / C;
    float* S = state + static_cast<long long>(h) * DK * dv;
    for (int e = tid; e < DK * NC; e += 256) {
        const int k = e / NC, cc = e - k * NC;
        Ss[e] = S[static_cast<long long>(k) * dv + col0 + cc];
    }
    const int ri = tid >> 2, rc = (tid & 3) * 8;    // D and O: row ri, 8 columns
    // S update: state row sk (< DK: threads past 2 * DK idle when DK = 64), 16 columns.
    const int sk = tid >> 1, sc = (tid & 1) * 16;
    const bool s_live = tid < 2 * DK;
    for (int c = 0; c < nchunks; ++c) {
        const float* R = rec + (static_cast<long long>(h) * nchunks + c) * gdn_record_floats(DK, dv);
        const float* U = R;
        const float* W = U + C * dv;
        const float* Qg = W + C * DK;
        const float* Kp = Qg + C * DK;
        const float* P = Kp + C * DK;
        const float gamma = P[C * C];
        __syncthreads();  // the previous chunk is done with the staged record
        // All of the chunk's staging copies in flight at once (16-byte cp.async), then one wait.
        for (int e = tid; e < C * DK / 4; e += 256) {
            const int i = (e * 4) / DK, d = (e * 4) - i * DK;
            cp_async16(&Ws[i * LW + d], W + 4 * e);
            cp_async16(&Qs[i * LW + d], Qg + 4 * e);
            cp_async16(&Ks[4 * e], Kp + 4 * e);
        }
        for (int e = tid; e < C * C / 4; e += 256) cp_async16(&Ps[4 * e], P + 4 * e);
        for (int e = tid; e < C * NC / 4; e += 256) {
            const int i = (e * 4) / NC, cc = (e * 4) - i * NC;
            cp_async16(&Us[4 * e], U + static_cast<long long>(i) * dv + col0 + cc);
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // D = U - W S0 (rows ri, columns rc .. rc + 7).
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = Us[ri * NC + rc + e];
        for (int k = 0; k < DK; ++k) {
            const float w = Ws[ri * LW + k];
            const float4 s0 = *reinterpret_cast<const float4*>(&Ss[k * NC + rc]);
            const float4 s1 = *reinterpret_cast<const float4*>(&Ss[k * NC + rc + 4]);
            acc[0] = fmaf(-w, s0.x, acc[0]);
            acc[1] = fmaf(-w, s0.y, acc[1]);
            acc[2] = fmaf(-w, s0.z, acc[2]);
            acc[3] = fmaf(-w, s0.w, acc[3]);
            acc[4] = fmaf(-w, s1.x, acc[4]);
            acc[5] = fmaf(-w, s1.y, acc[5]);
            acc[6] = fmaf(-w, s1.z, acc[6]);
            acc[7] = fmaf(-w, s1.w, acc[7]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) Ds[ri * NC + rc + e] = acc[e];
        __syncthreads();
        // O = (e^G Q) S0 + P D.
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
        for (int k = 0; k < DK; ++k) {
            const float q = Qs[ri * LW + k];
            const float4 s0 = *reinterpret_cast<const float4*>(&Ss[k * NC + rc]);
            const float4 s1 = *reinterpret_cast<const float4*>(&Ss[k * NC + rc + 4]);
            acc[0] = fmaf(q, s0.x, acc[0]);
            acc[1] = fmaf(q, s0.y, acc[1]);
            acc[2] = fmaf(q, s0.z, acc[2]);
            acc[3] = fmaf(q, s0.w, acc[3]);
            acc[4] = fmaf(q, s1.x, acc[4]);
            acc[5] = fmaf(q, s1.y, acc[5]);
            acc[6] = fmaf(q, s1.z, acc[6]);
            acc[7] = fmaf(q, s1.w, acc[7]);
        }
        for (int j = 0; j <= ri; ++j) {
            const float pj = Ps[ri * C + j];
            const float4 d0 = *reinterpret_cast<const float4*>(&Ds[j * NC + rc]);
            const float4 d1 = *reinterpret_cast<const float4*>(&Ds[j * NC + rc + 4]);
            acc[0] = fmaf(pj, d0.x, acc[0]);
            acc[1] = fmaf(pj, d0.y, acc[1]);
            acc[2] = fmaf(pj, d0.z, acc[2]);
            acc[3] = fmaf(pj, d0.w, acc[3]);
            acc[4] = fmaf(pj, d1.x, acc[4]);
            acc[5] = fmaf(pj, d1.y, acc[5]);
            acc[6] = fmaf(pj, d1.z, acc[6]);
            acc[7] = fmaf(pj, d1.w, acc[7]);
        }
        const int t = c * C + ri;
        if (t < tokens) {
            float* o = out + static_cast<long long>(t) * hv * dv + static_cast<long long>(h) * dv + col0 + rc;
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = acc[e];
        }
        // S_end = e^(G_last) S0 + K'^T D (state row sk, columns sc .. sc + 15), written after every read of S0.
        float sn[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) sn[e] = s_live ? gamma * Ss[sk * NC + sc + e] : 0.f;
        for (int j = 0; j < C && s_live; ++j) {
            const float kj = Ks[j * DK + sk];
#pragma unroll
            for (int e = 0; e < 16; e += 4) {
                const float4 d = *reinterpret_cast<const float4*>(&Ds[j * NC + sc + e]);
                sn[e] = fmaf(kj, d.x, sn[e]);
                sn[e + 1] = fmaf(kj, d.y, sn[e + 1]);
                sn[e + 2] = fmaf(kj, d.z, sn[e + 2]);
                sn[e + 3] = fmaf(kj, d.w, sn[e + 3]);
            }
        }
        __syncthreads();
        if (s_live) {
#pragma unroll
            for (int e = 0; e < 16; ++e) Ss[sk * NC + sc + e] = sn[e];
        }
    }
    __syncthreads();
    for (int e = tid; e < DK * NC; e += 256) {
        const int k = e / NC, cc = e - k * NC;
        S[static_cast<long long>(k) * dv + col0 + cc] = Ss[e];
    }
}

template <int DK>
size_t gdn_prep_smem() {
    // q, k rows of DK + 1; A rows of C + 4 starting 16-byte aligned (2 C (DK + 1) is a multiple of 4).
    return static_cast<size_t>(2 * kGdnChunk * (DK + 1) + kGdnChunk * (kGdnChunk + 4)) * sizeof(float);
}
template <int DK>
size_t gdn_scan_smem() {
    return static_cast<size_t>(2 * kGdnChunk * (DK + 4) + kGdnChunk * DK + kGdnChunk * kGdnChunk + 2 * kGdnChunk * kGdnCols +
                               DK * kGdnCols) * sizeof(float);
}

template <int DK>
l0b_status gdn_chunked(l0b_device* d, float* rec, const float* conv, const float* z, const float* b, const float* a,
                       const float* a_log, const float* dt_bias, const float* norm_w, float* state, float* out, int hk,
                       int hv, int dv, int tokens, float eps) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(gdn_prep_smem<DK>()));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gdn_chunk_scan_kernel<DK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(gdn_scan_smem<DK>()));
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        configured = true;
    }
    const int nchunks = (tokens + kGdnChunk - 1) / kGdnChunk;
    L0B_TRY(d->launch(gdn_chunk_prep_kernel<DK>, dim3(nchunks, hv), dim3(256), gdn_prep_smem<DK>(), conv, b, a, a_log,
                      dt_bias, rec, hk, hv, dv, tokens));
    L0B_TRY(d->launch(gdn_chunk_scan_kernel<DK>, dim3(hv, dv / kGdnCols), dim3(256), gdn_scan_smem<DK>(),
                      static_cast<const float*>(rec), state, out, hv, dv, tokens));
    const int threads = ((dv + 31) / 32) * 32;
    return d->launch(gated_norm_kernel, dim3(tokens * hv), dim3(threads), 0, out, z, norm_w, dv, eps);
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
                     tokens, 0LL, 0LL);
}

// One token of each of `batch` sequences: rows b of x / out, window b of the [batch, conv_dim, kernel - 1] states.
l0b_status k_causal_conv_batch(l0b_device* d, const float* x, float* states, const float* w, float* out, int conv_dim,
                               int kernel, int batch) {
    return d->launch(causal_conv_kernel, dim3((conv_dim + 127) / 128, batch), dim3(128), 0, x, states, w, out, conv_dim,
                     kernel, 1, static_cast<long long>(conv_dim), static_cast<long long>(conv_dim) * (kernel - 1));
}

// One token of each of `batch` sequences, states [batch, hv, dk, dv].
l0b_status k_gated_delta_batch(l0b_device* d, const float* conv, const float* z, const float* b, const float* a,
                               const float* a_log, const float* dt_bias, const float* norm_w, float* states, float* out,
                               int hk, int hv, int dk, int dv, int batch, float eps) {
    const int threads = ((dv + 31) / 32) * 32;
    if (dk == 128)
        return d->launch(gated_delta_kernel<128>, dim3(hv, batch), dim3(threads), 0, conv, z, b, a, a_log, dt_bias,
                         norm_w, states, out, hk, hv, dv, 1, eps);
    if (dk == 64)
        return d->launch(gated_delta_kernel<64>, dim3(hv, batch), dim3(threads), 0, conv, z, b, a, a_log, dt_bias,
                         norm_w, states, out, hk, hv, dv, 1, eps);
    return fail(L0B_ERR_UNSUPPORTED, "gated delta key head dim %d (64 or 128 are supported)", dk);
}

// Scratch of the chunked prefill: one record per (value head, chunk), grown on demand outside a
// recording (a recorded call that would need more runs on the per-token scan instead).
float* gdn_scratch(l0b_suite* s, long long floats) {
    if (floats <= s->gdn_floats) return s->gdn_rec;
    if (s->dev->recording) return nullptr;
    if (s->gdn_rec) {
        cudaStreamSynchronize(s->dev->stream);
        cudaFree(s->gdn_rec);
        s->gdn_rec = nullptr;
        s->gdn_floats = 0;
    }
    if (cudaMalloc(&s->gdn_rec, static_cast<size_t>(floats) * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        s->gdn_rec = nullptr;
        return nullptr;
    }
    s->gdn_floats = floats;
    return s->gdn_rec;
}

l0b_status k_gated_delta(l0b_suite* s, l0b_device* d, const float* conv, const float* z, const float* b, const float* a,
                         const float* a_log, const float* dt_bias, const float* norm_w, float* state, float* out, int hk,
                         int hv, int dk, int dv, int tokens, float eps) {
    const int threads = ((dv + 31) / 32) * 32;
    if (tokens >= 16 && g_gdn_chunked && (dk == 128 || dk == 64) && dv % kGdnCols == 0 && dv <= 256 - dk && s) {
        const long long nchunks = (tokens + kGdnChunk - 1) / kGdnChunk;
        float* rec = gdn_scratch(s, nchunks * hv * gdn_record_floats(dk, dv));
        if (rec) {
            if (dk == 128)
                return gdn_chunked<128>(d, rec, conv, z, b, a, a_log, dt_bias, norm_w, state, out, hk, hv, dv, tokens, eps);
            return gdn_chunked<64>(d, rec, conv, z, b, a, a_log, dt_bias, norm_w, state, out, hk, hv, dv, tokens, eps);
        }
    }
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
    return k_gated_delta(s, d, P(conv), P(z), P(b), P(a), P(a_log), P(dt_bias), P(norm_w), P(state), P(out), n_k_heads,
                         n_v_heads, key_dim, value_dim, tokens, eps);
}

L0B_API l0b_status l0b_causal_conv_execute_batch(l0b_suite* s, l0b_device* d, l0b_buffer* qkv, l0b_buffer* conv_states,
                                                 l0b_buffer* conv_w, l0b_buffer* out, int32_t conv_dim, int32_t kernel,
                                                 int32_t batch) {
    L0B_REQUIRE(s && d && s->dev == d, L0B_ERR_ARGUMENT, "suite/device mismatch");
    L0B_REQUIRE(conv_dim > 0 && kernel >= 1 && kernel <= 8 && batch > 0 && batch <= 65535, L0B_ERR_OUT_OF_RANGE,
                "convDim %d kernel %d batch %d (kernel 1..8)", conv_dim, kernel, batch);
    const long long n = static_cast<long long>(batch) * conv_dim;
    L0B_TRY(need_f32(qkv, "qkv", n));
    L0B_TRY(need_f32(out, "out", n));
    L0B_TRY(need_f32(conv_states, "convStates", n * (kernel - 1)));
    L0B_TRY(need_f32(conv_w, "convW", static_cast<long long>(conv_dim) * kernel));
    return k_causal_conv_batch(d, P(qkv), P(conv_states), P(conv_w), P(out), conv_dim, kernel, batch);
}

L0B_API l0b_status l0b_gated_delta_execute_batch(l0b_suite* s, l0b_device* d, l0b_buffer* conv, l0b_buffer* z,
                                                 l0b_buffer* b, l0b_buffer* a, l0b_buffer* a_log, l0b_buffer* dt_bias,
                                                 l0b_buffer* norm_w, l0b_buffer* states, l0b_buffer* out,
                                                 int32_t n_k_heads, int32_t n_v_heads, int32_t key_dim,
                                                 int32_t value_dim, int32_t batch, float eps) {
    L0B_REQUIRE(s && d && s->dev == d, L0B_ERR_ARGUMENT, "suite/device mismatch");
    L0B_REQUIRE(n_k_heads > 0 && n_v_heads > 0 && n_v_heads % n_k_heads == 0, L0B_ERR_ARGUMENT,
                "value heads %d must be a multiple of key heads %d", n_v_heads, n_k_heads);
    L0B_REQUIRE(value_dim > 0 && value_dim <= 256 && batch > 0 && batch <= 65535, L0B_ERR_OUT_OF_RANGE,
                "value dim %d batch %d", value_dim, batch);
    const long long conv_dim = 2LL * n_k_heads * key_dim + static_cast<long long>(n_v_heads) * value_dim;
    const long long vd = static_cast<long long>(n_v_heads) * value_dim;
    L0B_TRY(need_f32(conv, "conv", batch * conv_dim));
    L0B_TRY(need_f32(z, "z", batch * vd));
    L0B_TRY(need_f32(b, "b", static_cast<long long>(batch) * n_v_heads));
    L0B_TRY(need_f32(a, "a", static_cast<long long>(batch) * n_v_heads));
    L0B_TRY(need_f32(a_log, "A_log", n_v_heads));
    L0B_TRY(need_f32(dt_bias, "dt_bias", n_v_heads));
    L0B_TRY(need_f32(norm_w, "normW", value_dim));
    L0B_TRY(need_f32(states, "states", batch * vd * key_dim));
    L0B_TRY(need_f32(out, "out", batch * vd));
    return k_gated_delta_batch(d, P(conv), P(z), P(b), P(a), P(a_log), P(dt_bias), P(norm_w), P(states), P(out),
                               n_k_heads, n_v_heads, key_dim, value_dim, batch, eps);
}

// The DeltaNet part of the device-side fork: sequence dst's conv window and recurrent state become copies
// of sequence src's, in batched state buffers ([batch, conv_dim, kernel - 1] and [batch, hv, dk, dv]).
L0B_API l0b_status l0b_linear_state_fork(l0b_suite* s, l0b_device* d, l0b_buffer* conv_states, l0b_buffer* states,
                                         int32_t conv_dim, int32_t kernel, int32_t n_v_heads, int32_t key_dim,
                                         int32_t value_dim, int32_t src, int32_t dst) {
    L0B_REQUIRE(s && d && s->dev == d, L0B_ERR_ARGUMENT, "suite/device mismatch");
    L0B_REQUIRE(conv_dim > 0 && kernel >= 1 && n_v_heads > 0 && key_dim > 0 && value_dim > 0, L0B_ERR_OUT_OF_RANGE,
                "state shape");
    L0B_REQUIRE(src >= 0 && dst >= 0, L0B_ERR_OUT_OF_RANGE, "sequences %d -> %d", src, dst);
    L0B_REQUIRE(src != dst, L0B_ERR_ARGUMENT, "a sequence cannot be forked onto itself");
    const long long cw = static_cast<long long>(conv_dim) * (kernel - 1);
    const long long rs = static_cast<long long>(n_v_heads) * key_dim * value_dim;
    const long long hi = src > dst ? src : dst;
    L0B_TRY(need_f32(conv_states, "convStates", (hi + 1) * cw));
    L0B_TRY(need_f32(states, "states", (hi + 1) * rs));
    L0B_REQUIRE(!d->recording, L0B_ERR_INVALID_OPERATION, "fork the state outside a recording");
    L0B_CHECK_CUDA(cudaSetDevice(d->index));
    if (cw > 0)
        L0B_CHECK_CUDA(cudaMemcpyAsync(P(conv_states) + dst * cw, P(conv_states) + src * cw, cw * sizeof(float),
                                       cudaMemcpyDeviceToDevice, d->stream));
    L0B_CHECK_CUDA(cudaMemcpyAsync(P(states) + dst * rs, P(states) + src * rs, rs * sizeof(float),
                                   cudaMemcpyDeviceToDevice, d->stream));
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gated_delta_chunked(int32_t enable) {
    g_gdn_chunked = enable != 0;
    return L0B_OK;
}

L0B_API l0b_status l0b_gated_delta_execute(l0b_suite* s, l0b_device* d, l0b_buffer* conv, l0b_buffer* z, l0b_buffer* b,
                                           l0b_buffer* a, l0b_buffer* a_log, l0b_buffer* dt_bias, l0b_buffer* norm_w,
                                           l0b_buffer* state, l0b_buffer* out, int32_t n_v_heads, int32_t key_dim,
                                           int32_t value_dim, int32_t tokens, float eps) {
    return l0b_gated_delta_execute_grouped(s, d, conv, z, b, a, a_log, dt_bias, norm_w, state, out, n_v_heads,
                                           n_v_heads, key_dim, value_dim, tokens, eps);
}

}  // extern "C"
