// Tensor-core (tcgen05 / TMEM / TMA) GEMM for prefill and batched decode: Y[M, N] = X[M, K] W[N, K]^T.
#pragma once

#include "runtime.h"

namespace l0b {

struct TcGemmArgs {
    int M, N, K;           // tokens, weight rows, inner dimension
    const void* x16;       // [M, K] activations in the weight's 16-bit format (row stride K)
    const void* w;         // [N, K] weights, f16, bf16 or int8
    int wdtype;            // L0B_F16, L0B_BF16 or L0B_I8 (activations then f16)
    int epi;               // GemvEpi: STORE, ACCUM or SWIGLU (W = [gate; up], N = 2 * I)
    float* out;            // f32 output, row stride ld (SWIGLU: [M, N/2])
    int ld;
    const float* bias;     // STORE / ACCUM: f32 [N] or null
    // Split activations (cast_rows_split_launch): x16 is [M, 2 Kp], hi in columns [0, K) and the f16
    // residual lo in [Kp, Kp + K), Kp = 64 * ceil(K / 64); every weight tile meets both halves in the
    // same accumulator, and row t of the result is multiplied by rscale[t].
    int split = 0;
    const float* rscale = nullptr;
    const void* wscale = nullptr;  // int8: f16 [N], one scale per weight row
};

// Launches the GEMM on the device's stream (recorded when the device records).
l0b_status tc_gemm_launch(l0b_device* d, const TcGemmArgs& a);

// out16[m, :] = (RMSNorm(x[m, :]) if norm_w) in f16/bf16 for m < M; x row stride ld_x.
l0b_status cast_rows_launch(l0b_device* d, const float* x, long long ld_x, const float* norm_w, float eps, void* out16,
                            int dtype, int M, int K);

// out16 = the rows of x (RMS-normalised with norm_w when given) split as [hi | lo] in f16/bf16 with
// row stride 2 Kp (Kp = 64 * ceil(K / 64), padding zeroed); for f16 each row is first scaled by a power
// of two putting its largest value near 2^14, and rscale[m] receives the inverse.
l0b_status cast_rows_split_launch(l0b_device* d, const float* x, long long ld_x, const float* norm_w, float eps,
                                  void* out16, float* rscale, int dtype, int M, int K);

// True when the tensor-core path takes this shape: f16/bf16 weights with K % 8 == 0 or int8 weights
// (per-row scales) with K % 16 == 0, K >= 64; SwiGLU needs (N / 2) % 64 == 0.
bool tc_gemm_supported(int wdtype, int M, int N, int K, int epi);

}  // namespace l0b
