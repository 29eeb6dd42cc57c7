// Tensor-core (tcgen05 / TMEM / TMA) GEMM for prefill and batched decode: Y[M, N] = X[M, K] W[N, K]^T.
#pragma once

#include "runtime.h"

namespace l0b {

// Tile plan of one GEMM: BN accumulator columns per CTA, of which TB are tokens (TB = BN / 2 when the
// activations come as hi / lo pairs); tiles_x token tiles x tiles_y weight tiles, each split S ways
// along K. With S > 1 every split writes its partial tile to `part` and the last split of a tile to
// finish (an atomic counter per tile) sums them in split order and runs the epilogue.
struct TcPlan {
    int bn = 64, tb = 64, tiles_x = 1, tiles_y = 1, S = 1;
    size_t part_floats = 0;  // scratch the split needs (tiles * S * TB * 128)
    int counters = 0;        // tile counters the split needs
};

struct TcGemmArgs {
    int M, N, K;           // tokens, weight rows, inner dimension
    const void* x16;       // activations in the GEMM's 16-bit format (layout below)
    const void* w;         // [N, K] weights, f16, bf16 or int8
    int wdtype;            // L0B_F16, L0B_BF16 or L0B_I8 (activations then int8 digits)
    int epi;               // GemvEpi: STORE, ACCUM, SWIGLU (W = [gate; up], N = 2 * I) or ARGMAX
    float* out;            // f32 output, row stride ld (SWIGLU: [M, N/2])
    int ld;
    const float* bias;     // STORE / ACCUM: f32 [N] or null
    // Paired activations (cast_rows_split_launch): token t of token tile j = t / TB has its hi half in
    // x16 row j * BN + t % TB and its lo residual in row j * BN + TB + t % TB (row stride K); the two
    // accumulator columns are summed, and the result of token t is multiplied by rscale[t].
    // Unpaired: x16 is [M, K], one rounded row per token. int8 weights (split ignored): x16 holds four
    // int8 digit rows per token, digit dg of token t in row j * BN + dg * TB + t % TB (TB = BN / 4), and
    // rscale[t] = 2^-s of the token's scaling (cast_rows_split_launch with dtype L0B_I8).
    int split = 0;
    const float* rscale = nullptr;
    const void* wscale = nullptr;  // int8: f16 [N], one scale per weight row
    int kb = 0;                    // int8: > 0 when w is in the blocked layout (gemv.cuh), k per block
    // EPI_ARGMAX: logits to out (when not null) and, per token t, atomicMax of
    // argmax_key(value, row + argmax_base) into argmax[t].
    unsigned long long* argmax = nullptr;
    int argmax_base = 0;
    // Split-K scratch (may be null: no split): f32 partial tiles and zeroed tile counters, which the
    // GEMM leaves zeroed again.
    float* part = nullptr;
    size_t part_floats = 0;
    unsigned* counters = nullptr;
    int counter_count = 0;
};

// The tile plan tc_gemm_launch uses for this shape and weight type on `sm_count` SMs (pair = split
// 16-bit activations; int8 weights always take four digit columns per token).
TcPlan tc_gemm_plan(int M, int N, int K, int epi, bool pair, int wdtype, int sm_count);

// Rows of the paired x16 matrix for M tokens under `plan` (tiles_x * BN).
inline long long tc_pair_rows(const TcPlan& plan) { return static_cast<long long>(plan.tiles_x) * plan.bn; }

// Launches the GEMM on the device's stream (recorded when the device records).
l0b_status tc_gemm_launch(l0b_device* d, const TcGemmArgs& a);

// out16[m, :] = (RMSNorm(x[m, :]) if norm_w) in f16/bf16 for m < M; x row stride ld_x.
l0b_status cast_rows_launch(l0b_device* d, const float* x, long long ld_x, const float* norm_w, float eps, void* out16,
                            int dtype, int M, int K);

// out16 = the rows of x (RMS-normalised with norm_w when given) as hi / lo pairs in f16/bf16 in the
// paired layout of `plan` (row stride K); for f16 each token is first scaled by a power of two putting
// its largest value near 2^14, and rscale[m] receives the inverse (bf16: 1). dtype L0B_I8: four int8
// digit rows per token (the int8-weight layout), rscale[m] = 2^-s.
l0b_status cast_rows_split_launch(l0b_device* d, const float* x, long long ld_x, const float* norm_w, float eps,
                                  void* out16, float* rscale, int dtype, int M, int K, const TcPlan& plan);

// True when the tensor-core path takes this shape: f16/bf16 weights with K % 8 == 0 or int8 weights
// (per-row scales) with K % 16 == 0, K >= 64; SwiGLU needs (N / 2) % 64 == 0. Epilogues: store,
// residual add, SwiGLU, argmax.
bool tc_gemm_supported(int wdtype, int M, int N, int K, int epi);

// Upper bound on the K split of later plans (1..16; <= 0 restores 16). Launches already recorded into
// command lists keep their plan.
void tc_gemm_set_max_splits(int s);

// Split-K scratch that covers every plan on `sm_count` SMs: floats and counters.
size_t tc_gemm_part_floats(int sm_count);
constexpr int kTcCounters = 4096;

}  // namespace l0b
