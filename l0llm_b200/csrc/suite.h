// LlmKernelSuite state: the int8 activation scratch and cached RoPE tables.
#pragma once

#include <map>
#include <utility>

#include "runtime.h"

namespace l0b {
// LlmGemvKernel.MaxRows: rows per ExecuteRows call and per prefill chunk of the model.
constexpr int kMaxRows = 64;
// Tokens per prefill chunk of the model (activation rows it allocates).
constexpr int kPrefillRows = 512;
// 16-row tiles the suite's split-K GEMV scratch covers (N <= 65536 output rows).
constexpr int kSuiteSplitTiles = 4096;
// Output rows the suite's k-split GEMV row sums cover (l0b_linear_fused over blocked int8 weights).
constexpr int kSuiteKsRows = 16 * kSuiteSplitTiles;
}  // namespace l0b

struct l0b_suite {
    l0b_device* dev = nullptr;
    float* q8_x = nullptr;  // GemvQ8 activation scratch [q8_rows, q8_width] f32
    int q8_rows = 0;
    int q8_width = 0;
    int q8_k = 0;
    int* error_flag = nullptr;  // set by kernels that meet an out-of-range index (embedding ids)
    // Split-K scratch of the one-row bulk GEMV (l0b::kSuiteSplitTiles tiles), counters zero at rest.
    // Records of the chunked Gated DeltaNet prefill (floats), grown on demand.
    float* gdn_rec = nullptr;
    long long gdn_floats = 0;
    float* split_part = nullptr;
    unsigned* split_counters = nullptr;
    // Exact int64 row sums of the k-split GEMV [kSuiteKsRows], zero at rest (every launch leaves them
    // zero); its tile-group counters are split_counters.
    long long* ks_acc = nullptr;
    std::map<std::pair<int, double>, float*> rope_tables;
    ~l0b_suite();
};

namespace l0b {
// Device table of RoPE inverse frequencies for (rotary dim, theta), built once per suite.
l0b_status suite_rope_table(l0b_suite* s, int rot, double theta, const float** out);
}  // namespace l0b
