// C++ mirror of the reference decoder host (LlmModel / LlmDecoderLayer / LlmMatrix / LlmKvCache).
#pragma once

#include <cuda_fp16.h>

#include <string>
#include <vector>

#include "runtime.h"

namespace l0b {

// LlmMatrix: one projection in the [out = n, in = k] order, f32 / f16 / bf16 or int8 + f16 scales.
// Fused projections are stored stacked: q/k/v as [q; k; v] rows, gate/up as [gate; up] rows.
struct ModelMatrix {
    int n = 0, k = 0;
    int dtype = L0B_F16;
    void* w = nullptr;
    __half* scales = nullptr;
    int group = 0;  // int8 scale group (k = per output channel)
    int kb = 0;     // > 0: int8 weights in the blocked layout (gemv.cuh blocked_index), 0: row-major
    size_t bytes() const {
        size_t b = static_cast<size_t>(n) * k * dtype_size(static_cast<l0b_dtype>(dtype));
        if (dtype == L0B_I8) b += static_cast<size_t>(n) * (k / group) * 2;
        return b;
    }
};

struct ModelLayer {
    float* in_norm = nullptr;
    float* post_norm = nullptr;
    ModelMatrix qkv, o, gate_up, down;
    float* qkv_bias = nullptr;  // [q_dim + 2 kv_dim] or null
    float* q_norm = nullptr;
    float* k_norm = nullptr;
    void* kc = nullptr;  // [batch_cap, max_seq, kv_dim] (cache dtype)
    void* vc = nullptr;
    // Qwen3.5 Gated DeltaNet layer (LlmLinearAttentionWeights / LlmLinearState, L/LlmLinearAttention.cs):
    // in-projections stacked [qkv; z; b; a], out_proj, conv taps [conv_dim, k], A_log, dt_bias, the gated
    // norm weight, and the sequence's conv window [conv_dim, k - 1] and recurrent state [hv, dk, dv].
    bool linear = false;
    ModelMatrix lin_in, lin_out;
    float *conv_w = nullptr, *a_log = nullptr, *dt_bias = nullptr, *lin_norm = nullptr;
    float *conv_state = nullptr, *rec_state = nullptr;
};

// Rotary table per L/RopeFrequencies.cs:67-183 (default, linear, yarn, llama3).
l0b_status rope_frequencies(const l0b_model_config& c, std::vector<float>* inv_freq, float* attention_factor);

}  // namespace l0b
