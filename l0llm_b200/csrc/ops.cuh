// Host-side launchers of the op kernels (elementwise.cu, attention.cu, deltanet.cu).
#pragma once

#include <cuda_fp16.h>

#include "runtime.h"

namespace l0b {

l0b_status k_rmsnorm(l0b_device* d, float* x, const float* res, const float* w, float* out, float eps, int width,
                     int rows, int add_res);
l0b_status k_bias_add(l0b_device* d, float* x, const float* b, int width, int rows);
// q_stride / k_stride / in_stride: elements between tokens (<= 0: packed rows).
// RMSNorm of every head of the nq query and nk key heads of `rows` stacked q|k|v rows (row stride ld), in
// place, with the query / key norm weights.
l0b_status k_head_norm(l0b_device* d, float* qkv, long long ld, int nq, int nk, int hd, const float* wq,
                       const float* wk, float eps, int rows);
l0b_status k_rope(l0b_device* d, float* q, float* k, const int* positions, const float* inv_freq, int hd, int nh,
                  int nkv, float attn_scale, int rot, int tokens, long long q_stride = 0, long long k_stride = 0);
l0b_status k_kv_store(l0b_device* d, const float* k, const float* v, void* kc, void* vc, int cache_dtype, int pos0,
                      int kv_dim, int tokens, long long in_stride = 0);
l0b_status k_swiglu(l0b_device* d, float* gate, const float* up, long long n);
l0b_status k_add(l0b_device* d, float* a, const float* b, long long n);
l0b_status k_sigmoid_gate(l0b_device* d, float* x, const float* g, long long n);
l0b_status k_embedding(l0b_device* d, const int* ids, const void* table, int table_dtype, float* out, int h,
                       long long count, int vocab, int* error);
l0b_status k_copy(l0b_device* d, const float* src, float* dst, long long offset, long long n);
l0b_status k_sampling(l0b_device* d, const float* logits, int* sampled, float temperature, float random_val,
                      int vocab);
l0b_status k_quantize(l0b_device* d, const void* w, int w_dtype, int n, int k, int group, int8_t* q, __half* s);

// ------------------------------------------------------------------------------------------------
// Attention (attention.cu)
// ------------------------------------------------------------------------------------------------

struct AttnParams {
    const float* q;            // query rows: q + b * q_bstride, heads contiguous [nH * hd]
    long long q_bstride;
    // Fused decode: RoPE on q and on the new key (k_new) in-kernel, k/v of the query position
    // stored to the cache by the CTA that owns it. rope == 0: q is used as is, cache already filled.
    int rope;
    int store_new;
    const float* k_new;        // [nKv * hd] per b (pre-RoPE), stride new_bstride
    const float* v_new;
    long long new_bstride;
    const float* inv_freq;     // [rot / 2]
    int rot;                   // rotary dim
    float attn_scale;
    void* kc;                  // caches [maxSeq, kv_dim] per b, dtype cache_dtype, b stride cache_bstride
    void* vc;
    int cache_dtype;
    long long cache_bstride;
    int kv_dim;
    // Query position of row b: positions[b] when non-null, else pos_base + b * pos_step.
    const int* positions;
    int pos_base;
    int pos_step;
    float* out;                // out + b * out_bstride, [nH * hd]
    long long out_bstride;
    float* part;               // split partials [B, nH, max_splits, hd]
    float* part_ml;            // [B, nH, max_splits, 2]
    unsigned* counters;        // [B, nKv] zeroed, reset by the last CTA
    int nh, nkv, hd;
    int chunk;                 // positions per split (multiple of 32)
    int max_splits;
    float scale;               // head_dim^-0.5
};

// Launches the split-KV attention kernel over grid (nKv, max_splits, batch).
l0b_status attention_launch(l0b_device* d, const AttnParams& p, int batch);
// Raw-stream variant used by callers without a device handle.
l0b_status attention_launch_stream(cudaStream_t stream, const AttnParams& p, int batch);
// Decode attention in thread-block clusters of `splits` (1, 2, 4 or 8) CTAs per (row, KV head group) merged through
// distributed shared memory: needs no part/part_ml/counters. p.chunk is the minimum split length
// (a multiple of 32); the kernel derives the split length from each row's live sequence length.
l0b_status attention_cluster_launch(l0b_device* d, const AttnParams& p, int batch, int splits);
// Cluster size for a cache of max_seq positions and `work_items` (batch * KV head groups) rows.
int attention_cluster_splits(int max_seq, int work_items, int sm_count);
// Scratch floats / counters the kernel needs for (batch, nh, max_splits, hd).
size_t attention_part_floats(int batch, int nh, int max_splits, int hd);
// Picks the split length for a cache of max_seq positions and `work_items` (batch * nKv) rows.
void attention_pick_split(int max_seq, int work_items, int sm_count, int* chunk, int* max_splits);

// Device sampling (LlmSampler.Sample): validates the parameters (top_k within the select's 1024
// candidates when T > 0).
l0b_status sample_check(float temperature, float top_p, int top_k, float penalty, int vocab);
// p[0..n) = v.
l0b_status k_fill_u32(l0b_device* d, uint32_t* p, uint32_t v, int n);
// CausalConv / GatedDelta over raw device pointers (the checked entry points wrap these; deltanet.cu).
l0b_status k_causal_conv(l0b_device* d, const float* x, float* state, const float* w, float* out, int conv_dim,
                         int kernel, int tokens);
l0b_status k_gated_delta(l0b_suite* s, l0b_device* d, const float* conv, const float* z, const float* b, const float* a,
                         const float* a_log, const float* dt_bias, const float* norm_w, float* state, float* out, int hk,
                         int hv, int dk, int dv, int tokens, float eps);
// 32-bit words of a context bitmap over `vocab` tokens.
size_t sample_seen_words(int vocab);
// 32-bit words of the key scratch sample_step takes for `vocab` tokens (keys, the max word, which must
// be zero before the first draw and is left zero, and the normaliser partials).
size_t sample_keys_words(int vocab);
// bits = the set of ids[0..n) (one CTA; zeroes the bitmap first).
l0b_status seen_build(l0b_device* d, const int* ids, int n, int vocab, uint32_t* bits);
// One draw: keys scratch [vocab]; `seen` (or null) drives the repetition penalty. The draw is `u`, or
// when pos is given the seeded draw of the token at position *pos + pos_offset: 53 bits of
// splitmix64(seed ^ ((p + 1) * 0x9E3779B97F4A7C15)) scaled to [0, 1). The token goes to out_token and/or
// as an argmax key to out_key; seen_update (or null) records it.
l0b_status sample_step(l0b_device* d, const float* logits, int vocab, const uint32_t* seen, float temperature,
                       float top_p, int top_k, float penalty, uint32_t* keys, double u, unsigned long long seed,
                       const int* pos, int pos_offset, int* out_token, unsigned long long* out_key,
                       uint32_t* seen_update);

}  // namespace l0b
