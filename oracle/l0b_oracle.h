/*
 * l0b_oracle.h -- CPU restatement of the l0llm decoder hot path. TEST INFRASTRUCTURE ONLY.
 *
 * This is the checker the CUDA backend is compared against (tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference arm). Nothing in the product library links or calls it.
 *
 * The reference (hf-laboratories/l0llm) is C#; its GPU arithmetic lives in the external NuGet package
 * LevelZero.NET 2.0.0 (pinned in src/HFLabs.ML.LLM.LevelZero/HFLabs.ML.LLM.LevelZero.csproj:16), which is
 * absent here, and no .NET SDK exists, so nothing of the reference can be compiled or run. Each function
 * restates the semantics of the reference call site it names (`L/` = src/HFLabs.ML.LLM.LevelZero/,
 * `T/` = tests/HFLabs.ML.LLM.LevelZero.Tests/) and is pinned against the reference's own known-answer
 * tests and golden vectors: T/LlmMatrixTests.cs:99-130 (GEMV KAT), T/golden/rope.golden.json +
 * T/RopeFrequenciesTests.cs:25-47 (RoPE tables), T/RopeLlama3Tests.cs:8-38 (llama3 table),
 * T/LlmMatrixInt8Tests.cs:45-119 (int8 sizes and error bound). The int8 word/scale packing and the
 * quantizer rounding of LevelZero.NET are not visible in any source: that layout is an assumption
 * (documented in l0b200.h) and its parity is unpinned. Dot products accumulate in double, as the
 * reference's CPU checks do (T/LlmMatrixTests.cs:71-79); orc_gemm_fast (a model's fast mode) is the
 * fp32-accumulate timing build of the same products, used for the CPU baseline and to ingest long
 * prompts into the checker, with its error bound stated where it is defined.
 */
#ifndef L0B_ORACLE_H
#define L0B_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_I8 = 3 };
enum { ORC_ROPE_DEFAULT = 0, ORC_ROPE_LINEAR = 1, ORC_ROPE_YARN = 2, ORC_ROPE_LLAMA3 = 3 };
enum { ORC_SYN_NORMAL = 0, ORC_SYN_CONST = 1, ORC_SYN_I8 = 2, ORC_SYN_UNIFORM = 3 };

/* fp16 / bf16 conversions (round to nearest even). */
uint16_t orc_f32_to_f16(float v);
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float v);
float orc_bf16_to_f32(uint16_t h);
void orc_convert(const float* src, void* dst, int dtype, int64_t n);

/* y[m, n] = sum_k x[m, k] * W[n, k] with W [N, K] (HF [out, in]); int8 W dequantised with f16 scales
 * [N, K/group]. L/LlmMatrix.cs:122-171 (GemvQ8 for int8, Gemv for 16/32-bit). */
void orc_gemv_out_in(int M, int N, int K, const float* x, int wdtype, const void* w, const uint16_t* scales,
                     int group, float* y);
/* orc_gemv_out_in with fp32 fused multiply-add accumulation (AVX2, eight lanes per output), for timing. */
void orc_gemm_fast(int M, int N, int K, const float* x, int wdtype, const void* w, const uint16_t* scales, int group,
                   float* y);
/* Reference layout W [K, N] (f32 or f16): y[m, n] = sum_k x[m, k] * W[k, n]. T/LlmMatrixTests.cs:71-79. */
void orc_gemv_in_out(int M, int N, int K, const float* x, int w_is_half, const void* w, float* y);
/* Symmetric int8 quantisation of [N, K] with one scale per `group` inputs (L/LlmMatrix.cs:89-93). */
void orc_q8_quantize(const float* w, int N, int K, int group, int8_t* q, uint16_t* scales);

/* RMSNorm.Execute (L/LlmDecoderLayer.cs:167,183-184): [x += res]; out = x * rsqrt(mean(x^2) + eps) * w. */
void orc_rmsnorm(float* x, const float* res, const float* w, float* out, float eps, int width, int rows, int add_res);
void orc_bias_add(float* x, const float* b, int width, int rows);
void orc_swiglu(float* gate, const float* up, int64_t n);
void orc_add(float* a, const float* b, int64_t n);
void orc_sigmoid_gate(float* x, const float* g, int64_t n);
/* Embedding.Execute (L/LlmModel.cs:360,424), table f32/f16/bf16. */
void orc_embedding(const int* ids, const void* table, int table_dtype, float* out, int h, int64_t count);

/* RopeFrequencies.Compute (L/RopeFrequencies.cs:67-183). Returns the number of frequencies. */
int orc_rope_frequencies(int dim, double theta, int max_pos, int type, double factor, int original_max,
                         double low_freq, double high_freq, double beta_fast, double beta_slow, double attention_factor,
                         double mscale, double mscale_all_dim, int truncate, float* out, float* attention_out);
/* RoPE.Execute / ExecuteWithFrequencies (L/LlmDecoderLayer.cs:411-425): HF rotate-half pairs. */
void orc_rope(float* q, float* k, const int* positions, const float* inv_freq, int hd, int nh, int nkv,
              float attn_scale, int rot, int tokens);
/* KvCacheStore (L/LlmDecoderLayer.cs:322,368): rows stored at the cache dtype. */
void orc_kv_store(const float* k, const float* v, void* kc, void* vc, int cache_dtype, int pos0, int kv_dim, int tokens);
/* Attention.Execute / ExecutePrefill (L/LlmDecoderLayer.cs:325-327,369-371): query t sits at position
 * pos0 + t and attends to cache slots [0, pos0 + t]; softmax(q k / sqrt(hd)) v in double. */
void orc_attention(const float* q, const void* kc, const void* vc, int cache_dtype, float* out, int hd, int nh,
                   int nkv, int pos0, int tokens);
/* Sampling.Execute (L/LlmModel.cs:398): argmax (first maximum) or inverse-CDF sample. */
int orc_argmax(const float* x, int n);
int orc_sample(const float* logits, int vocab, float temperature, float random_val);
/* LlmSampler.Sample (src/HFLabs.ML.LLM.LevelZero/LlmAbstractions.cs:40-165) with its random draw passed
 * in (u = Random.NextDouble()): repetition penalty on the distinct ids of ctx, greedy argmax when T <= 0,
 * logits / T, softmax in double, descending sort (ties: lower index first; the reference's List.Sort is
 * unstable), top-k, top-p (shortest prefix reaching top_p), inverse CDF of the kept mass at u * mass. */
int orc_sampler(const float* logits, int vocab, const int* ctx, int n_ctx, float temperature, float top_p, int top_k,
                float repetition_penalty, double u);
/* The seeded draw the device sampled decode uses for the token at position p: 53 bits of
 * splitmix64(seed ^ ((p + 1) * 0x9E3779B97F4A7C15)) scaled to [0, 1). */
double orc_sample_uniform(uint64_t seed, int p);

/* Seeded synthetic tensors: restates the generator of the CUDA model (splitmix64 hashing, exactly
 * rounded float steps), so both sides hold identical weights. */
uint64_t orc_tensor_stream(uint64_t seed, uint64_t id);
void orc_synth_fill(void* dst, int dtype, int64_t count, uint64_t stream, int mode, float a, float b, int64_t row_len,
                    int64_t full_len, int64_t row0, int64_t col0);

/* CausalConv.Execute (L/LlmDecoderLayer.cs:392). state [conv_dim, k-1] oldest first; w [conv_dim, k]. */
void orc_causal_conv(const float* x, float* state, const float* w, float* out, int conv_dim, int kernel, int tokens);
/* GatedDelta.Execute (L/LlmDecoderLayer.cs:393-395), Hk key heads shared by Hv/Hk value heads each.
 * conv rows [q (Hk*dk) | k (Hk*dk) | v (Hv*dv)], state [Hv, dk, dv]. */
void orc_gated_delta(const float* conv, const float* z, const float* b, const float* a, const float* a_log,
                     const float* dt_bias, const float* norm_w, float* state, float* out, int hk, int hv, int dk,
                     int dv, int tokens, float eps);

/* ----------------------------------------------------------------------------------------------- */
/* Whole decoder (LlmModel.Step / LlmDecoderLayer.Forward, L/LlmModel.cs:402-444,                   */
/* L/LlmDecoderLayer.cs:129-196, 290-334), one token at a time.                                      */
/* ----------------------------------------------------------------------------------------------- */
typedef struct orc_config {
    int hidden, inter, layers, heads, kv_heads, head_dim, vocab, max_pos;
    float eps;
    double theta;
    int tie, bias, qk_norm;
    int rope_type;
    double rope_factor;
    int rope_original_max;
    double rope_low, rope_high, rope_beta_fast, rope_beta_slow, rope_attention;
    int wdtype, group, kv_dtype;
    /* Qwen3.5 hybrid (all zero: a standard decoder). Layer l is a Gated DeltaNet layer when bit l of
     * linear_mask is set (HfModelConfig.IsLinearLayer); attn_gate: q_proj carries a sigmoid output gate
     * per head (AttentionOutputGate); norm_offset is added to the input / post-attention / final / q / k
     * norm weights at load (RmsNormOffset); partial_rotary: fraction of head_dim rotated (0 = all). */
    uint64_t linear_mask;
    int lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim, lin_conv;
    int attn_gate;
    float norm_offset;
    double partial_rotary;
} orc_config;

typedef struct orc_model orc_model;
orc_model* orc_model_create(const orc_config* cfg, int max_seq);
/* `batch` sequences, each with its own KV cache rows [max_seq, kv_dim] per layer. */
orc_model* orc_model_create_batch(const orc_config* cfg, int max_seq, int batch);
/* 1: projections accumulate in fp32 (orc_gemm_fast); 0 (default): in double. */
void orc_model_set_fast(orc_model* m, int fast);
void orc_model_free(orc_model* m);
int orc_model_init_synthetic(orc_model* m, uint64_t seed, float std, float scale_lo, float scale_hi);
int orc_model_set_tensor(orc_model* m, const char* name, const float* data, int64_t count);
/* Feeds token `token` at `position` and writes the vocab logits of the next token. */
int orc_model_step(orc_model* m, int token, int position, float* logits);
/* `rows` tokens at once: row r is token tokens[r] at positions[r] of sequence seqs[r] (NULL: 0). All rows'
 * K/V are stored before attention, so consecutive positions of one sequence are a causal prefill chunk
 * (LlmModel.IngestPrompt) and rows of different sequences a decode batch (LlmModel.StepBatch).
 * logits: [rows, vocab], or the last row's only when last_only; may be NULL. */
int orc_model_forward(orc_model* m, int rows, const int* tokens, const int* positions, const int* seqs,
                      float* logits, int last_only);
/* Runs only `layers_to_run` layers (<= cfg.layers) for timing samples; 0 = all. */
void orc_model_set_layer_limit(orc_model* m, int layers_to_run);
/* Stage callback with the reference's probe stage names (L/LlmDecoderLayer.cs:113-119). */
typedef void (*orc_probe_fn)(void* user, int layer, const char* stage, const float* values, int64_t count);
void orc_model_set_probe(orc_model* m, orc_probe_fn fn, void* user);
/* Reads the K/V cache rows of a layer as f32. */
int orc_model_read_kv(orc_model* m, int layer, int row0, int rows, float* keys, float* values);
int orc_model_read_kv_seq(orc_model* m, int layer, int seq, int row0, int rows, float* keys, float* values);
/* Writes K/V cache rows (rounded to the cache dtype), e.g. a context filled by another prefill. */
int orc_model_write_kv_seq(orc_model* m, int layer, int seq, int row0, int rows, const float* keys,
                           const float* values);
/* Threads used by the oracle's parallel loops (OpenMP). */
int orc_num_threads(void);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
