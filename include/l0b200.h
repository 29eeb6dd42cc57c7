/*
 * l0b200.h -- C ABI of the B200 (sm_100a) backend for the l0llm decoder hot path.
 *
 * The library replaces the kernel surface that l0llm's C# decoder calls through the external
 * LevelZero.NET 2.0.0 package: LevelZeroRuntime / ComputeDevice / SharedBuffer<T> /
 * LlmKernelSuite and its ops. Each entry point names the reference call site it stands in for
 * (paths are relative to the l0llm repository; `L/` = src/HFLabs.ML.LLM.LevelZero/).
 *
 * Conventions
 *  - Every function returns an l0b_status; 0 (L0B_OK) is success. On failure l0b_last_error()
 *    returns a thread-local, human-readable message. Argument errors map to the exception types
 *    the reference throws (ArgumentException, ArgumentOutOfRangeException, NotSupportedException,
 *    InvalidOperationException), see l0b_status.
 *  - Handles are opaque. The caller owns them and frees them with the matching *_free call; the
 *    library never frees a buffer it did not allocate.
 *  - Buffers live in device memory (HBM). The reference's host-addressable USM pointer
 *    (SharedBuffer.Pointer) is replaced by l0b_buffer_read / l0b_buffer_write of element ranges.
 *  - Ops enqueue work on the device's stream. Between l0b_device_begin_recording and
 *    l0b_device_end_recording they are recorded into a command list instead; end_recording submits
 *    the list as one CUDA graph launch and waits (the reference's one submit + one wait per token).
 *    Buffer writes made while recording take effect before the list runs, as host writes to USM do.
 *  - One host thread per device. No entry point is re-entrant for the same device.
 *  - No CPU fallback: without a usable sm_100 device every op returns L0B_ERR_NO_DEVICE.
 */
#ifndef L0B200_H
#define L0B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define L0B_API __declspec(dllexport)
#else
#define L0B_API __attribute__((visibility("default")))
#endif

typedef enum l0b_status {
    L0B_OK = 0,
    L0B_ERR_ARGUMENT = 1,          /* ArgumentException / ArgumentNullException */
    L0B_ERR_OUT_OF_RANGE = 2,      /* ArgumentOutOfRangeException */
    L0B_ERR_UNSUPPORTED = 3,       /* NotSupportedException */
    L0B_ERR_INVALID_OPERATION = 4, /* InvalidOperationException */
    L0B_ERR_INVALID_DATA = 5,      /* InvalidDataException */
    L0B_ERR_CUDA = 6,              /* a CUDA runtime call failed */
    L0B_ERR_OUT_OF_MEMORY = 7,
    L0B_ERR_NO_DEVICE = 8,         /* no sm_100 device: LevelZeroRuntime.IsAvailable() == false */
    L0B_ERR_TIMEOUT = 9,           /* a bounded device-side wait gave up */
    L0B_ERR_NCCL = 10
} l0b_status;

typedef enum l0b_dtype {
    L0B_F32 = 0,
    L0B_F16 = 1,
    L0B_BF16 = 2,
    L0B_I8 = 3,
    L0B_I32 = 4,
    L0B_U8 = 5
} l0b_dtype;

typedef struct l0b_device l0b_device;
typedef struct l0b_buffer l0b_buffer;
typedef struct l0b_suite l0b_suite;
typedef struct l0b_model l0b_model;
typedef struct l0b_comm l0b_comm;

/* ------------------------------------------------------------------------------------------ */
/* Errors and versions                                                                         */
/* ------------------------------------------------------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). Valid until the next call. */
L0B_API const char* l0b_last_error(void);
/* Library ABI version, (major << 16) | minor. */
L0B_API int32_t l0b_version(void);
/* Number of device kernels this process has launched through the library (immediate launches and
 * kernel nodes of submitted command lists). Used by benchmarks to count launches. */
L0B_API int64_t l0b_kernel_launch_count(void);

/* ------------------------------------------------------------------------------------------ */
/* Runtime and device  (LevelZeroRuntime, ComputeDevice: src/l0llm/Program.cs:124,138-141,      */
/*                      L/LevelZeroLlmEngine.cs:355-361, L/LlmModel.cs:353-442)                 */
/* ------------------------------------------------------------------------------------------ */

/* LevelZeroRuntime.IsAvailable(): *available = 1 when an sm_100 device is present. */
L0B_API l0b_status l0b_runtime_is_available(int32_t* available);
/* LevelZeroRuntime.EnumerateDevices(): number of usable devices. */
L0B_API l0b_status l0b_device_count(int32_t* count);
/* DeviceInfo{Name}: writes a NUL-terminated name (truncated to name_len) and SM count. */
L0B_API l0b_status l0b_device_info(int32_t index, char* name, int32_t name_len, int32_t* sm_count,
                                   int64_t* total_bytes);
/* LevelZeroRuntime.GetDevice / GetDefaultDevice (index 0). */
L0B_API l0b_status l0b_device_create(int32_t index, l0b_device** out);
/* ComputeDevice.Dispose. Frees the stream, cached command lists and internal scratch. */
L0B_API l0b_status l0b_device_free(l0b_device* dev);
/* ComputeDevice.BeginRecording / EndRecording / AbortRecording / IsRecording. */
L0B_API l0b_status l0b_device_begin_recording(l0b_device* dev);
L0B_API l0b_status l0b_device_end_recording(l0b_device* dev);
L0B_API l0b_status l0b_device_abort_recording(l0b_device* dev);
L0B_API l0b_status l0b_device_is_recording(l0b_device* dev, int32_t* recording);
/* Waits until all work enqueued on the device's stream is done. */
L0B_API l0b_status l0b_device_synchronize(l0b_device* dev);
/* The device's cudaStream_t, for callers that interleave their own work (e.g. torch). */
L0B_API l0b_status l0b_device_stream(l0b_device* dev, void** stream);
/* Number of command lists built (captured + instantiated) and reused since creation. */
L0B_API l0b_status l0b_device_graph_stats(l0b_device* dev, int64_t* built, int64_t* reused,
                                          int64_t* updated);
/* Reads and clears the device's error flag: nonzero when a kernel's bounded wait (a pipeline barrier
 * that never completed) gave up instead of hanging; the results of that launch are invalid. */
L0B_API l0b_status l0b_device_error_status(l0b_device* dev, int32_t* code);
/* Enables (1) or disables (0) programmatic dependent launch between consecutive kernels. */
L0B_API l0b_status l0b_device_set_pdl(l0b_device* dev, int32_t enabled);

/* ------------------------------------------------------------------------------------------ */
/* Buffers  (SharedBuffer<T>: Write/ToArray/Pointer/Count/Dispose, L/LlmSequenceState.cs:60-80) */
/* ------------------------------------------------------------------------------------------ */

/* ComputeDevice.AllocShared<T>(count): zero-filled device buffer of count elements. */
L0B_API l0b_status l0b_buffer_alloc(l0b_device* dev, l0b_dtype dtype, int64_t count, l0b_buffer** out);
/* ComputeDevice.AllocShared<T>(T[] data). */
L0B_API l0b_status l0b_buffer_alloc_from(l0b_device* dev, l0b_dtype dtype, int64_t count,
                                         const void* host, l0b_buffer** out);
/* A buffer naming elements [offset, offset + count) of `base` (the C# side's Pointer + offset): it
 * owns nothing, l0b_buffer_free releases only the handle, and it must not outlive `base`. */
L0B_API l0b_status l0b_buffer_view(l0b_buffer* base, int64_t offset, int64_t count, l0b_buffer** out);
L0B_API l0b_status l0b_buffer_free(l0b_buffer* buf);
/* SharedBuffer.Write(T[]) at an element offset (Marshal.Copy into Pointer + offset). */
L0B_API l0b_status l0b_buffer_write(l0b_buffer* buf, int64_t offset, const void* host, int64_t count);
/* SharedBuffer.ToArray() / Marshal.Copy out of Pointer + offset. Waits for prior work. */
L0B_API l0b_status l0b_buffer_read(l0b_buffer* buf, int64_t offset, void* host, int64_t count);
/* Device-to-device copy of count elements (same dtype). */
L0B_API l0b_status l0b_buffer_copy(l0b_buffer* dst, int64_t dst_offset, l0b_buffer* src,
                                   int64_t src_offset, int64_t count);
/* Sets every element to zero (stream-ordered). */
L0B_API l0b_status l0b_buffer_zero(l0b_buffer* buf);
L0B_API l0b_status l0b_buffer_count(l0b_buffer* buf, int64_t* count);
L0B_API l0b_status l0b_buffer_dtype(l0b_buffer* buf, l0b_dtype* dtype);
/* Raw device address (for interop with other CUDA code in the same process). */
L0B_API l0b_status l0b_buffer_device_ptr(l0b_buffer* buf, void** ptr);

/* ------------------------------------------------------------------------------------------ */
/* Kernel suite  (LlmKernelSuite.Create/Dispose/EnsureQ8Scratch/Q8Scratch; statics of          */
/*                LlmGemvKernel / LlmGemvQ8Kernel: L/LlmModel.cs:131-144, L/LlmMatrix.cs:242-253) */
/* ------------------------------------------------------------------------------------------ */

L0B_API l0b_status l0b_suite_create(l0b_device* dev, l0b_suite** out);
L0B_API l0b_status l0b_suite_free(l0b_suite* suite);
/* LlmKernelSuite.GemvQ8 != null: this backend always has the int8 kernels (returns 1). */
L0B_API int32_t l0b_suite_has_q8(l0b_suite* suite);
/* LlmKernelSuite.EnsureQ8Scratch(device, rows, width): sizes the shared activation scratch. */
L0B_API l0b_status l0b_suite_ensure_q8_scratch(l0b_suite* suite, int32_t rows, int32_t width);
/* LlmQ8Activations.RowCapacity of the current scratch (0 when none). */
L0B_API int32_t l0b_suite_q8_scratch_rows(l0b_suite* suite);
/* LlmGemvKernel.Supports(N): N % 4 == 0. */
L0B_API int32_t l0b_gemv_supports(int32_t n);
/* LlmGemvKernel.MaxRows: rows one ExecuteRows call (and one prefill chunk) takes. */
L0B_API int32_t l0b_gemv_max_rows(void);
/* LlmGemvQ8Kernel.Supports(N, K): N % 4 == 0 && K % 32 == 0. */
L0B_API int32_t l0b_gemv_q8_supports(int32_t n, int32_t k);
/* LlmGemvQ8Kernel.GroupSize (32). */
L0B_API int32_t l0b_gemv_q8_group_size(void);

/* ------------------------------------------------------------------------------------------ */
/* Int8 weight format  (LlmQ8Quantizer.QuantizeOutIn, L/LlmMatrix.cs:89-93)                    */
/*                                                                                            */
/* Weights stay in the HuggingFace [out, in] order: words[o*K/4 + i/4] holds the int8 of input  */
/* i in byte (i % 4), i.e. a row-major int8 [N, K] array. One half scale per `group` inputs     */
/* per output: scales[o*(K/group) + i/group]; group == K gives per-output-channel scales.       */
/* Symmetric quantization: s = half(max|w| / 127) over the group, q = clamp(rint(w / s),        */
/* -127, 127) with rint rounding half to even; an all-zero group gets s = 0 and q = 0.          */
/* ------------------------------------------------------------------------------------------ */

/* Host quantizer: hf [N, K] fp32 -> words (N*K/4 int32) + scales (N*K/group fp16 bits). */
L0B_API l0b_status l0b_q8_quantize_out_in(const float* hf, int32_t n, int32_t k, int32_t group,
                                          int32_t* words, uint16_t* scales);
/* Device quantizer with the same result: w [N, K] (f32/f16/bf16 buffer) -> q (i8 buffer) + s (f16). */
L0B_API l0b_status l0b_q8_quantize_device(l0b_suite* suite, l0b_device* dev, int32_t n, int32_t k,
                                          int32_t group, l0b_buffer* w, l0b_buffer* q, l0b_buffer* s);

/* ------------------------------------------------------------------------------------------ */
/* Ops of LlmKernelSuite, argument orders as the reference calls them                          */
/* Activations are f32 buffers as in the reference unless a dtype is stated.                   */
/* ------------------------------------------------------------------------------------------ */

/* Embedding.Execute(dev, ids, table, out, h, count) -- L/LlmModel.cs:360,424.
 * out[e] = table[ids[e / h] * h + e % h] for e < count. table: f32/f16/bf16 [vocab, h]. */
L0B_API l0b_status l0b_embedding_execute(l0b_suite* s, l0b_device* d, l0b_buffer* ids, l0b_buffer* table,
                                         l0b_buffer* out, int32_t h, int32_t count);

/* RMSNorm.Execute(dev, x, res, w, out, eps, width, rows, addResidual) --
 * L/LlmDecoderLayer.cs:167,183-184,311-312; L/LlmModel.cs:394.
 * With add_residual: x += res (in place) first. Then out = x * rsqrt(mean(x^2) + eps) * w per row.
 * out may alias x (per-head QK-norm). res may be NULL when add_residual == 0. */
L0B_API l0b_status l0b_rmsnorm_execute(l0b_suite* s, l0b_device* d, l0b_buffer* x, l0b_buffer* res,
                                       l0b_buffer* w, l0b_buffer* out, float eps, int32_t width,
                                       int32_t rows, int32_t add_residual);

/* Gemv.Execute(dev, N, K, x, W, y) -- L/LlmMatrix.cs:134,138. W f32/f16 stored [in=K, out=N]
 * (the reference layout, L/LlmMatrix.cs:5). y[n] = sum_k x[k] * W[k, n]. Requires N % 4 == 0. */
L0B_API l0b_status l0b_gemv_execute(l0b_suite* s, l0b_device* d, int32_t n, int32_t k, l0b_buffer* x,
                                    l0b_buffer* w, l0b_buffer* y);
/* Gemv.ExecuteRows(dev, M, N, K, x, W, y) -- L/LlmMatrix.cs:161,165. X [M, K], Y [M, N]. */
L0B_API l0b_status l0b_gemv_execute_rows(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k,
                                         l0b_buffer* x, l0b_buffer* w, l0b_buffer* y);
/* Gemm.Execute(dev, M, N, K, A, B, C) -- L/LlmMatrix.cs:142,169. f32 C[M,N] = A[M,K] * B[K,N]. */
L0B_API l0b_status l0b_gemm_execute(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k,
                                    l0b_buffer* a, l0b_buffer* b, l0b_buffer* c);

/* GemvQ8.Quantize(dev, rows, K, x, scratch) -- L/LlmMatrix.cs:129,156,201. Stages `rows` rows of
 * the f32 activations x [rows, K] in the suite's activation scratch (sized by ensure_q8_scratch).
 * This backend multiplies int8 weights with 16/32-bit activations (W8A16 and wider), so staging
 * keeps the activations exact (f32) instead of quantizing them. */
L0B_API l0b_status l0b_gemv_q8_quantize(l0b_suite* s, l0b_device* d, int32_t rows, int32_t k, l0b_buffer* x);
/* GemvQ8.Execute / ExecuteRows(dev, [M,] N, K, scratch, words, scales, y) -- L/LlmMatrix.cs:130,157,
 * 235,239. words: i8 (or i32-packed) [N, K]; scales f16 [N, K/32]. Y [M, N] f32.
 * The reference's `scratch` argument is not taken: every reference call passes the suite's own
 * LlmQ8Activations (suite.Q8Scratch, via RequireScratch, L/LlmMatrix.cs:243-253), and these entries
 * always read the suite's scratch, i.e. the rows the last l0b_gemv_q8_quantize on this suite staged.
 * A facade holding any other LlmQ8Activations must quantize into the suite before calling. */
L0B_API l0b_status l0b_gemv_q8_execute(l0b_suite* s, l0b_device* d, int32_t n, int32_t k,
                                       l0b_buffer* words, l0b_buffer* scales, l0b_buffer* y);
L0B_API l0b_status l0b_gemv_q8_execute_rows(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k,
                                            l0b_buffer* words, l0b_buffer* scales, l0b_buffer* y);

/* BiasAdd.Execute(dev, x, b, width, rows) -- L/LlmDecoderLayer.cs:303-305,356-358. x[r,:] += b. */
L0B_API l0b_status l0b_bias_add_execute(l0b_suite* s, l0b_device* d, l0b_buffer* x, l0b_buffer* b,
                                        int32_t width, int32_t rows);

/* RoPE.Execute(dev, q, k, positions, hd, nH, nKv, theta, tokens) -- L/LlmDecoderLayer.cs:415-417.
 * HF rotate-half pairing (i, i + hd/2); inverse frequencies theta^(-2i/hd) computed in double and
 * rounded to f32 (L/RopeFrequencies.cs:75-80); angle = f32(position) * inv_freq in f32. */
L0B_API l0b_status l0b_rope_execute(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* k,
                                    l0b_buffer* positions, int32_t head_dim, int32_t n_heads,
                                    int32_t n_kv_heads, float theta, int32_t tokens);
/* RoPE.ExecuteWithFrequencies(dev, q, k, positions, invFreq, hd, nH, nKv, attnScale, tokens,
 * rotaryDim) -- L/LlmDecoderLayer.cs:421-423. Rotates the first rotary_dim elements of each head
 * with the table inv_freq [rotary_dim/2]; cos and sin are multiplied by attn_scale. */
L0B_API l0b_status l0b_rope_execute_with_frequencies(l0b_suite* s, l0b_device* d, l0b_buffer* q,
                                                     l0b_buffer* k, l0b_buffer* positions,
                                                     l0b_buffer* inv_freq, int32_t head_dim,
                                                     int32_t n_heads, int32_t n_kv_heads,
                                                     float attn_scale, int32_t tokens, int32_t rotary_dim);

/* KvCacheStore.Execute / ExecuteRows(dev, k, v, Kc, Vc, pos0, kvDim[, tokens]) --
 * L/LlmDecoderLayer.cs:322,368. Kc[pos0 + t, :] = k[t, :]; cache dtype f32/f16/bf16. */
L0B_API l0b_status l0b_kv_cache_store_execute(l0b_suite* s, l0b_device* d, l0b_buffer* k, l0b_buffer* v,
                                              l0b_buffer* kc, l0b_buffer* vc, int32_t pos0, int32_t kv_dim);
L0B_API l0b_status l0b_kv_cache_store_execute_rows(l0b_suite* s, l0b_device* d, l0b_buffer* k,
                                                   l0b_buffer* v, l0b_buffer* kc, l0b_buffer* vc,
                                                   int32_t pos0, int32_t kv_dim, int32_t tokens);

/* Attention.Execute(dev, q, Kc, Vc, out, hd, nH, nKv, seqLen, maxSeq) -- L/LlmDecoderLayer.cs:325-327.
 * One query token over cache slots [0, seq_len): out = softmax(q K^T / sqrt(hd)) V per head, query
 * head h reading kv head h / (nH / nKv). Split-KV with online softmax: no 15000-token cap. */
L0B_API l0b_status l0b_attention_execute(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* kc,
                                         l0b_buffer* vc, l0b_buffer* out, int32_t head_dim,
                                         int32_t n_heads, int32_t n_kv_heads, int32_t seq_len,
                                         int32_t max_seq);
/* Attention.ExecutePrefill(dev, q, Kc, Vc, out, hd, nH, nKv, pos0, tokens, maxSeq) --
 * L/LlmDecoderLayer.cs:369-371. Query t (position pos0 + t) attends to slots [0, pos0 + t]. */
L0B_API l0b_status l0b_attention_execute_prefill(l0b_suite* s, l0b_device* d, l0b_buffer* q,
                                                 l0b_buffer* kc, l0b_buffer* vc, l0b_buffer* out,
                                                 int32_t head_dim, int32_t n_heads, int32_t n_kv_heads,
                                                 int32_t pos0, int32_t tokens, int32_t max_seq);

/* Decode attention (the l0b_attention_execute computation, one query token over cache slots
 * [0, seq_len)) that allocates nothing, for callers that cannot allocate device memory during a call:
 * a server that plans all of HBM at start-up, code running while a pool or another runtime owns the
 * allocator, or a host that must never block in cudaMalloc mid-step. No counterpart in the reference.
 * Raw device pointers; cache_dtype is L0B_F32/F16/BF16; enqueued on `stream` (a cudaStream_t).
 * The split partials live in a fixed 4 MiB array and 4096 counters compiled into the library (every
 * GPU that loads it holds them until exit); n_heads * (head_dim + 2) must fit 1,048,576 floats and
 * n_kv_heads * ceil(group / 8) must fit 4096 counters, else L0B_ERR_OUT_OF_RANGE. All calls share that
 * scratch: calls that overlap on the GPU (other streams, other threads) race and must be serialised.
 * The first call on a device looks up the arrays' device addresses; make it before any stream capture. */
L0B_API l0b_status l0b_attention_decode_noalloc(void* stream, const float* q, const void* kc, const void* vc,
                                                int32_t cache_dtype, float* out, int32_t head_dim,
                                                int32_t n_heads, int32_t n_kv_heads, int32_t seq_len,
                                                int32_t max_seq);

/* Tuning: prefill attention (a block of query rows over f16 / bf16 caches, head dim 64 or 128) on the
 * tensor cores (1, default: flash-attention tiles on mma.sync with hi + lo 16-bit queries and
 * probabilities, about fp32 accuracy) or on the scalar kernel (0). No counterpart in the reference. */
L0B_API l0b_status l0b_set_attention_prefill_tensor_cores(int32_t enable);

/* Tuning: decode attention clusters of up to 16 split CTAs (1, default, where the device can hold
 * such non-portable clusters) or at most the portable 8 (0). More splits shorten each CTA's walk over
 * the cache when a step has few (sequence, KV head) items. No counterpart in the reference. */
L0B_API l0b_status l0b_set_attention_cluster16(int32_t enable);

/* Tuning: decode attention over f16 / bf16 caches (head dim 64 or 128) on the tensor cores (1, default:
 * the query heads of a KV head as the rows of mma.sync tiles, hi + lo 16-bit queries and probabilities,
 * about fp32 accuracy, the key and value of the new position as the cache stores them) or on the fp32
 * FMA kernel (0). Affects launches recorded after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_attention_decode_tensor_cores(int32_t enable);

/* SigmoidGate.Execute(dev, x, gate, n) -- L/LlmDecoderLayer.cs:330,374. x *= sigmoid(gate). */
L0B_API l0b_status l0b_sigmoid_gate_execute(l0b_suite* s, l0b_device* d, l0b_buffer* x, l0b_buffer* gate,
                                            int32_t n);
/* SwiGLU.Execute(dev, gate, up, n) -- L/LlmDecoderLayer.cs:189,265. gate = silu(gate) * up. */
L0B_API l0b_status l0b_swiglu_execute(l0b_suite* s, l0b_device* d, l0b_buffer* gate, l0b_buffer* up,
                                      int32_t n);
/* Add.Execute(dev, hidden, down, n) -- L/LlmDecoderLayer.cs:194,267. hidden += down. */
L0B_API l0b_status l0b_add_execute(l0b_suite* s, l0b_device* d, l0b_buffer* hidden, l0b_buffer* down,
                                   int32_t n);
/* Copy.Execute(dev, src, dst, offset, n) -- L/LlmModel.cs:368. dst[0, n) = src[offset, offset + n). */
L0B_API l0b_status l0b_copy_execute(l0b_suite* s, l0b_device* d, l0b_buffer* src, l0b_buffer* dst,
                                    int32_t offset, int32_t n);
/* Sampling.Execute(dev, logits, sampled, temperature, randomVal, vocab) -- L/LlmModel.cs:398.
 * temperature == 0: argmax (lowest index on ties). Otherwise the smallest index whose cumulative
 * softmax(logits / temperature) mass reaches random_val * total. */
L0B_API l0b_status l0b_sampling_execute(l0b_suite* s, l0b_device* d, l0b_buffer* logits,
                                        l0b_buffer* sampled, float temperature, float random_val,
                                        int32_t vocab);
/* LlmSampler.Sample (src/HFLabs.ML.LLM.LevelZero/LlmAbstractions.cs:40-165) on the device, the token
 * written to out_token (i32 [1]) with no logits readback: repetition penalty over the distinct ids of
 * `context` (i32 [n_context], may be NULL), greedy when temperature <= 0, else softmax(logits / T) cut to
 * the top_k most likely tokens and to the shortest prefix reaching top_p, sampled at random_value * (kept
 * mass) (random_value in [0, 1): the reference's Random.NextDouble()). Ties order by token index. top_k
 * must lie in [1, 1024] when temperature > 0 (L0B_ERR_UNSUPPORTED otherwise); vocab may be smaller than
 * the logits buffer (the reference's usable tokenizer vocabulary). */
L0B_API l0b_status l0b_sample_execute(l0b_suite* s, l0b_device* d, l0b_buffer* logits, int32_t vocab,
                                      l0b_buffer* context, int32_t n_context, float temperature, float top_p,
                                      int32_t top_k, float repetition_penalty, double random_value,
                                      l0b_buffer* out_token);

/* CausalConv.Execute(dev, qkv, convState, convW, out, convDim, k, tokens) -- L/LlmDecoderLayer.cs:392.
 * Depthwise causal conv1d over [history (k-1 taps, oldest first) ++ tokens], then SiLU; the history
 * is shifted to hold the last k-1 inputs. convW [convDim, k]. */
L0B_API l0b_status l0b_causal_conv_execute(l0b_suite* s, l0b_device* d, l0b_buffer* qkv,
                                           l0b_buffer* conv_state, l0b_buffer* conv_w, l0b_buffer* out,
                                           int32_t conv_dim, int32_t kernel, int32_t tokens);
/* GatedDelta.Execute(dev, conv, z, b, a, A_log, dt_bias, normW, S, out, Hv, dk, dv, tokens, eps) --
 * L/LlmDecoderLayer.cs:393-395. Per token in order: q,k L2-normalised (eps 1e-6), beta = sigmoid(b),
 * g = -exp(A_log) * softplus(a + dt_bias), S = e^g S, S += k (beta (v - S^T k))^T, o = S^T q / sqrt(dk),
 * out = rmsnorm(o) * normW * silu(z) per head. The reference requires Hk == Hv. */
L0B_API l0b_status l0b_gated_delta_execute(l0b_suite* s, l0b_device* d, l0b_buffer* conv, l0b_buffer* z,
                                           l0b_buffer* b, l0b_buffer* a, l0b_buffer* a_log,
                                           l0b_buffer* dt_bias, l0b_buffer* norm_w, l0b_buffer* state,
                                           l0b_buffer* out, int32_t n_v_heads, int32_t key_dim,
                                           int32_t value_dim, int32_t tokens, float eps);
/* Same with Hk < Hv (Qwen3.5 grouping: value head h reads key head h / (Hv / Hk)); conv rows are
 * [q (Hk*dk) | k (Hk*dk) | v (Hv*dv)]. No reference counterpart (the reference rejects Hk != Hv,
 * L/HfModelConfig.cs:367-370); needed by the Hk=16, Hv=32 DeltaNet configuration. */
L0B_API l0b_status l0b_gated_delta_execute_grouped(l0b_suite* s, l0b_device* d, l0b_buffer* conv,
                                                   l0b_buffer* z, l0b_buffer* b, l0b_buffer* a,
                                                   l0b_buffer* a_log, l0b_buffer* dt_bias,
                                                   l0b_buffer* norm_w, l0b_buffer* state, l0b_buffer* out,
                                                   int32_t n_k_heads, int32_t n_v_heads, int32_t key_dim,
                                                   int32_t value_dim, int32_t tokens, float eps);
/* Tuning: calls of 16 or more tokens (prefill) run the recurrence in chunks of 64 tokens (1, default:
 * the WY form -- per-chunk products built for every chunk in parallel, then one pass over the chunks
 * per group of state columns; key head dim 64 or 128, value head dim a multiple of 32; scratch of
 * ~150 KB per (value head, chunk) kept by the suite, grown outside recording) or token by token (0).
 * No counterpart in the reference. */
L0B_API l0b_status l0b_set_gated_delta_chunked(int32_t enable);
/* Batched decode of the DeltaNet ops (no counterpart in the reference, whose MixLinear runs one sequence
 * at a time, L/LlmDecoderLayer.cs:381-397): one token of each of `batch` sequences in one launch.
 * CausalConv: qkv / out [batch, convDim], convStates [batch, convDim, kernel - 1]. GatedDelta: conv
 * [batch, convDim], z / out [batch, Hv * dv], b / a [batch, Hv], states [batch, Hv, dk, dv]. Row b of
 * each equals the single-sequence op on sequence b's buffers. */
L0B_API l0b_status l0b_causal_conv_execute_batch(l0b_suite* s, l0b_device* d, l0b_buffer* qkv,
                                                 l0b_buffer* conv_states, l0b_buffer* conv_w, l0b_buffer* out,
                                                 int32_t conv_dim, int32_t kernel, int32_t batch);
L0B_API l0b_status l0b_gated_delta_execute_batch(l0b_suite* s, l0b_device* d, l0b_buffer* conv, l0b_buffer* z,
                                                 l0b_buffer* b, l0b_buffer* a, l0b_buffer* a_log,
                                                 l0b_buffer* dt_bias, l0b_buffer* norm_w, l0b_buffer* states,
                                                 l0b_buffer* out, int32_t n_k_heads, int32_t n_v_heads,
                                                 int32_t key_dim, int32_t value_dim, int32_t batch, float eps);
/* The DeltaNet part of the device-side fork (replaces the LlmLinearState half of LlmModel.CaptureState +
 * RestoreState, L/LlmModel.cs:257-306 and L/LlmSequenceState.cs:14-80, which copy the conv window and the
 * recurrent state through host arrays): sequence dst's conv window and recurrent state in the batched
 * state buffers become device copies of sequence src's. Stream-ordered; not while recording. */
L0B_API l0b_status l0b_linear_state_fork(l0b_suite* s, l0b_device* d, l0b_buffer* conv_states, l0b_buffer* states,
                                         int32_t conv_dim, int32_t kernel, int32_t n_v_heads, int32_t key_dim,
                                         int32_t value_dim, int32_t src, int32_t dst);

/* ------------------------------------------------------------------------------------------ */
/* Linear layers in the [out, in] layout, and the fused decode ops                              */
/*                                                                                            */
/* These take weights in the HuggingFace [out=N, in=K] order for every precision, which is the  */
/* order the int8 path already uses (L/LlmMatrix.cs:89-93): each output row is one contiguous   */
/* stream that a warp reads with 128-bit loads and reduces with shuffles.                       */
/* w dtype: L0B_F32, L0B_F16, L0B_BF16 or L0B_I8 (then `scales` f16 [N, K/group]).             */
/* ------------------------------------------------------------------------------------------ */

/* Ordering note for the linear ops below: the decode GEMVs start streaming W before they wait for the
 * previous kernel on the stream (weights are parameters), and the GEMVs, GEMMs and attention let the
 * next kernel start early. So W must not be an output of the linear / attention op launched just before
 * on the same stream; weights written by uploads, l0b_q8_quantize_device or the other ops are ordered.
 *
 * Y[M, N] = X[M, K] * W^T (+ bias). X f32/f16/bf16, Y f32/f16/bf16; bias f32 [N] or NULL.
 * group: int8 scale group (32, or K for per-channel); ignored for 16/32-bit weights.
 * Any M: the weights stream once per 8 rows (tensor-core GEMV); l0b_linear_tc runs a prefill-sized M
 * as one tcgen05 GEMM. */
L0B_API l0b_status l0b_linear(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                              l0b_buffer* w, l0b_buffer* scales, int32_t group, l0b_buffer* bias,
                              l0b_buffer* y);

/* LlmMatrix.ProjectShared(dev, suite, rows, x, W1, y1, ..., W4, y4) -- L/LlmMatrix.cs:177-218 -- for up
 * to four projections of the same x whose weights are stored stacked in one matrix W = [W1; W2; ...]
 * ([out, in] order, sum(seg_rows) rows; int8 with scales stacked the same way): one launch streams W
 * once and writes Y_i [m, seg_rows[i]] (+ biases[i] f32 when biases and biases[i] are non-null). The
 * outputs share one dtype (f32/f16/bf16). Gated DeltaNet's in-projections (qkv, z, b, a) and the
 * attention's q/k/v are the reference's uses. */
L0B_API l0b_status l0b_linear_shared(l0b_suite* s, l0b_device* d, int32_t m, int32_t k, l0b_buffer* x,
                                     l0b_buffer* w, l0b_buffer* scales, int32_t group, int32_t nseg,
                                     const int32_t* seg_rows, l0b_buffer* const* biases, l0b_buffer* const* outs);

typedef enum l0b_epilogue {
    L0B_EPI_STORE = 0,  /* out[m, n] = y[m, n] (+ bias) */
    L0B_EPI_ACCUM = 1,  /* out[m, n] += y[m, n] (+ bias): the residual add of o_proj / down_proj */
    L0B_EPI_SWIGLU = 2, /* W = [gate; up] (N = 2 * I rows): out[m, i] = silu(y[m, i]) * y[m, i + I] */
    /* l0b_linear_tc only, OR'ed into the epilogue: the x rows enter as hi + lo 16-bit halves (each row
     * scaled by a power of two for f16's range) so the products keep about f32 activation precision,
     * at twice the tensor-core work; the mode the model's prefill uses. */
    L0B_EPI_F32_ACTIVATIONS = 0x100,
    /* l0b_linear_fused only, OR'ed into the epilogue: W is int8 with one f16 scale per row (group = K)
     * stored in the blocked layout [N/16][K/512][16][512] bytes (N % 16 == 0, K % 512 == 0) -- the
     * 16 rows x 512 k of one (row tile, k block) are one contiguous 8 KB block, the layout a model keeps
     * its q/k/v, o_proj and down projections in. One activation row runs on the k-split GEMV (each CTA
     * one k block of a group of row tiles, exact integer row sums in the suite's scratch); more rows on
     * the tensor-core GEMV with blocked addressing. N <= 65536. */
    L0B_EPI_BLOCKED_WEIGHTS = 0x200
} l0b_epilogue;

/* Fused linear layer of the decode path: optional RMSNorm of each x row with norm_w (eps) as the
 * prologue (the input / post-attention norm, L/LlmDecoderLayer.cs:167,183-184), then the projection,
 * then the epilogue. Replaces RMSNorm + ProjectShared(gate, up) + SwiGLU (L/LlmDecoderLayer.cs:183-189)
 * or Project + Add (:190-194) with one kernel. out is f32. */
L0B_API l0b_status l0b_linear_fused(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                    l0b_buffer* w, l0b_buffer* scales, int32_t group, l0b_buffer* norm_w, float eps,
                                    int32_t epilogue, l0b_buffer* bias, l0b_buffer* out);

/* Prefill-sized linear layer on the tensor cores (tcgen05.mma, accumulator in TMEM, TMA-fed): the x
 * rows are (RMS-normalised with norm_w when given and) rounded to the weight's 16-bit format, then
 * out = epilogue(x16 W^T) with fp32 accumulation. w: f16 or bf16 [N, K], K % 8 == 0; SwiGLU needs
 * (N/2) % 64 == 0. The multi-row GEMV of Gemv.ExecuteRows (L/LlmMatrix.cs:149-171) replaced by a GEMM. */
L0B_API l0b_status l0b_linear_tc(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                 l0b_buffer* w, l0b_buffer* norm_w, float eps, int32_t epilogue, l0b_buffer* bias,
                                 l0b_buffer* out);
/* l0b_linear_tc for int8 weights: W int8 [N, K] (K % 16 == 0) with one f16 scale per row (scales [N],
 * group = K or <= 0). TMA stages the raw bytes, two warps convert them to f16 in shared memory (exact),
 * the MMA runs in f16 (activations rounded to f16, or split into hi + lo f16 halves with
 * L0B_EPI_F32_ACTIVATIONS), and the epilogue applies the row scale. Group-wise scales are refused
 * (L0B_ERR_UNSUPPORTED): they stay on the GEMV. f16/bf16 W are accepted and scales ignored. */
L0B_API l0b_status l0b_linear_tc_scaled(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                        l0b_buffer* w, l0b_buffer* scales, int32_t group, l0b_buffer* norm_w,
                                        float eps, int32_t epilogue, l0b_buffer* bias, l0b_buffer* out);

/* ------------------------------------------------------------------------------------------ */
/* Tensor parallelism (one process per GPU, NCCL over NVLink/NVSwitch)                           */
/* ------------------------------------------------------------------------------------------ */

/* A 128-byte NCCL unique id, made on one rank and handed to the others by the caller (any channel).
 * No counterpart in the reference (single-GPU); LevelZeroLlmEngine would pass it at start-up. */
L0B_API l0b_status l0b_comm_unique_id(uint8_t* id, int32_t bytes);
/* Joins communicator `id` as `rank` of `nranks`, bound to `dev`'s stream. Collective: every rank
 * calls it. Models created with cfg.tp_size = nranks, cfg.tp_rank = rank take it (l0b_model_create). */
L0B_API l0b_status l0b_comm_create(l0b_device* dev, const uint8_t* id, int32_t bytes, int32_t nranks, int32_t rank,
                                   l0b_comm** out);
L0B_API l0b_status l0b_comm_free(l0b_comm* comm);
/* In-place sum of the first `count` elements of `buf` over the ranks, on the device stream (recorded
 * into the current command list when the device is recording). */
L0B_API l0b_status l0b_comm_allreduce(l0b_comm* comm, l0b_buffer* buf, int64_t count);
/* Tensor-parallel all-reduces of f32 sums (the row-split o_proj / down partials, up to 131072 values)
 * and u64 maxima (the vocab-split argmax keys, up to 2 MB) run as one kernel over peer memory: every
 * rank's mailbox is mapped into the others by CUDA IPC when the communicator is made. f32 sums: each rank
 * writes every value into every mailbox as one 64-bit word that also carries the call's epoch, and reads
 * the others' words from its own mailbox as they arrive (bounded wait, ~2 s, then the device error
 * flag), summing in rank order, so all ranks hold the same bits; no fence and no separate flag. u64
 * maxima: partials, a system-scope fence and an epoch flag per rank. No multicast loads. Larger or other
 * collectives, and communicators made after l0b_comm_set_peer_allreduce(0), use NCCL. No counterpart in
 * the reference (single device). */
L0B_API l0b_status l0b_comm_set_peer_allreduce(int32_t enable);
/* *enabled = 1 when this communicator's small all-reduces run over peer memory (every rank agrees). */
L0B_API l0b_status l0b_comm_uses_peer_allreduce(l0b_comm* comm, int32_t* enabled);
/* With peer memory, a model's row-split decode projections (o_proj, down on the register-streamed
 * tensor-core GEMV: 16-bit or row-major int8 weights) fold the all-reduce into the GEMV (1, default):
 * each CTA sends its tiles' partial sums, tagged with the call's epoch, to every rank's mailbox, reads
 * (bounded wait) the same tiles from the other ranks and adds them to the residual stream in rank order
 * -- the bits of the GEMV + all-reduce pair, one launch instead of two. 0: the pair. Process-wide;
 * affects steps recorded after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_comm_set_fused_allreduce(int32_t enable);

/* Tuning: the largest K split the tensor-core GEMM may use for narrow projections (1..16, default 16;
 * <= 0 restores the default). Affects plans made after the call. */
L0B_API l0b_status l0b_tc_set_max_splits(int32_t splits);
/* Tuning: one-row int8 projections on the GEMV that streams weights by bulk copies (1, default) -- whole
 * 16-row tiles for projections with at least 8 tiles per SM (gate/up, LM head), units of up to four
 * 512-k blocks of a tile for projections stored in the blocked layout (q/k/v, o_proj, down) -- or on the
 * register-streamed one (0). Affects launches made after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_bulk(int32_t enable);
/* Tuning: largest K split (1, 2, 4 or 8; default 2) the register-streamed tensor-core GEMV takes only to
 * fill SMs that its 16-row tiles would leave idle (fewer tiles than SMs, slices of at least 2048 k);
 * 1 disables it. Affects launches made after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_fill_split(int32_t max_splits);
/* Tuning: blocked int8 projections with short rows (fewer than 16 blocks of 512 k: q/k/v and o_proj of
 * a 3584-wide model) on the bulk-copy GEMV as well (1) or on the register-streamed one (0, default).
 * Affects launches made after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_bulk_short_rows(int32_t enable);
/* Tuning: one-row blocked int8 projections of a model (q/k/v, o_proj, down) on the k-split GEMV (1,
 * default: each CTA multiplies one 512-k block of a group of row tiles on the integer tensor cores and
 * adds exact int64 row sums; the last CTA of a group runs the epilogue) or on the bulk / register GEMVs
 * (0). Affects launches made after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_ksplit(int32_t enable);
/* Tuning: stages (32 KB each, 2..6, default 4) of the k-split GEMV's bulk-copy ring. Fewer stages leave
 * room on an SM for the next kernel's CTAs to start early (config 2 bs1: 6 stages 448, 4 stages 453, 2
 * stages 446 tok/s). Affects launches made after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_ksplit_stages(int32_t stages);
/* Tuning: L2 prefetch in the one-row decode step of a single-GPU model (0 = off). With gate_up_mb > 0
 * the k-split GEMVs, whose latency-bound launches leave HBM mostly idle, prefetch constant weights of the
 * projections that follow into L2 (cp.async.bulk.prefetch.L2): q/k/v prefetches o_proj's weights, o_proj
 * the first gate_up_mb MB of the [gate; up] weights (half from each), down the next layer's q/k/v.
 * Results are unchanged (a prefetch only moves data into the cache). Affects steps recorded after the
 * call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_l2_prefetch(int32_t gate_up_mb);
/* Tuning: the bulk-copy GEMV's ring of whole 16-row tiles (row-major int8: gate/up, LM head; units of
 * blocked k blocks are not affected). 0 (default): at most 120 KB of tiles, at least two -- two at K = 3584,
 * which leaves room on an SM for the next k-split GEMV's CTAs (config 2 bs1: 2.192 ms per step, 2.231 with
 * three), eight at K = 896; 2..8: at most that many tiles; 1: as many as its shared-memory budget holds.
 * Affects launches made after the call. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_bulk_stages(int32_t stages);
/* Layout of the int8 weights of models created after the call: with blocking on (1, default), int8
 * projections with one scale per row, K % 512 == 0, N % 16 == 0 and fewer than 8 tiles of 16 rows per
 * SM (q/k/v, o_proj, down at Qwen2.5-7B widths) are stored as [N/16][K/512][16][512] bytes, so the k
 * blocks of a 16-row tile are contiguous 8 KB blocks; 0 keeps every matrix row-major [N, K].
 * l0b_model_read_weight returns the [out, in] order either way. No counterpart in the reference. */
L0B_API l0b_status l0b_set_weight_blocking(int32_t enable);
/* Process-wide choice of the decode GEMV kernel for shapes both take: 1 (default) = tensor-core
 * mma.sync streaming kernel, 0 = fp32-FMA streaming kernel. Used by tests to cover both; recorded
 * command lists keep the kernel they were recorded with. No counterpart in the reference. */
L0B_API l0b_status l0b_set_gemv_tensor_cores(int32_t enable);

/* Raw-pointer int8 GEMV for callers that manage device memory themselves (config 0 shape:
 * y[M,N] = x[M,K] * (q * s)^T with fp16 x and y). x_dtype/y_dtype from l0b_dtype. Enqueued on
 * `stream` (a cudaStream_t, NULL = legacy default stream); returns immediately. */
L0B_API l0b_status l0b_gemv_w8a16_raw(void* stream, int32_t m, int32_t n, int32_t k, const void* x,
                                      int32_t x_dtype, const int8_t* q, const uint16_t* scales,
                                      int32_t group, void* y, int32_t y_dtype);

/* ------------------------------------------------------------------------------------------ */
/* Decoder model  (C++ mirror of LlmModel / LlmDecoderLayer / LlmMatrix / LlmKvCache,            */
/*                 L/LlmModel.cs:15-481, L/LlmDecoderLayer.cs:19-534)                          */
/* ------------------------------------------------------------------------------------------ */

typedef enum l0b_precision {
    L0B_PRECISION_AUTO = 0,    /* LlmWeightPrecision.Auto -> Int8 (this backend has the int8 kernels) */
    L0B_PRECISION_FLOAT32 = 1, /* LlmWeightPrecision.Float32 */
    L0B_PRECISION_FLOAT16 = 2, /* LlmWeightPrecision.Float16 */
    L0B_PRECISION_INT8 = 3,    /* LlmWeightPrecision.Int8 (scale group: l0b_model_config.q8_group) */
    L0B_PRECISION_BFLOAT16 = 4 /* bf16 storage (no reference counterpart; Llama-3-70B configuration) */
} l0b_precision;

typedef enum l0b_rope_type {
    L0B_ROPE_DEFAULT = 0,
    L0B_ROPE_LINEAR = 1,
    L0B_ROPE_YARN = 2,
    L0B_ROPE_LLAMA3 = 3
} l0b_rope_type;

/* The fields of HfModelConfig the decoder reads (L/HfModelConfig.cs:132-205). */
typedef struct l0b_model_config {
    int32_t hidden_size;
    int32_t intermediate_size;
    int32_t num_layers;
    int32_t num_attention_heads;
    int32_t num_key_value_heads;
    int32_t head_dim;
    int32_t vocab_size;
    int32_t max_position_embeddings;
    float rms_norm_eps;
    double rope_theta;
    int32_t tie_word_embeddings;
    int32_t attention_bias;      /* qwen2: q/k/v bias */
    int32_t qk_norm;             /* qwen3: per-head RMSNorm on q and k */
    int32_t rope_type;           /* l0b_rope_type */
    double rope_factor;
    int32_t rope_original_max_position;
    double rope_low_freq_factor;
    double rope_high_freq_factor;
    double rope_beta_fast;
    double rope_beta_slow;
    double rope_attention_factor; /* <= 0: derive (YaRN mscale) */
    double rope_mscale;           /* YaRN mscale, <= 0 when absent */
    double rope_mscale_all_dim;   /* YaRN mscale_all_dim, <= 0 when absent */
    int32_t rope_truncate;        /* YaRN: round the correction range to whole dims (default 1) */
    double partial_rotary_factor; /* 1.0 = full rotary */
    int32_t kv_dtype;            /* l0b_dtype of the KV cache: F32 (reference), F16 or BF16 */
    int32_t q8_group;            /* int8 scale group: 32 (reference) or 0 = per output channel */
    int32_t tp_size;             /* tensor-parallel ranks (1 = none) */
    int32_t tp_rank;
    int32_t max_batch;           /* sequences decoded together (KV cache rows); default 1, at most 64 */
    /* Qwen3.5 hybrid decoders (L/HfModelConfig.cs:186-205, 340-370); all zero for the other families.
     * Layer l is a Gated DeltaNet (linear attention) layer when bit l of linear_layer_mask is set
     * (IsLinearLayer); such a model runs on one GPU, one sequence, on the reference op sequence. */
    uint64_t linear_layer_mask;
    int32_t linear_num_key_heads;
    int32_t linear_num_value_heads;
    int32_t linear_key_head_dim;   /* 64 or 128 */
    int32_t linear_value_head_dim; /* <= 256 */
    int32_t linear_conv_kernel;    /* 2..8 */
    int32_t attention_output_gate; /* q_proj holds [query | gate] rows per head (AttentionOutputGate) */
    float rms_norm_offset;         /* added to the input / post-attention / final / q / k norm weights at
                                      load (RmsNormOffset: 1 for Qwen3.5) */
} l0b_model_config;

/* Fills a config with the defaults HfModelConfig.Parse applies. */
L0B_API l0b_status l0b_model_config_init(l0b_model_config* cfg);

/* RopeFrequencies.Compute(config) -- L/RopeFrequencies.cs:60-107: the inverse frequencies of the
 * rotary table (rotary_dim / 2 values, written when inv_freq is non-null) and the factor that
 * multiplies cos and sin, for default / linear / yarn / llama3 scaling. */
L0B_API l0b_status l0b_rope_frequencies(const l0b_model_config* cfg, float* inv_freq, int32_t capacity,
                                        int32_t* count, float* attention_factor);

/* Allocates the model (weights, KV caches, per-layer buffers) for max_seq_len positions.
 * Weights are zero until loaded with l0b_model_set_tensor or l0b_model_init_synthetic.
 * comm: NULL, or the tensor-parallel communicator when cfg->tp_size > 1. */
L0B_API l0b_status l0b_model_create(l0b_device* dev, l0b_suite* suite, const l0b_model_config* cfg,
                                    int32_t max_seq_len, l0b_precision precision, l0b_comm* comm,
                                    l0b_model** out);
L0B_API l0b_status l0b_model_free(l0b_model* model);
/* Loads one HuggingFace-named tensor from host memory (fp32 values in the HF [out, in] order), with
 * the reference's load-time rules: norm offset, int8 quantization or 16-bit storage, q/gate split
 * (L/LlmLayerWeights.cs:110-212, L/LlmMatrix.cs:80-106). Names: model.embed_tokens.weight,
 * model.norm.weight, lm_head.weight, model.layers.{i}.{input_layernorm,post_attention_layernorm}.weight,
 * model.layers.{i}.self_attn.{q,k,v,o}_proj.weight, ...{q,k,v}_proj.bias, ...{q,k}_norm.weight,
 * model.layers.{i}.mlp.{gate,up,down}_proj.weight. With tensor parallelism pass the full tensor; the
 * model keeps its rank's shard. */
L0B_API l0b_status l0b_model_set_tensor(l0b_model* model, const char* name, const float* data,
                                        int64_t count);

/* Where l0b_model_set_tensor puts checkpoint tensor `name` for rank cfg->tp_rank of cfg->tp_size: the
 * model's tensor-parallel split as plain host arithmetic (no device, no model), the plan set_tensor
 * itself follows. Column-split projections (q/k/v by whole heads, gate/up, lm_head) keep output rows
 * [row0, row0 + rows) of the [full_rows, full_cols] tensor and place them at row dst_row of the rank's
 * stacked matrix ([q; k; v] or [gate; up]); row-split projections (o_proj, down) keep input columns
 * [col0, col0 + cols) of every row; a vector keeps elements [col0, col0 + cols) at element dst_row of its
 * destination (the q/k/v biases follow their projection's rows); norms and the embedding are whole on every
 * rank. The layout is this backend's; the reference runs one device (L/LlmLayerWeights.cs:110-212 loads the
 * same names unsplit). Unknown or unused names fail with L0B_ERR_INVALID_DATA, as l0b_model_set_tensor. */
typedef enum l0b_shard_kind {
    L0B_SHARD_MATRIX = 0,
    L0B_SHARD_VECTOR = 1,
    L0B_SHARD_EMBEDDING = 2,
    /* a Qwen3.5 q_proj with its output gate: per head, head_dim query rows then head_dim gate rows
     * (SplitQueryAndGate, L/LlmLayerWeights.cs:282-297). The `rows` query rows land at dst_row of the
     * stacked [q; k; v; gate] matrix, the gate rows after v. */
    L0B_SHARD_QUERY_GATE = 3
} l0b_shard_kind;
typedef enum l0b_shard_slot {
    /* matrices */
    L0B_SLOT_QKV = 0, L0B_SLOT_O = 1, L0B_SLOT_GATE_UP = 2, L0B_SLOT_DOWN = 3, L0B_SLOT_LM_HEAD = 4,
    L0B_SLOT_LIN_IN = 5,  /* Gated DeltaNet in-projections stacked [qkv; z; b; a] */
    L0B_SLOT_LIN_OUT = 6, /* Gated DeltaNet out_proj */
    /* vectors */
    L0B_SLOT_IN_NORM = 0, L0B_SLOT_POST_NORM = 1, L0B_SLOT_QKV_BIAS = 2, L0B_SLOT_Q_NORM = 3,
    L0B_SLOT_K_NORM = 4, L0B_SLOT_FINAL_NORM = 5, L0B_SLOT_LIN_CONV = 6, L0B_SLOT_LIN_A_LOG = 7,
    L0B_SLOT_LIN_DT_BIAS = 8, L0B_SLOT_LIN_NORM = 9
} l0b_shard_slot;
typedef struct l0b_shard_plan {
    int32_t kind;                 /* l0b_shard_kind */
    int32_t layer;                /* decoder layer, -1 for model-level tensors */
    int32_t slot;                 /* l0b_shard_slot of the destination */
    int32_t full_rows, full_cols; /* the checkpoint tensor ([1, n] for a vector) */
    int32_t row0, rows;           /* rows kept */
    int32_t col0, cols;           /* columns (vector: elements) kept */
    int32_t dst_row;              /* first destination row (vector: element) */
} l0b_shard_plan;
L0B_API l0b_status l0b_model_shard_plan(const l0b_model_config* cfg, const char* name, l0b_shard_plan* out);
/* A checkpoint tensor's raw 16-bit payload (dtype L0B_F16 or L0B_BF16, count values, HF [out, in] order) --
 * the bytes a safetensors F16 / BF16 entry holds -- uploaded as is and widened, range-checked (Float16
 * storage), converted or quantized on the device, with the rules of l0b_model_set_tensor. Replaces the
 * host-side BF16 -> f32 conversion before upload (L/SafetensorsReader.cs:262-277) and halves the bytes that
 * cross PCIe. */
L0B_API l0b_status l0b_model_set_tensor_raw(l0b_model* model, const char* name, const void* data, int32_t dtype,
                                            int64_t count);
/* Seeded synthetic weights generated on the device (no host copy): projections N(0, std) (an
 * Irwin-Hall(4) approximation of the normal), or for Int8 precision uniform int8 in [-127, 127]
 * with fp16 scales uniform on [scale_lo, scale_hi]; biases N(0, std); norms 1. */
L0B_API l0b_status l0b_model_init_synthetic(l0b_model* model, uint64_t seed, float std, float scale_lo,
                                            float scale_hi);
/* LlmModel.Prefill(promptIds): resets the sequence, ingests the prompt in chunks of up to 512 tokens
 * (each projection of a chunk one tensor-core GEMM that reads the weights once; the reference chunks by
 * LlmGemvKernel.MaxRows) and writes the logits of the next token (vocab f32, may be NULL). */
L0B_API l0b_status l0b_model_prefill(l0b_model* model, const int32_t* ids, int32_t count, float* logits);
/* LlmModel.Decode(tokenId): one token at Position; writes its logits (may be NULL). */
L0B_API l0b_status l0b_model_decode(l0b_model* model, int32_t token, float* logits);
/* LlmModel.ComputeLogits(tokenId, position). */
L0B_API l0b_status l0b_model_compute_logits(l0b_model* model, int32_t token, int32_t position, float* logits);
/* LlmModel.GenerateGreedy(promptIds, maxNewTokens, stopTokenIds): tokens (without the prompt) to
 * out[0, *out_count). The argmax is taken on the device; only token ids cross to the host. */
L0B_API l0b_status l0b_model_generate_greedy(l0b_model* model, const int32_t* ids, int32_t count,
                                             int32_t max_new, const int32_t* stop_ids, int32_t n_stop,
                                             int32_t* out, int32_t* out_count);
/* LlmModel.Position / ResetSequence / MaxSeqLen / ProjectionBytes. */
/* Batched decoding of independent sequences (a capability the reference's engine lacks: it serialises
 * one request at a time, L/LevelZeroLlmEngine.cs:22,55). A model created with cfg.max_batch = B keeps B
 * KV-cache rows; sequence 0 is also the one the single-sequence calls above use.
 *
 * Prefill of sequence `seq` (LlmModel.Prefill semantics, L/LlmModel.cs:224-239, into cache row seq);
 * logits (may be NULL) receive the last position's logits; the greedy next token and position are kept
 * on the device for l0b_model_decode_greedy_device_batch. */
L0B_API l0b_status l0b_model_prefill_sequence(l0b_model* model, int32_t seq, const int32_t* ids, int32_t count,
                                              float* logits);
/* One decode step of sequences 0..count-1: row b takes tokens[b] at positions[b] (cache row b).
 * logits (may be NULL): [count, vocab]. Fused path only. */
L0B_API l0b_status l0b_model_decode_batch(l0b_model* model, const int32_t* tokens, const int32_t* positions,
                                          int32_t count, float* logits);
/* `steps` greedy steps of sequences 0..count-1 entirely on the device (one CUDA graph per step), each
 * sequence continuing from its own token and position; out (may be NULL): [steps, count] tokens. */
L0B_API l0b_status l0b_model_decode_greedy_device_batch(l0b_model* model, int32_t steps, int32_t count,
                                                        int32_t* out);
/* Next position of sequence `seq` (its prefilled and decoded length). */
L0B_API l0b_status l0b_model_sequence_position(l0b_model* model, int32_t seq, int32_t* position);
/* Device-side fork for beam search (replaces LlmModel.CaptureState + RestoreState,
 * src/HFLabs.ML.LLM.LevelZero/LlmModel.cs:257-306, which copy the KV tail through host arrays): sequence
 * dst becomes a copy of sequence src. KV-cache rows [base_position, length of src) of every layer are
 * copied device to device (rows below base_position, a shared prompt, are assumed equal), and dst takes
 * src's length and its device-side next token and position. Stream-ordered: no host synchronisation. */
L0B_API l0b_status l0b_model_fork_sequence(l0b_model* model, int32_t src, int32_t dst, int32_t base_position);
L0B_API l0b_status l0b_model_position(l0b_model* model, int32_t* position);
L0B_API l0b_status l0b_model_reset_sequence(l0b_model* model);
L0B_API l0b_status l0b_model_projection_bytes(l0b_model* model, int64_t* bytes);
/* Runs `steps` greedy decode steps entirely on the device (each step's input is the previous step's
 * argmax, no host round trip), starting from the last sampled token. Tokens to out (may be NULL).
 * This is the device-resident throughput path that benchmarks time. */
L0B_API l0b_status l0b_model_decode_greedy_device(l0b_model* model, int32_t steps, int32_t* out);
/* Debug mode: run ops without command-list recording (the reference's Probe path). */
L0B_API l0b_status l0b_model_set_recording(l0b_model* model, int32_t enabled);
/* Selects the fused decode kernels (1, default) or the one-op-per-reference-call sequence (0). */
L0B_API l0b_status l0b_model_set_fused(l0b_model* model, int32_t enabled);
/* Projections over at least `min_rows` activation rows (prefill chunks) with f16/bf16 weights, or int8
 * weights with one scale per row, run on the tcgen05 GEMM (weights read once per chunk, activations as
 * hi + lo 16-bit halves); fewer rows, group-wise int8 and min_rows = 0 use the GEMV. Default 8. */
L0B_API l0b_status l0b_model_set_gemm_rows(l0b_model* model, int32_t min_rows);
/* LlmDecoderLayer.Probe (L/LlmDecoderLayer.cs:113-119): when set, steps run the reference op sequence
 * without command-list recording and call `fn` after each stage of each layer with a host copy of the
 * stage's buffer (row 0 of the step). Stages: input_norm, q, k, v (after bias, before RoPE), attn_out
 * (after o_proj), post_norm, mlp_out, output. The host copy is reused: copy what you need inside the
 * callback. fn = NULL removes the probe. */
typedef void (*l0b_probe_fn)(void* user, int32_t layer, const char* stage, const float* values, int64_t count);
L0B_API l0b_status l0b_model_set_probe(l0b_model* model, l0b_probe_fn fn, void* user);
/* Copies raw weight storage of layer `layer` (-1 = LM head) for inspection: kind 0 = stacked q/k/v,
 * 1 = o_proj, 2 = stacked gate/up, 3 = down_proj (weights in the model precision's dtype, [out, in]);
 * kind 4..7 = the int8 scales of the same matrices. bytes must equal the storage size. */
L0B_API l0b_status l0b_model_read_weight(l0b_model* model, int32_t layer, int32_t kind, void* out, int64_t bytes);
/* Reads layer `layer`'s KV cache rows [row0, row0 + rows) as f32 (CaptureState's KV part,
 * L/LlmModel.cs:257-281). keys/values hold rows * kvDim floats. */
L0B_API l0b_status l0b_model_read_kv(l0b_model* model, int32_t layer, int32_t row0, int32_t rows,
                                     float* keys, float* values);

#ifdef __cplusplus
}
#endif

#endif /* L0B200_H */
