// C ABI of LlmKernelSuite: argument validation (mirroring the reference's exceptions) and dispatch to
// the kernels. Every op accepts the device the suite was created on.
#include <cmath>
#include <map>
#include <memory>
#include <vector>

#include <cuda_fp16.h>

#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "ops.cuh"
#include "suite.h"

using namespace l0b;

namespace l0b {

l0b_status suite_rope_table(l0b_suite* s, int rot, double theta, const float** out) {
    auto key = std::make_pair(rot, theta);
    auto it = s->rope_tables.find(key);
    if (it == s->rope_tables.end()) {
        // L/RopeFrequencies.cs:75-80: 1 / theta^(2i / dim) in double, rounded to float.
        std::vector<float> t(rot / 2);
        for (int i = 0; i < rot / 2; ++i) t[i] = static_cast<float>(1.0 / std::pow(theta, 2.0 * i / rot));
        float* dptr = nullptr;
        L0B_CHECK_CUDA(cudaMalloc(&dptr, t.size() * sizeof(float)));
        L0B_CHECK_CUDA(copy_sync(s->dev->stream, dptr, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice));
        it = s->rope_tables.emplace(key, dptr).first;
    }
    *out = it->second;
    return L0B_OK;
}

}  // namespace l0b

l0b_suite::~l0b_suite() {
    if (dev) cudaSetDevice(dev->index);
    if (dev && dev->stream) cudaStreamSynchronize(dev->stream);
    for (auto& kv : rope_tables) cudaFree(kv.second);
    if (q8_x) cudaFree(q8_x);
    if (error_flag) cudaFree(error_flag);
    if (split_part) cudaFree(split_part);
    if (gdn_rec) cudaFree(gdn_rec);
    if (split_counters) cudaFree(split_counters);
    if (ks_acc) cudaFree(ks_acc);
}

namespace {

l0b_status check_suite(l0b_suite* s, l0b_device* d) {
    L0B_REQUIRE(s, L0B_ERR_ARGUMENT, "suite is null");
    L0B_REQUIRE(d, L0B_ERR_ARGUMENT, "device is null");
    L0B_REQUIRE(s->dev == d, L0B_ERR_ARGUMENT, "the suite belongs to another device");
    return L0B_OK;
}

l0b_status need(l0b_buffer* b, const char* name, l0b_dtype t, long long count) {
    L0B_REQUIRE(b, L0B_ERR_ARGUMENT, "%s is null", name);
    L0B_REQUIRE(b->dtype == t, L0B_ERR_ARGUMENT, "%s must be a %s buffer, got %s", name, dtype_name(t),
                dtype_name(b->dtype));
    L0B_REQUIRE(b->count >= count, L0B_ERR_ARGUMENT, "%s holds %lld elements, need %lld", name,
                (long long)b->count, count);
    return L0B_OK;
}

l0b_status need_float(l0b_buffer* b, const char* name, long long count) {
    L0B_REQUIRE(b, L0B_ERR_ARGUMENT, "%s is null", name);
    L0B_REQUIRE(b->dtype == L0B_F32 || b->dtype == L0B_F16 || b->dtype == L0B_BF16, L0B_ERR_ARGUMENT,
                "%s must be an f32/f16/bf16 buffer, got %s", name, dtype_name(b->dtype));
    L0B_REQUIRE(b->count >= count, L0B_ERR_ARGUMENT, "%s holds %lld elements, need %lld", name,
                (long long)b->count, count);
    return L0B_OK;
}

float* F(l0b_buffer* b) { return b ? static_cast<float*>(b->ptr) : nullptr; }

}  // namespace

#define GUARD_BEGIN try {
#define GUARD_END                                                                                  \
    }                                                                                              \
    catch (const std::bad_alloc&) {                                                                \
        return fail(L0B_ERR_OUT_OF_MEMORY, "host allocation failed");                              \
    }                                                                                              \
    catch (const std::exception& e) {                                                              \
        return fail(L0B_ERR_INVALID_OPERATION, "%s", e.what());                                    \
    }

extern "C" {

L0B_API l0b_status l0b_suite_create(l0b_device* dev, l0b_suite** out) {
    GUARD_BEGIN
    L0B_REQUIRE(dev && out, L0B_ERR_ARGUMENT, "null argument");
    std::unique_ptr<l0b_suite> s(new l0b_suite());
    s->dev = dev;
    L0B_CHECK_CUDA(cudaSetDevice(dev->index));
    L0B_CHECK_CUDA(cudaMalloc(&s->error_flag, sizeof(int)));
    L0B_CHECK_CUDA(cudaMemsetAsync(s->error_flag, 0, sizeof(int), dev->stream));
    L0B_CHECK_CUDA(cudaMalloc(&s->split_part, sizeof(float) * 64 * kSuiteSplitTiles));
    L0B_CHECK_CUDA(cudaMalloc(&s->split_counters, sizeof(unsigned) * kSuiteSplitTiles));
    L0B_CHECK_CUDA(cudaMemsetAsync(s->split_counters, 0, sizeof(unsigned) * kSuiteSplitTiles, dev->stream));
    L0B_CHECK_CUDA(cudaMalloc(&s->ks_acc, sizeof(long long) * kSuiteKsRows));
    L0B_CHECK_CUDA(cudaMemsetAsync(s->ks_acc, 0, sizeof(long long) * kSuiteKsRows, dev->stream));
    L0B_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
    *out = s.release();
    return L0B_OK;
    GUARD_END
}

L0B_API l0b_status l0b_suite_free(l0b_suite* suite) {
    delete suite;
    return L0B_OK;
}

L0B_API int32_t l0b_suite_has_q8(l0b_suite* suite) { return suite ? 1 : 0; }

L0B_API l0b_status l0b_suite_ensure_q8_scratch(l0b_suite* s, int32_t rows, int32_t width) {
    L0B_REQUIRE(s, L0B_ERR_ARGUMENT, "suite is null");
    L0B_REQUIRE(rows > 0 && width > 0, L0B_ERR_OUT_OF_RANGE, "scratch of %d rows x %d", rows, width);
    if (rows <= s->q8_rows && width <= s->q8_width) return L0B_OK;
    L0B_REQUIRE(!s->dev->recording, L0B_ERR_INVALID_OPERATION,
                "the activation scratch must be sized before a command list is recorded");
    const int r = rows > s->q8_rows ? rows : s->q8_rows;
    const int w = width > s->q8_width ? width : s->q8_width;
    if (s->q8_x) {
        L0B_CHECK_CUDA(cudaStreamSynchronize(s->dev->stream));
        L0B_CHECK_CUDA(cudaFree(s->q8_x));
        s->q8_x = nullptr;
    }
    L0B_CHECK_CUDA(cudaMalloc(&s->q8_x, static_cast<size_t>(r) * w * sizeof(float)));
    s->q8_rows = r;
    s->q8_width = w;
    return L0B_OK;
}

L0B_API int32_t l0b_suite_q8_scratch_rows(l0b_suite* s) { return s ? s->q8_rows : 0; }

L0B_API int32_t l0b_gemv_supports(int32_t n) { return n > 0 && n % 4 == 0; }
L0B_API int32_t l0b_gemv_max_rows(void) { return kMaxRows; }
L0B_API int32_t l0b_gemv_q8_supports(int32_t n, int32_t k) { return n > 0 && k > 0 && n % 4 == 0 && k % 32 == 0; }
L0B_API int32_t l0b_gemv_q8_group_size(void) { return 32; }

L0B_API l0b_status l0b_q8_quantize_out_in(const float* hf, int32_t n, int32_t k, int32_t group, int32_t* words,
                                          uint16_t* scales) {
    L0B_REQUIRE(hf && words && scales, L0B_ERR_ARGUMENT, "null argument");
    L0B_REQUIRE(n > 0 && k > 0 && group > 0 && k % group == 0 && k % 4 == 0, L0B_ERR_ARGUMENT,
                "quantization needs K %% group == 0 and K %% 4 == 0 (N=%d K=%d group=%d)", n, k, group);
    int8_t* q = reinterpret_cast<int8_t*>(words);
    const int gpr = k / group;
    for (int o = 0; o < n; ++o) {
        for (int g = 0; g < gpr; ++g) {
            const float* src = hf + static_cast<long long>(o) * k + static_cast<long long>(g) * group;
            float mx = 0.f;
            for (int i = 0; i < group; ++i) mx = std::fmax(mx, std::fabs(src[i]));
            const __half sh = __float2half_rn(mx / 127.0f);
            const float sf = __half2float(sh);
            for (int i = 0; i < group; ++i) {
                float r = 0.f;
                if (sf > 0.f) r = std::fmin(127.f, std::fmax(-127.f, std::nearbyint(src[i] / sf)));
                q[static_cast<long long>(o) * k + static_cast<long long>(g) * group + i] = static_cast<int8_t>(r);
            }
            __half_raw raw = sh;
            scales[static_cast<long long>(o) * gpr + g] = raw.x;
        }
    }
    return L0B_OK;
}

L0B_API l0b_status l0b_q8_quantize_device(l0b_suite* s, l0b_device* d, int32_t n, int32_t k, int32_t group,
                                          l0b_buffer* w, l0b_buffer* q, l0b_buffer* sc) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(n > 0 && k > 0 && group > 0 && k % group == 0, L0B_ERR_ARGUMENT, "bad quantization shape");
    const long long nk = static_cast<long long>(n) * k;
    L0B_TRY(need_float(w, "w", nk));
    L0B_REQUIRE(q && (q->dtype == L0B_I8 || q->dtype == L0B_I32) && static_cast<long long>(q->bytes()) >= nk,
                L0B_ERR_ARGUMENT, "q must hold N*K int8 values");
    L0B_TRY(need(sc, "scales", L0B_F16, nk / group));
    return k_quantize(d, w->ptr, w->dtype, n, k, group, static_cast<int8_t*>(q->ptr), static_cast<__half*>(sc->ptr));
}

L0B_API l0b_status l0b_embedding_execute(l0b_suite* s, l0b_device* d, l0b_buffer* ids, l0b_buffer* table,
                                         l0b_buffer* out, int32_t h, int32_t count) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(h > 0 && count >= 0 && count % h == 0, L0B_ERR_OUT_OF_RANGE, "count %d is not a multiple of h %d",
                count, h);
    L0B_TRY(need(ids, "ids", L0B_I32, count / h));
    L0B_TRY(need_float(table, "table", h));
    L0B_TRY(need(out, "out", L0B_F32, count));
    const int vocab = static_cast<int>(table->count / h);
    return k_embedding(d, static_cast<const int*>(ids->ptr), table->ptr, table->dtype, F(out), h, count, vocab,
                       s->error_flag);
}

L0B_API l0b_status l0b_rmsnorm_execute(l0b_suite* s, l0b_device* d, l0b_buffer* x, l0b_buffer* res, l0b_buffer* w,
                                       l0b_buffer* out, float eps, int32_t width, int32_t rows, int32_t add_residual) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(width > 0 && rows > 0, L0B_ERR_OUT_OF_RANGE, "width %d rows %d", width, rows);
    const long long n = static_cast<long long>(width) * rows;
    L0B_TRY(need(x, "x", L0B_F32, n));
    L0B_TRY(need(w, "w", L0B_F32, width));
    L0B_TRY(need(out, "out", L0B_F32, n));
    if (add_residual) L0B_TRY(need(res, "res", L0B_F32, n));
    return k_rmsnorm(d, F(x), add_residual ? F(res) : nullptr, F(w), F(out), eps, width, rows, add_residual ? 1 : 0);
}

L0B_API l0b_status l0b_gemv_execute(l0b_suite* s, l0b_device* d, int32_t n, int32_t k, l0b_buffer* x, l0b_buffer* w,
                                    l0b_buffer* y) {
    return l0b_gemv_execute_rows(s, d, 1, n, k, x, w, y);
}

L0B_API l0b_status l0b_gemv_execute_rows(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                         l0b_buffer* w, l0b_buffer* y) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(m > 0 && n > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d N=%d K=%d", m, n, k);
    L0B_REQUIRE(n % 4 == 0, L0B_ERR_UNSUPPORTED, "Gemv needs N %% 4 == 0 (N=%d); use Gemm", n);
    L0B_REQUIRE(m <= kMaxRows, L0B_ERR_OUT_OF_RANGE, "ExecuteRows takes at most %d rows, got %d", kMaxRows, m);
    L0B_TRY(need(x, "x", L0B_F32, static_cast<long long>(m) * k));
    L0B_REQUIRE(w && (w->dtype == L0B_F32 || w->dtype == L0B_F16), L0B_ERR_ARGUMENT, "W must be f32 or f16");
    L0B_REQUIRE(w->count >= static_cast<long long>(n) * k, L0B_ERR_ARGUMENT, "W holds %lld elements, need %lld",
                (long long)w->count, static_cast<long long>(n) * k);
    L0B_TRY(need(y, "y", L0B_F32, static_cast<long long>(m) * n));
    return gemv_kn_launch(d, w->dtype, m, n, k, F(x), w->ptr, F(y));
}

L0B_API l0b_status l0b_gemm_execute(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* a,
                                    l0b_buffer* b, l0b_buffer* c) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(m > 0 && n > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d N=%d K=%d", m, n, k);
    L0B_TRY(need(a, "A", L0B_F32, static_cast<long long>(m) * k));
    L0B_TRY(need(b, "B", L0B_F32, static_cast<long long>(k) * n));
    L0B_TRY(need(c, "C", L0B_F32, static_cast<long long>(m) * n));
    return gemm_f32_launch(d, m, n, k, F(a), F(b), F(c));
}

L0B_API l0b_status l0b_gemv_q8_quantize(l0b_suite* s, l0b_device* d, int32_t rows, int32_t k, l0b_buffer* x) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(s->q8_x, L0B_ERR_INVALID_OPERATION,
                "Int8 weights need the int8 kernels and activation scratch (see LlmKernelSuite.EnsureQ8Scratch).");
    L0B_REQUIRE(rows > 0 && rows <= s->q8_rows, L0B_ERR_INVALID_OPERATION,
                "Activation scratch holds %d rows but %d were requested.", s->q8_rows, rows);
    L0B_REQUIRE(k > 0 && k <= s->q8_width, L0B_ERR_INVALID_OPERATION, "Activation scratch is %d wide, K is %d",
                s->q8_width, k);
    L0B_TRY(need(x, "x", L0B_F32, static_cast<long long>(rows) * k));
    s->q8_k = k;
    return k_copy(d, F(x), s->q8_x, 0, static_cast<long long>(rows) * k);
}

static l0b_status q8_exec(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* words,
                          l0b_buffer* scales, l0b_buffer* y) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(l0b_gemv_q8_supports(n, k), L0B_ERR_UNSUPPORTED, "GemvQ8 needs N %% 4 == 0 and K %% 32 == 0 (N=%d K=%d)",
                n, k);
    L0B_REQUIRE(s->q8_x && m <= s->q8_rows && k <= s->q8_width, L0B_ERR_INVALID_OPERATION,
                "the activation scratch does not hold %d rows of %d", m, k);
    L0B_REQUIRE(m <= kMaxRows, L0B_ERR_OUT_OF_RANGE, "ExecuteRows takes at most %d rows, got %d", kMaxRows, m);
    const long long nk = static_cast<long long>(n) * k;
    L0B_REQUIRE(words && (words->dtype == L0B_I8 || words->dtype == L0B_I32) &&
                    static_cast<long long>(words->bytes()) >= nk,
                L0B_ERR_ARGUMENT, "words must hold N*K int8 values");
    L0B_REQUIRE(scales && scales->dtype == L0B_F16, L0B_ERR_ARGUMENT, "scales must be an f16 buffer");
    int group;
    if (scales->count == n) group = k;
    else if (scales->count >= nk / 32) group = 32;
    else return fail(L0B_ERR_ARGUMENT, "scales hold %lld values: need N*K/32 (=%lld) or N (=%d)",
                     (long long)scales->count, nk / 32, n);
    L0B_TRY(need(y, "y", L0B_F32, static_cast<long long>(m) * n));
    GemvParams p = {};
    p.w = words->ptr;
    p.scales = scales->ptr;
    p.group = group;
    p.N = n;
    p.K = k;
    p.M = m;
    p.x = s->q8_x;
    p.x_dtype = L0B_F32;
    p.x_ld = k;
    p.epi = EPI_STORE;
    p.out_dtype = L0B_F32;
    p.nseg = 1;
    p.seg[0].out = y->ptr;
    p.seg[0].row_end = n;
    p.seg[0].ld = n;
    p.prefetch = 1;
    p.part = s->split_part;
    p.counters = s->split_counters;
    p.counter_count = kSuiteSplitTiles;
    return gemv_nk_launch(d, L0B_I8, p);
}

L0B_API l0b_status l0b_gemv_q8_execute(l0b_suite* s, l0b_device* d, int32_t n, int32_t k, l0b_buffer* words,
                                       l0b_buffer* scales, l0b_buffer* y) {
    return q8_exec(s, d, 1, n, k, words, scales, y);
}

L0B_API l0b_status l0b_gemv_q8_execute_rows(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k,
                                            l0b_buffer* words, l0b_buffer* scales, l0b_buffer* y) {
    return q8_exec(s, d, m, n, k, words, scales, y);
}

L0B_API l0b_status l0b_bias_add_execute(l0b_suite* s, l0b_device* d, l0b_buffer* x, l0b_buffer* b, int32_t width,
                                        int32_t rows) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(width > 0 && rows > 0, L0B_ERR_OUT_OF_RANGE, "width %d rows %d", width, rows);
    L0B_TRY(need(x, "x", L0B_F32, static_cast<long long>(width) * rows));
    L0B_TRY(need(b, "b", L0B_F32, width));
    return k_bias_add(d, F(x), F(b), width, rows);
}

static l0b_status rope_common(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* k, l0b_buffer* positions,
                              const float* table, int hd, int nh, int nkv, float attn_scale, int tokens, int rot) {
    L0B_REQUIRE(hd > 0 && hd % 2 == 0, L0B_ERR_OUT_OF_RANGE, "head_dim %d must be positive and even", hd);
    L0B_REQUIRE(rot > 0 && rot % 2 == 0 && rot <= hd, L0B_ERR_OUT_OF_RANGE, "rotary dim %d", rot);
    L0B_REQUIRE(nh > 0 && nkv > 0 && tokens > 0, L0B_ERR_OUT_OF_RANGE, "heads %d/%d tokens %d", nh, nkv, tokens);
    L0B_TRY(need(q, "q", L0B_F32, static_cast<long long>(tokens) * nh * hd));
    L0B_TRY(need(k, "k", L0B_F32, static_cast<long long>(tokens) * nkv * hd));
    L0B_TRY(need(positions, "positions", L0B_I32, tokens));
    return k_rope(d, F(q), F(k), static_cast<const int*>(positions->ptr), table, hd, nh, nkv, attn_scale, rot, tokens);
}

L0B_API l0b_status l0b_rope_execute(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* k, l0b_buffer* positions,
                                    int32_t head_dim, int32_t n_heads, int32_t n_kv_heads, float theta, int32_t tokens) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(head_dim > 0 && head_dim % 2 == 0, L0B_ERR_OUT_OF_RANGE, "head_dim %d", head_dim);
    L0B_REQUIRE(theta > 0.f, L0B_ERR_OUT_OF_RANGE, "theta must be positive");
    const float* table = nullptr;
    L0B_TRY(suite_rope_table(s, head_dim, static_cast<double>(theta), &table));
    return rope_common(s, d, q, k, positions, table, head_dim, n_heads, n_kv_heads, 1.0f, tokens, head_dim);
}

L0B_API l0b_status l0b_rope_execute_with_frequencies(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* k,
                                                     l0b_buffer* positions, l0b_buffer* inv_freq, int32_t head_dim,
                                                     int32_t n_heads, int32_t n_kv_heads, float attn_scale,
                                                     int32_t tokens, int32_t rotary_dim) {
    L0B_TRY(check_suite(s, d));
    L0B_TRY(need(inv_freq, "invFreq", L0B_F32, rotary_dim / 2));
    return rope_common(s, d, q, k, positions, F(inv_freq), head_dim, n_heads, n_kv_heads, attn_scale, tokens,
                       rotary_dim);
}

static l0b_status kv_store(l0b_suite* s, l0b_device* d, l0b_buffer* k, l0b_buffer* v, l0b_buffer* kc, l0b_buffer* vc,
                           int pos0, int kv_dim, int tokens) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(pos0 >= 0 && kv_dim > 0 && tokens > 0, L0B_ERR_OUT_OF_RANGE, "pos0 %d kvDim %d tokens %d", pos0,
                kv_dim, tokens);
    const long long n = static_cast<long long>(tokens) * kv_dim;
    L0B_TRY(need(k, "k", L0B_F32, n));
    L0B_TRY(need(v, "v", L0B_F32, n));
    const long long end = static_cast<long long>(pos0 + tokens) * kv_dim;
    L0B_TRY(need_float(kc, "Kc", end));
    L0B_TRY(need_float(vc, "Vc", end));
    L0B_REQUIRE(kc->dtype == vc->dtype, L0B_ERR_ARGUMENT, "K and V caches differ in dtype");
    return k_kv_store(d, F(k), F(v), kc->ptr, vc->ptr, kc->dtype, pos0, kv_dim, tokens);
}

L0B_API l0b_status l0b_kv_cache_store_execute(l0b_suite* s, l0b_device* d, l0b_buffer* k, l0b_buffer* v,
                                              l0b_buffer* kc, l0b_buffer* vc, int32_t pos0, int32_t kv_dim) {
    return kv_store(s, d, k, v, kc, vc, pos0, kv_dim, 1);
}

L0B_API l0b_status l0b_kv_cache_store_execute_rows(l0b_suite* s, l0b_device* d, l0b_buffer* k, l0b_buffer* v,
                                                   l0b_buffer* kc, l0b_buffer* vc, int32_t pos0, int32_t kv_dim,
                                                   int32_t tokens) {
    return kv_store(s, d, k, v, kc, vc, pos0, kv_dim, tokens);
}

static l0b_status attention_common(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* kc, l0b_buffer* vc,
                                   l0b_buffer* out, int hd, int nh, int nkv, int pos_base, int pos_step, int batch,
                                   int max_seq, bool prefill) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(hd > 0 && nh > 0 && nkv > 0 && nh % nkv == 0, L0B_ERR_ARGUMENT, "heads %d/%d head_dim %d", nh, nkv, hd);
    const int last = pos_base + (batch - 1) * pos_step;
    L0B_REQUIRE(pos_base >= 0 && last < max_seq, L0B_ERR_OUT_OF_RANGE, "positions up to %d exceed maxSeq %d", last,
                max_seq);
    const int kv_dim = nkv * hd;
    L0B_TRY(need(q, "q", L0B_F32, static_cast<long long>(batch) * nh * hd));
    L0B_TRY(need(out, "out", L0B_F32, static_cast<long long>(batch) * nh * hd));
    L0B_TRY(need_float(kc, "Kc", static_cast<long long>(max_seq) * kv_dim));
    L0B_TRY(need_float(vc, "Vc", static_cast<long long>(max_seq) * kv_dim));
    L0B_REQUIRE(kc->dtype == vc->dtype, L0B_ERR_ARGUMENT, "K and V caches differ in dtype");
    AttnParams p = {};
    p.q = F(q);
    p.q_bstride = static_cast<long long>(nh) * hd;
    p.kc = kc->ptr;
    p.vc = vc->ptr;
    p.cache_dtype = kc->dtype;
    p.cache_bstride = 0;
    p.kv_dim = kv_dim;
    p.pos_base = pos_base;
    p.pos_step = pos_step;
    p.out = F(out);
    p.out_bstride = static_cast<long long>(nh) * hd;
    p.nh = nh;
    p.nkv = nkv;
    p.hd = hd;
    p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
    if (prefill) {
        // One CTA per (query, KV head) over the whole causal prefix: no partials needed.
        p.chunk = ((last + 1) + 31) / 32 * 32;
        p.max_splits = 1;
        return attention_launch(d, p, batch);
    }
    // Decode: split-KV in thread-block clusters merged on chip (no scratch).
    const int seq = last + 1;
    const int groups = batch * nkv * ((nh / nkv + 7) / 8);
    p.chunk = 32;
    return attention_cluster_launch(d, p, batch, attention_cluster_splits(seq, groups, d->sm_count));
}

L0B_API l0b_status l0b_attention_execute(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* kc, l0b_buffer* vc,
                                         l0b_buffer* out, int32_t head_dim, int32_t n_heads, int32_t n_kv_heads,
                                         int32_t seq_len, int32_t max_seq) {
    L0B_REQUIRE(seq_len > 0, L0B_ERR_OUT_OF_RANGE, "seqLen %d must be positive", seq_len);
    return attention_common(s, d, q, kc, vc, out, head_dim, n_heads, n_kv_heads, seq_len - 1, 0, 1, max_seq, false);
}

L0B_API l0b_status l0b_attention_execute_prefill(l0b_suite* s, l0b_device* d, l0b_buffer* q, l0b_buffer* kc,
                                                 l0b_buffer* vc, l0b_buffer* out, int32_t head_dim, int32_t n_heads,
                                                 int32_t n_kv_heads, int32_t pos0, int32_t tokens, int32_t max_seq) {
    L0B_REQUIRE(tokens > 0, L0B_ERR_OUT_OF_RANGE, "tokens %d must be positive", tokens);
    return attention_common(s, d, q, kc, vc, out, head_dim, n_heads, n_kv_heads, pos0, 1, tokens, max_seq, true);
}

L0B_API l0b_status l0b_sigmoid_gate_execute(l0b_suite* s, l0b_device* d, l0b_buffer* x, l0b_buffer* gate, int32_t n) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(n >= 0, L0B_ERR_OUT_OF_RANGE, "n %d", n);
    L0B_TRY(need(x, "x", L0B_F32, n));
    L0B_TRY(need(gate, "gate", L0B_F32, n));
    return k_sigmoid_gate(d, F(x), F(gate), n);
}

L0B_API l0b_status l0b_swiglu_execute(l0b_suite* s, l0b_device* d, l0b_buffer* gate, l0b_buffer* up, int32_t n) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(n >= 0, L0B_ERR_OUT_OF_RANGE, "n %d", n);
    L0B_TRY(need(gate, "gate", L0B_F32, n));
    L0B_TRY(need(up, "up", L0B_F32, n));
    return k_swiglu(d, F(gate), F(up), n);
}

L0B_API l0b_status l0b_add_execute(l0b_suite* s, l0b_device* d, l0b_buffer* hidden, l0b_buffer* down, int32_t n) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(n >= 0, L0B_ERR_OUT_OF_RANGE, "n %d", n);
    L0B_TRY(need(hidden, "hidden", L0B_F32, n));
    L0B_TRY(need(down, "down", L0B_F32, n));
    return k_add(d, F(hidden), F(down), n);
}

L0B_API l0b_status l0b_copy_execute(l0b_suite* s, l0b_device* d, l0b_buffer* src, l0b_buffer* dst, int32_t offset,
                                    int32_t n) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(offset >= 0 && n >= 0, L0B_ERR_OUT_OF_RANGE, "offset %d n %d", offset, n);
    L0B_TRY(need(src, "src", L0B_F32, static_cast<long long>(offset) + n));
    L0B_TRY(need(dst, "dst", L0B_F32, n));
    return k_copy(d, F(src), F(dst), offset, n);
}

L0B_API l0b_status l0b_sampling_execute(l0b_suite* s, l0b_device* d, l0b_buffer* logits, l0b_buffer* sampled,
                                        float temperature, float random_val, int32_t vocab) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(vocab > 0, L0B_ERR_OUT_OF_RANGE, "vocab %d", vocab);
    L0B_REQUIRE(temperature >= 0.f, L0B_ERR_OUT_OF_RANGE, "temperature must be >= 0");
    L0B_TRY(need(logits, "logits", L0B_F32, vocab));
    L0B_TRY(need(sampled, "sampled", L0B_I32, 1));
    return k_sampling(d, F(logits), static_cast<int*>(sampled->ptr), temperature, random_val, vocab);
}

L0B_API l0b_status l0b_sample_execute(l0b_suite* s, l0b_device* d, l0b_buffer* logits, int32_t vocab,
                                      l0b_buffer* context, int32_t n_context, float temperature, float top_p,
                                      int32_t top_k, float repetition_penalty, double random_value,
                                      l0b_buffer* out_token) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(vocab > 0, L0B_ERR_ARGUMENT, "Logits array cannot be null or empty.");
    L0B_REQUIRE(random_value >= 0.0 && random_value < 1.0, L0B_ERR_OUT_OF_RANGE, "random value %g outside [0, 1)",
                random_value);
    L0B_TRY(need(logits, "logits", L0B_F32, vocab));
    L0B_TRY(need(out_token, "out_token", L0B_I32, 1));
    L0B_REQUIRE(n_context >= 0, L0B_ERR_OUT_OF_RANGE, "n_context %d", n_context);
    if (n_context > 0) L0B_TRY(need(context, "context", L0B_I32, n_context));
    L0B_TRY(sample_check(temperature, top_p, top_k, repetition_penalty, vocab));
    const size_t words = sample_seen_words(vocab), kwords = sample_keys_words(vocab);
    void* scratch = nullptr;
    L0B_TRY(d->ensure_scratch((kwords + words) * sizeof(uint32_t), &scratch, 0));
    uint32_t* keys = static_cast<uint32_t*>(scratch);
    // The max word starts at zero (the scratch may hold anything); the select kernel leaves it zero.
    L0B_TRY(k_fill_u32(d, keys + vocab, 0u, 1));
    uint32_t* seen = nullptr;
    if (n_context > 0 && repetition_penalty != 1.0f) {
        seen = keys + kwords;
        L0B_TRY(seen_build(d, static_cast<const int*>(context->ptr), n_context, vocab, seen));
    }
    return sample_step(d, F(logits), vocab, seen, temperature, top_p, top_k, repetition_penalty, keys, random_value,
                       0, nullptr, 0, static_cast<int*>(out_token->ptr), nullptr, nullptr);
}

L0B_API l0b_status l0b_linear(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                              l0b_buffer* w, l0b_buffer* scales, int32_t group, l0b_buffer* bias, l0b_buffer* y) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(m > 0 && n > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d N=%d K=%d", m, n, k);
    L0B_TRY(need_float(x, "x", static_cast<long long>(m) * k));
    L0B_TRY(need_float(y, "y", static_cast<long long>(m) * n));
    L0B_REQUIRE(w, L0B_ERR_ARGUMENT, "W is null");
    const long long nk = static_cast<long long>(n) * k;
    int wdt = w->dtype;
    if (wdt == L0B_I32) wdt = L0B_I8;
    L0B_REQUIRE(static_cast<long long>(w->bytes()) >= nk * static_cast<long long>(dtype_size((l0b_dtype)wdt)),
                L0B_ERR_ARGUMENT, "W is smaller than N*K");
    if (wdt == L0B_I8) {
        if (group <= 0) group = k;
        L0B_REQUIRE(k % group == 0, L0B_ERR_ARGUMENT, "group %d does not divide K %d", group, k);
        L0B_TRY(need(scales, "scales", L0B_F16, nk / group));
    }
    if (bias) L0B_TRY(need(bias, "bias", L0B_F32, n));
    GemvParams p = {};
    p.w = w->ptr;
    p.scales = scales ? scales->ptr : nullptr;
    p.group = group;
    p.N = n;
    p.K = k;
    p.M = m;
    p.x = x->ptr;
    p.x_dtype = x->dtype;
    p.x_ld = k;
    p.epi = EPI_STORE;
    p.out_dtype = y->dtype;
    p.nseg = 1;
    p.seg[0].out = y->ptr;
    p.seg[0].bias = bias ? F(bias) : nullptr;
    p.seg[0].row_end = n;
    p.seg[0].ld = n;
    p.prefetch = 1;
    p.part = s->split_part;
    p.counters = s->split_counters;
    p.counter_count = kSuiteSplitTiles;
    return gemv_nk_launch(d, wdt, p);
}

L0B_API l0b_status l0b_linear_shared(l0b_suite* s, l0b_device* d, int32_t m, int32_t k, l0b_buffer* x, l0b_buffer* w,
                                     l0b_buffer* scales, int32_t group, int32_t nseg, const int32_t* seg_rows,
                                     l0b_buffer* const* biases, l0b_buffer* const* outs) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(nseg >= 1 && nseg <= 4, L0B_ERR_ARGUMENT, "1..4 projections share x, got %d", nseg);
    L0B_REQUIRE(seg_rows && outs, L0B_ERR_ARGUMENT, "seg_rows and outs are required");
    L0B_REQUIRE(m > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d K=%d", m, k);
    L0B_TRY(need_float(x, "x", static_cast<long long>(m) * k));
    L0B_REQUIRE(w, L0B_ERR_ARGUMENT, "W is null");
    GemvParams p = {};
    long long n = 0;
    for (int i = 0; i < nseg; ++i) {
        L0B_REQUIRE(seg_rows[i] > 0, L0B_ERR_OUT_OF_RANGE, "projection %d has %d rows", i, seg_rows[i]);
        L0B_TRY(need_float(outs[i], "output", static_cast<long long>(m) * seg_rows[i]));
        L0B_REQUIRE(outs[i]->dtype == outs[0]->dtype, L0B_ERR_ARGUMENT, "the outputs must share one dtype");
        l0b_buffer* b = biases ? biases[i] : nullptr;
        if (b) L0B_TRY(need(b, "bias", L0B_F32, seg_rows[i]));
        n += seg_rows[i];
        L0B_REQUIRE(n <= INT32_MAX, L0B_ERR_OUT_OF_RANGE, "stacked rows exceed int32");
        p.seg[i].out = outs[i]->ptr;
        p.seg[i].bias = b ? F(b) : nullptr;
        p.seg[i].row_end = static_cast<int>(n);
        p.seg[i].ld = seg_rows[i];
    }
    const long long nk = n * k;
    int wdt = w->dtype == L0B_I32 ? L0B_I8 : w->dtype;
    L0B_REQUIRE(static_cast<long long>(w->bytes()) >= nk * static_cast<long long>(dtype_size((l0b_dtype)wdt)),
                L0B_ERR_ARGUMENT, "W is smaller than (sum of rows) * K");
    if (wdt == L0B_I8) {
        if (group <= 0) group = k;
        L0B_REQUIRE(k % group == 0, L0B_ERR_ARGUMENT, "group %d does not divide K %d", group, k);
        L0B_TRY(need(scales, "scales", L0B_F16, nk / group));
    }
    p.w = w->ptr;
    p.scales = scales ? scales->ptr : nullptr;
    p.group = group;
    p.N = static_cast<int>(n);
    p.K = k;
    p.M = m;
    p.x = x->ptr;
    p.x_dtype = x->dtype;
    p.x_ld = k;
    p.epi = EPI_STORE;
    p.out_dtype = outs[0]->dtype;
    p.nseg = nseg;
    p.prefetch = 1;
    p.part = s->split_part;
    p.counters = s->split_counters;
    p.counter_count = kSuiteSplitTiles;
    return gemv_nk_launch(d, wdt, p);
}

L0B_API l0b_status l0b_linear_fused(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                    l0b_buffer* w, l0b_buffer* scales, int32_t group, l0b_buffer* norm_w, float eps,
                                    int32_t epilogue, l0b_buffer* bias, l0b_buffer* out) {
    L0B_TRY(check_suite(s, d));
    L0B_REQUIRE(m > 0 && n > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d N=%d K=%d", m, n, k);
    const bool blocked = (epilogue & L0B_EPI_BLOCKED_WEIGHTS) != 0;
    epilogue &= ~L0B_EPI_BLOCKED_WEIGHTS;
    L0B_REQUIRE(epilogue >= L0B_EPI_STORE && epilogue <= L0B_EPI_SWIGLU, L0B_ERR_ARGUMENT, "epilogue %d", epilogue);
    L0B_REQUIRE(epilogue != L0B_EPI_SWIGLU || n % 2 == 0, L0B_ERR_ARGUMENT, "SwiGLU needs an even N");
    L0B_REQUIRE(epilogue != L0B_EPI_SWIGLU || !bias, L0B_ERR_ARGUMENT, "the SwiGLU epilogue takes no bias");
    const int out_cols = epilogue == L0B_EPI_SWIGLU ? n / 2 : n;
    L0B_TRY(need_float(x, "x", static_cast<long long>(m) * k));
    L0B_TRY(need(out, "out", L0B_F32, static_cast<long long>(m) * out_cols));
    L0B_REQUIRE(w, L0B_ERR_ARGUMENT, "W is null");
    const long long nk = static_cast<long long>(n) * k;
    int wdt = w->dtype == L0B_I32 ? L0B_I8 : w->dtype;
    L0B_REQUIRE(static_cast<long long>(w->bytes()) >= nk * static_cast<long long>(dtype_size((l0b_dtype)wdt)),
                L0B_ERR_ARGUMENT, "W is smaller than N*K");
    if (wdt == L0B_I8) {
        if (group <= 0) group = k;
        L0B_REQUIRE(k % group == 0, L0B_ERR_ARGUMENT, "group %d does not divide K %d", group, k);
        L0B_TRY(need(scales, "scales", L0B_F16, nk / group));
    }
    if (blocked) {
        L0B_REQUIRE(wdt == L0B_I8 && group >= k, L0B_ERR_ARGUMENT,
                    "blocked weights must be int8 with one scale per row");
        L0B_REQUIRE(n % 16 == 0 && k % kWeightBlock == 0, L0B_ERR_ARGUMENT,
                    "blocked weights need N %% 16 == 0 and K %% %d == 0 (N=%d K=%d)", kWeightBlock, n, k);
        L0B_REQUIRE(n <= kSuiteKsRows, L0B_ERR_OUT_OF_RANGE, "blocked weights with N=%d > %d rows", n, kSuiteKsRows);
        L0B_REQUIRE(epilogue != L0B_EPI_SWIGLU || (n / 2) % 16 == 0, L0B_ERR_ARGUMENT,
                    "blocked [gate; up] needs N/2 %% 16 == 0");
    }
    if (norm_w) L0B_TRY(need(norm_w, "norm_w", L0B_F32, k));
    if (bias) L0B_TRY(need(bias, "bias", L0B_F32, out_cols));
    GemvParams p = {};
    p.w = w->ptr;
    p.scales = scales ? scales->ptr : nullptr;
    p.group = group;
    p.N = n;
    p.K = k;
    p.M = m;
    p.x = x->ptr;
    p.x_dtype = x->dtype;
    p.x_ld = k;
    p.norm_w = norm_w ? F(norm_w) : nullptr;
    p.eps = eps;
    p.epi = epilogue == L0B_EPI_ACCUM ? EPI_ACCUM : epilogue == L0B_EPI_SWIGLU ? EPI_SWIGLU : EPI_STORE;
    p.out_dtype = L0B_F32;
    p.nseg = 1;
    p.seg[0].out = out->ptr;
    p.seg[0].bias = bias ? F(bias) : nullptr;
    p.seg[0].row_end = out_cols;
    p.seg[0].ld = out_cols;
    p.prefetch = 1;
    p.part = s->split_part;
    p.counters = s->split_counters;
    p.counter_count = kSuiteSplitTiles;
    if (blocked) {
        p.kb = kWeightBlock;
        p.acc = s->ks_acc;
        p.acc_count = kSuiteKsRows;
    }
    return gemv_nk_launch(d, wdt, p);
}

namespace {

l0b_status linear_tc(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x, l0b_buffer* w,
                     l0b_buffer* scales, int32_t group, l0b_buffer* norm_w, float eps, int32_t epilogue,
                     l0b_buffer* bias, l0b_buffer* out) {
    L0B_TRY(check_suite(s, d));
    const bool split = (epilogue & L0B_EPI_F32_ACTIVATIONS) != 0;
    epilogue &= ~L0B_EPI_F32_ACTIVATIONS;
    L0B_REQUIRE(m > 0 && n > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d N=%d K=%d", m, n, k);
    L0B_REQUIRE(w && (w->dtype == L0B_F16 || w->dtype == L0B_BF16 || w->dtype == L0B_I8), L0B_ERR_ARGUMENT,
                "W must be f16, bf16 or int8");
    L0B_REQUIRE(w->count >= static_cast<long long>(n) * k, L0B_ERR_ARGUMENT, "W is smaller than N*K");
    const bool q8 = w->dtype == L0B_I8;
    if (q8) {
        L0B_REQUIRE(group <= 0 || group >= k, L0B_ERR_UNSUPPORTED,
                    "the tensor-core GEMM takes int8 weights with one scale per row (group = K), not group %d", group);
        L0B_TRY(need(scales, "scales", L0B_F16, n));
    }
    const int epi = epilogue == L0B_EPI_ACCUM ? EPI_ACCUM : epilogue == L0B_EPI_SWIGLU ? EPI_SWIGLU : EPI_STORE;
    L0B_REQUIRE(tc_gemm_supported(w->dtype, m, n, k, epi), L0B_ERR_UNSUPPORTED,
                "the tensor-core GEMM needs K >= 64, K %% 8 == 0 (int8: %% 16) and for SwiGLU (N/2) %% 64 == 0");
    L0B_REQUIRE(epi != EPI_SWIGLU || !bias, L0B_ERR_ARGUMENT, "the SwiGLU epilogue takes no bias");
    const int out_cols = epi == EPI_SWIGLU ? n / 2 : n;
    L0B_TRY(need(x, "x", L0B_F32, static_cast<long long>(m) * k));
    L0B_TRY(need(out, "out", L0B_F32, static_cast<long long>(m) * out_cols));
    if (norm_w) L0B_TRY(need(norm_w, "norm_w", L0B_F32, k));
    if (bias) L0B_TRY(need(bias, "bias", L0B_F32, n));
    const int xdtype = w->dtype;  // int8 weights: the activations as int8 digits (always near-f32)
    const TcPlan plan = tc_gemm_plan(m, n, k, epi, split, w->dtype, d->sm_count);
    void* x16 = nullptr;
    float* rscale = nullptr;
    if (split || q8) {
        const size_t x_bytes = (static_cast<size_t>(tc_pair_rows(plan)) * k * (q8 ? 1 : 2) + 255) / 256 * 256;
        L0B_TRY(d->ensure_scratch(x_bytes + static_cast<size_t>(m) * sizeof(float), &x16, 1));
        rscale = reinterpret_cast<float*>(static_cast<char*>(x16) + x_bytes);
        L0B_TRY(cast_rows_split_launch(d, F(x), k, norm_w ? F(norm_w) : nullptr, eps, x16, rscale, xdtype, m, k,
                                       plan));
    } else {
        L0B_TRY(d->ensure_scratch(static_cast<size_t>(m) * k * 2, &x16, 1));
        L0B_TRY(cast_rows_launch(d, F(x), k, norm_w ? F(norm_w) : nullptr, eps, x16, xdtype, m, k));
    }
    TcGemmArgs a;
    if (plan.S > 1) {
        void* part = nullptr;
        L0B_TRY(d->ensure_scratch(plan.part_floats * sizeof(float), &part, 0));
        L0B_TRY(d->ensure_counters(kTcCounters, &a.counters));
        a.part = static_cast<float*>(part);
        a.part_floats = plan.part_floats;
        a.counter_count = kTcCounters;
    }
    a.split = split ? 1 : 0;
    a.rscale = rscale;
    a.wscale = q8 ? scales->ptr : nullptr;
    a.M = m;
    a.N = n;
    a.K = k;
    a.x16 = x16;
    a.w = w->ptr;
    a.wdtype = w->dtype;
    a.epi = epi;
    a.out = F(out);
    a.ld = out_cols;
    a.bias = bias ? F(bias) : nullptr;
    return tc_gemm_launch(d, a);
}

}  // namespace

L0B_API l0b_status l0b_linear_tc(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                 l0b_buffer* w, l0b_buffer* norm_w, float eps, int32_t epilogue, l0b_buffer* bias,
                                 l0b_buffer* out) {
    L0B_REQUIRE(!w || w->dtype != L0B_I8, L0B_ERR_ARGUMENT, "int8 weights go through l0b_linear_tc_scaled");
    return linear_tc(s, d, m, n, k, x, w, nullptr, 0, norm_w, eps, epilogue, bias, out);
}

L0B_API l0b_status l0b_linear_tc_scaled(l0b_suite* s, l0b_device* d, int32_t m, int32_t n, int32_t k, l0b_buffer* x,
                                        l0b_buffer* w, l0b_buffer* scales, int32_t group, l0b_buffer* norm_w,
                                        float eps, int32_t epilogue, l0b_buffer* bias, l0b_buffer* out) {
    return linear_tc(s, d, m, n, k, x, w, scales, group, norm_w, eps, epilogue, bias, out);
}

L0B_API l0b_status l0b_tc_set_max_splits(int32_t splits) {
    tc_gemm_set_max_splits(splits);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_bulk(int32_t enable) {
    gemv_set_bulk(enable != 0);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_ksplit(int32_t enable) {
    gemv_set_ksplit(enable != 0);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_bulk_stages(int32_t stages) {
    gemv_set_bulk_stages(stages);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_l2_prefetch(int32_t gate_up_mb) {
    gemv_set_l2_prefetch_mb(gate_up_mb);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_ksplit_stages(int32_t stages) {
    gemv_set_ksplit_stages(stages);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_bulk_short_rows(int32_t enable) {
    gemv_set_bulk_short_rows(enable != 0);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_fill_split(int32_t max_splits) {
    gemv_set_fill_split(max_splits);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_weight_blocking(int32_t enable) {
    set_weight_blocking(enable != 0);
    return L0B_OK;
}

L0B_API l0b_status l0b_set_gemv_tensor_cores(int32_t enable) {
    gemv_set_tensor_cores(enable != 0);
    return L0B_OK;
}

L0B_API l0b_status l0b_gemv_w8a16_raw(void* stream, int32_t m, int32_t n, int32_t k, const void* x, int32_t x_dtype,
                                      const int8_t* q, const uint16_t* scales, int32_t group, void* y,
                                      int32_t y_dtype) {
    L0B_REQUIRE(x && q && scales && y, L0B_ERR_ARGUMENT, "null pointer");
    L0B_REQUIRE(m > 0 && n > 0 && k > 0, L0B_ERR_OUT_OF_RANGE, "shape M=%d N=%d K=%d", m, n, k);
    if (group <= 0) group = k;
    L0B_REQUIRE(k % group == 0, L0B_ERR_ARGUMENT, "group %d does not divide K %d", group, k);
    L0B_REQUIRE(x_dtype == L0B_F32 || x_dtype == L0B_F16 || x_dtype == L0B_BF16, L0B_ERR_ARGUMENT, "x dtype");
    L0B_REQUIRE(y_dtype == L0B_F32 || y_dtype == L0B_F16 || y_dtype == L0B_BF16, L0B_ERR_ARGUMENT, "y dtype");
    static int sm_count = 0;
    if (!sm_count) {
        int dev = 0;
        L0B_CHECK_CUDA(cudaGetDevice(&dev));
        L0B_CHECK_CUDA(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev));
    }
    GemvParams p = {};
    p.w = q;
    p.scales = scales;
    p.group = group;
    p.N = n;
    p.K = k;
    p.M = m;
    p.x = x;
    p.x_dtype = x_dtype;
    p.x_ld = k;
    p.epi = EPI_STORE;
    p.out_dtype = y_dtype;
    p.nseg = 1;
    p.seg[0].out = y;
    p.seg[0].row_end = n;
    p.seg[0].ld = n;
    p.prefetch = 1;
    return gemv_nk_launch_stream(static_cast<cudaStream_t>(stream), sm_count, L0B_I8, p);
}

}  // extern "C"
