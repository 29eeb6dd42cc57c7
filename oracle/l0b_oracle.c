/*
 * l0b_oracle.c -- CPU restatement of the l0llm decoder hot path. TEST INFRASTRUCTURE ONLY: the
 * checker for the CUDA backend (see l0b_oracle.h for what pins it). Build with -ffp-contract=off so
 * float steps round exactly as written. Parallel loops use OpenMP over independent output rows.
 */
#include "l0b_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------------ */
/* Number formats                                                                                    */
/* ------------------------------------------------------------------------------------------------ */

static uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static float u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary16, round to nearest even (subnormals and overflow to inf handled). */
uint16_t orc_f32_to_f16(float v) {
    uint32_t x = f2u(v);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mag = x & 0x7FFFFFFFu;
    if (mag >= 0x7F800000u) return (uint16_t)(sign | (mag > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (mag >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
    if (mag < 0x38800000u) {                                   /* below 2^-14: subnormal half */
        if (mag < 0x33000000u) return (uint16_t)sign;          /* < 2^-25: rounds to 0 */
        uint32_t e = mag >> 23;
        uint32_t m = (mag & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14 - (e - 127) + 13 - 1 ... yields the half subnormal */
        uint32_t r = m >> (shift);
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) r += 1;
        return (uint16_t)(sign | r);
    }
    uint32_t e = (mag >> 23) - 127 + 15;
    uint32_t m = mag & 0x7FFFFFu;
    uint32_t r = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1;
    return (uint16_t)(sign | r);
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return u2f(sign);
        float f = (float)m * (1.0f / 16777216.0f); /* m * 2^-24 */
        return sign ? -f : f;
    }
    if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
    return u2f(sign | ((e - 15 + 127) << 23) | (m << 13));
}

uint16_t orc_f32_to_bf16(float v) {
    uint32_t x = f2u(v);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float orc_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

static float load_elem(const void* p, int dtype, int64_t i) {
    switch (dtype) {
        case ORC_F16: return orc_f16_to_f32(((const uint16_t*)p)[i]);
        case ORC_BF16: return orc_bf16_to_f32(((const uint16_t*)p)[i]);
        case ORC_I8: return (float)((const int8_t*)p)[i];
        default: return ((const float*)p)[i];
    }
}

static void store_elem(void* p, int dtype, int64_t i, float v) {
    switch (dtype) {
        case ORC_F16: ((uint16_t*)p)[i] = orc_f32_to_f16(v); break;
        case ORC_BF16: ((uint16_t*)p)[i] = orc_f32_to_bf16(v); break;
        case ORC_I8: ((int8_t*)p)[i] = (int8_t)v; break;
        default: ((float*)p)[i] = v; break;
    }
}

static size_t dtype_bytes(int dtype) { return dtype == ORC_F32 ? 4 : dtype == ORC_I8 ? 1 : 2; }

void orc_convert(const float* src, void* dst, int dtype, int64_t n) {
    for (int64_t i = 0; i < n; ++i) store_elem(dst, dtype, i, src[i]);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------------------------------ */
/* Linear layers                                                                                      */
/* ------------------------------------------------------------------------------------------------ */

void orc_gemv_out_in(int M, int N, int K, const float* x, int wdtype, const void* w, const uint16_t* scales, int group,
                     float* y) {
    if (wdtype == ORC_I8 && group <= 0) group = K;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int m = 0; m < M; ++m) {
            const float* xr = x + (int64_t)m * K;
            double acc = 0.0;
            if (wdtype == ORC_I8) {
                const int8_t* row = (const int8_t*)w + (int64_t)n * K;
                const int gpr = K / group;
                for (int g = 0; g < gpr; ++g) {
                    const float s = orc_f16_to_f32(scales[(int64_t)n * gpr + g]);
                    double part = 0.0;
                    for (int i = g * group; i < (g + 1) * group; ++i) part += (double)row[i] * (double)xr[i];
                    acc += part * (double)s;
                }
            } else if (wdtype == ORC_F16) {
                const uint16_t* row = (const uint16_t*)w + (int64_t)n * K;
                for (int i = 0; i < K; ++i) acc += (double)orc_f16_to_f32(row[i]) * (double)xr[i];
            } else if (wdtype == ORC_BF16) {
                const uint16_t* row = (const uint16_t*)w + (int64_t)n * K;
                for (int i = 0; i < K; ++i) acc += (double)orc_bf16_to_f32(row[i]) * (double)xr[i];
            } else {
                const float* row = (const float*)w + (int64_t)n * K;
                for (int i = 0; i < K; ++i) acc += (double)row[i] * (double)xr[i];
            }
            y[(int64_t)m * N + n] = (float)acc;
        }
    }
}

void orc_gemv_in_out(int M, int N, int K, const float* x, int w_is_half, const void* w, float* y) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                const float wv = w_is_half ? orc_f16_to_f32(((const uint16_t*)w)[(int64_t)k * N + n])
                                           : ((const float*)w)[(int64_t)k * N + n];
                acc += (double)x[(int64_t)m * K + k] * (double)wv;
            }
            y[(int64_t)m * N + n] = (float)acc;
        }
}

/* Timing build of orc_gemv_out_in: the same products accumulated in fp32 with fused multiply-adds in
 * eight AVX2 lanes per (row, token) pair (each lane sums K/8 products; the lanes meet in double), two
 * weight rows x up to six activation rows per register block, activation rows in blocks of 24 so a
 * block stays in the core's L2 while the weights stream. Relative error ~sqrt(K/8) * 2^-24 per output
 * (about 1e-6 at K = 18944), far below the 1e-2 parity tolerance. */
#define ORC_RB 2
#define ORC_TB 6
#define ORC_TBIG 24

static inline __attribute__((always_inline)) __m256 ld8w(const void* w, int dt, int64_t i) {
    if (dt == ORC_I8) return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)((const int8_t*)w + i))));
    if (dt == ORC_F16) return _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)((const uint16_t*)w + i)));
    if (dt == ORC_BF16)
        return _mm256_castsi256_ps(
            _mm256_slli_epi32(_mm256_cvtepu16_epi32(_mm_loadu_si128((const __m128i*)((const uint16_t*)w + i))), 16));
    return _mm256_loadu_ps((const float*)w + i);
}

static inline double hsum8(__m256 v) {
    const __m256d a = _mm256_add_pd(_mm256_cvtps_pd(_mm256_castps256_ps128(v)), _mm256_cvtps_pd(_mm256_extractf128_ps(v, 1)));
    const __m128d s = _mm_add_pd(_mm256_castpd256_pd128(a), _mm256_extractf128_pd(a, 1));
    return _mm_cvtsd_f64(_mm_add_sd(s, _mm_unpackhi_pd(s, s)));
}

/* Rows n0 and n1 (n1 may repeat n0 when N is odd; its result is then not stored) x tokens [t0, t0 + tb). */
static inline __attribute__((always_inline)) void fast_block(int dt, int K, int group, const void* w,
                                                             const uint16_t* sc, int n0, int n1, int store1,
                                                             const float* x, int t0, int tb, int N, float* y) {
    __m256 acc[ORC_RB][ORC_TB];
    double tail[ORC_RB][ORC_TB];
    for (int r = 0; r < ORC_RB; ++r)
        for (int t = 0; t < tb; ++t) {
            acc[r][t] = _mm256_setzero_ps();
            tail[r][t] = 0.0;
        }
    const int64_t w0 = (int64_t)n0 * K, w1 = (int64_t)n1 * K;
    const int grouped = dt == ORC_I8 && group < K;
    const int kv = K & ~7;
    if (!grouped) {
        for (int k = 0; k < kv; k += 8) {
            const __m256 a0 = ld8w(w, dt, w0 + k), a1 = ld8w(w, dt, w1 + k);
            for (int t = 0; t < tb; ++t) {
                const __m256 xv = _mm256_loadu_ps(x + (int64_t)(t0 + t) * K + k);
                acc[0][t] = _mm256_fmadd_ps(a0, xv, acc[0][t]);
                acc[1][t] = _mm256_fmadd_ps(a1, xv, acc[1][t]);
            }
        }
        for (int k = kv; k < K; ++k)
            for (int t = 0; t < tb; ++t) {
                const double xv = x[(int64_t)(t0 + t) * K + k];
                tail[0][t] += (double)load_elem(w, dt, w0 + k) * xv;
                tail[1][t] += (double)load_elem(w, dt, w1 + k) * xv;
            }
        const double s0 = dt == ORC_I8 ? (double)orc_f16_to_f32(sc[n0]) : 1.0;
        const double s1 = dt == ORC_I8 ? (double)orc_f16_to_f32(sc[n1]) : 1.0;
        for (int t = 0; t < tb; ++t) {
            y[(int64_t)(t0 + t) * N + n0] = (float)((hsum8(acc[0][t]) + tail[0][t]) * s0);
            if (store1) y[(int64_t)(t0 + t) * N + n1] = (float)((hsum8(acc[1][t]) + tail[1][t]) * s1);
        }
        return;
    }
    /* int8 with group-wise scales (group a multiple of 8): each group's partial sum times its scale. */
    const int gpr = K / group;
    for (int g = 0; g < gpr; ++g) {
        __m256 part[ORC_RB][ORC_TB];
        for (int r = 0; r < ORC_RB; ++r)
            for (int t = 0; t < tb; ++t) part[r][t] = _mm256_setzero_ps();
        for (int k = g * group; k < (g + 1) * group; k += 8) {
            const __m256 a0 = ld8w(w, dt, w0 + k), a1 = ld8w(w, dt, w1 + k);
            for (int t = 0; t < tb; ++t) {
                const __m256 xv = _mm256_loadu_ps(x + (int64_t)(t0 + t) * K + k);
                part[0][t] = _mm256_fmadd_ps(a0, xv, part[0][t]);
                part[1][t] = _mm256_fmadd_ps(a1, xv, part[1][t]);
            }
        }
        const __m256 s0 = _mm256_set1_ps(orc_f16_to_f32(sc[(int64_t)n0 * gpr + g]));
        const __m256 s1 = _mm256_set1_ps(orc_f16_to_f32(sc[(int64_t)n1 * gpr + g]));
        for (int t = 0; t < tb; ++t) {
            acc[0][t] = _mm256_fmadd_ps(part[0][t], s0, acc[0][t]);
            acc[1][t] = _mm256_fmadd_ps(part[1][t], s1, acc[1][t]);
        }
    }
    for (int t = 0; t < tb; ++t) {
        y[(int64_t)(t0 + t) * N + n0] = (float)hsum8(acc[0][t]);
        if (store1) y[(int64_t)(t0 + t) * N + n1] = (float)hsum8(acc[1][t]);
    }
}

static void fast_rows(int dt, int M, int N, int K, const float* x, const void* w, const uint16_t* sc, int group,
                      float* y) {
    for (int m0 = 0; m0 < M; m0 += ORC_TBIG) {
        const int mb = M - m0 < ORC_TBIG ? M - m0 : ORC_TBIG;
#pragma omp parallel for schedule(static)
        for (int np = 0; np < (N + 1) / 2; ++np) {
            const int n0 = 2 * np, has1 = n0 + 1 < N, n1 = has1 ? n0 + 1 : n0;
            int t = m0;
            for (; t + ORC_TB <= m0 + mb; t += ORC_TB) fast_block(dt, K, group, w, sc, n0, n1, has1, x, t, ORC_TB, N, y);
            for (; t < m0 + mb; ++t) fast_block(dt, K, group, w, sc, n0, n1, has1, x, t, 1, N, y);
        }
    }
}

void orc_gemm_fast(int M, int N, int K, const float* x, int wdtype, const void* w, const uint16_t* scales, int group,
                   float* y) {
    if (wdtype == ORC_I8 && group <= 0) group = K;
    if (wdtype == ORC_I8 && group < K && group % 8 != 0) {
        orc_gemv_out_in(M, N, K, x, wdtype, w, scales, group, y);
        return;
    }
    switch (wdtype) {
        case ORC_I8: fast_rows(ORC_I8, M, N, K, x, w, scales, group, y); break;
        case ORC_F16: fast_rows(ORC_F16, M, N, K, x, w, scales, group, y); break;
        case ORC_BF16: fast_rows(ORC_BF16, M, N, K, x, w, scales, group, y); break;
        default: fast_rows(ORC_F32, M, N, K, x, w, scales, group, y); break;
    }
}

void orc_q8_quantize(const float* w, int N, int K, int group, int8_t* q, uint16_t* scales) {
    if (group <= 0) group = K;
    const int gpr = K / group;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int g = 0; g < gpr; ++g) {
            const float* src = w + (int64_t)n * K + (int64_t)g * group;
            float mx = 0.f;
            for (int i = 0; i < group; ++i) mx = fmaxf(mx, fabsf(src[i]));
            const uint16_t sh = orc_f32_to_f16(mx / 127.0f);
            const float sf = orc_f16_to_f32(sh);
            for (int i = 0; i < group; ++i) {
                float r = 0.f;
                if (sf > 0.f) r = fminf(127.f, fmaxf(-127.f, nearbyintf(src[i] / sf)));
                q[(int64_t)n * K + (int64_t)g * group + i] = (int8_t)r;
            }
            scales[(int64_t)n * gpr + g] = sh;
        }
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Elementwise                                                                                        */
/* ------------------------------------------------------------------------------------------------ */

void orc_rmsnorm(float* x, const float* res, const float* w, float* out, float eps, int width, int rows, int add_res) {
    for (int r = 0; r < rows; ++r) {
        float* xr = x + (int64_t)r * width;
        double ss = 0.0;
        for (int i = 0; i < width; ++i) {
            float v = xr[i];
            if (add_res) {
                v = v + res[(int64_t)r * width + i];
                xr[i] = v;
            }
            ss += (double)v * (double)v;
        }
        const float rstd = (float)(1.0 / sqrt(ss / width + (double)eps));
        for (int i = 0; i < width; ++i) out[(int64_t)r * width + i] = (xr[i] * rstd) * w[i];
    }
}

void orc_bias_add(float* x, const float* b, int width, int rows) {
    for (int r = 0; r < rows; ++r)
        for (int i = 0; i < width; ++i) x[(int64_t)r * width + i] += b[i];
}

static float silu_f(float x) { return (float)((double)x / (1.0 + exp(-(double)x))); }

void orc_swiglu(float* gate, const float* up, int64_t n) {
    for (int64_t i = 0; i < n; ++i) gate[i] = silu_f(gate[i]) * up[i];
}

void orc_add(float* a, const float* b, int64_t n) {
    for (int64_t i = 0; i < n; ++i) a[i] += b[i];
}

void orc_sigmoid_gate(float* x, const float* g, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = x[i] * (float)(1.0 / (1.0 + exp(-(double)g[i])));
}

void orc_embedding(const int* ids, const void* table, int table_dtype, float* out, int h, int64_t count) {
    for (int64_t e = 0; e < count; ++e) {
        const int64_t t = e / h;
        out[e] = load_elem(table, table_dtype, (int64_t)ids[t] * h + (e - t * h));
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Rotary embeddings                                                                                  */
/* ------------------------------------------------------------------------------------------------ */

static double mscale_of(double scale, double m) { return scale <= 1.0 ? 1.0 : 0.1 * m * log(scale) + 1.0; }

int orc_rope_frequencies(int dim, double theta, int max_pos, int type, double factor, int original_max,
                         double low_freq, double high_freq, double beta_fast, double beta_slow, double attention_factor,
                         double mscale, double mscale_all_dim, int truncate, float* out, float* attention_out) {
    if (dim <= 0 || dim % 2) return -1;
    const int half = dim / 2;
    double attention = 1.0;
    const double original = original_max > 0 ? (double)original_max : (double)max_pos;
    double low = 0, high = 0;
    if (type == ORC_ROPE_YARN) {
        if (attention_factor > 0) attention = attention_factor;
        else if (mscale > 0 && mscale_all_dim > 0) attention = mscale_of(factor, mscale) / mscale_of(factor, mscale_all_dim);
        else attention = mscale_of(factor, 1.0);
        low = dim * log(original / (beta_fast * 2 * M_PI)) / (2 * log(theta));
        high = dim * log(original / (beta_slow * 2 * M_PI)) / (2 * log(theta));
        if (truncate) {
            low = floor(low);
            high = ceil(high);
        }
        if (low < 0) low = 0;
        if (high > dim - 1) high = dim - 1;
        if (low == high) high += 0.001;
    }
    for (int i = 0; i < half; ++i) {
        const double base = 1.0 / pow(theta, 2.0 * i / dim);
        double r = base;
        if (type == ORC_ROPE_LINEAR) {
            r = base / factor;
        } else if (type == ORC_ROPE_YARN) {
            double ramp = (i - low) / (high - low);
            ramp = ramp < 0 ? 0 : ramp > 1 ? 1 : ramp;
            const double extra = 1.0 - ramp;
            r = (base / factor) * (1.0 - extra) + base * extra;
        } else if (type == ORC_ROPE_LLAMA3) {
            const double wl = 2 * M_PI / base;
            const double low_wl = original / low_freq, high_wl = original / high_freq;
            if (wl < high_wl) r = base;
            else if (wl > low_wl) r = base / factor;
            else {
                const double smooth = (original / wl - low_freq) / (high_freq - low_freq);
                r = (1 - smooth) * base / factor + smooth * base;
            }
        }
        out[i] = (float)r;
    }
    if (attention_out) *attention_out = (float)attention;
    return half;
}

void orc_rope(float* q, float* k, const int* positions, const float* inv_freq, int hd, int nh, int nkv, float attn_scale,
              int rot, int tokens) {
    const int half = rot / 2;
    for (int t = 0; t < tokens; ++t) {
        for (int head = 0; head < nh + nkv; ++head) {
            float* v = head < nh ? q + ((int64_t)t * nh + head) * hd : k + ((int64_t)t * nkv + head - nh) * hd;
            for (int j = 0; j < half; ++j) {
                const float ang = (float)positions[t] * inv_freq[j];
                float c = (float)cos((double)ang), s = (float)sin((double)ang);
                c = c * attn_scale;
                s = s * attn_scale;
                const float x1 = v[j], x2 = v[j + half];
                v[j] = x1 * c - x2 * s;
                v[j + half] = x2 * c + x1 * s;
            }
        }
    }
}

void orc_kv_store(const float* k, const float* v, void* kc, void* vc, int cache_dtype, int pos0, int kv_dim, int tokens) {
    for (int64_t i = 0; i < (int64_t)tokens * kv_dim; ++i) {
        store_elem(kc, cache_dtype, (int64_t)pos0 * kv_dim + i, k[i]);
        store_elem(vc, cache_dtype, (int64_t)pos0 * kv_dim + i, v[i]);
    }
}

void orc_attention(const float* q, const void* kc, const void* vc, int cache_dtype, float* out, int hd, int nh, int nkv,
                   int pos0, int tokens) {
    const int group = nh / nkv, kv_dim = nkv * hd;
    const double scale = (double)(float)(1.0 / sqrt((double)hd));
#pragma omp parallel for schedule(static) collapse(2)
    for (int t = 0; t < tokens; ++t) {
        for (int h = 0; h < nh; ++h) {
            const int seq = pos0 + t + 1;
            const int kvh = h / group;
            const float* qh = q + ((int64_t)t * nh + h) * hd;
            double* sc = (double*)malloc(sizeof(double) * (size_t)seq);
            double mx = -INFINITY;
            for (int p = 0; p < seq; ++p) {
                double a = 0.0;
                for (int d = 0; d < hd; ++d)
                    a += (double)qh[d] * (double)load_elem(kc, cache_dtype, (int64_t)p * kv_dim + (int64_t)kvh * hd + d);
                sc[p] = a * scale;
                if (sc[p] > mx) mx = sc[p];
            }
            double sum = 0.0;
            for (int p = 0; p < seq; ++p) {
                sc[p] = exp(sc[p] - mx);
                sum += sc[p];
            }
            for (int d = 0; d < hd; ++d) {
                double o = 0.0;
                for (int p = 0; p < seq; ++p)
                    o += sc[p] * (double)load_elem(vc, cache_dtype, (int64_t)p * kv_dim + (int64_t)kvh * hd + d);
                out[((int64_t)t * nh + h) * hd + d] = (float)(o / sum);
            }
            free(sc);
        }
    }
}

int orc_argmax(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

int orc_sample(const float* logits, int vocab, float temperature, float random_val) {
    const int arg = orc_argmax(logits, vocab);
    if (temperature <= 0.f) return arg;
    const double mx = logits[arg];
    double total = 0.0;
    for (int i = 0; i < vocab; ++i) total += exp(((double)logits[i] - mx) / temperature);
    const double target = (double)random_val * total;
    double run = 0.0;
    for (int i = 0; i < vocab; ++i) {
        run += exp(((double)logits[i] - mx) / temperature);
        if (run >= target) return i;
    }
    return vocab - 1;
}

typedef struct {
    double p;
    int idx;
} orc_prob;

/* Descending probability, then ascending index. */
static int orc_prob_cmp(const void* a, const void* b) {
    const orc_prob* x = (const orc_prob*)a;
    const orc_prob* y = (const orc_prob*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

int orc_sampler(const float* logits, int vocab, const int* ctx, int n_ctx, float temperature, float top_p, int top_k,
                float repetition_penalty, double u) {
    if (!logits || vocab <= 0) return -1;
    float* c = (float*)malloc(sizeof(float) * (size_t)vocab);
    memcpy(c, logits, sizeof(float) * (size_t)vocab);
    /* 1. Repetition penalty, once per distinct context id (LlmAbstractions.cs:60-78). */
    if (repetition_penalty != 1.0f && ctx && n_ctx > 0) {
        unsigned char* done = (unsigned char*)calloc((size_t)vocab, 1);
        for (int i = 0; i < n_ctx; ++i) {
            const int t = ctx[i];
            if (t < 0 || t >= vocab || done[t]) continue;
            done[t] = 1;
            const float l = c[t];
            c[t] = l >= 0.0f ? l / repetition_penalty : l * repetition_penalty;
        }
        free(done);
    }
    /* 2. Greedy when T <= 0 (:81-94). */
    if (temperature <= 0.0f) {
        int best = 0;
        for (int i = 1; i < vocab; ++i)
            if (c[i] > c[best]) best = i;
        free(c);
        return best;
    }
    /* 3-4. Temperature, softmax in double (:97-113). */
    for (int i = 0; i < vocab; ++i) c[i] /= temperature;
    float mx = c[0];
    for (int i = 1; i < vocab; ++i)
        if (c[i] > mx) mx = c[i];
    orc_prob* pr = (orc_prob*)malloc(sizeof(orc_prob) * (size_t)vocab);
    double sum = 0.0;
    for (int i = 0; i < vocab; ++i) {
        const float d = c[i] - mx;
        pr[i].p = exp((double)d);
        pr[i].idx = i;
        sum += pr[i].p;
    }
    for (int i = 0; i < vocab; ++i) pr[i].p /= sum;
    /* 5. Sort, top-k, top-p (:116-146). */
    qsort(pr, (size_t)vocab, sizeof(orc_prob), orc_prob_cmp);
    int count = vocab;
    if (top_k > 0 && top_k < count) count = top_k;
    if (top_p > 0.0f && top_p < 1.0f) {
        double cum = 0.0;
        int keep = 0;
        for (int i = 0; i < count; ++i) {
            cum += pr[i].p;
            ++keep;
            if (cum >= (double)top_p) break;
        }
        if (keep < count) count = keep;
    }
    /* 6. Inverse CDF over the kept mass (:148-164). */
    double kept = 0.0;
    for (int i = 0; i < count; ++i) kept += pr[i].p;
    int chosen = pr[count - 1].idx;
    if (kept <= 0.0) {
        chosen = pr[0].idx;
    } else {
        const double r = u * kept;
        double cur = 0.0;
        for (int i = 0; i < count; ++i) {
            cur += pr[i].p;
            if (r <= cur) {
                chosen = pr[i].idx;
                break;
            }
        }
    }
    free(pr);
    free(c);
    return chosen;
}

/* ------------------------------------------------------------------------------------------------ */
/* Synthetic tensors (restates synth_kernel of the CUDA model)                                        */
/* ------------------------------------------------------------------------------------------------ */

static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ULL;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ULL;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBULL;
    return x ^ (x >> 31);
}

uint64_t orc_tensor_stream(uint64_t seed, uint64_t id) { return splitmix64(seed ^ (id * 0x9E3779B97F4A7C15ULL)); }

double orc_sample_uniform(uint64_t seed, int p) {
    const uint64_t h = splitmix64(seed ^ ((uint64_t)(p + 1) * 0x9E3779B97F4A7C15ULL));
    return (double)(h >> 11) * (1.0 / 9007199254740992.0);
}

void orc_synth_fill(void* dst, int dtype, int64_t count, uint64_t stream, int mode, float a, float b, int64_t row_len,
                    int64_t full_len, int64_t row0, int64_t col0) {
    if (row_len <= 0) row_len = count;
    if (full_len <= 0) full_len = row_len;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < count; ++i) {
        const int64_t r = i / row_len;
        const int64_t idx = (row0 + r) * full_len + col0 + (i - r * row_len);
        const uint64_t bits = splitmix64(stream + (uint64_t)idx * 0xD1B54A32D192ED03ULL);
        if (mode == ORC_SYN_I8) {
            ((int8_t*)dst)[i] = (int8_t)((int)(bits % 255ULL) - 127);
            continue;
        }
        float v;
        if (mode == ORC_SYN_NORMAL) {
            const uint32_t s = (uint32_t)(bits & 0xFFFF) + (uint32_t)((bits >> 16) & 0xFFFF) +
                               (uint32_t)((bits >> 32) & 0xFFFF) + (uint32_t)(bits >> 48);
            const float u = (float)s * (1.0f / 65536.0f);
            const float z = (u - 2.0f) * 1.7320508f;
            v = z * a;
        } else if (mode == ORC_SYN_UNIFORM) {
            const float u = (float)(bits >> 40) * (1.0f / 16777216.0f);
            const float span = b - a;
            v = a + u * span;
        } else {
            v = a;
        }
        store_elem(dst, dtype, i, v);
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Gated DeltaNet                                                                                     */
/* ------------------------------------------------------------------------------------------------ */

void orc_causal_conv(const float* x, float* state, const float* w, float* out, int conv_dim, int kernel, int tokens) {
    const int hist = kernel - 1;
    for (int c = 0; c < conv_dim; ++c) {
        float* st = state + (int64_t)c * hist;
        const float* wc = w + (int64_t)c * kernel;
        float* win = (float*)malloc(sizeof(float) * (size_t)(hist + tokens));
        for (int j = 0; j < hist; ++j) win[j] = st[j];
        for (int t = 0; t < tokens; ++t) win[hist + t] = x[(int64_t)t * conv_dim + c];
        for (int t = 0; t < tokens; ++t) {
            double acc = 0.0;
            for (int j = 0; j < kernel; ++j) acc += (double)wc[j] * (double)win[t + j];
            out[(int64_t)t * conv_dim + c] = silu_f((float)acc);
        }
        for (int j = 0; j < hist; ++j) st[j] = win[tokens + j];
        free(win);
    }
}

void orc_gated_delta(const float* conv, const float* z, const float* b, const float* a, const float* a_log,
                     const float* dt_bias, const float* norm_w, float* state, float* out, int hk, int hv, int dk, int dv,
                     int tokens, float eps) {
    const int conv_dim = 2 * hk * dk + hv * dv;
    const int rep = hv / hk;
    const double qscale = 1.0 / sqrt((double)dk);
    /* Value heads are independent (each owns its state and output columns): one per OpenMP iteration,
     * its tokens in order. */
#pragma omp parallel for schedule(dynamic)
    for (int h = 0; h < hv; ++h) {
        double* q = (double*)malloc(sizeof(double) * (size_t)dk);
        double* k = (double*)malloc(sizeof(double) * (size_t)dk);
        double* o = (double*)malloc(sizeof(double) * (size_t)dv);
        double* kv = (double*)malloc(sizeof(double) * (size_t)dv);
        for (int t = 0; t < tokens; ++t) {
            const float* row = conv + (int64_t)t * conv_dim;
            const int kh = h / rep;
            const float* qs = row + (int64_t)kh * dk;
            const float* ks = row + (int64_t)hk * dk + (int64_t)kh * dk;
            const float* vs = row + 2 * (int64_t)hk * dk + (int64_t)h * dv;
            double nq = 0, nk = 0;
            for (int i = 0; i < dk; ++i) {
                nq += (double)qs[i] * qs[i];
                nk += (double)ks[i] * ks[i];
            }
            const double iq = 1.0 / sqrt(nq + 1e-6), ik = 1.0 / sqrt(nk + 1e-6);
            for (int i = 0; i < dk; ++i) {
                q[i] = qs[i] * iq * qscale;
                k[i] = ks[i] * ik;
            }
            const double beta = 1.0 / (1.0 + exp(-(double)b[(int64_t)t * hv + h]));
            const double xa = (double)a[(int64_t)t * hv + h] + (double)dt_bias[h];
            const double softplus = xa > 20.0 ? xa : log1p(exp(xa));
            const double g = -exp((double)a_log[h]) * softplus;
            const double decay = exp(g);
            float* S = state + (int64_t)h * dk * dv;
            for (int64_t i = 0; i < (int64_t)dk * dv; ++i) S[i] = (float)(S[i] * decay);
            for (int j = 0; j < dv; ++j) {
                double acc = 0;
                for (int i = 0; i < dk; ++i) acc += (double)S[(int64_t)i * dv + j] * k[i];
                kv[j] = ((double)vs[j] - acc) * beta;
            }
            for (int i = 0; i < dk; ++i)
                for (int j = 0; j < dv; ++j) S[(int64_t)i * dv + j] = (float)(S[(int64_t)i * dv + j] + k[i] * kv[j]);
            double ss = 0;
            for (int j = 0; j < dv; ++j) {
                double acc = 0;
                for (int i = 0; i < dk; ++i) acc += (double)S[(int64_t)i * dv + j] * q[i];
                o[j] = acc;
                ss += acc * acc;
            }
            const double rstd = 1.0 / sqrt(ss / dv + (double)eps);
            for (int j = 0; j < dv; ++j) {
                const double zz = z[(int64_t)t * hv * dv + (int64_t)h * dv + j];
                const double gate = zz / (1.0 + exp(-zz));
                out[(int64_t)t * hv * dv + (int64_t)h * dv + j] = (float)((double)(float)(o[j] * rstd) * norm_w[j] * gate);
            }
        }
        free(q);
        free(k);
        free(o);
        free(kv);
    }
}

/* ------------------------------------------------------------------------------------------------ */
/* Whole decoder                                                                                     */
/* ------------------------------------------------------------------------------------------------ */

typedef struct {
    int n, k, dtype, group;
    void* w;
    uint16_t* s;
} orc_mat;

typedef struct {
    float *in_norm, *post_norm, *qb, *kb, *vb, *qn, *kn;
    orc_mat q, k, v, o, gate, up, down;
    void *kc, *vc;
    /* Qwen3.5: attention output gate rows (split from q_proj), and a Gated DeltaNet layer's weights
     * (L/LlmLinearAttention.cs:7-40) and per-sequence state (conv window, recurrent state; :42-90). */
    orc_mat qg;
    int linear;
    orc_mat in_qkv, in_z, in_b, in_a, out;
    float *conv_w, *a_log, *dt_bias, *lin_norm;
    float *conv_state, *rec_state;
} orc_layer;

struct orc_model {
    orc_config c;
    int max_seq, qd, kvd, rot, layer_limit;
    int batch;  /* sequences: KV caches are [batch, max_seq, kv_dim] */
    int fast;   /* 1: projections on the fp32 timing GEMM (orc_gemm_fast); 0: double accumulation */
    float attn_scale;
    float* inv_freq;
    float* embed;
    float* final_norm;
    orc_mat lm_head;
    orc_layer* L;
    /* row scratch, [rows_cap, width] */
    int rows_cap;
    float *hidden, *normed, *q, *k, *v, *attn, *proj, *gate, *up, *down;
    /* Qwen3.5 row scratch: the attention gate [rows, qd]; linear layers' projections and outputs */
    int lin_cap;
    float *ag, *lq, *lz, *lb, *la, *lc, *lo;
    int conv_dim, lin_vd;
    orc_probe_fn probe;
    void* probe_user;
};

void orc_model_set_probe(orc_model* m, orc_probe_fn fn, void* user) {
    m->probe = fn;
    m->probe_user = user;
}

static void emit(orc_model* m, int l, const char* stage, const float* v, int64_t n) {
    if (m->probe) m->probe(m->probe_user, l, stage, v, n);
}

static int mat_alloc(orc_mat* m, int n, int k, int dtype, int group) {
    m->n = n;
    m->k = k;
    m->dtype = dtype;
    m->group = dtype == ORC_I8 ? (group > 0 ? group : k) : 0;
    m->w = calloc((size_t)n * k, dtype_bytes(dtype));
    m->s = dtype == ORC_I8 ? (uint16_t*)calloc((size_t)n * (k / m->group), 2) : NULL;
    return m->w != NULL;
}

static void mat_free(orc_mat* m) {
    free(m->w);
    free(m->s);
}

static void mat_set_f32(orc_mat* m, const float* src) {
    if (m->dtype == ORC_I8) orc_q8_quantize(src, m->n, m->k, m->group, (int8_t*)m->w, m->s);
    else orc_convert(src, m->w, m->dtype, (int64_t)m->n * m->k);
}

static void mat_apply_rows(const orc_model* om, const orc_mat* m, int rows, const float* x, float* y) {
    if (om->fast) orc_gemm_fast(rows, m->n, m->k, x, m->dtype, m->w, m->s, m->group, y);
    else orc_gemv_out_in(rows, m->n, m->k, x, m->dtype, m->w, m->s, m->group, y);
}

static void free_rows(orc_model* m) {
    free(m->hidden);
    free(m->normed);
    free(m->q);
    free(m->k);
    free(m->v);
    free(m->attn);
    free(m->proj);
    free(m->gate);
    free(m->up);
    free(m->down);
    m->hidden = m->normed = m->q = m->k = m->v = m->attn = m->proj = m->gate = m->up = m->down = NULL;
    m->rows_cap = 0;
    free(m->ag);
    free(m->lq);
    free(m->lz);
    free(m->lb);
    free(m->la);
    free(m->lc);
    free(m->lo);
    m->ag = m->lq = m->lz = m->lb = m->la = m->lc = m->lo = NULL;
    m->lin_cap = 0;
}

/* Row scratch of the Qwen3.5 layers (attention gate, Gated DeltaNet projections), grown with rows. */
static int ensure_hybrid_rows(orc_model* m, int rows) {
    if (rows <= m->lin_cap) return 0;
    const size_t r = (size_t)rows, hv = (size_t)(m->c.lin_v_heads > 0 ? m->c.lin_v_heads : 1);
    free(m->ag);
    free(m->lq);
    free(m->lz);
    free(m->lb);
    free(m->la);
    free(m->lc);
    free(m->lo);
    m->ag = (float*)calloc(r * (size_t)m->qd, sizeof(float));
    m->lq = (float*)calloc(r * (size_t)(m->conv_dim + 1), sizeof(float));
    m->lc = (float*)calloc(r * (size_t)(m->conv_dim + 1), sizeof(float));
    m->lz = (float*)calloc(r * (size_t)(m->lin_vd + 1), sizeof(float));
    m->lo = (float*)calloc(r * (size_t)(m->lin_vd + 1), sizeof(float));
    m->lb = (float*)calloc(r * hv, sizeof(float));
    m->la = (float*)calloc(r * hv, sizeof(float));
    if (!m->ag || !m->lq || !m->lc || !m->lz || !m->lo || !m->lb || !m->la) return -1;
    m->lin_cap = rows;
    return 0;
}

static int ensure_rows(orc_model* m, int rows) {
    if (rows <= m->rows_cap) return 0;
    free_rows(m);
    const size_t r = (size_t)rows, H = (size_t)m->c.hidden, I = (size_t)m->c.inter;
    m->hidden = (float*)calloc(r * H, sizeof(float));
    m->normed = (float*)calloc(r * H, sizeof(float));
    m->q = (float*)calloc(r * (size_t)m->qd, sizeof(float));
    m->k = (float*)calloc(r * (size_t)m->kvd, sizeof(float));
    m->v = (float*)calloc(r * (size_t)m->kvd, sizeof(float));
    m->attn = (float*)calloc(r * (size_t)m->qd, sizeof(float));
    m->proj = (float*)calloc(r * H, sizeof(float));
    m->gate = (float*)calloc(r * I, sizeof(float));
    m->up = (float*)calloc(r * I, sizeof(float));
    m->down = (float*)calloc(r * H, sizeof(float));
    if (!m->hidden || !m->normed || !m->q || !m->k || !m->v || !m->attn || !m->proj || !m->gate || !m->up || !m->down) {
        free_rows(m);
        return -1;
    }
    m->rows_cap = rows;
    return 0;
}

/* KV cache rows of sequence `seq`. */
static void* seq_cache(const orc_model* m, void* cache, int seq) {
    return (char*)cache + (size_t)seq * m->max_seq * m->kvd * dtype_bytes(m->c.kv_dtype);
}

orc_model* orc_model_create(const orc_config* cfg, int max_seq) { return orc_model_create_batch(cfg, max_seq, 1); }

orc_model* orc_model_create_batch(const orc_config* cfg, int max_seq, int batch) {
    if (batch < 1) return NULL;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    if (!m) return NULL;
    m->c = *cfg;
    m->max_seq = max_seq;
    m->batch = batch;
    m->qd = cfg->heads * cfg->head_dim;
    m->kvd = cfg->kv_heads * cfg->head_dim;
    m->inv_freq = (float*)calloc((size_t)cfg->head_dim, sizeof(float));
    const int rope_dim = cfg->partial_rotary > 0.0 && cfg->partial_rotary < 1.0
                             ? (int)(cfg->head_dim * cfg->partial_rotary)
                             : cfg->head_dim;
    m->conv_dim = 2 * cfg->lin_k_heads * cfg->lin_k_dim + cfg->lin_v_heads * cfg->lin_v_dim;
    m->lin_vd = cfg->lin_v_heads * cfg->lin_v_dim;
    m->rot = 2 * orc_rope_frequencies(rope_dim, cfg->theta, cfg->max_pos, cfg->rope_type, cfg->rope_factor,
                                      cfg->rope_original_max, cfg->rope_low, cfg->rope_high, cfg->rope_beta_fast,
                                      cfg->rope_beta_slow, cfg->rope_attention, 0, 0, 1, m->inv_freq, &m->attn_scale);
    const int H = cfg->hidden, I = cfg->inter;
    m->embed = (float*)calloc((size_t)cfg->vocab * H, sizeof(float));
    m->final_norm = (float*)malloc(sizeof(float) * (size_t)H);
    for (int i = 0; i < H; ++i) m->final_norm[i] = 1.f;
    mat_alloc(&m->lm_head, cfg->vocab, H, cfg->wdtype, cfg->group);
    m->L = (orc_layer*)calloc((size_t)cfg->layers, sizeof(orc_layer));
    const size_t kvb = dtype_bytes(cfg->kv_dtype);
    for (int l = 0; l < cfg->layers; ++l) {
        orc_layer* L = &m->L[l];
        L->in_norm = (float*)malloc(sizeof(float) * (size_t)H);
        L->post_norm = (float*)malloc(sizeof(float) * (size_t)H);
        for (int i = 0; i < H; ++i) L->in_norm[i] = L->post_norm[i] = 1.f;
        mat_alloc(&L->q, m->qd, H, cfg->wdtype, cfg->group);
        mat_alloc(&L->k, m->kvd, H, cfg->wdtype, cfg->group);
        mat_alloc(&L->v, m->kvd, H, cfg->wdtype, cfg->group);
        mat_alloc(&L->o, H, m->qd, cfg->wdtype, cfg->group);
        mat_alloc(&L->gate, I, H, cfg->wdtype, cfg->group);
        mat_alloc(&L->up, I, H, cfg->wdtype, cfg->group);
        mat_alloc(&L->down, H, I, cfg->wdtype, cfg->group);
        if (cfg->bias) {
            L->qb = (float*)calloc((size_t)m->qd, sizeof(float));
            L->kb = (float*)calloc((size_t)m->kvd, sizeof(float));
            L->vb = (float*)calloc((size_t)m->kvd, sizeof(float));
        }
        if (cfg->qk_norm) {
            L->qn = (float*)malloc(sizeof(float) * (size_t)cfg->head_dim);
            L->kn = (float*)malloc(sizeof(float) * (size_t)cfg->head_dim);
            for (int i = 0; i < cfg->head_dim; ++i) L->qn[i] = L->kn[i] = 1.f;
        }
        if (cfg->attn_gate) mat_alloc(&L->qg, m->qd, H, cfg->wdtype, cfg->group);
        L->linear = l < 64 && ((cfg->linear_mask >> l) & 1ULL);
        if (L->linear) {
            const int hv = cfg->lin_v_heads, cd = m->conv_dim, vd = m->lin_vd, km1 = cfg->lin_conv - 1;
            if (hv < 1 || cfg->lin_k_heads < 1 || hv % cfg->lin_k_heads || cfg->lin_conv < 2) {
                m->c.layers = l + 1;
                orc_model_free(m);
                return NULL;
            }
            mat_alloc(&L->in_qkv, cd, H, cfg->wdtype, cfg->group);
            mat_alloc(&L->in_z, vd, H, cfg->wdtype, cfg->group);
            mat_alloc(&L->in_b, hv, H, cfg->wdtype, cfg->group);
            mat_alloc(&L->in_a, hv, H, cfg->wdtype, cfg->group);
            mat_alloc(&L->out, H, vd, cfg->wdtype, cfg->group);
            L->conv_w = (float*)calloc((size_t)cd * cfg->lin_conv, sizeof(float));
            L->a_log = (float*)calloc((size_t)hv, sizeof(float));
            L->dt_bias = (float*)calloc((size_t)hv, sizeof(float));
            L->lin_norm = (float*)malloc(sizeof(float) * (size_t)cfg->lin_v_dim);
            for (int i = 0; i < cfg->lin_v_dim; ++i) L->lin_norm[i] = 1.f;
            L->conv_state = (float*)calloc((size_t)batch * cd * km1, sizeof(float));
            L->rec_state = (float*)calloc((size_t)batch * hv * cfg->lin_k_dim * cfg->lin_v_dim, sizeof(float));
        }
        L->kc = calloc((size_t)batch * max_seq * m->kvd, kvb);
        L->vc = calloc((size_t)batch * max_seq * m->kvd, kvb);
        if (!L->kc || !L->vc || !L->q.w || !L->gate.w || !L->down.w) {
            m->c.layers = l + 1;
            orc_model_free(m);
            return NULL;
        }
    }
    (void)I;
    if (!m->embed || !m->lm_head.w || ensure_rows(m, 1) != 0) {
        orc_model_free(m);
        return NULL;
    }
    return m;
}

void orc_model_set_fast(orc_model* m, int fast) { m->fast = fast != 0; }

void orc_model_free(orc_model* m) {
    if (!m) return;
    for (int l = 0; l < m->c.layers; ++l) {
        orc_layer* L = &m->L[l];
        free(L->in_norm);
        free(L->post_norm);
        free(L->qb);
        free(L->kb);
        free(L->vb);
        free(L->qn);
        free(L->kn);
        mat_free(&L->q);
        mat_free(&L->k);
        mat_free(&L->v);
        mat_free(&L->o);
        mat_free(&L->gate);
        mat_free(&L->up);
        mat_free(&L->down);
        free(L->kc);
        free(L->vc);
        mat_free(&L->qg);
        mat_free(&L->in_qkv);
        mat_free(&L->in_z);
        mat_free(&L->in_b);
        mat_free(&L->in_a);
        mat_free(&L->out);
        free(L->conv_w);
        free(L->a_log);
        free(L->dt_bias);
        free(L->lin_norm);
        free(L->conv_state);
        free(L->rec_state);
    }
    free(m->L);
    mat_free(&m->lm_head);
    free(m->embed);
    free(m->final_norm);
    free(m->inv_freq);
    free_rows(m);
    free(m);
}

void orc_model_set_layer_limit(orc_model* m, int layers_to_run) { m->layer_limit = layers_to_run; }

/* Synthetic tensor ids: the same table as the CUDA model. */
enum { K_IN_NORM = 0, K_POST_NORM, K_Q, K_K, K_V, K_O, K_GATE, K_UP, K_DOWN, K_QB, K_KB, K_VB, K_QN, K_KN, K_SCALE = 16 };
static uint64_t layer_id(int l, int kind) { return 1000ULL + (uint64_t)l * 64 + (uint64_t)kind; }

static void synth_mat(orc_mat* mt, uint64_t seed, uint64_t id, uint64_t sid, float std, float lo, float hi) {
    const int64_t count = (int64_t)mt->n * mt->k;
    if (mt->dtype == ORC_I8) {
        orc_synth_fill(mt->w, ORC_I8, count, orc_tensor_stream(seed, id), ORC_SYN_I8, 0, 0, count, count, 0, 0);
        const int64_t ns = (int64_t)mt->n * (mt->k / mt->group);
        orc_synth_fill(mt->s, ORC_F16, ns, orc_tensor_stream(seed, sid), ORC_SYN_UNIFORM, lo, hi, ns, ns, 0, 0);
    } else {
        orc_synth_fill(mt->w, mt->dtype, count, orc_tensor_stream(seed, id), ORC_SYN_NORMAL, std, 0, count, count, 0, 0);
    }
}

int orc_model_init_synthetic(orc_model* m, uint64_t seed, float std, float lo, float hi) {
    const orc_config* c = &m->c;
    const int64_t ne = (int64_t)c->vocab * c->hidden;
    orc_synth_fill(m->embed, ORC_F32, ne, orc_tensor_stream(seed, 1), ORC_SYN_NORMAL, std, 0, ne, ne, 0, 0);
    if (c->tie) mat_set_f32(&m->lm_head, m->embed);
    else synth_mat(&m->lm_head, seed, 3, 4, std, lo, hi);
    for (int l = 0; l < c->layers; ++l) {
        orc_layer* L = &m->L[l];
        synth_mat(&L->q, seed, layer_id(l, K_Q), layer_id(l, K_SCALE + K_Q), std, lo, hi);
        synth_mat(&L->k, seed, layer_id(l, K_K), layer_id(l, K_SCALE + K_K), std, lo, hi);
        synth_mat(&L->v, seed, layer_id(l, K_V), layer_id(l, K_SCALE + K_V), std, lo, hi);
        synth_mat(&L->o, seed, layer_id(l, K_O), layer_id(l, K_SCALE + K_O), std, lo, hi);
        synth_mat(&L->gate, seed, layer_id(l, K_GATE), layer_id(l, K_SCALE + K_GATE), std, lo, hi);
        synth_mat(&L->up, seed, layer_id(l, K_UP), layer_id(l, K_SCALE + K_UP), std, lo, hi);
        synth_mat(&L->down, seed, layer_id(l, K_DOWN), layer_id(l, K_SCALE + K_DOWN), std, lo, hi);
        if (c->bias) {
            orc_synth_fill(L->qb, ORC_F32, m->qd, orc_tensor_stream(seed, layer_id(l, K_QB)), ORC_SYN_NORMAL, std, 0,
                           m->qd, m->qd, 0, 0);
            orc_synth_fill(L->kb, ORC_F32, m->kvd, orc_tensor_stream(seed, layer_id(l, K_KB)), ORC_SYN_NORMAL, std, 0,
                           m->kvd, m->kvd, 0, 0);
            orc_synth_fill(L->vb, ORC_F32, m->kvd, orc_tensor_stream(seed, layer_id(l, K_VB)), ORC_SYN_NORMAL, std, 0,
                           m->kvd, m->kvd, 0, 0);
        }
    }
    return 0;
}

int orc_model_set_tensor(orc_model* m, const char* name, const float* data, int64_t count) {
    const orc_config* c = &m->c;
    const int H = c->hidden;
    if (!strcmp(name, "model.embed_tokens.weight")) {
        if (count != (int64_t)c->vocab * H) return -2;
        memcpy(m->embed, data, sizeof(float) * (size_t)count);
        if (c->tie) mat_set_f32(&m->lm_head, m->embed);
        return 0;
    }
    if (!strcmp(name, "model.norm.weight")) {
        for (int i = 0; i < H; ++i) m->final_norm[i] = data[i] + c->norm_offset;
        return 0;
    }
    if (!strcmp(name, "lm_head.weight")) {
        mat_set_f32(&m->lm_head, data);
        return 0;
    }
    int l = -1;
    char rest[128];
    if (sscanf(name, "model.layers.%d.%127s", &l, rest) != 2 || l < 0 || l >= c->layers) return -1;
    orc_layer* L = &m->L[l];
    const float off = c->norm_offset;
    if (L->linear) {
        /* LlmLayerWeights.Load, linear branch (L/LlmLayerWeights.cs:146-163): the gated norm weight is
         * loaded as is (no offset); conv1d.weight [conv_dim, 1, k] is [conv_dim, k]. */
        const int hv = c->lin_v_heads;
        if (!strcmp(rest, "linear_attn.in_proj_qkv.weight")) mat_set_f32(&L->in_qkv, data);
        else if (!strcmp(rest, "linear_attn.in_proj_z.weight")) mat_set_f32(&L->in_z, data);
        else if (!strcmp(rest, "linear_attn.in_proj_b.weight")) mat_set_f32(&L->in_b, data);
        else if (!strcmp(rest, "linear_attn.in_proj_a.weight")) mat_set_f32(&L->in_a, data);
        else if (!strcmp(rest, "linear_attn.out_proj.weight")) mat_set_f32(&L->out, data);
        else if (!strcmp(rest, "linear_attn.conv1d.weight"))
            memcpy(L->conv_w, data, sizeof(float) * (size_t)m->conv_dim * c->lin_conv);
        else if (!strcmp(rest, "linear_attn.A_log")) memcpy(L->a_log, data, sizeof(float) * (size_t)hv);
        else if (!strcmp(rest, "linear_attn.dt_bias")) memcpy(L->dt_bias, data, sizeof(float) * (size_t)hv);
        else if (!strcmp(rest, "linear_attn.norm.weight")) memcpy(L->lin_norm, data, sizeof(float) * (size_t)c->lin_v_dim);
        else goto common;
        return 0;
    }
    if (c->attn_gate && !strcmp(rest, "self_attn.q_proj.weight")) {
        /* SplitQueryAndGate (L/LlmLayerWeights.cs:282-297): per head, hd query rows then hd gate rows. */
        const size_t blk = (size_t)c->head_dim * H;
        float* qr = (float*)malloc(sizeof(float) * blk * (size_t)c->heads);
        float* gr = (float*)malloc(sizeof(float) * blk * (size_t)c->heads);
        if (!qr || !gr) {
            free(qr);
            free(gr);
            return -2;
        }
        for (int h = 0; h < c->heads; ++h) {
            memcpy(qr + h * blk, data + (2 * (size_t)h) * blk, sizeof(float) * blk);
            memcpy(gr + h * blk, data + (2 * (size_t)h + 1) * blk, sizeof(float) * blk);
        }
        mat_set_f32(&L->q, qr);
        mat_set_f32(&L->qg, gr);
        free(qr);
        free(gr);
        return 0;
    }
common:
    if (!strcmp(rest, "input_layernorm.weight")) {
        for (int i = 0; i < H; ++i) L->in_norm[i] = data[i] + off;
    } else if (!strcmp(rest, "post_attention_layernorm.weight")) {
        for (int i = 0; i < H; ++i) L->post_norm[i] = data[i] + off;
    } else if (L->linear && strncmp(rest, "mlp.", 4) != 0) {
        return -1;
    } else if (!strcmp(rest, "self_attn.q_proj.weight")) mat_set_f32(&L->q, data);
    else if (!strcmp(rest, "self_attn.k_proj.weight")) mat_set_f32(&L->k, data);
    else if (!strcmp(rest, "self_attn.v_proj.weight")) mat_set_f32(&L->v, data);
    else if (!strcmp(rest, "self_attn.o_proj.weight")) mat_set_f32(&L->o, data);
    else if (!strcmp(rest, "mlp.gate_proj.weight")) mat_set_f32(&L->gate, data);
    else if (!strcmp(rest, "mlp.up_proj.weight")) mat_set_f32(&L->up, data);
    else if (!strcmp(rest, "mlp.down_proj.weight")) mat_set_f32(&L->down, data);
    else if (!strcmp(rest, "self_attn.q_proj.bias") && L->qb) memcpy(L->qb, data, sizeof(float) * (size_t)m->qd);
    else if (!strcmp(rest, "self_attn.k_proj.bias") && L->kb) memcpy(L->kb, data, sizeof(float) * (size_t)m->kvd);
    else if (!strcmp(rest, "self_attn.v_proj.bias") && L->vb) memcpy(L->vb, data, sizeof(float) * (size_t)m->kvd);
    else if (!strcmp(rest, "self_attn.q_norm.weight") && L->qn) {
        for (int i = 0; i < c->head_dim; ++i) L->qn[i] = data[i] + off;
    } else if (!strcmp(rest, "self_attn.k_norm.weight") && L->kn) {
        for (int i = 0; i < c->head_dim; ++i) L->kn[i] = data[i] + off;
    } else return -1;
    return 0;
}

/* LlmDecoderLayer.MixLinear (L/LlmDecoderLayer.cs:381-397) for `rows` tokens: the four in-projections of the
 * normed rows, then row by row in order the causal conv and the gated delta step on the row's sequence
 * state (reset when the row is at position 0, as MixLinear resets at a chunk starting at 0), then
 * out_proj into m->proj. */
static void mix_linear(orc_model* m, orc_layer* L, int rows, const int* positions, const int* seqs) {
    const orc_config* c = &m->c;
    const int cd = m->conv_dim, vd = m->lin_vd, hv = c->lin_v_heads, km1 = c->lin_conv - 1;
    const size_t st = (size_t)hv * c->lin_k_dim * c->lin_v_dim;
    mat_apply_rows(m, &L->in_qkv, rows, m->normed, m->lq);
    mat_apply_rows(m, &L->in_z, rows, m->normed, m->lz);
    mat_apply_rows(m, &L->in_b, rows, m->normed, m->lb);
    mat_apply_rows(m, &L->in_a, rows, m->normed, m->la);
    for (int r = 0; r < rows; ++r) {
        const int sq = seqs ? seqs[r] : 0;
        float* cs = L->conv_state + (size_t)sq * cd * km1;
        float* rs = L->rec_state + (size_t)sq * st;
        if (positions[r] == 0) {
            memset(cs, 0, sizeof(float) * (size_t)cd * km1);
            memset(rs, 0, sizeof(float) * st);
        }
        orc_causal_conv(m->lq + (int64_t)r * cd, cs, L->conv_w, m->lc + (int64_t)r * cd, cd, c->lin_conv, 1);
        orc_gated_delta(m->lc + (int64_t)r * cd, m->lz + (int64_t)r * vd, m->lb + (int64_t)r * hv,
                        m->la + (int64_t)r * hv, L->a_log, L->dt_bias, L->lin_norm, rs, m->lo + (int64_t)r * vd,
                        c->lin_k_heads, hv, c->lin_k_dim, c->lin_v_dim, 1, c->eps);
    }
    mat_apply_rows(m, &L->out, rows, m->lo, m->proj);
}

/* LlmModel.Step / StepBatch / IngestPrompt + LlmDecoderLayer.Forward / ForwardBatch (L/LlmModel.cs:156-251,
 * 320-444; L/LlmDecoderLayer.cs:129-196, 290-378): `rows` tokens through the decoder at once. Row r feeds
 * tokens[r] at positions[r] of sequence seqs[r] (NULL: sequence 0). Every row's K/V is stored before any
 * attention, so consecutive positions of one sequence form a causal prefill chunk and rows of distinct
 * sequences a decode batch. logits: [rows, vocab], or only the last row's when last_only; may be NULL. */
int orc_model_forward(orc_model* m, int rows, const int* tokens, const int* positions, const int* seqs,
                      float* logits, int last_only) {
    const orc_config* c = &m->c;
    const int H = c->hidden, I = c->inter, hd = c->head_dim;
    if (rows < 1) return -1;
    for (int r = 0; r < rows; ++r) {
        const int sq = seqs ? seqs[r] : 0;
        if (tokens[r] < 0 || tokens[r] >= c->vocab || positions[r] < 0 || positions[r] >= m->max_seq || sq < 0 ||
            sq >= m->batch)
            return -1;
    }
    if (ensure_rows(m, rows) != 0) return -2;
    for (int r = 0; r < rows; ++r)
        memcpy(m->hidden + (int64_t)r * H, m->embed + (int64_t)tokens[r] * H, sizeof(float) * (size_t)H);
    const int nl = m->layer_limit > 0 && m->layer_limit < c->layers ? m->layer_limit : c->layers;
    if ((c->linear_mask || c->attn_gate) && ensure_hybrid_rows(m, rows) != 0) return -2;
    for (int l = 0; l < nl; ++l) {
        orc_layer* L = &m->L[l];
        orc_rmsnorm(m->hidden, NULL, L->in_norm, m->normed, c->eps, H, rows, 0);
        emit(m, l, "input_norm", m->normed, H);
        if (L->linear) {
            mix_linear(m, L, rows, positions, seqs);
            goto mlp;
        }
        mat_apply_rows(m, &L->q, rows, m->normed, m->q);
        if (c->attn_gate) mat_apply_rows(m, &L->qg, rows, m->normed, m->ag);
        mat_apply_rows(m, &L->k, rows, m->normed, m->k);
        mat_apply_rows(m, &L->v, rows, m->normed, m->v);
        if (c->bias) {
            orc_bias_add(m->q, L->qb, m->qd, rows);
            orc_bias_add(m->k, L->kb, m->kvd, rows);
            orc_bias_add(m->v, L->vb, m->kvd, rows);
        }
        if (c->qk_norm) {
            orc_rmsnorm(m->q, NULL, L->qn, m->q, c->eps, hd, rows * c->heads, 0);
            orc_rmsnorm(m->k, NULL, L->kn, m->k, c->eps, hd, rows * c->kv_heads, 0);
        }
        emit(m, l, "q", m->q, m->qd);
        emit(m, l, "k", m->k, m->kvd);
        emit(m, l, "v", m->v, m->kvd);
        orc_rope(m->q, m->k, positions, m->inv_freq, hd, c->heads, c->kv_heads, m->attn_scale, m->rot, rows);
        for (int r = 0; r < rows; ++r) {
            const int sq = seqs ? seqs[r] : 0;
            orc_kv_store(m->k + (int64_t)r * m->kvd, m->v + (int64_t)r * m->kvd, seq_cache(m, L->kc, sq),
                         seq_cache(m, L->vc, sq), c->kv_dtype, positions[r], m->kvd, 1);
        }
        for (int r = 0; r < rows; ++r) {
            const int sq = seqs ? seqs[r] : 0;
            orc_attention(m->q + (int64_t)r * m->qd, seq_cache(m, L->kc, sq), seq_cache(m, L->vc, sq), c->kv_dtype,
                          m->attn + (int64_t)r * m->qd, hd, c->heads, c->kv_heads, positions[r], 1);
        }
        /* MixFull (L/LlmDecoderLayer.cs:328-331): the optional sigmoid output gate before o_proj. */
        if (c->attn_gate) orc_sigmoid_gate(m->attn, m->ag, (int64_t)rows * m->qd);
        mat_apply_rows(m, &L->o, rows, m->attn, m->proj);
    mlp:
        emit(m, l, "attn_out", m->proj, H);
        orc_rmsnorm(m->hidden, m->proj, L->post_norm, m->normed, c->eps, H, rows, 1);
        emit(m, l, "post_norm", m->normed, H);
        mat_apply_rows(m, &L->gate, rows, m->normed, m->gate);
        mat_apply_rows(m, &L->up, rows, m->normed, m->up);
        orc_swiglu(m->gate, m->up, (int64_t)rows * I);
        mat_apply_rows(m, &L->down, rows, m->gate, m->down);
        emit(m, l, "mlp_out", m->down, H);
        orc_add(m->hidden, m->down, (int64_t)rows * H);
        emit(m, l, "output", m->hidden, H);
    }
    if (!logits) return 0;
    if (last_only) {
        orc_rmsnorm(m->hidden + (int64_t)(rows - 1) * H, NULL, m->final_norm, m->normed, c->eps, H, 1, 0);
        mat_apply_rows(m, &m->lm_head, 1, m->normed, logits);
    } else {
        orc_rmsnorm(m->hidden, NULL, m->final_norm, m->normed, c->eps, H, rows, 0);
        mat_apply_rows(m, &m->lm_head, rows, m->normed, logits);
    }
    return 0;
}

/* LlmModel.Step (L/LlmModel.cs:402-444): one token of sequence 0. */
int orc_model_step(orc_model* m, int token, int position, float* logits) {
    return orc_model_forward(m, 1, &token, &position, NULL, logits, 0);
}

int orc_model_read_kv_seq(orc_model* m, int layer, int seq, int row0, int rows, float* keys, float* values) {
    if (layer < 0 || layer >= m->c.layers || seq < 0 || seq >= m->batch || row0 < 0 || row0 + rows > m->max_seq) return -1;
    const void* kc = seq_cache(m, m->L[layer].kc, seq);
    const void* vc = seq_cache(m, m->L[layer].vc, seq);
    for (int64_t i = 0; i < (int64_t)rows * m->kvd; ++i) {
        keys[i] = load_elem(kc, m->c.kv_dtype, (int64_t)row0 * m->kvd + i);
        values[i] = load_elem(vc, m->c.kv_dtype, (int64_t)row0 * m->kvd + i);
    }
    return 0;
}

int orc_model_write_kv_seq(orc_model* m, int layer, int seq, int row0, int rows, const float* keys,
                           const float* values) {
    if (layer < 0 || layer >= m->c.layers || seq < 0 || seq >= m->batch || row0 < 0 || row0 + rows > m->max_seq) return -1;
    orc_kv_store(keys, values, seq_cache(m, m->L[layer].kc, seq), seq_cache(m, m->L[layer].vc, seq), m->c.kv_dtype, row0,
                 m->kvd, rows);
    return 0;
}

int orc_model_read_kv(orc_model* m, int layer, int row0, int rows, float* keys, float* values) {
    if (layer < 0 || layer >= m->c.layers || row0 < 0 || row0 + rows > m->max_seq) return -1;
    for (int64_t i = 0; i < (int64_t)rows * m->kvd; ++i) {
        keys[i] = load_elem(m->L[layer].kc, m->c.kv_dtype, (int64_t)row0 * m->kvd + i);
        values[i] = load_elem(m->L[layer].vc, m->c.kv_dtype, (int64_t)row0 * m->kvd + i);
    }
    return 0;
}
