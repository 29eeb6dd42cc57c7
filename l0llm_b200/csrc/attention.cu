// Decode / prefill attention over the KV cache (sm_100a, CUDA cores).
//
// One CTA owns one KV head (and the up-to-8 query heads that share it, GQA), one split of the
// positions and one query row. K/V tiles of 32 positions are staged in shared memory as fp32 (K rows
// padded to HD+1 floats so the per-position dot products are bank-conflict free); each warp scores
// 32 positions for its heads and keeps an online softmax (running max, running sum, rescaled
// accumulator), so no score buffer grows with the sequence and there is no length cap (the
// reference's fused kernel stops at 15000 tokens, L/LlmDecoderLayer.cs:21-22).
//
// Splits write (m, l, acc) partials; the last CTA of a (query, KV head) to finish -- found with an
// atomic counter that it resets afterwards -- merges them. With rope/store_new set the kernel also
// applies RoPE to the query and to the new key, and the CTA owning the query position writes the
// new key/value row into the cache, replacing the separate RoPE and KvCacheStore launches.
#include <cmath>
#include <mutex>

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "ops.cuh"

namespace l0b {

namespace {

constexpr int kT = 32;     // positions per tile
constexpr int kMaxG = 8;   // query heads per CTA
constexpr int kClusterThreads = 256;  // threads of the cluster decode kernel
constexpr int kMaxClusterSplits = 16;  // CTAs per cluster of the cluster decode kernel (16 is non-portable)

// Element d of a rotated head (HF rotate-half pairs) from the per-position cos/sin table.
__device__ __forceinline__ float rope_elem(const float* head, int d, int rot, const float* cs, const float* sn) {
    const float v = head[d];
    if (d >= rot) return v;
    const int half = rot >> 1;
    const int i = d < half ? d : d - half;
    const float c = cs[i], s = sn[i];
    if (d < half) return __fsub_rn(__fmul_rn(v, c), __fmul_rn(head[d + half], s));
    return __fadd_rn(__fmul_rn(v, c), __fmul_rn(head[d - half], s));
}

// Eight consecutive cache elements as fp32 (one 16-byte load for f16/bf16, two for f32).
__device__ __forceinline__ void load8(const void* base, int dtype, long long off, float (&o)[8]) {
    if (dtype == L0B_F32) {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + off + 4);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
        return;
    }
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + off);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = dtype == L0B_F16 ? half2_bits_to_float2(w[i]) : bf162_bits_to_float2(w[i]);
        o[2 * i] = f.x;
        o[2 * i + 1] = f.y;
    }
}

template <int HD>
__global__ void __launch_bounds__(128) attn_kernel(const AttnParams p) {
    constexpr int HPT = 128 / HD;          // head lanes per dim in the PV phase
    constexpr int JPT = kMaxG / HPT;       // heads per thread in the PV phase
    __shared__ float qs[kMaxG][HD];
    __shared__ float ks[kT][HD + 1];
    __shared__ __align__(16) float vs[kT][HD];
    __shared__ float ps[kMaxG][kT];
    __shared__ float m_s[kMaxG], l_s[kMaxG], corr_s[kMaxG];
    __shared__ float knew[HD], vnew[HD];
    __shared__ float cs_s[HD / 2], sn_s[HD / 2];
    __shared__ int last_s;

    const int G = p.nh / p.nkv;
    const int gparts = (G + kMaxG - 1) / kMaxG;
    const int kvh = blockIdx.x / gparts, gp = blockIdx.x - (blockIdx.x / gparts) * gparts;
    const int h0 = kvh * G + gp * kMaxG;
    const int ng = min(kMaxG, G - gp * kMaxG);
    const int split = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    pdl_wait();
    const int qpos = p.positions ? p.positions[b] : p.pos_base + b * p.pos_step;
    const int seq = qpos + 1;
    const int nact = (seq + p.chunk - 1) / p.chunk;
    if (split >= nact) return;
    pdl_launch_dependents();

    // cos/sin of this query position, once per CTA: angle = f32(pos) * inv_freq (as RoPE.Execute).
    if (p.rope) {
        for (int i = tid; i < p.rot / 2; i += 128) {
            const float ang = __fmul_rn(static_cast<float>(qpos), p.inv_freq[i]);
            float s, c;
            sincosf(ang, &s, &c);
            cs_s[i] = __fmul_rn(c, p.attn_scale);
            sn_s[i] = __fmul_rn(s, p.attn_scale);
        }
        __syncthreads();
    }
    const float* qb = p.q + b * p.q_bstride + static_cast<long long>(h0) * HD;
    for (int idx = tid; idx < kMaxG * HD; idx += 128) {
        const int j = idx / HD, d = idx - (idx / HD) * HD;
        float v = 0.f;
        if (j < ng) v = p.rope ? rope_elem(qb + j * HD, d, p.rot, cs_s, sn_s) : qb[j * HD + d];
        qs[j][d] = v;
    }
    if (tid < kMaxG) {
        m_s[tid] = kNegInf;
        l_s[tid] = 0.f;
    }
    const bool owns_new = p.store_new && split == nact - 1;
    if (owns_new) {
        const float* kb = p.k_new + b * p.new_bstride + static_cast<long long>(kvh) * HD;
        const float* vb = p.v_new + b * p.new_bstride + static_cast<long long>(kvh) * HD;
        for (int d = tid; d < HD; d += 128) {
            const float kv = p.rope ? rope_elem(kb, d, p.rot, cs_s, sn_s) : kb[d];
            knew[d] = kv;
            vnew[d] = vb[d];
            if (gp == 0) {
                const long long off = b * p.cache_bstride + static_cast<long long>(qpos) * p.kv_dim +
                                      static_cast<long long>(kvh) * HD + d;
                store_from_float(p.kc, p.cache_dtype, off, kv);
                store_from_float(p.vc, p.cache_dtype, off, vb[d]);
            }
        }
    }
    __syncthreads();

    float acc[JPT];
#pragma unroll
    for (int i = 0; i < JPT; ++i) acc[i] = 0.f;
    const int dim = tid % HD, jb = tid / HD;

    const int p_begin = split * p.chunk;
    const int p_end = min(seq, p_begin + p.chunk);
    const long long cache_base = b * p.cache_bstride + static_cast<long long>(kvh) * HD;
    for (int t0 = p_begin; t0 < p_end; t0 += kT) {
        // 16-byte loads: HD/8 threads per row, each owning 8 consecutive dims.
        constexpr int TPR = HD / 8;
        for (int idx = tid; idx < kT * TPR; idx += 128) {
            const int t = idx / TPR, d0 = (idx - t * TPR) * 8;
            const int pos = t0 + t;
            float kv[8], vv[8];
            if (pos < p_end && !(owns_new && pos == qpos)) {
                const long long off = cache_base + static_cast<long long>(pos) * p.kv_dim + d0;
                load8(p.kc, p.cache_dtype, off, kv);
                load8(p.vc, p.cache_dtype, off, vv);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const bool mine = pos < p_end;
                    kv[e] = mine ? knew[d0 + e] : 0.f;
                    vv[e] = mine ? vnew[d0 + e] : 0.f;
                }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) ks[t][d0 + e] = kv[e];
            *reinterpret_cast<float4*>(&vs[t][d0]) = make_float4(vv[0], vv[1], vv[2], vv[3]);
            *reinterpret_cast<float4*>(&vs[t][d0 + 4]) = make_float4(vv[4], vv[5], vv[6], vv[7]);
        }
        __syncthreads();
        for (int j = warp; j < ng; j += 4) {
            float s = kNegInf;
            if (t0 + lane < p_end) {
                float a = 0.f;
#pragma unroll 16
                for (int d = 0; d < HD; ++d) a = fmaf(qs[j][d], ks[lane][d], a);
                s = a * p.scale;
            }
            const float mx = warp_max(s);
            const float m_old = m_s[j];
            const float m_new = fmaxf(m_old, mx);
            const float pj = s == kNegInf ? 0.f : expf(s - m_new);
            const float sum = warp_sum(pj);
            ps[j][lane] = pj;
            __syncwarp();
            if (lane == 0) {
                const float corr = expf(m_old - m_new);
                corr_s[j] = corr;
                l_s[j] = l_s[j] * corr + sum;
                m_s[j] = m_new;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < JPT; ++i) {
            const int j = jb + i * HPT;
            if (j < ng) {
                float a = acc[i] * corr_s[j];
#pragma unroll 8
                for (int t = 0; t < kT; ++t) a = fmaf(ps[j][t], vs[t][dim], a);
                acc[i] = a;
            }
        }
        __syncthreads();
    }

    if (nact == 1) {
#pragma unroll
        for (int i = 0; i < JPT; ++i) {
            const int j = jb + i * HPT;
            if (j < ng) p.out[b * p.out_bstride + static_cast<long long>(h0 + j) * HD + dim] = acc[i] / l_s[j];
        }
        return;
    }

    const long long row = static_cast<long long>(b) * p.nh;
#pragma unroll
    for (int i = 0; i < JPT; ++i) {
        const int j = jb + i * HPT;
        if (j < ng) p.part[((row + h0 + j) * p.max_splits + split) * HD + dim] = acc[i];
    }
    if (tid < ng) {
        float* ml = p.part_ml + ((row + h0 + tid) * p.max_splits + split) * 2;
        ml[0] = m_s[tid];
        ml[1] = l_s[tid];
    }
    __threadfence();
    __syncthreads();
    unsigned* counter = p.counters + (static_cast<long long>(b) * p.nkv + kvh) * gparts + gp;
    if (tid == 0) last_s = atomicAdd(counter, 1u) == static_cast<unsigned>(nact - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
#pragma unroll
    for (int i = 0; i < JPT; ++i) {
        const int j = jb + i * HPT;
        if (j >= ng) continue;
        const float* ml = p.part_ml + (row + h0 + j) * p.max_splits * 2;
        const float* pa = p.part + (row + h0 + j) * p.max_splits * HD;
        float mmax = kNegInf;
        for (int s = 0; s < nact; ++s) mmax = fmaxf(mmax, __ldcg(ml + 2 * s));
        float lsum = 0.f, o = 0.f;
        for (int s = 0; s < nact; ++s) {
            const float w = expf(__ldcg(ml + 2 * s) - mmax);
            lsum = fmaf(w, __ldcg(ml + 2 * s + 1), lsum);
            o = fmaf(w, __ldcg(pa + static_cast<long long>(s) * HD + dim), o);
        }
        p.out[b * p.out_bstride + static_cast<long long>(h0 + j) * HD + dim] = o / lsum;
    }
    if (tid == 0) *counter = 0u;
}

// ---------------------------------------------------------------------------------------------
// Decode attention in thread-block clusters (no global partials, no counters).
//
// The S splits of one (query row, KV head group) form one cluster of (1, S, 1) CTAs, S <= 16. Each
// CTA walks its share of the positions -- chunk = max(p.chunk, 32 * ceil(seq / (32 S))) computed from
// the live sequence length, so short contexts leave the tail CTAs idle instead of launching more --
// with the next 32-position K/V tile loaded into registers while the current one is scored. Its
// (running max, running sum, unnormalised output) stay in its shared memory; after one cluster
// barrier CTA r merges head dimensions [r HD / S, (r + 1) HD / S) of every head by reading the S
// partials straight from the peers' shared memory (distributed shared memory over the cluster), and
// a second barrier keeps every CTA's shared memory alive until its peers have read it.
// ---------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(kClusterThreads) attn_cluster_kernel(const AttnParams p) {
    namespace cg = cooperative_groups;
    constexpr int NT = kClusterThreads;
    constexpr int HPT = NT / HD;             // threads per head dimension in the PV phase
    constexpr int JPT = kMaxG / HPT;         // heads per thread in the PV phase
    constexpr int TPR = HD / 8;              // threads per cached row, 8 dims each
    constexpr int ITEMS = kT * TPR / NT;     // row pieces per thread per tile
    // K tile as float4 columns: dims [4 c, 4 c + 4) of position t at ks4[c][t ^ kswz(c)], so a warp
    // scoring 32 positions reads one conflict-free 16-byte word per lane and the staging stores of
    // one row spread over the banks.
    __shared__ __align__(16) float qs[kMaxG][HD];
    __shared__ float4 ks4[HD / 4][kT];
    __shared__ __align__(16) float vs[kT][HD];
    __shared__ __align__(16) float ps[kMaxG][kT];
    __shared__ float m_s[kMaxG], l_s[kMaxG], corr_s[kMaxG];
    __shared__ float knew[HD], vnew[HD];
    __shared__ float cs_s[HD / 2], sn_s[HD / 2];
    __shared__ float acc_s[kMaxG][HD];

    cg::cluster_group cluster = cg::this_cluster();
    const int G = p.nh / p.nkv;
    const int gparts = (G + kMaxG - 1) / kMaxG;
    const int kvh = blockIdx.x / gparts, gp = blockIdx.x - (blockIdx.x / gparts) * gparts;
    const int h0 = kvh * G + gp * kMaxG;
    const int ng = min(kMaxG, G - gp * kMaxG);
    const int S = gridDim.y, split = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    auto kswz = [](int c) { return (c >> 1) & (kT - 1); };

    pdl_wait();
    const int qpos = p.positions ? p.positions[b] : p.pos_base + b * p.pos_step;
    const int seq = qpos + 1;
    int chunk = ((seq + S - 1) / S + kT - 1) / kT * kT;
    chunk = max(chunk, p.chunk);
    const int nact = (seq + chunk - 1) / chunk;
    const bool active = split < nact;
    pdl_launch_dependents();
    const int p_begin = split * chunk;
    const int p_end = min(seq, p_begin + chunk);
    const bool owns_new = p.store_new && split == nact - 1;
    const long long cache_base = b * p.cache_bstride + static_cast<long long>(kvh) * HD;
    const bool f32c = p.cache_dtype == L0B_F32;

    // Raw 16-byte pieces of the K and V rows of one tile (two per piece for an fp32 cache).
    uint4 kr[ITEMS][2], vr[ITEMS][2];
    auto load_tile = [&](int t0) {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int idx = tid + it * NT;
            const int t = idx / TPR, d0 = (idx - t * TPR) * 8;
            const int pos = t0 + t;
            kr[it][0] = kr[it][1] = vr[it][0] = vr[it][1] = make_uint4(0, 0, 0, 0);
            if (pos < p_end && !(owns_new && pos == qpos)) {
                const long long off = cache_base + static_cast<long long>(pos) * p.kv_dim + d0;
                if (f32c) {
                    const uint4* k4 = reinterpret_cast<const uint4*>(static_cast<const float*>(p.kc) + off);
                    const uint4* v4 = reinterpret_cast<const uint4*>(static_cast<const float*>(p.vc) + off);
                    kr[it][0] = k4[0], kr[it][1] = k4[1], vr[it][0] = v4[0], vr[it][1] = v4[1];
                } else {
                    kr[it][0] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.kc) + off);
                    vr[it][0] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.vc) + off);
                }
            }
        }
    };
    auto unpack = [&](const uint4 (&r)[2], float (&o)[8]) {
        if (f32c) {
            o[0] = __uint_as_float(r[0].x), o[1] = __uint_as_float(r[0].y), o[2] = __uint_as_float(r[0].z);
            o[3] = __uint_as_float(r[0].w), o[4] = __uint_as_float(r[1].x), o[5] = __uint_as_float(r[1].y);
            o[6] = __uint_as_float(r[1].z), o[7] = __uint_as_float(r[1].w);
            return;
        }
        const uint32_t w[4] = {r[0].x, r[0].y, r[0].z, r[0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = p.cache_dtype == L0B_F16 ? half2_bits_to_float2(w[i]) : bf162_bits_to_float2(w[i]);
            o[2 * i] = f.x;
            o[2 * i + 1] = f.y;
        }
    };
    if (active) load_tile(p_begin);

    if (p.rope) {
        for (int i = tid; i < p.rot / 2; i += NT) {
            const float ang = __fmul_rn(static_cast<float>(qpos), p.inv_freq[i]);
            float s, c;
            sincosf(ang, &s, &c);
            cs_s[i] = __fmul_rn(c, p.attn_scale);
            sn_s[i] = __fmul_rn(s, p.attn_scale);
        }
        __syncthreads();
    }
    const float* qb = p.q + b * p.q_bstride + static_cast<long long>(h0) * HD;
    for (int idx = tid; idx < kMaxG * HD; idx += NT) {
        const int j = idx / HD, d = idx - (idx / HD) * HD;
        float v = 0.f;
        if (j < ng) v = p.rope ? rope_elem(qb + j * HD, d, p.rot, cs_s, sn_s) : qb[j * HD + d];
        qs[j][d] = v;
    }
    if (tid < kMaxG) {
        m_s[tid] = kNegInf;
        l_s[tid] = 0.f;
        corr_s[tid] = 1.f;
    }
    for (int idx = tid; idx < kMaxG * kT; idx += NT) ps[idx / kT][idx % kT] = 0.f;  // head slots past ng stay 0
    if (owns_new) {
        const float* kb = p.k_new + b * p.new_bstride + static_cast<long long>(kvh) * HD;
        const float* vb = p.v_new + b * p.new_bstride + static_cast<long long>(kvh) * HD;
        for (int d = tid; d < HD; d += NT) {
            const float kv = p.rope ? rope_elem(kb, d, p.rot, cs_s, sn_s) : kb[d];
            knew[d] = kv;
            vnew[d] = vb[d];
            if (gp == 0) {
                const long long off = b * p.cache_bstride + static_cast<long long>(qpos) * p.kv_dim +
                                      static_cast<long long>(kvh) * HD + d;
                store_from_float(p.kc, p.cache_dtype, off, kv);
                store_from_float(p.vc, p.cache_dtype, off, vb[d]);
            }
        }
    }
    __syncthreads();

    float acc[JPT];
#pragma unroll
    for (int i = 0; i < JPT; ++i) acc[i] = 0.f;
    const int dim = tid % HD, jb = tid / HD;
    for (int t0 = p_begin; active && t0 < p_end; t0 += kT) {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int idx = tid + it * NT;
            const int t = idx / TPR, d0 = (idx - t * TPR) * 8;
            const int pos = t0 + t;
            float kv[8], vv[8];
            if (owns_new && pos == qpos) {
#pragma unroll
                for (int e = 0; e < 8; ++e) kv[e] = knew[d0 + e], vv[e] = vnew[d0 + e];
            } else {
                unpack(kr[it], kv);
                unpack(vr[it], vv);
            }
            const int c0 = d0 >> 2;
            ks4[c0][t ^ kswz(c0)] = make_float4(kv[0], kv[1], kv[2], kv[3]);
            ks4[c0 + 1][t ^ kswz(c0 + 1)] = make_float4(kv[4], kv[5], kv[6], kv[7]);
            *reinterpret_cast<float4*>(&vs[t][d0]) = make_float4(vv[0], vv[1], vv[2], vv[3]);
            *reinterpret_cast<float4*>(&vs[t][d0 + 4]) = make_float4(vv[4], vv[5], vv[6], vv[7]);
        }
        __syncthreads();
        if (t0 + kT < p_end) load_tile(t0 + kT);  // next tile in flight during the math
        for (int j = warp; j < ng; j += NT / 32) {
            float s = kNegInf;
            if (t0 + lane < p_end) {
                float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
                const float4* q4 = reinterpret_cast<const float4*>(qs[j]);
#pragma unroll 8
                for (int c = 0; c < HD / 4; ++c) {
                    const float4 kk = ks4[c][lane ^ kswz(c)];
                    const float4 qq = q4[c];
                    a0 = fmaf(qq.x, kk.x, a0);
                    a1 = fmaf(qq.y, kk.y, a1);
                    a2 = fmaf(qq.z, kk.z, a2);
                    a3 = fmaf(qq.w, kk.w, a3);
                }
                s = ((a0 + a1) + (a2 + a3)) * p.scale;
            }
            const float mx = warp_max(s);
            const float m_old = m_s[j];
            const float m_new = fmaxf(m_old, mx);
            const float pj = s == kNegInf ? 0.f : expf(s - m_new);
            const float sum = warp_sum(pj);
            ps[j][lane] = pj;
            __syncwarp();
            if (lane == 0) {
                const float corr = expf(m_old - m_new);
                corr_s[j] = corr;
                l_s[j] = l_s[j] * corr + sum;
                m_s[j] = m_new;
            }
        }
        __syncthreads();
        // Positions outer, heads inner: each V value is read once for all of this thread's heads.
#pragma unroll
        for (int i = 0; i < JPT; ++i) acc[i] *= corr_s[jb + i * HPT];
#pragma unroll 2
        for (int t = 0; t < kT; t += 4) {
            const float v0 = vs[t][dim], v1 = vs[t + 1][dim], v2 = vs[t + 2][dim], v3 = vs[t + 3][dim];
#pragma unroll
            for (int i = 0; i < JPT; ++i) {
                const float4 pp = *reinterpret_cast<const float4*>(&ps[jb + i * HPT][t]);
                acc[i] = fmaf(pp.x, v0, fmaf(pp.y, v1, fmaf(pp.z, v2, fmaf(pp.w, v3, acc[i]))));
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < JPT; ++i) acc_s[jb + i * HPT][dim] = acc[i];

    // A single split needs no cluster: its own shared memory and a block barrier.
    auto peer = [&](float* ptr, int s) { return S > 1 ? cluster.map_shared_rank(ptr, s) : ptr; };
    if (S > 1) cluster.sync();
    else __syncthreads();
    // Merge this CTA's slice of head dimensions from the nact active partials of the cluster.
    const int dper = HD / S;
    for (int o = tid; o < ng * dper; o += NT) {
        const int j = o / dper, d = split * dper + (o - (o / dper) * dper);
        float mv[kMaxClusterSplits], lv[kMaxClusterSplits], av[kMaxClusterSplits];
        float mmax = kNegInf;
#pragma unroll
        for (int s = 0; s < kMaxClusterSplits; ++s) {
            mv[s] = kNegInf, lv[s] = 0.f, av[s] = 0.f;
            if (s < nact) {
                mv[s] = *peer(&m_s[j], s);
                lv[s] = *peer(&l_s[j], s);
                av[s] = *peer(&acc_s[j][d], s);
            }
        }
#pragma unroll
        for (int s = 0; s < kMaxClusterSplits; ++s) mmax = fmaxf(mmax, mv[s]);
        float lsum = 0.f, y = 0.f;
#pragma unroll
        for (int s = 0; s < kMaxClusterSplits; ++s) {
            if (s < nact) {
                const float w = expf(mv[s] - mmax);
                lsum = fmaf(w, lv[s], lsum);
                y = fmaf(w, av[s], y);
            }
        }
        p.out[b * p.out_bstride + static_cast<long long>(h0 + j) * HD + d] = y / lsum;
    }
    if (S > 1) cluster.sync();
}

template <typename F>
l0b_status launch_attn(l0b_device* d, cudaStream_t stream, F kernel, dim3 grid, const AttnParams& p) {
    if (d) return d->launch(kernel, grid, dim3(128), 0, p);
    kernel<<<grid, 128, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    add_launches(1);
    return L0B_OK;
}

// ---------------------------------------------------------------------------------------------
// Prefill attention on the tensor cores (mma.sync m16n8k16, fp32 accumulators), flash-attention style.
//
// A CTA takes 64 query rows of one query head (four warps of 16 rows) and walks the key tiles of its
// KV head up to the largest position among its rows, 64 slots a tile, double-buffered in shared memory
// by cp.async (16-byte chunks of a row XOR-swizzled by the row index, so the fragment reads hit 32
// distinct banks). S = Q K^T: the query rows are scaled by softmax_scale * log2(e) and split into hi +
// lo 16-bit halves held in registers for the whole walk, each against the exact 16-bit key, so the
// scores keep about 22 bits (f16) or 16 bits (bf16) of the f32 query. The mask keeps slot <= the row's
// position; the softmax is online in exp2 (running max and sum per row, rows with nothing seen yet
// kept at zero). O += P V: P enters as the A operand straight from the score registers, again as hi +
// lo halves; V fragments come transposed by ldmatrix. Finally O / sum goes to the row's output.
// K / V caches f16 or bf16 (f32 caches take the scalar kernel).
// ---------------------------------------------------------------------------------------------
constexpr int kPfBM = 64, kPfBN = 64;
bool g_attn_prefill_mma = true;  // l0b_set_attention_prefill_tensor_cores
bool g_attn_cluster16 = true;    // l0b_set_attention_cluster16
bool g_attn_decode_mma = true;   // l0b_set_attention_decode_tensor_cores

__device__ __forceinline__ uint32_t pf_pack(float a, float b, bool bf) {
    if (bf) {
        const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&v);
    }
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float2 pf_unpack(uint32_t u, bool bf) {
    if (bf) return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
// hi = 16-bit (a, b); lo = 16-bit residuals.
__device__ __forceinline__ void pf_split(float a, float b, bool bf, uint32_t& hi, uint32_t& lo) {
    hi = pf_pack(a, b, bf);
    const float2 h = pf_unpack(hi, bf);
    lo = pf_pack(a - h.x, b - h.y, bf);
}
__device__ __forceinline__ void pf_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1, bool bf) {
    if (bf)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int HD, bool BF>
__global__ void __launch_bounds__(128) attn_prefill_mma_kernel(const AttnParams p, int rows) {
    constexpr int NT = HD / 8;    // 8-column tiles of the output
    constexpr int KS = HD / 16;   // 16-deep steps of Q K^T
    constexpr int RB = HD * 2;    // bytes per tile row
    constexpr int TILE = kPfBN * RB;
    extern __shared__ __align__(128) unsigned char pf_smem[];
    unsigned char* Ks = pf_smem;             // [2][kPfBN][HD] 16-bit, swizzled
    unsigned char* Vs = pf_smem + 2 * TILE;  // [2][kPfBN][HD]
    __shared__ int pmax_s[4];
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int h = blockIdx.y, kvh = h / (p.nh / p.nkv);
    const int r0 = blockIdx.x * kPfBM, wr = r0 + warp * 16;
    auto pos_of = [&](int b) { return b < rows ? (p.positions ? p.positions[b] : p.pos_base + b * p.pos_step) : -1; };
    // The largest position among the CTA's rows bounds the key walk.
    {
        int pm = -1;
        for (int b = r0 + threadIdx.x; b < r0 + kPfBM; b += 128) pm = max(pm, pos_of(b));
        for (int o = 16; o > 0; o >>= 1) pm = max(pm, __shfl_xor_sync(0xffffffffu, pm, o));
        if (lane == 0) pmax_s[warp] = pm;
    }
    __syncthreads();
    const int pmax = max(max(pmax_s[0], pmax_s[1]), max(pmax_s[2], pmax_s[3]));
    if (pmax < 0) return;
    const int pa = pos_of(wr + g), pb = pos_of(wr + g + 8);
    const int ntiles = pmax / kPfBN + 1;
    const char* kbase = static_cast<const char*>(p.kc) + static_cast<long long>(kvh) * HD * 2;
    const char* vbase = static_cast<const char*>(p.vc) + static_cast<long long>(kvh) * HD * 2;
    const long long row_stride = static_cast<long long>(p.kv_dim) * 2;
    // One key tile (and value tile) into stage st: 16-byte chunks, rows past pmax zero-filled.
    auto load_tile = [&](int j, int st) {
        for (int e = threadIdx.x; e < kPfBN * (HD / 8); e += 128) {
            const int r = e / (HD / 8), c = e - r * (HD / 8);
            const int slot = j * kPfBN + r;
            const uint32_t off = static_cast<uint32_t>(r * RB + ((c ^ (r & 7)) * 16));
            unsigned char* kd = Ks + st * TILE + off;
            unsigned char* vd = Vs + st * TILE + off;
            if (slot <= pmax) {
                const long long go = static_cast<long long>(slot) * row_stride + c * 16;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                                 __cvta_generic_to_shared(kd))),
                             "l"(kbase + go)
                             : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                                 __cvta_generic_to_shared(vd))),
                             "l"(vbase + go)
                             : "memory");
            } else {
                *reinterpret_cast<uint4*>(kd) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(vd) = make_uint4(0, 0, 0, 0);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_tile(0, 0);
    // Query fragments (rows g and g + 8 of this warp), scaled for exp2 and split into hi / lo halves.
    const float qs = p.scale * 1.4426950408889634f;
    uint32_t qh[KS][4], ql[KS][4];
    {
        const float* qa = pa >= 0 ? p.q + static_cast<long long>(wr + g) * p.q_bstride + static_cast<long long>(h) * HD : nullptr;
        const float* qb = pb >= 0 ? p.q + static_cast<long long>(wr + g + 8) * p.q_bstride + static_cast<long long>(h) * HD : nullptr;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            const int c0 = 16 * kk + 2 * t, c1 = c0 + 8;
            const float2 x0 = qa ? *reinterpret_cast<const float2*>(qa + c0) : make_float2(0.f, 0.f);
            const float2 x1 = qb ? *reinterpret_cast<const float2*>(qb + c0) : make_float2(0.f, 0.f);
            const float2 x2 = qa ? *reinterpret_cast<const float2*>(qa + c1) : make_float2(0.f, 0.f);
            const float2 x3 = qb ? *reinterpret_cast<const float2*>(qb + c1) : make_float2(0.f, 0.f);
            pf_split(x0.x * qs, x0.y * qs, BF, qh[kk][0], ql[kk][0]);
            pf_split(x1.x * qs, x1.y * qs, BF, qh[kk][1], ql[kk][1]);
            pf_split(x2.x * qs, x2.y * qs, BF, qh[kk][2], ql[kk][2]);
            pf_split(x3.x * qs, x3.y * qs, BF, qh[kk][3], ql[kk][3]);
        }
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
    // This warp's rows need tiles up to wmax / kPfBN. The skip test must be the same for every lane: the
    // MMA and ldmatrix below are warp-collective (.sync.aligned), so the bound is the warp-wide maximum.
    int wmax = max(pa, pb);
    for (int o = 16; o > 0; o >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (j + 1 < ntiles) {
            load_tile(j + 1, st ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        if (j * kPfBN <= wmax) {
            const unsigned char* kt = Ks + st * TILE;
            const unsigned char* vt = Vs + st * TILE;
            // S = Q K^T for the 64 slots of the tile: 8 tiles of 8 slots.
            float sc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
                const int r = nt * 8 + g;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kt + r * RB + (((2 * kk) ^ (r & 7)) * 16) + 4 * t);
                    const uint32_t b1 =
                        *reinterpret_cast<const uint32_t*>(kt + r * RB + (((2 * kk + 1) ^ (r & 7)) * 16) + 4 * t);
                    pf_mma(sc[nt], qh[kk][0], qh[kk][1], qh[kk][2], qh[kk][3], b0, b1, BF);
                    pf_mma(sc[nt], ql[kk][0], ql[kk][1], ql[kk][2], ql[kk][3], b0, b1, BF);
                }
            }
            // Mask and online softmax (rows g: sc[.][0..1], g + 8: sc[.][2..3]).
            float ta = -INFINITY, tb = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int s0 = j * kPfBN + nt * 8 + 2 * t;
                if (s0 > pa) sc[nt][0] = -INFINITY;
                if (s0 + 1 > pa) sc[nt][1] = -INFINITY;
                if (s0 > pb) sc[nt][2] = -INFINITY;
                if (s0 + 1 > pb) sc[nt][3] = -INFINITY;
                ta = fmaxf(ta, fmaxf(sc[nt][0], sc[nt][1]));
                tb = fmaxf(tb, fmaxf(sc[nt][2], sc[nt][3]));
            }
            ta = fmaxf(ta, __shfl_xor_sync(0xffffffffu, ta, 1));
            ta = fmaxf(ta, __shfl_xor_sync(0xffffffffu, ta, 2));
            tb = fmaxf(tb, __shfl_xor_sync(0xffffffffu, tb, 1));
            tb = fmaxf(tb, __shfl_xor_sync(0xffffffffu, tb, 2));
            const float na = fmaxf(ma, ta), nb = fmaxf(mb, tb);
            const float aa = na == -INFINITY ? 1.f : exp2f(ma - na);
            const float ab = nb == -INFINITY ? 1.f : exp2f(mb - nb);
            ma = na;
            mb = nb;
            float sa = 0.f, sb = 0.f;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                sc[nt][0] = na == -INFINITY ? 0.f : exp2f(sc[nt][0] - na);
                sc[nt][1] = na == -INFINITY ? 0.f : exp2f(sc[nt][1] - na);
                sc[nt][2] = nb == -INFINITY ? 0.f : exp2f(sc[nt][2] - nb);
                sc[nt][3] = nb == -INFINITY ? 0.f : exp2f(sc[nt][3] - nb);
                sa += sc[nt][0] + sc[nt][1];
                sb += sc[nt][2] + sc[nt][3];
            }
            la = la * aa + sa;
            lb = lb * ab + sb;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                o[n][0] *= aa;
                o[n][1] *= aa;
                o[n][2] *= ab;
                o[n][3] *= ab;
            }
            // O += P V: P of slots 16 kk .. 16 kk + 15 from score tiles 2 kk and 2 kk + 1.
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t ph[4], pl[4];
                pf_split(sc[2 * kk][0], sc[2 * kk][1], BF, ph[0], pl[0]);
                pf_split(sc[2 * kk][2], sc[2 * kk][3], BF, ph[1], pl[1]);
                pf_split(sc[2 * kk + 1][0], sc[2 * kk + 1][1], BF, ph[2], pl[2]);
                pf_split(sc[2 * kk + 1][2], sc[2 * kk + 1][3], BF, ph[3], pl[3]);
#pragma unroll
                for (int n = 0; n < NT; n += 2) {
                    // Transposed fragments of V rows 16 kk .. + 15, columns of output tiles n and n + 1.
                    const int r = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8;
                    const int c = n + (lane >> 4);
                    const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(vt + r * RB + ((c ^ (r & 7)) * 16)));
                    uint32_t v0, v1, v2, v3;
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                                 : "r"(addr));
                    pf_mma(o[n], ph[0], ph[1], ph[2], ph[3], v0, v1, BF);
                    pf_mma(o[n], pl[0], pl[1], pl[2], pl[3], v0, v1, BF);
                    pf_mma(o[n + 1], ph[0], ph[1], ph[2], ph[3], v2, v3, BF);
                    pf_mma(o[n + 1], pl[0], pl[1], pl[2], pl[3], v2, v3, BF);
                }
            }
        }
        __syncthreads();  // stage st is refilled by the next iteration's prefetch
    }
    la += __shfl_xor_sync(0xffffffffu, la, 1);
    la += __shfl_xor_sync(0xffffffffu, la, 2);
    lb += __shfl_xor_sync(0xffffffffu, lb, 1);
    lb += __shfl_xor_sync(0xffffffffu, lb, 2);
    const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
    float* oa = pa >= 0 ? p.out + static_cast<long long>(wr + g) * p.out_bstride + static_cast<long long>(h) * HD : nullptr;
    float* ob = pb >= 0 ? p.out + static_cast<long long>(wr + g + 8) * p.out_bstride + static_cast<long long>(h) * HD : nullptr;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const int c = n * 8 + 2 * t;
        if (oa) *reinterpret_cast<float2*>(oa + c) = make_float2(o[n][0] * ia, o[n][1] * ia);
        if (ob) *reinterpret_cast<float2*>(ob + c) = make_float2(o[n][2] * ib, o[n][3] * ib);
    }
}

// ---------------------------------------------------------------------------------------------
// Decode attention on the tensor cores (mma.sync m16n8k16, fp32 accumulators), in thread-block
// clusters like attn_cluster_kernel.
//
// CTA (KV head group of up to 16 query heads, split, sequence) walks its share of the positions in
// 64-position tiles (K and V rows copied raw by cp.async into two swizzled stages). The query heads are
// the MMA rows: warp w scores positions [16 w, 16 w + 16) of the tile for all of them (Q in hi + lo
// 16-bit fragments, scaled by log2 e for exp2), keeps its own online softmax (running max, sum and
// unnormalised output in registers) and adds P V with P split into hi + lo halves and V read by
// ldmatrix.trans -- about fp32 accuracy from 16-bit operands, as in the prefill kernel. The new
// position's key and value (RoPE applied, rounded to the cache type as the cache stores them) are
// written into the tile by the CTA that owns the position. After the walk the four warps' states meet
// in shared memory, then the cluster's splits meet through distributed shared memory as in the
// FMA kernel (CTA r merges head dimensions [r HD / S, (r + 1) HD / S)).
// ---------------------------------------------------------------------------------------------
constexpr int kDmBN = 64;      // positions per tile
constexpr int kDmHeads = 16;   // query heads per CTA (MMA rows)

template <int HD>
constexpr size_t decode_mma_smem() {
    return 4ull * kDmBN * HD * 2;  // two stages of K and V tiles (16-bit)
}

template <int HD, bool BF>
__global__ void __launch_bounds__(128) attn_decode_mma_kernel(const AttnParams p) {
    namespace cg = cooperative_groups;
    constexpr int NT = HD / 8;    // 8-column output tiles
    constexpr int KS = HD / 16;   // 16-deep steps of Q K^T
    constexpr int RB = HD * 2;    // bytes per tile row
    constexpr int TILE = kDmBN * RB;
    extern __shared__ __align__(128) unsigned char dm_smem[];
    unsigned char* Ks = dm_smem;             // [2][kDmBN][HD] 16-bit, 16-byte chunks swizzled by row
    unsigned char* Vs = dm_smem + 2 * TILE;  // [2][kDmBN][HD]
    __shared__ __align__(16) float qn_s[kDmHeads][HD];   // rotated queries; after the walk, the CTA output
    __shared__ float m_s[kDmHeads], l_s[kDmHeads];      // CTA state (log2 units) for the cluster merge
    __shared__ float wm_s[4][kDmHeads], wl_s[4][kDmHeads];
    __shared__ float cs_s[HD / 2], sn_s[HD / 2];
    __shared__ __align__(16) uint16_t knew_s[HD], vnew_s[HD];

    cg::cluster_group cluster = cg::this_cluster();
    const int G = p.nh / p.nkv;
    const int gparts = (G + kDmHeads - 1) / kDmHeads;
    const int kvh = blockIdx.x / gparts, gp = blockIdx.x - (blockIdx.x / gparts) * gparts;
    const int h0 = kvh * G + gp * kDmHeads;
    const int ng = min(kDmHeads, G - gp * kDmHeads);
    const int S = gridDim.y, split = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;

    pdl_wait();
    const int qpos = p.positions ? p.positions[b] : p.pos_base + b * p.pos_step;
    const int seq = qpos + 1;
    int chunk = ((seq + S - 1) / S + kDmBN - 1) / kDmBN * kDmBN;
    chunk = max(chunk, p.chunk);
    const int nact = (seq + chunk - 1) / chunk;
    const bool active = split < nact;
    pdl_launch_dependents();
    const int p_begin = split * chunk;
    const int p_end = active ? min(seq, p_begin + chunk) : p_begin;
    const bool owns_new = p.store_new && active && split == nact - 1;
    const int ntiles = (p_end - p_begin + kDmBN - 1) / kDmBN;
    const long long row_stride = static_cast<long long>(p.kv_dim) * 2;
    const char* kbase = static_cast<const char*>(p.kc) + (b * p.cache_bstride + static_cast<long long>(kvh) * HD) * 2;
    const char* vbase = static_cast<const char*>(p.vc) + (b * p.cache_bstride + static_cast<long long>(kvh) * HD) * 2;

    // One K tile and V tile into stage st: 16-byte chunks, slots past the split zero-filled. The new
    // position's row is left alone in tile 0 (patched from knew_s / vnew_s once they exist, before the
    // first barrier that publishes the tile) and copied from them in later tiles.
    const int qslot = owns_new ? qpos - p_begin : -1;  // the new position's slot in the CTA's range
    auto load_tile = [&](int j, int st) {
        for (int e = tid; e < kDmBN * (HD / 8); e += 128) {
            const int r = e / (HD / 8), c = e - (e / (HD / 8)) * (HD / 8);
            const int pos = p_begin + j * kDmBN + r;
            const uint32_t off = static_cast<uint32_t>(r * RB + ((c ^ (r & 7)) * 16));
            unsigned char* kd = Ks + st * TILE + off;
            unsigned char* vd = Vs + st * TILE + off;
            if (j * kDmBN + r == qslot) {
                if (j > 0) {
                    *reinterpret_cast<uint4*>(kd) = *reinterpret_cast<const uint4*>(knew_s + 8 * c);
                    *reinterpret_cast<uint4*>(vd) = *reinterpret_cast<const uint4*>(vnew_s + 8 * c);
                }
            } else if (pos < p_end) {
                const long long go = static_cast<long long>(pos) * row_stride + c * 16;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                                 __cvta_generic_to_shared(kd))),
                             "l"(kbase + go)
                             : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(
                                 __cvta_generic_to_shared(vd))),
                             "l"(vbase + go)
                             : "memory");
            } else {
                *reinterpret_cast<uint4*>(kd) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(vd) = make_uint4(0, 0, 0, 0);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (ntiles > 0) load_tile(0, 0);  // in flight during the prologue

    // Raw queries of the group (rows past ng zero), one 16-byte load each, all issued before any store.
    const float* qb = p.q + b * p.q_bstride + static_cast<long long>(h0) * HD;
    {
        constexpr int PER = kDmHeads * HD / 4 / 128;  // float4s per thread
        float4 v[PER];
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int idx = tid + i * 128, j = idx / (HD / 4);
            v[i] = j < ng ? *reinterpret_cast<const float4*>(qb + 4 * idx) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int i = 0; i < PER; ++i) reinterpret_cast<float4*>(&qn_s[0][0])[tid + i * 128] = v[i];
    }
    if (p.rope) {
        for (int i = tid; i < p.rot / 2; i += 128) {
            const float ang = __fmul_rn(static_cast<float>(qpos), p.inv_freq[i]);
            float sv, cv;
            sincosf(ang, &sv, &cv);
            cs_s[i] = __fmul_rn(cv, p.attn_scale);
            sn_s[i] = __fmul_rn(sv, p.attn_scale);
        }
    }
    __syncthreads();
    // RoPE on the queries in place, one (d, d + rot / 2) pair per step.
    if (p.rope) {
        const int half = p.rot >> 1;
        for (int idx = tid; idx < ng * half; idx += 128) {
            const int j = idx / half, i = idx - (idx / half) * half;
            const float x1 = qn_s[j][i], x2 = qn_s[j][i + half], c = cs_s[i], sn = sn_s[i];
            qn_s[j][i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
            qn_s[j][i + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
        }
    }
    // The new key (rotated) and value, rounded to the cache type; the group-0 CTA stores them, and the
    // owner patches tile 0's slot when the new position lies in it.
    if (owns_new) {
        const float* kb = p.k_new + b * p.new_bstride + static_cast<long long>(kvh) * HD;
        const float* vb = p.v_new + b * p.new_bstride + static_cast<long long>(kvh) * HD;
        for (int d = tid; d < HD; d += 128) {
            const float kv = p.rope ? rope_elem(kb, d, p.rot, cs_s, sn_s) : kb[d];
            const float vv = vb[d];
            uint16_t kbits, vbits;
            if (BF) {
                const __nv_bfloat16 kh = __float2bfloat16_rn(kv), vh = __float2bfloat16_rn(vv);
                kbits = *reinterpret_cast<const uint16_t*>(&kh);
                vbits = *reinterpret_cast<const uint16_t*>(&vh);
            } else {
                const __half kh = __float2half_rn(kv), vh = __float2half_rn(vv);
                kbits = *reinterpret_cast<const uint16_t*>(&kh);
                vbits = *reinterpret_cast<const uint16_t*>(&vh);
            }
            knew_s[d] = kbits;
            vnew_s[d] = vbits;
            if (gp == 0) {
                const long long off = b * p.cache_bstride + static_cast<long long>(qpos) * p.kv_dim +
                                      static_cast<long long>(kvh) * HD + d;
                static_cast<uint16_t*>(p.kc)[off] = kbits;
                static_cast<uint16_t*>(p.vc)[off] = vbits;
            }
        }
        __syncthreads();
        if (qslot < kDmBN) {
            for (int c = tid; c < HD / 8; c += 128) {
                const uint32_t off = static_cast<uint32_t>(qslot * RB + ((c ^ (qslot & 7)) * 16));
                *reinterpret_cast<uint4*>(Ks + off) = *reinterpret_cast<const uint4*>(knew_s + 8 * c);
                *reinterpret_cast<uint4*>(Vs + off) = *reinterpret_cast<const uint4*>(vnew_s + 8 * c);
            }
        }
    }
    __syncthreads();
    const float qsc = p.scale * 1.4426950408889634f;
    uint32_t qh[KS][4], ql[KS][4];
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
        const int c0 = 16 * kk + 2 * t, c1 = c0 + 8;
        pf_split(qn_s[g][c0] * qsc, qn_s[g][c0 + 1] * qsc, BF, qh[kk][0], ql[kk][0]);
        pf_split(qn_s[g + 8][c0] * qsc, qn_s[g + 8][c0 + 1] * qsc, BF, qh[kk][1], ql[kk][1]);
        pf_split(qn_s[g][c1] * qsc, qn_s[g][c1 + 1] * qsc, BF, qh[kk][2], ql[kk][2]);
        pf_split(qn_s[g + 8][c1] * qsc, qn_s[g + 8][c1 + 1] * qsc, BF, qh[kk][3], ql[kk][3]);
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
    for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        if (j + 1 < ntiles) {
            load_tile(j + 1, st ^ 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int w0 = p_begin + j * kDmBN + 16 * warp;  // this warp's first position (warp-uniform)
        if (w0 < p_end) {
            const unsigned char* kt = Ks + st * TILE;
            const unsigned char* vt = Vs + st * TILE;
            // S = Q K^T for the warp's 16 positions: two tiles of 8.
            float sc[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
                const int r = 16 * warp + nt * 8 + g;
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kt + r * RB + (((2 * kk) ^ (r & 7)) * 16) + 4 * t);
                    const uint32_t b1 =
                        *reinterpret_cast<const uint32_t*>(kt + r * RB + (((2 * kk + 1) ^ (r & 7)) * 16) + 4 * t);
                    pf_mma(sc[nt], qh[kk][0], qh[kk][1], qh[kk][2], qh[kk][3], b0, b1, BF);
                    pf_mma(sc[nt], ql[kk][0], ql[kk][1], ql[kk][2], ql[kk][3], b0, b1, BF);
                }
            }
            // Positions past the split; online softmax over heads g (sc[.][0..1]) and g + 8 (sc[.][2..3]).
            float ta = -INFINITY, tb = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const int s0 = w0 + nt * 8 + 2 * t;
                if (s0 >= p_end) sc[nt][0] = sc[nt][2] = -INFINITY;
                if (s0 + 1 >= p_end) sc[nt][1] = sc[nt][3] = -INFINITY;
                ta = fmaxf(ta, fmaxf(sc[nt][0], sc[nt][1]));
                tb = fmaxf(tb, fmaxf(sc[nt][2], sc[nt][3]));
            }
            ta = fmaxf(ta, __shfl_xor_sync(0xffffffffu, ta, 1));
            ta = fmaxf(ta, __shfl_xor_sync(0xffffffffu, ta, 2));
            tb = fmaxf(tb, __shfl_xor_sync(0xffffffffu, tb, 1));
            tb = fmaxf(tb, __shfl_xor_sync(0xffffffffu, tb, 2));
            const float na = fmaxf(ma, ta), nb = fmaxf(mb, tb);
            const float aa = na == -INFINITY ? 1.f : exp2f(ma - na);
            const float ab = nb == -INFINITY ? 1.f : exp2f(mb - nb);
            ma = na;
            mb = nb;
            float sa = 0.f, sb = 0.f;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                sc[nt][0] = na == -INFINITY ? 0.f : exp2f(sc[nt][0] - na);
                sc[nt][1] = na == -INFINITY ? 0.f : exp2f(sc[nt][1] - na);
                sc[nt][2] = nb == -INFINITY ? 0.f : exp2f(sc[nt][2] - nb);
                sc[nt][3] = nb == -INFINITY ? 0.f : exp2f(sc[nt][3] - nb);
                sa += sc[nt][0] + sc[nt][1];
                sb += sc[nt][2] + sc[nt][3];
            }
            la = la * aa + sa;
            lb = lb * ab + sb;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                o[n][0] *= aa;
                o[n][1] *= aa;
                o[n][2] *= ab;
                o[n][3] *= ab;
            }
            // O += P V over the warp's 16 positions (one 16-deep step).
            uint32_t ph[4], pl[4];
            pf_split(sc[0][0], sc[0][1], BF, ph[0], pl[0]);
            pf_split(sc[0][2], sc[0][3], BF, ph[1], pl[1]);
            pf_split(sc[1][0], sc[1][1], BF, ph[2], pl[2]);
            pf_split(sc[1][2], sc[1][3], BF, ph[3], pl[3]);
#pragma unroll
            for (int n = 0; n < NT; n += 2) {
                const int r = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int c = n + (lane >> 4);
                const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(vt + r * RB + ((c ^ (r & 7)) * 16)));
                uint32_t v0, v1, v2, v3;
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                             : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                             : "r"(addr));
                pf_mma(o[n], ph[0], ph[1], ph[2], ph[3], v0, v1, BF);
                pf_mma(o[n], pl[0], pl[1], pl[2], pl[3], v0, v1, BF);
                pf_mma(o[n + 1], ph[0], ph[1], ph[2], ph[3], v2, v3, BF);
                pf_mma(o[n + 1], pl[0], pl[1], pl[2], pl[3], v2, v3, BF);
            }
        }
        __syncthreads();  // stage st is refilled by the next iteration's prefetch
    }
    // The four warps' states meet in shared memory: (max, sum) per head, and each warp's output scaled by
    // its weight 2^(m_w - M) into the free stage buffers (every copy has landed; the loop ended on a
    // barrier), summed in warp order into qn_s, the CTA's unnormalised output.
    la += __shfl_xor_sync(0xffffffffu, la, 1);
    la += __shfl_xor_sync(0xffffffffu, la, 2);
    lb += __shfl_xor_sync(0xffffffffu, lb, 1);
    lb += __shfl_xor_sync(0xffffffffu, lb, 2);
    if (t == 0) {
        wm_s[warp][g] = ma;
        wm_s[warp][g + 8] = mb;
        wl_s[warp][g] = la;
        wl_s[warp][g + 8] = lb;
    }
    __syncthreads();
    {
        float Ma = -INFINITY, Mb = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) Ma = fmaxf(Ma, wm_s[w][g]), Mb = fmaxf(Mb, wm_s[w][g + 8]);
        const float wa = ma == -INFINITY ? 0.f : exp2f(ma - Ma);
        const float wb = mb == -INFINITY ? 0.f : exp2f(mb - Mb);
        if (warp == 0 && t == 0) {
            float La = 0.f, Lb = 0.f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                if (wm_s[w][g] != -INFINITY) La = fmaf(exp2f(wm_s[w][g] - Ma), wl_s[w][g], La);
                if (wm_s[w][g + 8] != -INFINITY) Lb = fmaf(exp2f(wm_s[w][g + 8] - Mb), wl_s[w][g + 8], Lb);
            }
            m_s[g] = Ma;
            m_s[g + 8] = Mb;
            l_s[g] = La;
            l_s[g + 8] = Lb;
        }
        float* wo = reinterpret_cast<float*>(dm_smem) + static_cast<size_t>(warp) * kDmHeads * HD;  // [16][HD]
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int c = n * 8 + 2 * t;
            *reinterpret_cast<float2*>(wo + g * HD + c) = make_float2(wa * o[n][0], wa * o[n][1]);
            *reinterpret_cast<float2*>(wo + (g + 8) * HD + c) = make_float2(wb * o[n][2], wb * o[n][3]);
        }
    }
    __syncthreads();
    {
        const float4* w4 = reinterpret_cast<const float4*>(dm_smem);
        constexpr int Q4 = kDmHeads * HD / 4;  // float4s per warp's output
        for (int i = tid; i < Q4; i += 128) {
            const float4 a0 = w4[i], a1 = w4[Q4 + i], a2 = w4[2 * Q4 + i], a3 = w4[3 * Q4 + i];
            reinterpret_cast<float4*>(&qn_s[0][0])[i] = make_float4(((a0.x + a1.x) + a2.x) + a3.x, ((a0.y + a1.y) + a2.y) + a3.y,
                                                                     ((a0.z + a1.z) + a2.z) + a3.z, ((a0.w + a1.w) + a2.w) + a3.w);
        }
    }
    __syncthreads();
    // Merge the cluster's splits: this CTA's slice of head dimensions from the nact active partials.
    auto peer = [&](float* ptr, int s) { return S > 1 ? cluster.map_shared_rank(ptr, s) : ptr; };
    if (S > 1) cluster.sync();
    const int dper = HD / S;
    for (int o2 = tid; o2 < ng * dper; o2 += 128) {
        const int j = o2 / dper, d = split * dper + (o2 - (o2 / dper) * dper);
        float mv[kMaxClusterSplits], lv[kMaxClusterSplits], av[kMaxClusterSplits];
        float mmax = -INFINITY;
#pragma unroll
        for (int s2 = 0; s2 < kMaxClusterSplits; ++s2) {
            mv[s2] = -INFINITY, lv[s2] = 0.f, av[s2] = 0.f;
            if (s2 < nact) {
                mv[s2] = *peer(&m_s[j], s2);
                lv[s2] = *peer(&l_s[j], s2);
                av[s2] = *peer(&qn_s[j][d], s2);
            }
        }
#pragma unroll
        for (int s2 = 0; s2 < kMaxClusterSplits; ++s2) mmax = fmaxf(mmax, mv[s2]);
        float lsum = 0.f, y = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < kMaxClusterSplits; ++s2) {
            if (s2 < nact && mv[s2] != -INFINITY) {
                const float w = exp2f(mv[s2] - mmax);
                lsum = fmaf(w, lv[s2], lsum);
                y = fmaf(w, av[s2], y);
            }
        }
        p.out[b * p.out_bstride + static_cast<long long>(h0 + j) * HD + d] = y / lsum;
    }
    if (S > 1) cluster.sync();
}

template <int HD, bool BF>
l0b_status launch_prefill_mma(l0b_device* d, cudaStream_t stream, const AttnParams& p, int rows) {
    constexpr size_t smem = 4ull * kPfBN * HD * 2;
    auto kernel = attn_prefill_mma_kernel<HD, BF>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        configured = true;
    }
    const dim3 grid((rows + kPfBM - 1) / kPfBM, p.nh);
    if (d) return d->launch(kernel, grid, dim3(128), smem, p, rows);
    kernel<<<grid, 128, smem, stream>>>(p, rows);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    add_launches(1);
    return L0B_OK;
}

// The tensor-core prefill kernel applies: f16 / bf16 caches with 16-byte aligned rows, head dim 64 or
// 128, query rows 8-byte aligned (float2 reads), and a query block (prefill, not one decode row).
bool prefill_mma_applies(const AttnParams& p, int rows) {
    if (!g_attn_prefill_mma || rows < 2 || p.rope || p.store_new || p.cache_bstride != 0) return false;
    if (p.cache_dtype != L0B_F16 && p.cache_dtype != L0B_BF16) return false;
    if (p.hd != 64 && p.hd != 128) return false;
    if ((p.kv_dim * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(p.kc) % 16 || reinterpret_cast<uintptr_t>(p.vc) % 16)
        return false;
    if (reinterpret_cast<uintptr_t>(p.q) % 8 || p.q_bstride % 2 || reinterpret_cast<uintptr_t>(p.out) % 8 ||
        p.out_bstride % 2)
        return false;
    return true;
}

l0b_status attention_prefill_mma(l0b_device* d, cudaStream_t stream, const AttnParams& p, int rows) {
    const bool bf = p.cache_dtype == L0B_BF16;
    if (p.hd == 64) return bf ? launch_prefill_mma<64, true>(d, stream, p, rows) : launch_prefill_mma<64, false>(d, stream, p, rows);
    return bf ? launch_prefill_mma<128, true>(d, stream, p, rows) : launch_prefill_mma<128, false>(d, stream, p, rows);
}

l0b_status attention_any(l0b_device* d, cudaStream_t stream, const AttnParams& p, int batch) {
    L0B_REQUIRE(p.nkv > 0 && p.nh % p.nkv == 0, L0B_ERR_ARGUMENT, "heads %d not a multiple of kv heads %d", p.nh,
                p.nkv);
    L0B_REQUIRE(p.chunk > 0 && p.max_splits > 0, L0B_ERR_ARGUMENT, "bad split configuration");
    if (p.max_splits == 1 && prefill_mma_applies(p, batch)) return attention_prefill_mma(d, stream, p, batch);
    const int G = p.nh / p.nkv;
    const int gparts = (G + kMaxG - 1) / kMaxG;
    dim3 grid(p.nkv * gparts, p.max_splits, batch);
    switch (p.hd) {
        case 64: return launch_attn(d, stream, attn_kernel<64>, grid, p);
        case 128: return launch_attn(d, stream, attn_kernel<128>, grid, p);
        default: return fail(L0B_ERR_UNSUPPORTED, "attention head_dim %d is not supported (64, 128)", p.hd);
    }
}

// Whether clusters of 16 CTAs (beyond the portable 8) of the cluster kernel can be resident: sets the
// non-portable attribute on both instantiations and asks the occupancy calculator once per process.
bool cluster16_ok() {
    static std::once_flag once;
    static bool ok = false;
    std::call_once(once, [] {
        const void* fns[2] = {reinterpret_cast<const void*>(attn_cluster_kernel<64>),
                              reinterpret_cast<const void*>(attn_cluster_kernel<128>)};
        bool all = true;
        for (const void* f : fns) {
            if (cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
                all = false;
                break;
            }
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(1, kMaxClusterSplits, 1);
            cfg.blockDim = dim3(kClusterThreads);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 1;
            attr[0].val.clusterDim.y = kMaxClusterSplits;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, f, &cfg) != cudaSuccess || clusters < 1) {
                all = false;
                break;
            }
        }
        cudaGetLastError();
        ok = all;
    });
    return ok;
}

template <typename F>
l0b_status launch_attn_cluster(l0b_device* d, cudaStream_t stream, F kernel, dim3 grid, int S, const AttnParams& p) {
    if (d) return d->launch_cluster(kernel, grid, dim3(kClusterThreads), 0, S, p);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kClusterThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (S > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = S;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
    if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    add_launches(1);
    return L0B_OK;
}

// The tensor-core decode kernel: its shared-memory limit set per device, then launched in clusters of S.
template <int HD, bool BF>
l0b_status launch_decode_mma(l0b_device* d, cudaStream_t stream, const AttnParams& p, int batch, int S) {
    constexpr size_t smem = decode_mma_smem<HD>();
    auto kernel = attn_decode_mma_kernel<HD, BF>;
    {
        static bool configured[64] = {};
        static std::mutex mu;
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[dev]) {
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
            configured[dev] = true;
        }
    }
    const int gparts = (p.nh / p.nkv + kDmHeads - 1) / kDmHeads;
    const dim3 grid(p.nkv * gparts, S, batch);
    if (d) return d->launch_cluster(kernel, grid, dim3(128), smem, S, p);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (S > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = S;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
    if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    add_launches(1);
    return L0B_OK;
}

// Decode on the tensor-core kernel: f16 / bf16 caches, head dim 64 or 128, 16-byte aligned rows.
bool decode_mma_applies(const AttnParams& p) {
    if (!g_attn_decode_mma || (p.cache_dtype != L0B_F16 && p.cache_dtype != L0B_BF16)) return false;
    if (p.hd != 64 && p.hd != 128) return false;
    if ((p.kv_dim * 2) % 16 != 0 || (p.cache_bstride * 2) % 16 != 0) return false;
    return (reinterpret_cast<uintptr_t>(p.kc) | reinterpret_cast<uintptr_t>(p.vc)) % 16 == 0;
}

l0b_status attention_cluster_any(l0b_device* d, cudaStream_t stream, const AttnParams& p, int batch, int splits) {
    L0B_REQUIRE(p.nkv > 0 && p.nh % p.nkv == 0, L0B_ERR_ARGUMENT, "heads %d not a multiple of kv heads %d", p.nh,
                p.nkv);
    L0B_REQUIRE(splits == 1 || splits == 2 || splits == 4 || splits == 8 || (splits == 16 && cluster16_ok()),
                L0B_ERR_ARGUMENT, "cluster splits %d (1, 2, 4, 8, or 16 where the device runs such clusters)", splits);
    if (decode_mma_applies(p)) {
        const bool bf = p.cache_dtype == L0B_BF16;
        if (p.hd == 64) return bf ? launch_decode_mma<64, true>(d, stream, p, batch, splits)
                                  : launch_decode_mma<64, false>(d, stream, p, batch, splits);
        return bf ? launch_decode_mma<128, true>(d, stream, p, batch, splits)
                  : launch_decode_mma<128, false>(d, stream, p, batch, splits);
    }
    const int G = p.nh / p.nkv;
    const int gparts = (G + kMaxG - 1) / kMaxG;
    dim3 grid(p.nkv * gparts, splits, batch);
    switch (p.hd) {
        case 64: return launch_attn_cluster(d, stream, attn_cluster_kernel<64>, grid, splits, p);
        case 128: return launch_attn_cluster(d, stream, attn_cluster_kernel<128>, grid, splits, p);
        default: return fail(L0B_ERR_UNSUPPORTED, "attention head_dim %d is not supported (64, 128)", p.hd);
    }
}

}  // namespace

l0b_status attention_launch(l0b_device* d, const AttnParams& p, int batch) {
    return attention_any(d, d->stream, p, batch);
}

l0b_status attention_launch_stream(cudaStream_t stream, const AttnParams& p, int batch) {
    return attention_any(nullptr, stream, p, batch);
}

l0b_status attention_cluster_launch(l0b_device* d, const AttnParams& p, int batch, int splits) {
    return attention_cluster_any(d, d->stream, p, batch, splits);
}

int attention_cluster_splits(int max_seq, int work_items, int sm_count) {
    // Enough CTAs for about two per SM, and no split that the longest sequence cannot reach; at most
    // 16 (the non-portable cluster size) where the device can hold such clusters, else the portable 8.
    int s = g_attn_cluster16 && cluster16_ok() ? kMaxClusterSplits : 8;
    while (s > 1 && (static_cast<long long>(work_items) * s > 2LL * sm_count || 32LL * (s / 2) >= max_seq)) s >>= 1;
    return s;
}

size_t attention_part_floats(int batch, int nh, int max_splits, int hd) {
    return static_cast<size_t>(batch) * nh * max_splits * (hd + 2);
}

// ---------------------------------------------------------------------------------------------
// Decode attention for callers that cannot allocate device memory.
//
// The split-KV kernel needs scratch for its per-split partials and its merge counters. The regular
// entry point takes it from the device's scratch, which grows with cudaMalloc. Some callers cannot let
// a call allocate: a serving process that plans every byte of HBM at start-up, code that runs while a
// memory pool or another runtime owns the allocator, or a host (such as a managed-language façade)
// that must not have a call block in the allocator mid-step. This variant keeps its scratch in fixed
// arrays compiled into the library instead: 4 MiB of partials and 4096 counters per GPU that loads the
// library, held until the process exits.
// ---------------------------------------------------------------------------------------------

constexpr int kNoAllocPartFloats = 1 << 20;  // 4 MiB
constexpr int kNoAllocCounters = 4096;

static __device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
static __device__ __align__(256) unsigned g_noalloc_counters[kNoAllocCounters];

}  // namespace l0b

namespace {

// Device addresses of the two arrays, looked up once per device (the names are host stand-ins). The
// lookup runs under a mutex so two host threads making their first call on one device do not race.
struct NoAllocAddrs {
    bool ready = false;
    float* part = nullptr;
    unsigned* counters = nullptr;
};
NoAllocAddrs g_noalloc_addrs[64];
std::mutex g_noalloc_mutex;

}  // namespace

extern "C" L0B_API l0b_status l0b_set_attention_prefill_tensor_cores(int32_t enable) {
    l0b::g_attn_prefill_mma = enable != 0;
    return L0B_OK;
}

extern "C" L0B_API l0b_status l0b_set_attention_decode_tensor_cores(int32_t enable) {
    l0b::g_attn_decode_mma = enable != 0;
    return L0B_OK;
}

extern "C" L0B_API l0b_status l0b_set_attention_cluster16(int32_t enable) {
    l0b::g_attn_cluster16 = enable != 0;
    return L0B_OK;
}

extern "C" L0B_API l0b_status l0b_attention_decode_noalloc(void* stream, const float* q, const void* kc, const void* vc,
                                                         int32_t cache_dtype, float* out, int32_t head_dim,
                                                         int32_t n_heads, int32_t n_kv_heads, int32_t seq_len,
                                                         int32_t max_seq) {
    using namespace l0b;
    L0B_REQUIRE(q && kc && vc && out, L0B_ERR_ARGUMENT, "null pointer");
    L0B_REQUIRE(head_dim == 64 || head_dim == 128, L0B_ERR_UNSUPPORTED, "head_dim %d (64 or 128)", head_dim);
    L0B_REQUIRE(n_kv_heads > 0 && n_heads > 0 && n_heads % n_kv_heads == 0, L0B_ERR_ARGUMENT,
                "heads %d / kv heads %d", n_heads, n_kv_heads);
    L0B_REQUIRE(seq_len > 0 && seq_len <= max_seq, L0B_ERR_OUT_OF_RANGE, "seqLen %d outside (0, maxSeq %d]", seq_len,
                max_seq);
    L0B_REQUIRE(cache_dtype == L0B_F32 || cache_dtype == L0B_F16 || cache_dtype == L0B_BF16, L0B_ERR_ARGUMENT,
                "cache dtype %d", cache_dtype);
    const int gparts = (n_heads / n_kv_heads + kMaxG - 1) / kMaxG;
    const long long per_split = static_cast<long long>(n_heads) * (head_dim + 2);
    L0B_REQUIRE(per_split <= kNoAllocPartFloats && static_cast<long long>(n_kv_heads) * gparts <= kNoAllocCounters,
                L0B_ERR_OUT_OF_RANGE,
                "the fixed scratch holds %d partial floats and %d counters; %d heads of dim %d need %lld and %lld",
                kNoAllocPartFloats, kNoAllocCounters, n_heads, head_dim, per_split,
                static_cast<long long>(n_kv_heads) * gparts);
    int dev = 0;
    L0B_CHECK_CUDA(cudaGetDevice(&dev));
    L0B_REQUIRE(dev >= 0 && dev < 64, L0B_ERR_OUT_OF_RANGE, "device ordinal %d", dev);
    NoAllocAddrs a;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        NoAllocAddrs& slot = g_noalloc_addrs[dev];
        if (!slot.ready) {
            // First call on this device: resolve the arrays' device addresses (no allocation; the module
            // is already loaded). Make this first call before any stream capture on the device.
            float* part = nullptr;
            unsigned* counters = nullptr;
            L0B_CHECK_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&part), g_noalloc_part));
            L0B_CHECK_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&counters), g_noalloc_counters));
            slot.part = part;
            slot.counters = counters;
            slot.ready = true;
        }
        a = slot;
    }
    // As many splits as fit the fixed partials (and no more than the positions need).
    int chunk = 64;
    while (true) {
        const long long splits = (seq_len + chunk - 1) / chunk;
        if (splits * per_split <= kNoAllocPartFloats) break;
        chunk *= 2;
    }
    const int splits = (seq_len + chunk - 1) / chunk;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The counters must start at zero; a call that stopped early could have left them set.
    L0B_CHECK_CUDA(cudaMemsetAsync(a.counters, 0, sizeof(unsigned) * n_kv_heads * gparts, s));
    AttnParams p = {};
    p.q = q;
    p.q_bstride = static_cast<long long>(n_heads) * head_dim;
    p.kc = const_cast<void*>(kc);
    p.vc = const_cast<void*>(vc);
    p.cache_dtype = cache_dtype;
    p.kv_dim = n_kv_heads * head_dim;
    p.pos_base = seq_len - 1;
    p.out = out;
    p.out_bstride = static_cast<long long>(n_heads) * head_dim;
    p.part = a.part;
    p.part_ml = a.part + static_cast<long long>(n_heads) * splits * head_dim;
    p.counters = a.counters;
    p.nh = n_heads;
    p.nkv = n_kv_heads;
    p.hd = head_dim;
    p.chunk = chunk;
    p.max_splits = splits;
    p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)));
    return attention_launch_stream(s, p, 1);
}

namespace l0b {

void attention_pick_split(int max_seq, int work_items, int sm_count, int* chunk, int* max_splits) {
    (void)work_items;
    (void)sm_count;
    // One 32-position tile per CTA up to 4096 positions (most CTAs, shortest critical path), longer
    // splits beyond so the merge stays short.
    int c = max_seq <= 4096 ? 32 : max_seq <= 16384 ? 64 : 128;
    *chunk = c;
    *max_splits = (max_seq + c - 1) / c;
}

}  // namespace l0b
