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

#include "common.cuh"
#include "ops.cuh"

namespace l0b {

namespace {

constexpr int kT = 32;     // positions per tile
constexpr int kMaxG = 8;   // query heads per CTA
constexpr int kClusterThreads = 256;  // threads of the cluster decode kernel

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
// The S splits of one (query row, KV head group) form one cluster of (1, S, 1) CTAs, S <= 8. Each
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
        float mv[8], lv[8], av[8];
        float mmax = kNegInf;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            mv[s] = kNegInf, lv[s] = 0.f, av[s] = 0.f;
            if (s < nact) {
                mv[s] = *peer(&m_s[j], s);
                lv[s] = *peer(&l_s[j], s);
                av[s] = *peer(&acc_s[j][d], s);
            }
        }
#pragma unroll
        for (int s = 0; s < 8; ++s) mmax = fmaxf(mmax, mv[s]);
        float lsum = 0.f, y = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
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

l0b_status attention_any(l0b_device* d, cudaStream_t stream, const AttnParams& p, int batch) {
    L0B_REQUIRE(p.nkv > 0 && p.nh % p.nkv == 0, L0B_ERR_ARGUMENT, "heads %d not a multiple of kv heads %d", p.nh,
                p.nkv);
    L0B_REQUIRE(p.chunk > 0 && p.max_splits > 0, L0B_ERR_ARGUMENT, "bad split configuration");
    const int G = p.nh / p.nkv;
    const int gparts = (G + kMaxG - 1) / kMaxG;
    dim3 grid(p.nkv * gparts, p.max_splits, batch);
    switch (p.hd) {
        case 64: return launch_attn(d, stream, attn_kernel<64>, grid, p);
        case 128: return launch_attn(d, stream, attn_kernel<128>, grid, p);
        default: return fail(L0B_ERR_UNSUPPORTED, "attention head_dim %d is not supported (64, 128)", p.hd);
    }
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

l0b_status attention_cluster_any(l0b_device* d, cudaStream_t stream, const AttnParams& p, int batch, int splits) {
    L0B_REQUIRE(p.nkv > 0 && p.nh % p.nkv == 0, L0B_ERR_ARGUMENT, "heads %d not a multiple of kv heads %d", p.nh,
                p.nkv);
    L0B_REQUIRE(splits == 1 || splits == 2 || splits == 4 || splits == 8, L0B_ERR_ARGUMENT,
                "cluster splits %d (1, 2, 4 or 8)", splits);
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
    // the portable cluster size of 8.
    int s = 8;
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
