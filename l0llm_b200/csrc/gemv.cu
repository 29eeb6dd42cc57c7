// Weight-streaming linear layers for decode and small batches (sm_100a).
//
// Layout: W is [N, K] row-major (HuggingFace [out, in]); every output row is one contiguous stream.
// Two kernels. The tensor-core kernel further below (gemv_mma_kernel) takes 16-bit weights and int8
// with one scale per row, up to 8 activation rows; the fp32-FMA kernel described here takes the rest
// (fp32 weights, int8 with group scales, longer activation rows).
//
// A warp owns RPW rows (for SwiGLU a gate row and its up row); each lane reads 16 bytes per row per
// step with a no-L1-allocate 128-bit load, so a warp step moves 512 contiguous bytes per row. int8
// weights are dequantised in registers (exact byte -> fp32 trick, see dequant4) and multiplied with
// scalar fp32 FMAs; per-lane partial sums are reduced with warp shuffles. Activations are
// staged once per CTA in shared memory as fp32, permuted lane-major so the 128-bit shared loads are
// conflict-free, and optionally RMS-normalised on the way in (fused input/post-attention norm).
//
// The grid is persistent (CTAs = SMs x resident CTAs per SM) and each warp walks its row blocks as one
// flattened stream of (block, 512-byte chunk) steps through a register ring D steps deep: the loads of
// step s + D are issued while step s is multiplied, and row-block epilogues run in the stream. The
// first D steps are issued before griddepcontrol.wait -- weights never depend on the previous kernel
// -- so under programmatic dependent launch the weight stream starts while the producer of x drains.
#include <climits>
#include <cooperative_groups.h>
#include <cstring>

#include "common.cuh"
#include "gemv.cuh"

namespace l0b {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRing = 4;  // weight steps in flight per warp

// Position of element r (0 <= r < 32*VEC) of a 32*VEC-element chunk in the lane-major smem layout:
// the j-th float4 of lane l lives at j*128 + l*4.
template <int VEC>
__device__ __forceinline__ int xs_perm(int r) {
    const int l = r / VEC, j = (r % VEC) >> 2, e = r & 3;
    return j * 128 + l * 4 + e;
}

// Stores output row n of activation row m through the segment table and returns the value after the
// bias. `fold` = false leaves the argmax to the caller (which reduces keys across lanes first).
__device__ __forceinline__ float epilogue_store(const GemvParams& p, int n, int m, float v, bool fold = true) {
    int s = 0;
    while (s < p.nseg - 1 && n >= p.seg[s].row_end) ++s;
    const int begin = s ? p.seg[s - 1].row_end : 0;
    const int local = n - begin;
    const GemvSeg& g = p.seg[s];
    if (g.bias) v += g.bias[local];
    const long long idx = static_cast<long long>(m) * g.ld + local;
    if (p.epi == EPI_ACCUM) {
        float* o = static_cast<float*>(g.out);
        o[idx] += v;
    } else if (p.epi == EPI_ARGMAX) {
        if (g.out) store_from_float(g.out, p.out_dtype, idx, v);
        if (fold) atomicMax(p.argmax + m, argmax_key(v, n + p.argmax_base));
    } else {
        store_from_float(g.out, p.out_dtype, idx, v);
    }
    return v;
}

// Rows of row block `blk` owned by `warp`: RPW consecutive rows, or for SwiGLU pairs (i, i + N/2).
template <int RPW>
struct BlockRows {
    int unit0;
    int row[RPW];
    bool valid[RPW];
    __device__ __forceinline__ BlockRows(int blk, int warp, bool swiglu, int per_cta, int half_n, int N) {
        unit0 = swiglu ? blk * per_cta + warp * (RPW / 2) : blk * kWarps * RPW + warp * RPW;
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            row[r] = swiglu ? unit0 + (r & 1) * half_n + (r >> 1) : unit0 + r;
            valid[r] = swiglu ? unit0 + (r >> 1) < half_n : row[r] < N;
        }
    }
};

// Exact int8 -> fp32 of the four signed bytes of a word: byte b biased to u = b ^ 0x80 (0..255) sits in
// the mantissa of 2^23 (the float 0x4B0000uu = 8388608 + u), and subtracting 8388608 + 128 gives b.
__device__ __forceinline__ void dequant4(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
    const uint32_t u = w ^ 0x80808080u;
    f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
    f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
    f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
    f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}

// a += dot(4 weights of word w, x) with two independent accumulators (a.x, a.y) for ILP.
__device__ __forceinline__ void dot4_i8(uint32_t w, const float4& x, float2& a) {
    float f0, f1, f2, f3;
    dequant4(w, f0, f1, f2, f3);
    a.x = fmaf(f0, x.x, a.x);
    a.y = fmaf(f1, x.y, a.y);
    a.x = fmaf(f2, x.z, a.x);
    a.y = fmaf(f3, x.w, a.y);
}

template <typename WT>
__device__ __forceinline__ float2 w2_to_f2(uint32_t w) {
    if constexpr (DT<WT>::id == L0B_F16) return half2_bits_to_float2(w);
    else return bf162_bits_to_float2(w);
}

// acc[r][m] += W[row r, chunk] . x[m, chunk] for one 16-byte weight vector per row. xb points at the
// lane's first float4 of the chunk for activation row 0; rows of x are kt floats apart.
template <typename WT, int MR, int RPW>
__device__ __forceinline__ void mac_step(const uint4 (&w)[RPW], const float (&s)[RPW], const float* xb, int kt,
                                         bool per_channel, float2 (&acc)[RPW][MR]) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
        const float* xm = xb + m * kt;
        if constexpr (sizeof(WT) == 1) {
            const float4 x0 = *reinterpret_cast<const float4*>(xm);
            const float4 x1 = *reinterpret_cast<const float4*>(xm + 128);
            const float4 x2 = *reinterpret_cast<const float4*>(xm + 256);
            const float4 x3 = *reinterpret_cast<const float4*>(xm + 384);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                if (per_channel) {
                    dot4_i8(w[r].x, x0, acc[r][m]);
                    dot4_i8(w[r].y, x1, acc[r][m]);
                    dot4_i8(w[r].z, x2, acc[r][m]);
                    dot4_i8(w[r].w, x3, acc[r][m]);
                } else {
                    float2 a = make_float2(0.f, 0.f);
                    dot4_i8(w[r].x, x0, a);
                    dot4_i8(w[r].y, x1, a);
                    dot4_i8(w[r].z, x2, a);
                    dot4_i8(w[r].w, x3, a);
                    acc[r][m].x = fmaf(a.x + a.y, s[r], acc[r][m].x);
                }
            }
        } else if constexpr (sizeof(WT) == 2) {
            const float4 x0 = *reinterpret_cast<const float4*>(xm);
            const float4 x1 = *reinterpret_cast<const float4*>(xm + 128);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                const float2 w0 = w2_to_f2<WT>(w[r].x), w1 = w2_to_f2<WT>(w[r].y);
                const float2 w2 = w2_to_f2<WT>(w[r].z), w3 = w2_to_f2<WT>(w[r].w);
                float2& a = acc[r][m];
                a.x = fmaf(w0.x, x0.x, a.x);
                a.y = fmaf(w0.y, x0.y, a.y);
                a.x = fmaf(w1.x, x0.z, a.x);
                a.y = fmaf(w1.y, x0.w, a.y);
                a.x = fmaf(w2.x, x1.x, a.x);
                a.y = fmaf(w2.y, x1.y, a.y);
                a.x = fmaf(w3.x, x1.z, a.x);
                a.y = fmaf(w3.y, x1.w, a.y);
            }
        } else {
            const float4 x0 = *reinterpret_cast<const float4*>(xm);
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                float2& a = acc[r][m];
                a.x = fmaf(__uint_as_float(w[r].x), x0.x, a.x);
                a.y = fmaf(__uint_as_float(w[r].y), x0.y, a.y);
                a.x = fmaf(__uint_as_float(w[r].z), x0.z, a.x);
                a.y = fmaf(__uint_as_float(w[r].w), x0.w, a.y);
            }
        }
    }
}

// Warp reduction of a finished row block and its epilogue; results spread over lanes for the stores.
template <int MR, int RPW>
__device__ __forceinline__ void finish_block(const GemvParams& p, float2 (&acc)[RPW][MR], const BlockRows<RPW>& g,
                                             const float (&rscale)[RPW], bool per_channel, bool swiglu, int lane) {
    float res[RPW][MR];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            float v = warp_sum(acc[r][m].x + acc[r][m].y);
            if (per_channel) v *= rscale[r];
            res[r][m] = v;
            acc[r][m] = make_float2(0.f, 0.f);
        }
    if (swiglu) {
#pragma unroll
        for (int r = 0; r < RPW; r += 2)
#pragma unroll
            for (int m = 0; m < MR; ++m)
                if (lane == ((r * MR + m) & 31) && m < p.M && g.valid[r])
                    epilogue_store(p, g.unit0 + (r >> 1), m, silu(res[r][m]) * res[r + 1][m]);
    } else {
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < MR; ++m)
                if (lane == ((r * MR + m) & 31) && m < p.M && g.valid[r]) epilogue_store(p, g.row[r], m, res[r][m]);
    }
}

template <typename WT, int MR, int RPW>
__global__ void __launch_bounds__(kThreads, MR >= 4 ? 1 : 2) gemv_nk_kernel(const GemvParams p) {
    extern __shared__ float4 smem_f4[];
    float* xs = reinterpret_cast<float*>(smem_f4);
    __shared__ float rstd_s[MR];
    constexpr int VEC = 16 / sizeof(WT);
    constexpr int CH = 32 * VEC;  // elements per warp step
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = p.N, K = p.K, M = p.M, kt = p.kt;
    const bool swiglu = p.epi == EPI_SWIGLU;
    const int half_n = N >> 1;
    const int units = swiglu ? half_n : N;
    const int per_cta = swiglu ? kWarps * (RPW / 2) : kWarps * RPW;
    const int nblocks = (units + per_cta - 1) / per_cta;
    const bool per_channel = sizeof(WT) == 1 && p.group >= K;
    const int gpr = sizeof(WT) == 1 ? K / p.group : 0;
    const __half* scales = static_cast<const __half*>(p.scales);
    const WT* W = static_cast<const WT*>(p.w);
    const bool single_tile = K <= kt;

    if (p.prefetch && threadIdx.x == 0 && blockIdx.x < nblocks) {
        const long long u0 = static_cast<long long>(blockIdx.x) * per_cta;
        const long long u1 = min(u0 + per_cta, static_cast<long long>(units));
        const long long row_bytes = K * static_cast<long long>(sizeof(WT));
        for (int part = 0; part < (swiglu ? 2 : 1); ++part) {
            const char* base = static_cast<const char*>(p.w) + (u0 + part * half_n) * row_bytes;
            const long long bytes = (u1 - u0) * row_bytes;
            for (long long off = 0; off < bytes; off += 32768) {
                const long long len = min(32768LL, bytes - off);
                prefetch_l2_bulk(base + off, static_cast<uint32_t>(len));
            }
        }
    }

    // Weight stream state (single-tile path): steps (block, chunk) of this CTA in order.
    const int nchunks = (K + CH - 1) / CH;
    const int my_blocks = blockIdx.x < nblocks ? (nblocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = single_tile ? my_blocks * nchunks : 0;
    uint4 ring[kRing][RPW];
    float sring[kRing][RPW];
    // Row starts (null past N) and scale rows of the block being issued; updated at block changes only.
    const WT* i_ptr[RPW];
    const __half* i_sc[RPW];
    const int gshift = __ffs(p.group > 0 ? p.group : 1) - 1;
    const bool gpow2 = p.group > 0 && (1 << gshift) == p.group;
    int i_step = 0, i_blk = blockIdx.x, i_c = 0;
    auto set_issue_block = [&](int blk) {
        const BlockRows<RPW> g(blk, warp, swiglu, per_cta, half_n, N);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            i_ptr[r] = g.valid[r] ? W + static_cast<long long>(g.row[r]) * K : nullptr;
            i_sc[r] = (sizeof(WT) == 1 && g.valid[r]) ? scales + static_cast<long long>(g.row[r]) * gpr : nullptr;
        }
    };
    set_issue_block(blockIdx.x);
    auto issue = [&](uint4 (&slot)[RPW], float (&ss)[RPW]) {
        if (i_step < total) {
            const int kk = i_c * CH + lane * VEC;
            const bool in_k = kk < K;
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                slot[r] = (i_ptr[r] && in_k) ? ld_stream_v4(i_ptr[r] + kk) : make_uint4(0, 0, 0, 0);
                if constexpr (sizeof(WT) == 1) {
                    if (!per_channel)
                        ss[r] = (i_sc[r] && in_k) ? __half2float(i_sc[r][gpow2 ? kk >> gshift : kk / p.group]) : 0.f;
                    else if (i_c == 0)
                        ss[r] = i_sc[r] ? __half2float(i_sc[r][0]) : 0.f;
                }
            }
            if (++i_c == nchunks) {
                i_c = 0;
                i_blk += gridDim.x;
                set_issue_block(i_blk);
            }
        }
        ++i_step;
    };
#pragma unroll
    for (int d = 0; d < kRing; ++d) issue(ring[d], sring[d]);

    pdl_wait();
    pdl_launch_dependents();

    // fp32 activations in 16-byte aligned rows take the vector path of the prologue.
    const bool xvec = p.x_dtype == L0B_F32 && (K & 3) == 0 && (p.x_ld & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    const float* xf = static_cast<const float*>(p.x);

    // RMS of each activation row (fused norm): a block-wide reduction per row.
    if (p.norm_w) {
        __shared__ float red[32];
        for (int m = 0; m < MR; ++m) {
            float ss = 0.f;
            if (m < M) {
                if (xvec) {
                    for (int k = threadIdx.x * 4; k < K; k += kThreads * 4) {
                        const float4 v = *reinterpret_cast<const float4*>(xf + m * p.x_ld + k);
                        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    }
                } else {
                    for (int k = threadIdx.x; k < K; k += kThreads) {
                        const float v = load_as_float(p.x, p.x_dtype, m * p.x_ld + k);
                        ss += v * v;
                    }
                }
            }
            ss = block_sum(ss, red);
            if (threadIdx.x == 0) rstd_s[m] = 1.0f / sqrtf(ss / static_cast<float>(K) + p.eps);
        }
        __syncthreads();
    }

    auto stage = [&](int k0) {
        if (xvec) {
            // Four consecutive elements stay consecutive in the lane-major layout (VEC is a multiple of 4).
            const int quads = kt >> 2;
            for (int m = 0; m < MR; ++m) {
                for (int qi = threadIdx.x; qi < quads; qi += kThreads) {
                    const int r = qi << 2, k = k0 + r;
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (m < M && k < K) {
                        v = *reinterpret_cast<const float4*>(xf + m * p.x_ld + k);
                        if (p.norm_w) {
                            const float rs = rstd_s[m];
                            const float4 w4 = *reinterpret_cast<const float4*>(p.norm_w + k);
                            v = make_float4((v.x * rs) * w4.x, (v.y * rs) * w4.y, (v.z * rs) * w4.z, (v.w * rs) * w4.w);
                        }
                    }
                    const int c = r / CH, rr = r - c * CH;
                    *reinterpret_cast<float4*>(xs + m * kt + c * CH + xs_perm<VEC>(rr)) = v;
                }
            }
            return;
        }
        const int span = MR * kt;
        for (int idx = threadIdx.x; idx < span; idx += kThreads) {
            const int m = idx / kt, r = idx - m * kt;
            const int k = k0 + r;
            float v = 0.f;
            if (m < M && k < K) {
                v = load_as_float(p.x, p.x_dtype, m * p.x_ld + k);
                if (p.norm_w) v = (v * rstd_s[m]) * p.norm_w[k];
            }
            const int c = r / CH;
            xs[m * kt + c * CH + xs_perm<VEC>(r - c * CH)] = v;
        }
    };

    float2 acc[RPW][MR];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int m = 0; m < MR; ++m) acc[r][m] = make_float2(0.f, 0.f);
    float rscale[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) rscale[r] = 0.f;

    if (single_tile) {
        stage(0);
        __syncthreads();
        int c_blk = blockIdx.x, c_c = 0;
        for (int s = 0; s < total; s += kRing) {
#pragma unroll
            for (int d = 0; d < kRing; ++d) {
                if (s + d < total) {
                    mac_step<WT, MR, RPW>(ring[d], sring[d], xs + c_c * CH + lane * 4, kt, per_channel, acc);
                    if (per_channel && c_c == 0) {
#pragma unroll
                        for (int r = 0; r < RPW; ++r) rscale[r] = sring[d][r];
                    }
                    issue(ring[d], sring[d]);
                    if (++c_c == nchunks) {
                        finish_block<MR, RPW>(p, acc, BlockRows<RPW>(c_blk, warp, swiglu, per_cta, half_n, N), rscale,
                                              per_channel, swiglu, lane);
                        c_c = 0;
                        c_blk += gridDim.x;
                    }
                }
            }
        }
        return;
    }

    // Multi-tile path (activation rows too long for shared memory): stage each K tile, then stream.
    for (int blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
        const BlockRows<RPW> g(blk, warp, swiglu, per_cta, half_n, N);
        for (int k0 = 0; k0 < K; k0 += kt) {
            __syncthreads();
            stage(k0);
            __syncthreads();
            const int klen = min(kt, K - k0);
            for (int kk = lane * VEC; kk < klen; kk += CH) {
                uint4 w[RPW];
                float sc[RPW];
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    w[r] = g.valid[r] ? ld_stream_v4(W + static_cast<long long>(g.row[r]) * K + k0 + kk)
                                      : make_uint4(0, 0, 0, 0);
                    if constexpr (sizeof(WT) == 1)
                        sc[r] = g.valid[r]
                                    ? __half2float(scales[static_cast<long long>(g.row[r]) * gpr + (k0 + kk) / p.group])
                                    : 0.f;
                    else
                        sc[r] = 0.f;
                    rscale[r] = sc[r];
                }
                mac_step<WT, MR, RPW>(w, sc, xs + (kk / CH) * CH + lane * 4, kt, per_channel, acc);
            }
        }
        finish_block<MR, RPW>(p, acc, g, rscale, per_channel, swiglu, lane);
    }
}

// Generic fallback for shapes the vector kernel does not take (K not a multiple of the vector
// width or unaligned rows): one warp per (row, activation row), scalar loads.
template <typename WT>
__global__ void __launch_bounds__(kThreads) gemv_nk_scalar_kernel(const GemvParams p) {
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long gw = static_cast<long long>(blockIdx.x) * kWarps + warp;
    const int pairs = p.epi == EPI_SWIGLU;
    const long long outs = pairs ? p.N / 2 : p.N;
    if (gw >= outs * p.M) return;
    const int m = static_cast<int>(gw / outs);
    const int n = static_cast<int>(gw - static_cast<long long>(m) * outs);
    float rstd = 1.f;
    if (p.norm_w) {
        float ss = 0.f;
        for (int k = lane; k < p.K; k += 32) {
            const float v = load_as_float(p.x, p.x_dtype, m * p.x_ld + k);
            ss += v * v;
        }
        ss = warp_sum(ss);
        rstd = 1.0f / sqrtf(ss / static_cast<float>(p.K) + p.eps);
    }
    const __half* scales = static_cast<const __half*>(p.scales);
    float res[2];
    for (int t = 0; t <= pairs; ++t) {
        const int row = pairs ? n + t * (p.N / 2) : n;
        const WT* w = static_cast<const WT*>(p.w) + static_cast<long long>(row) * p.K;
        float acc = 0.f;
        for (int k = lane; k < p.K; k += 32) {
            float xv = load_as_float(p.x, p.x_dtype, m * p.x_ld + k);
            if (p.norm_w) xv = (xv * rstd) * p.norm_w[k];
            float wv;
            if constexpr (sizeof(WT) == 1) {
                const int gpr = p.K / p.group;
                wv = static_cast<float>(w[k]) * __half2float(scales[static_cast<long long>(row) * gpr + k / p.group]);
            } else if constexpr (DT<WT>::id == L0B_F16) {
                wv = __half2float(w[k]);
            } else if constexpr (DT<WT>::id == L0B_BF16) {
                wv = __bfloat162float(w[k]);
            } else {
                wv = w[k];
            }
            acc = fmaf(wv, xv, acc);
        }
        res[t] = warp_sum(acc);
    }
    if (lane == 0) epilogue_store(p, n, m, pairs ? silu(res[0]) * res[1] : res[0]);
}

// ---------------------------------------------------------------------------------------------
// Tensor-core weight streaming for up to 8 activation rows (decode, small batches).
//
// One mma.sync.m16n8k16 (fp32 accumulate) takes a 16-row x 16-k weight tile as its A operand and
// eight activation columns as B. Column 2m of B holds hi = half(x[m] * 2^e) and column 2m + 1 the
// fp16 residual half(x[m] * 2^e - hi), with 2^e a per-row power of two that puts the row's largest
// value near 2^14; the two products summed (and scaled back by 2^-e) give the dot product with x to
// ~22 bits -- fp32 activations in all but name -- using B columns a single row leaves idle.
// int8 weights become exact f16 integers with two byte permutes into the 0x64 exponent (1024 + u)
// and one f16x2 subtract of 1152; f16 and bf16 weights feed the MMA as loaded. The MMA reduces
// across the k of its tile, so no warp shuffles are needed and the instruction count per weight
// byte is a fraction of the fp32 FMA form.
//
// A tile is 16 output rows (SwiGLU: 8 gate rows and their 8 up rows, so the epilogue pairs them in
// one lane). Each row is read in 16-byte pieces (64 int8 or 32 16-bit k); four pieces make a chunk,
// and quad lane t loads piece bytes [16 t, 16 t + 16) of rows lane / 4 and lane / 4 + 8, so every row
// is streamed in 256-byte runs per quad -- the granularity at which the HBM keeps its pages busy (64-
// byte runs per row measured at about half the bandwidth). Warp w of a CTA takes the w-th eighth of
// each row's pieces, so the warps of a CTA finish a tile together at its barrier.
// The k order inside the MMA is a permutation of the real k, applied identically to A (weights) and B
// (activations staged in that order), which the dot product does not see. Per-warp partial sums meet
// in shared memory once per tile (double-buffered, one barrier) and one warp, rotating by tile, runs
// the epilogue. Weights stream through a register ring across tiles as in the FMA kernel above.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1, bool bf16) {
    if (bf16)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four signed bytes -> two f16x2 (bytes 0,1 and bytes 2,3), exact: u = b ^ 0x80 placed in the low
// mantissa of 1024.0 (0x64uu) is 1024 + u, and subtracting 1152 leaves b.
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t p0 = __byte_perm(u, 0x64646464u, 0x5140);
    const uint32_t p1 = __byte_perm(u, 0x64646464u, 0x5342);
    asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(p0), "r"(0x64806480u));
    asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(p1), "r"(0x64806480u));
}

__device__ __forceinline__ uint32_t u4_get(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Activation pair (hi, lo) of 8 consecutive values as two 16-byte rows of 16-bit words.
template <bool BF16>
__device__ __forceinline__ void split_hi_lo(const float (&v)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (BF16) {
            const __nv_bfloat16 a = __float2bfloat16_rn(v[2 * i]), b = __float2bfloat16_rn(v[2 * i + 1]);
            const __nv_bfloat16 c = __float2bfloat16_rn(v[2 * i] - __bfloat162float(a));
            const __nv_bfloat16 d = __float2bfloat16_rn(v[2 * i + 1] - __bfloat162float(b));
            h[i] = static_cast<uint32_t>(__bfloat16_as_ushort(a)) | (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
            l[i] = static_cast<uint32_t>(__bfloat16_as_ushort(c)) | (static_cast<uint32_t>(__bfloat16_as_ushort(d)) << 16);
        } else {
            const __half a = __float2half_rn(v[2 * i]), b = __float2half_rn(v[2 * i + 1]);
            const __half c = __float2half_rn(v[2 * i] - __half2float(a));
            const __half d = __float2half_rn(v[2 * i + 1] - __half2float(b));
            h[i] = static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
            l[i] = static_cast<uint32_t>(__half_as_ushort(c)) | (static_cast<uint32_t>(__half_as_ushort(d)) << 16);
        }
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Weight pieces: int8 = 64 k (16 bytes per lane, 4 MMAs), 16-bit = 32 k (16 bytes per lane, 2 MMAs).
// D += A B on the integer tensor cores: A 16 x 32 s8 (rows g, g + 8; k 4 t .. 4 t + 3 in a0 / a1 and
// 16 + 4 t .. in a2 / a3), B 32 x 8 s8 (column g; k 4 t .. in b0, 16 + 4 t .. in b1), s32 accumulators.
__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Peer-sum mailbox addressing (layout in gemv.cuh) and the system-scope flag accesses.
__device__ __forceinline__ unsigned long long* peer_sum_slot(char* mb, int par, int src) {
    return reinterpret_cast<unsigned long long*>(mb) + (static_cast<long long>(par) * kMaxPeerRanks + src) * kPeerSumSlotElems;
}
__device__ __forceinline__ unsigned* peer_sum_counter(char* mb, int i) {  // 0: epoch, 1: CTAs done
    return reinterpret_cast<unsigned*>(mb + kPeerSumDataBytes) + 32 * i;
}
// One tagged value: a single 64-bit store / load, so the tag and the value are seen together.
__device__ __forceinline__ void st_tagged_sys(unsigned long long* p, unsigned tag, float v) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
constexpr long long kPeerSumWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz, then the error flag

template <typename WT>
struct MmaPiece {
    static constexpr int kK = sizeof(WT) == 1 ? 64 : 32;  // k per piece
    static constexpr int kUnits = kK / 32;                // 32-k activation units per piece
};
constexpr int kMmaLoads = 4;  // pieces per chunk: 256 contiguous bytes of each row per quad
constexpr int kMmaRing = 2;   // chunks in flight per warp

// NG groups of 4 activation rows (8 B columns each, NG <= 4: up to 16 rows). Shared memory holds the
// split activations of this CTA's K range in 32-k units: unit u (relative to the range start), column
// col, quad lane t at (u * 2M + col) * 64 + t * 16, eight 16-bit values. For int8 unit u = 2p + j holds
// x[64 p + 16 t + 8 j, +8) (the 16 values lane t multiplies in piece p), for 16-bit weights
// x[32 u + 8 t, +8). Lane (g, t) reads column g with conflict-free loads; columns past 2M are never read.
//
// Split-K (gridDim.y = S > 1): the S CTAs of a thread-block cluster (1, S, 1) share the tiles of
// cluster blockIdx.x and each takes the ks-th S-th of every row's pieces, so each stages only its slice
// of x. Per-row sums of squares (for the fused RMSNorm) are exchanged through distributed shared memory
// before the split, and per tile the ranks' partial sums meet in rank 0, which reads them from the
// peers' shared memory in rank order one tile later (deterministic, no global scratch, no atomics).
template <typename WT, int NG>
__global__ void __launch_bounds__(kThreads, 2) gemv_mma_kernel(const GemvParams p) {
    namespace cg = cooperative_groups;
    extern __shared__ float4 smem_f4[];
    char* xs = reinterpret_cast<char*>(smem_f4);
    __shared__ float2 red[2][kWarps][NG][32];
    __shared__ float2 cpart[2][NG][32];  // this CTA's finished tile partial (split-K)
    __shared__ float oscale_s[4 * NG];
    __shared__ float ssq_s[4 * NG][kWarps], amax_s[4 * NG][kWarps];
    constexpr bool kI8 = sizeof(WT) == 1;
    constexpr bool kBF = DT<WT>::id == L0B_BF16;
    constexpr int PE = MmaPiece<WT>::kK;
    constexpr int KU = MmaPiece<WT>::kUnits;
    cg::cluster_group cluster = cg::this_cluster();
    const int S = gridDim.y, ks = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int N = p.N, K = p.K, M = p.M;
    const int C2 = 2 * M;
    const bool swiglu = p.epi == EPI_SWIGLU;
    const int half_n = N >> 1;
    const int units = swiglu ? half_n : N;
    const int ntiles = (units + (swiglu ? 7 : 15)) / (swiglu ? 8 : 16);
    // This CTA's pieces [kp0, kp1) of every row; warp w owns [p0, p1) of them (counts differ by <= 1).
    const int npieces = K / PE;
    const int kp0 = ks * npieces / S, kp1 = (ks + 1) * npieces / S;
    const int p0 = kp0 + warp * (kp1 - kp0) / kWarps, p1 = kp0 + (warp + 1) * (kp1 - kp0) / kWarps;
    const int nq = (p1 - p0 + kMmaLoads - 1) / kMmaLoads;  // chunks of this warp per tile
    const int u_lo = kp0 * KU, nunits = (kp1 - kp0) * KU;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = my_tiles * nq;
    const WT* W = static_cast<const WT*>(p.w);
    const __half* scales = static_cast<const __half*>(p.scales);
    auto cluster_barrier = [&]() {
        if (S > 1) cluster.sync();
        else __syncthreads();
    };

    auto tile_rows = [&](int tile, int& r0, int& r1, bool& v0, bool& v1) {
        if (swiglu) {
            r0 = tile * 8 + g;
            r1 = r0 + half_n;
            v0 = v1 = r0 < half_n;
        } else {
            r0 = tile * 16 + g;
            r1 = r0 + 8;
            v0 = r0 < N;
            v1 = r1 < N;
        }
    };

    if (p.prefetch && S == 1 && threadIdx.x == 0 && blockIdx.x < ntiles) {
        const long long row_bytes = K * static_cast<long long>(sizeof(WT));
        const int per = swiglu ? 8 : 16;
        const long long u0 = static_cast<long long>(blockIdx.x) * per;
        const long long u1 = min(u0 + per, static_cast<long long>(units));
        for (int part = 0; part < (swiglu ? 2 : 1); ++part) {
            const char* base = static_cast<const char*>(p.w) + (u0 + part * half_n) * row_bytes;
            const long long bytes = (u1 - u0) * row_bytes;
            for (long long off = 0; off < bytes; off += 32768)
                prefetch_l2_bulk(base + off, static_cast<uint32_t>(min(32768LL, bytes - off)));
        }
    }

    // Weight stream: steps (tile, chunk q of this warp) in order, kMmaRing steps ahead of the math.
    // Chunk q covers pieces p0 + 4q .. p0 + 4q + 3; a piece at or past p1 is neither loaded nor used.
    uint4 ring[kMmaRing][2][kMmaLoads];
    float sring[kMmaRing][2];
    const WT* i_p[2];
    const __half* i_s[2];
    int i_step = 0, i_tile = blockIdx.x, i_q = 0;
    // Blocked int8 layout (p.kb > 0): piece pc of row r lies in block pc / ppb of the row's tile, at
    // (r % 16) * kb + (pc % ppb) * PE within it.
    const int kbk = kI8 ? p.kb : 0;  // 0 or kWeightBlock (8 pieces of 64 k)
    auto set_issue_tile = [&](int tile) {
        int r0, r1;
        bool v0, v1;
        tile_rows(tile, r0, r1, v0, v1);
        if (kbk > 0) {
            const long long tb = static_cast<long long>(t) * (PE / 4);
            i_p[0] = v0 ? W + static_cast<long long>(r0 >> 4) * 16 * K + (r0 & 15) * kbk + tb : nullptr;
            i_p[1] = v1 ? W + static_cast<long long>(r1 >> 4) * 16 * K + (r1 & 15) * kbk + tb : nullptr;
        } else {
            const long long off = static_cast<long long>(p0) * PE + t * (PE / 4);
            i_p[0] = v0 ? W + static_cast<long long>(r0) * K + off : nullptr;
            i_p[1] = v1 ? W + static_cast<long long>(r1) * K + off : nullptr;
        }
        i_s[0] = (kI8 && v0) ? scales + r0 : nullptr;
        i_s[1] = (kI8 && v1) ? scales + r1 : nullptr;
    };
    set_issue_tile(i_tile);
    // Piece l of the chunk at the issue cursor (step i_step), then the cursor's scale and advance.
    auto issue_piece = [&](uint4 (&slot)[2][kMmaLoads], int l) {
        if (i_step < total) {
            const int pc = p0 + kMmaLoads * i_q + l;
            const bool in_k = pc < p1;
            const long long off = kbk > 0 ? static_cast<long long>(pc >> 3) * (16 * kWeightBlock) + (pc & 7) * PE
                                          : static_cast<long long>(i_q) * (kMmaLoads * PE) + l * PE;
#pragma unroll
            for (int r = 0; r < 2; ++r)
                slot[r][l] = (i_p[r] && in_k) ? ld_stream_v4(i_p[r] + off) : make_uint4(0, 0, 0, 0);
        }
    };
    auto issue_finish = [&](float (&ss)[2]) {
        if (i_step < total) {
            if (kI8 && i_q == 0) {
#pragma unroll
                for (int r = 0; r < 2; ++r) ss[r] = i_s[r] ? __half2float(*i_s[r]) : 0.f;
            }
            if (++i_q == nq) {
                i_q = 0;
                i_tile += gridDim.x;
                set_issue_tile(i_tile);
            }
        }
        ++i_step;
    };
    // The whole ring goes out before griddepcontrol.wait: weights never depend on the previous kernel.
    // (Issuing the second slot only after staging, to free its registers there, measured 20-25% slower.)
#pragma unroll
    for (int d = 0; d < kMmaRing; ++d) {
#pragma unroll
        for (int l = 0; l < kMmaLoads; ++l) issue_piece(ring[d], l);
        issue_finish(sring[d]);
    }

    pdl_wait();
    pdl_launch_dependents();
    // Peer-sum epilogue: this call's epoch (the previous call's last CTA advanced it before that kernel
    // ended, and pdl_wait has waited for it) and mailbox parity.
    const bool psum = p.epi == EPI_PEER_SUM;
    const unsigned ep =
        psum ? *reinterpret_cast<const volatile unsigned*>(peer_sum_counter(p.peer->mbox[p.peer->rank], 0)) + 1u : 0u;
    const int par = static_cast<int>(ep & 1u);

    const bool xvec = p.x_dtype == L0B_F32 && (p.x_ld & 3) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    const float* xf = static_cast<const float*>(p.x);
    // Stage this CTA's slice of x in two passes over shared memory, one global read. Pass 1: each thread
    // loads its items (32-k unit u, quad lane t: 8 consecutive k), applies the RMS-norm weight, stores
    // the fp32 values into the 32 bytes their hi/lo pair will occupy, and accumulates the row's sum of
    // squares and largest magnitude. Pass 2 (after one barrier; with split-K a cluster barrier, and the
    // sums of squares of all ranks are added so the norm covers the whole row): the same thread rereads
    // its values, applies the row's 1/RMS and a power-of-two scale 2^e that puts this slice's maximum
    // near 2^14 (so the f16 split neither overflows nor loses small values to subnormals), and splits them
    // into hi + lo. The epilogue multiplies by the exact 2^-e.
    {
        const int items = nunits * 4;  // per activation row
        constexpr int kSB = 2;
        auto item_slot = [&](int it, int m, int& k) {
            const int ur = it >> 2, tt = it & 3, u = u_lo + ur;
            k = kI8 ? (u >> 1) * 64 + 16 * tt + 8 * (u & 1) : 32 * u + 8 * tt;
            return xs + static_cast<size_t>(ur) * C2 * 64 + tt * 16 + (2 * m) * 64;  // lo slot is +64
        };
        for (int m = 0; m < M; ++m) {
            float ss = 0.f, amax = 0.f;
            for (int it0 = threadIdx.x; it0 < items; it0 += kThreads * kSB) {
                float v[kSB][8], nw[kSB][8];
#pragma unroll
                for (int b = 0; b < kSB; ++b) {
                    const int it = it0 + b * kThreads;
                    int k;
                    item_slot(it, m, k);
                    if (it < items) {
                        if (xvec) {
                            const float4 a = *reinterpret_cast<const float4*>(xf + m * p.x_ld + k);
                            const float4 c = *reinterpret_cast<const float4*>(xf + m * p.x_ld + k + 4);
                            v[b][0] = a.x, v[b][1] = a.y, v[b][2] = a.z, v[b][3] = a.w;
                            v[b][4] = c.x, v[b][5] = c.y, v[b][6] = c.z, v[b][7] = c.w;
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) v[b][e] = load_as_float(p.x, p.x_dtype, m * p.x_ld + k + e);
                        }
                        if (p.norm_w) {
                            const float4 a = *reinterpret_cast<const float4*>(p.norm_w + k);
                            const float4 c = *reinterpret_cast<const float4*>(p.norm_w + k + 4);
                            nw[b][0] = a.x, nw[b][1] = a.y, nw[b][2] = a.z, nw[b][3] = a.w;
                            nw[b][4] = c.x, nw[b][5] = c.y, nw[b][6] = c.z, nw[b][7] = c.w;
                        }
                    }
                }
#pragma unroll
                for (int b = 0; b < kSB; ++b) {
                    const int it = it0 + b * kThreads;
                    if (it >= items) break;
                    int k;
                    char* slot = item_slot(it, m, k);
                    if (p.norm_w) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            ss = fmaf(v[b][e], v[b][e], ss);
                            v[b][e] *= nw[b][e];
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[b][e]));
                    *reinterpret_cast<float4*>(slot) = make_float4(v[b][0], v[b][1], v[b][2], v[b][3]);
                    *reinterpret_cast<float4*>(slot + 64) = make_float4(v[b][4], v[b][5], v[b][6], v[b][7]);
                }
            }
            ss = warp_sum(ss);
            amax = warp_max(amax);
            if (lane == 0) {
                ssq_s[m][warp] = ss;
                amax_s[m][warp] = amax;
            }
        }
        cluster_barrier();
        for (int m = 0; m < M; ++m) {
            float ss = 0.f, amax = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) amax = fmaxf(amax, amax_s[m][w]);
            if (p.norm_w) {
                for (int r = 0; r < S; ++r) {
                    const float* q = S > 1 ? cluster.map_shared_rank(&ssq_s[m][0], r) : &ssq_s[m][0];
#pragma unroll
                    for (int w = 0; w < kWarps; ++w) ss += q[w];
                }
            }
            const float rs = p.norm_w ? 1.0f / sqrtf(ss / static_cast<float>(K) + p.eps) : 1.0f;
            // Power of two 2^e with (amax * rs) * 2^e in [2^13, 2^14); bf16 keeps the fp32 range (e = 0).
            int e = 0;
            if (!kBF && amax * rs > 0.f && isfinite(amax * rs)) {
                int ex;
                frexpf(amax * rs, &ex);  // amax * rs = f * 2^ex, f in [0.5, 1)
                e = min(max(14 - ex, -100), 100);
            }
            const float in_scale = rs * ldexpf(1.0f, e);
            if (threadIdx.x == 0) oscale_s[m] = ldexpf(1.0f, -e);
            for (int it = threadIdx.x; it < items; it += kThreads) {
                int k;
                char* slot = item_slot(it, m, k);
                const float4 a = *reinterpret_cast<const float4*>(slot);
                const float4 c = *reinterpret_cast<const float4*>(slot + 64);
                float v[8] = {a.x * in_scale, a.y * in_scale, a.z * in_scale, a.w * in_scale,
                              c.x * in_scale, c.y * in_scale, c.z * in_scale, c.w * in_scale};
                uint4 hi, lo;
                split_hi_lo<kBF>(v, hi, lo);
                *reinterpret_cast<uint4*>(slot) = hi;
                *reinterpret_cast<uint4*>(slot + 64) = lo;
            }
        }
    }
    __syncthreads();
    // oscale_s[m] = 2^-e of row m, applied to this CTA's partial sums.

    // Store / argmax / SwiGLU epilogue of a finished tile; y[ng] = (row g, row g + 8) of row 4 ng + t.
    auto epilogue = [&](int tile, const float2 (&y)[NG]) {
        int r0, r1;
        bool v0, v1;
        tile_rows(tile, r0, r1, v0, v1);
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
            const float y0 = y[ng].x, y1 = y[ng].y;
            const int m = 4 * ng + t;
            const bool live = m < M;
            if (psum) {
                // This rank's partial of rows (r0, r1) into its slot of every rank's mailbox.
                if (live) {
                    const PeerSum* ps = p.peer;
                    const long long i0 = static_cast<long long>(m) * N + r0, i1 = static_cast<long long>(m) * N + r1;
                    for (int d = 0; d < ps->nranks; ++d) {
                        unsigned long long* dst = peer_sum_slot(ps->mbox[d], par, ps->rank);
                        if (v0) st_tagged_sys(dst + i0, ep, y0);
                        if (v1) st_tagged_sys(dst + i1, ep, y1);
                    }
                }
            } else if (p.epi == EPI_ARGMAX) {
                unsigned long long key = 0;
                if (live && v0) key = argmax_key(epilogue_store(p, r0, m, y0, false), r0 + p.argmax_base);
                if (live && v1) key = max(key, argmax_key(epilogue_store(p, r1, m, y1, false), r1 + p.argmax_base));
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
                if (live && g == 0 && key) atomicMax(p.argmax + m, key);
            } else if (live) {
                if (swiglu) {
                    if (v0) epilogue_store(p, r0, m, silu(y0) * y1);
                } else {
                    if (v0) epilogue_store(p, r0, m, y0);
                    if (v1) epilogue_store(p, r1, m, y1);
                }
            }
        }
    };
    // This CTA's partial of tile iteration i: the warps' partials in red[i & 1], scaled back by 2^-e.
    auto local_tile = [&](int i, float2 (&y)[NG]) {
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
            float y0 = 0.f, y1 = 0.f;
            for (int w = 0; w < kWarps; ++w) {
                const float2 q = red[i & 1][w][ng][lane];
                y0 += q.x;
                y1 += q.y;
            }
            const int m = 4 * ng + t;
            const float f = m < M ? oscale_s[m] : 1.0f;
            y[ng] = make_float2(y0 * f, y1 * f);
        }
    };
    // Rank 0: tile iteration i summed over the cluster's ranks (in rank order), then its epilogue.
    auto cluster_epilogue = [&](int i) {
        float2 y[NG];
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) {
            float y0 = 0.f, y1 = 0.f;
            for (int r = 0; r < S; ++r) {
                const float2 q = *cluster.map_shared_rank(&cpart[i & 1][ng][lane], r);
                y0 += q.x;
                y1 += q.y;
            }
            y[ng] = make_float2(y0, y1);
        }
        epilogue(blockIdx.x + i * gridDim.x, y);
    };
    auto reducer = [&](int i) { return kWarps - 1 - (i & (kWarps - 1)); };
    // After the barrier of tile iteration i: its local partial, and (split-K, rank 0) the previous
    // iteration's cluster sum, whose peer partials the barrier has made visible.
    auto finish_tile = [&](int i) {
        if (warp == reducer(i)) {
            float2 y[NG];
            local_tile(i, y);
            if (S == 1) {
                epilogue(blockIdx.x + i * gridDim.x, y);
            } else {
#pragma unroll
                for (int ng = 0; ng < NG; ++ng) cpart[i & 1][ng][lane] = y[ng];
            }
        }
        if (S > 1 && ks == 0 && i > 0 && warp == reducer(i - 1)) cluster_epilogue(i - 1);
    };

    if (nq == 0) {  // no pieces for this warp (a short K range): zero partials, barriers, epilogues
        for (int i = 0; i < my_tiles; ++i) {
#pragma unroll
            for (int ng = 0; ng < NG; ++ng) red[i & 1][warp][ng][lane] = make_float2(0.f, 0.f);
            cluster_barrier();
            finish_tile(i);
        }
    } else {
        float acc[NG][4];
#pragma unroll
        for (int ng = 0; ng < NG; ++ng) acc[ng][0] = acc[ng][1] = acc[ng][2] = acc[ng][3] = 0.f;
        float rs2[2] = {1.f, 1.f};
        int c_q = 0, c_i = 0;
        const int col_off = g * 64 + t * 16;  // this lane's column g, quad slot t inside a unit
        for (int s = 0; s < total; s += kMmaRing) {
#pragma unroll
            for (int d = 0; d < kMmaRing; ++d) {
                if (s + d < total) {
#pragma unroll
                    for (int l = 0; l < kMmaLoads; ++l) {
                        const int piece = p0 + kMmaLoads * c_q + l;
                        if (piece < p1) {
                            const char* ub = xs + static_cast<size_t>(piece * KU - u_lo) * C2 * 64 + col_off;
                            if constexpr (NG <= 2) {
                                // B fragments of the whole piece: KU 16-byte loads per column group.
                                uint32_t b[NG][8];
#pragma unroll
                                for (int ng = 0; ng < NG; ++ng) {
                                    const bool col_ok = 8 * ng + g < C2;
#pragma unroll
                                    for (int j = 0; j < KU; ++j) {
                                        uint4 q = make_uint4(0, 0, 0, 0);
                                        if (col_ok)
                                            q = *reinterpret_cast<const uint4*>(ub + static_cast<size_t>(j) * C2 * 64 +
                                                                                ng * 8 * 64);
                                        b[ng][4 * j] = q.x, b[ng][4 * j + 1] = q.y, b[ng][4 * j + 2] = q.z,
                                        b[ng][4 * j + 3] = q.w;
                                    }
                                }
                                if constexpr (kI8) {
#pragma unroll
                                    for (int jj = 0; jj < 4; ++jj) {
                                        uint32_t a0, a1, a2, a3;
                                        i8x4_to_h2x2(u4_get(ring[d][0][l], jj), a0, a2);
                                        i8x4_to_h2x2(u4_get(ring[d][1][l], jj), a1, a3);
#pragma unroll
                                        for (int ng = 0; ng < NG; ++ng)
                                            mma_16816(acc[ng], a0, a1, a2, a3, b[ng][2 * jj], b[ng][2 * jj + 1], false);
                                    }
                                } else {
#pragma unroll
                                    for (int jj = 0; jj < 2; ++jj) {
                                        const uint32_t a0 = u4_get(ring[d][0][l], 2 * jj), a2 = u4_get(ring[d][0][l], 2 * jj + 1);
                                        const uint32_t a1 = u4_get(ring[d][1][l], 2 * jj), a3 = u4_get(ring[d][1][l], 2 * jj + 1);
#pragma unroll
                                        for (int ng = 0; ng < NG; ++ng)
                                            mma_16816(acc[ng], a0, a1, a2, a3, b[ng][2 * jj], b[ng][2 * jj + 1], kBF);
                                    }
                                }
                            } else {
                                // Four column groups: B fragments loaded per MMA (8 bytes) to bound registers.
#pragma unroll
                                for (int jj = 0; jj < (kI8 ? 4 : 2); ++jj) {
                                    uint32_t a0, a1, a2, a3;
                                    if constexpr (kI8) {
                                        i8x4_to_h2x2(u4_get(ring[d][0][l], jj), a0, a2);
                                        i8x4_to_h2x2(u4_get(ring[d][1][l], jj), a1, a3);
                                    } else {
                                        a0 = u4_get(ring[d][0][l], 2 * jj), a2 = u4_get(ring[d][0][l], 2 * jj + 1);
                                        a1 = u4_get(ring[d][1][l], 2 * jj), a3 = u4_get(ring[d][1][l], 2 * jj + 1);
                                    }
                                    const char* jb = ub + static_cast<size_t>(kI8 ? (jj >> 1) : 0) * C2 * 64 +
                                                     (kI8 ? (jj & 1) : jj) * 8;
#pragma unroll
                                    for (int ng = 0; ng < NG; ++ng) {
                                        uint2 q = make_uint2(0, 0);
                                        if (8 * ng + g < C2) q = *reinterpret_cast<const uint2*>(jb + ng * 8 * 64);
                                        mma_16816(acc[ng], a0, a1, a2, a3, q.x, q.y, kBF);
                                    }
                                }
                            }
                        }
                        issue_piece(ring[d], l);  // piece l of this slot is free again: refill it now
                    }
                    if (kI8 && c_q == 0) rs2[0] = sring[d][0], rs2[1] = sring[d][1];
                    issue_finish(sring[d]);
                    if (++c_q == nq) {
#pragma unroll
                        for (int ng = 0; ng < NG; ++ng) {
                            red[c_i & 1][warp][ng][lane] =
                                make_float2((acc[ng][0] + acc[ng][1]) * rs2[0], (acc[ng][2] + acc[ng][3]) * rs2[1]);
                            acc[ng][0] = acc[ng][1] = acc[ng][2] = acc[ng][3] = 0.f;
                        }
                        cluster_barrier();
                        finish_tile(c_i);
                        c_q = 0;
                        ++c_i;
                    }
                }
            }
        }
    }
    if (S > 1) {
        // The last tile's partials are complete after this barrier; the second keeps every CTA's shared
        // memory alive until rank 0 has read it.
        cluster.sync();
        if (ks == 0 && my_tiles > 0 && warp == reducer(my_tiles - 1)) cluster_epilogue(my_tiles - 1);
        cluster.sync();
    }
    if (psum && ks == 0) {
        // Every partial of this CTA's tiles is on its way: read every rank's values of the same tiles (the
        // same CTA index on every rank) as they arrive, and add them in rank order.
        const PeerSum* ps = p.peer;
        const int nr = ps->nranks, me = ps->rank;
        char* mine = ps->mbox[me];
        __syncthreads();
        float* out = static_cast<float*>(p.seg[0].out);
        const long long ld = p.seg[0].ld;
        const int per = 16 * M;
        const long long t0 = clock64();
        bool late = false;
        for (int idx = threadIdx.x; idx < my_tiles * per; idx += kThreads) {
            const int i = idx / per, rem = idx - (idx / per) * per, m = rem >> 4;
            const int r = (blockIdx.x + i * gridDim.x) * 16 + (rem & 15);
            if (r >= N) continue;
            const long long si = static_cast<long long>(m) * N + r;
            float v = out[m * ld + r];
            for (int src = 0; src < nr; ++src) {
                const unsigned long long* q = peer_sum_slot(mine, par, src) + si;
                unsigned long long w = ld_tagged_sys(q);
                while (static_cast<unsigned>(w >> 32) != ep && !late) {
                    if (clock64() - t0 > kPeerSumWaitCycles) {
                        late = true;
                        if (ps->error) atomicExch(ps->error, 1);
                    }
                    w = ld_tagged_sys(q);
                }
                v += __uint_as_float(static_cast<unsigned>(w));
            }
            out[m * ld + r] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            // The last CTA of the call advances the epoch for the next one.
            __threadfence();
            unsigned* done = peer_sum_counter(mine, 1);
            if (atomicAdd(done, 1u) == gridDim.x - 1) {
                *done = 0u;
                __threadfence();
                *reinterpret_cast<volatile unsigned*>(peer_sum_counter(mine, 0)) = ep;
            }
        }
    }
}

bool g_gemv_mma = true;
bool g_gemv_bulk = true;  // the bulk-copy one-row kernel where it applies (l0b_set_gemv_bulk)
int g_gemv_fill_split = 2;  // largest split-K taken only to fill idle SMs (l0b_set_gemv_fill_split)
bool g_gemv_bulk_short = false;  // blocked projections with short rows on the bulk GEMV too
bool g_gemv_ksplit = true;  // blocked one-row int8 projections on the k-split GEMV (l0b_set_gemv_ksplit)
int g_ksplit_stages = 4;     // stages of the k-split GEMV's ring (l0b_set_gemv_ksplit_stages)
int g_l2_prefetch_mb = 0;    // gate/up megabytes prefetched into L2 by the decode step (l0b_set_l2_prefetch)

template <typename F, typename... A>
l0b_status launch_on(l0b_device* dev, cudaStream_t stream, F kernel, dim3 g, dim3 b, size_t smem, A... args) {
    if (dev) return dev->launch(kernel, g, b, smem, args...);
    kernel<<<g, b, smem, stream>>>(args...);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
    add_launches(1);
    return L0B_OK;
}

// ---------------------------------------------------------------------------------------------
// Bulk-streamed tensor-core GEMV for one activation row (decode at batch 1), int8 weights.
//
// A tile's 16 weight rows are one contiguous block of HBM (8 gate + 8 up rows for SwiGLU: two blocks),
// so a whole tile arrives in shared memory with one 1-D bulk copy (cp.async.bulk, completing on an
// mbarrier) of 16 K bytes (57 KB at K = 3584). Large contiguous copies are what the copy engine streams
// fastest: a read-only probe of 8-64 KB copies measured 7.1-7.3 TB/s on B200, while copies of 512-byte
// row segments (one per row) and 3-D tensor-map boxes of 128-byte lines were bound by the engine's cost
// per operation and per line (0.5 and 2 TB/s). A producer warp keeps 2-4 stages in flight per SM
// (issued before the dependency wait: weights never depend on the previous kernel). The weights go to
// the integer tensor cores as they are (mma.sync m16n8k32 s8, no conversion): the activation row enters
// as four balanced base-128 int8 digits of x 2^e (|x 2^e| < 2^26, about 27 bits of the row's largest
// value), four B columns of one MMA, so the s32 sums are exact (|sum| < 2^31 for K < 2^18) and the
// digit columns join in int64 and f64 before one rounding. Sixteen consumer warps split each unit's
// pieces; their partial sums meet (exact integers: any order gives the same bits) in double-buffered
// shared memory, and a reducer warp rotating by tile runs the epilogue while the others go on.
// ---------------------------------------------------------------------------------------------
constexpr int kBulkCW = 16;                      // consumer warps
constexpr int kBulkConsumers = kBulkCW * 32;
constexpr int kBulkThreads = kBulkConsumers + 32;  // consumers + 1 producer warp
constexpr int kBulkMaxStages = 8;
constexpr int kBulkSmemBudget = 206 * 1024;  // dynamic; the static arrays take ~17 KB of the 227 KB
constexpr long long kBulkWaitCycles = 4000000000LL;

__device__ __forceinline__ uint32_t bulk_smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Bounded mbarrier wait (~2 s): false on timeout.
__device__ __forceinline__ bool bulk_wait(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bulk_smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > kBulkWaitCycles) return false;
    }
}

__device__ __forceinline__ void bulk_consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kBulkConsumers) : "memory"); }

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     bulk_smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(bulk_smem_u32(bar))
                 : "memory");
}

// Activations staged as hi/lo pairs (bytes) and the ring of `stages` units of 16 rows x UK bytes.
__host__ __device__ inline size_t bulk_xs_bytes(int K) { return (static_cast<size_t>(K) * 4 + 1023) & ~static_cast<size_t>(1023); }
inline size_t bulk_smem_bytes(int K, int stages, int UK) {
    return 1024 + bulk_xs_bytes(K) + static_cast<size_t>(stages) * 16 * UK + 2 * kBulkMaxStages * 8;
}
// Ring of whole tiles (row-major weights; units of blocked k blocks keep every stage that fits). By default
// it holds at most kBulkRingBytes of tiles (at least two): two 57 KB tiles at K = 3584 (gate/up, LM head)
// leave an SM room for the next k-split GEMV's CTAs, which then start their weight copies while this
// kernel drains (config 2 bs1: 2.192 ms per step against 2.231 with three stages), and short rows keep a
// deep ring (eight 14 KB tiles at K = 896). l0b_set_gemv_bulk_stages: n >= 2 caps the ring at n tiles, 1
// takes as many as the shared-memory budget holds, 0 restores the default.
constexpr int kBulkRingBytes = 120 * 1024;
int g_bulk_max_stages = 0;
inline int bulk_stages(int K, int UK, bool whole_tiles) {
    int top = kBulkMaxStages;
    if (whole_tiles && g_bulk_max_stages >= 2) {
        top = g_bulk_max_stages < kBulkMaxStages ? g_bulk_max_stages : kBulkMaxStages;
    } else if (whole_tiles && g_bulk_max_stages == 0) {
        const int by_bytes = kBulkRingBytes / (16 * UK);
        top = by_bytes < 2 ? 2 : (by_bytes < kBulkMaxStages ? by_bytes : kBulkMaxStages);
    }
    for (int s = top; s >= 2; --s)
        if (bulk_smem_bytes(K, s, UK) <= static_cast<size_t>(kBulkSmemBudget)) return s;
    return 0;
}

// Split-K units (projections with few row tiles -- o_proj, down, q/k/v -- stored in the blocked layout,
// p.kb > 0): a unit is up to p.ugroup consecutive k blocks of one 16-row tile, which the blocked layout
// keeps contiguous, so a unit is one bulk copy of up to ugroup * 16 * kb bytes. A CTA's copies complete
// one stage at a time, at about one DRAM latency each (a probe of copies alone: 8 KB stages 3.0 TB/s,
// 16 KB 6.0, 32 KB and more 7.0 on B200), so units are made large enough to stream at full rate.
// Units are taken in (tile, group) order -- their order in HBM -- and each CTA a contiguous range of
// them, so the work per SM differs by at most one unit. A warp keeps its sums across the units of a
// tile in registers; at the end of the tile (or of the CTA's range) the warps' sums meet once. A tile
// whose units two CTAs share (the host keeps every range at least units-per-tile - 1 long, so never
// more than two) is finished by the second CTA to get there: each writes its 16 partial sums to
// p.part[tile][first unit == 0 ? 0 : 1] and bumps p.counters[tile]; the one that finds the other's
// partial adds the two (a + b == b + a: the result does not depend on arrival order), runs the
// epilogue and re-arms the counter.
template <bool BLK>
__global__ void __launch_bounds__(kBulkThreads, 1) gemv_bulk_kernel(const GemvParams p, int stages, int* error) {
    extern __shared__ char bulk_smem[];
    constexpr int PE = 64;  // k per piece: lane t holds bytes [16 t, 16 t + 16) of rows g and g + 8
    __shared__ int4 red[2][kBulkCW][32];
    __shared__ float ssq_s[kBulkCW], amax_s[kBulkCW];
    __shared__ double oscale_s;
    // After one timed-out wait the rest of the launch only drains: abort_s is set and units from
    // issued_s on (never copied, or stuck) are not waited for, so the kernel returns after one timeout.
    __shared__ int abort_s, issued_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int N = p.N, K = p.K;
    const bool swiglu = p.epi == EPI_SWIGLU;
    const int half_n = N >> 1;
    constexpr bool blocked = BLK;
    const int kb = blocked ? kWeightBlock : K;  // k per block (row-major: the whole row)
    const int nb = K / kb;                      // blocks per row
    const int G = blocked ? p.ugroup : 1;       // blocks per unit
    const int ug = blocked ? (nb + G - 1) / G : 1;  // units per tile
    const int ppb = kb / PE;                    // pieces per block
    const int npieces = K / PE;                // pieces of a whole row (x staging)
    const int ntiles = swiglu ? (half_n + 7) / 8 : (N + 15) / 16;
    const int nunits = ntiles * ug;
    const int u_begin = static_cast<int>(static_cast<long long>(nunits) * blockIdx.x / gridDim.x);
    const int u_end = static_cast<int>(static_cast<long long>(nunits) * (blockIdx.x + 1) / gridDim.x);
    char* const base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(bulk_smem) + 1023) & ~uintptr_t(1023));
    char* xs = base;
    char* ring = base + bulk_xs_bytes(K);
    const size_t stage_bytes = static_cast<size_t>(16) * kb * G;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + stages * stage_bytes);
    uint64_t* empty = full + kBulkMaxStages;
    const char* W = static_cast<const char*>(p.w);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bulk_smem_u32(&full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bulk_smem_u32(&empty[s])), "r"(kBulkCW)
                         : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_s = 0;
        issued_s = INT_MAX;
    }
    __syncthreads();

    if (warp == kBulkCW) {
        // Producer: unit i's rows as one contiguous copy (S = 1; SwiGLU: two), or one copy per row of its
        // segment (S > 1). Rows past the matrix are not copied (their stage bytes are stale and their
        // outputs are never stored).
        if (lane == 0) {
            for (int u = u_begin, i = 0; u < u_end; ++u, ++i) {
                const int s = i % stages;
                if (i >= stages && !bulk_wait(&empty[s], ((i / stages) & 1) ^ 1)) {
                    if (error) atomicExch(error, 1);
                    atomicMin(&issued_s, i);
                    __threadfence_block();
                    atomicExch(&abort_s, 1);
                    break;
                }
                char* dst = ring + s * stage_bytes;
                const int tile = u / ug, uj = u - tile * ug;
                if (swiglu) {
                    const int r0 = tile * 8, nr = min(8, half_n - r0);
                    const uint32_t bytes = static_cast<uint32_t>(nr) * K;
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bulk_smem_u32(&full[s])),
                                 "r"(2 * bytes)
                                 : "memory");
                    bulk_copy(dst, W + static_cast<long long>(r0) * K, bytes, &full[s]);
                    bulk_copy(dst + 8 * K, W + static_cast<long long>(half_n + r0) * K, bytes, &full[s]);
                } else if constexpr (!blocked) {
                    const int r0 = tile * 16, nr = min(16, N - r0);
                    const uint32_t bytes = static_cast<uint32_t>(nr) * K;
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bulk_smem_u32(&full[s])),
                                 "r"(bytes)
                                 : "memory");
                    bulk_copy(dst, W + static_cast<long long>(r0) * K, bytes, &full[s]);
                } else {
                    // Blocks [uj * G, uj * G + nblk) of the tile: contiguous in the blocked layout.
                    const int nblk = min(G, nb - uj * G);
                    const uint32_t bytes = static_cast<uint32_t>(nblk) * 16 * kb;
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bulk_smem_u32(&full[s])),
                                 "r"(bytes)
                                 : "memory");
                    bulk_copy(dst, W + static_cast<long long>(tile) * 16 * K + static_cast<long long>(uj) * G * 16 * kb,
                              bytes, &full[s]);
                }
            }
        }
        return;
    }

    // Consumers.
    pdl_wait();
    pdl_launch_dependents();
    // Stage x as int8 digits: item (piece pc, lane t) is x[64 pc + 16 t, + 16) -- the k of the 16 weight
    // bytes lane t loads from each row -- and its slot (pc * 16 + t * 4 + dg) * 16 holds digit dg of those
    // 16 values (byte i <-> k 64 pc + 16 t + i). Pass 1 keeps the raw values (times the RMS-norm weight)
    // in the item's 64 bytes and forms the row's sum of squares and largest magnitude; pass 2 applies
    // 1/RMS and 2^e (largest |x| 2^e just below 2^26) and writes the four balanced base-128 digits.
    {
        const int items = npieces * 4;
        const float* xf = static_cast<const float*>(p.x);
        const bool xvec = p.x_dtype == L0B_F32 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
        float ss = 0.f, amax = 0.f;
        for (int it = threadIdx.x; it < items; it += kBulkConsumers) {
            const int k0 = it * 16;  // (pc, t) = (it / 4, it % 4): 64 pc + 16 t
            float4* slot = reinterpret_cast<float4*>(xs + static_cast<size_t>(it) * 64);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float4 a;
                if (xvec) {
                    a = *reinterpret_cast<const float4*>(xf + k0 + 4 * q);
                } else {
                    a = make_float4(load_as_float(p.x, p.x_dtype, k0 + 4 * q), load_as_float(p.x, p.x_dtype, k0 + 4 * q + 1),
                                    load_as_float(p.x, p.x_dtype, k0 + 4 * q + 2), load_as_float(p.x, p.x_dtype, k0 + 4 * q + 3));
                }
                if (p.norm_w) {
                    ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
                    const float4 w = *reinterpret_cast<const float4*>(p.norm_w + k0 + 4 * q);
                    a.x *= w.x, a.y *= w.y, a.z *= w.z, a.w *= w.w;
                }
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
                slot[q] = a;
            }
        }
        ss = warp_sum(ss);
        amax = warp_max(amax);
        if (lane == 0) {
            ssq_s[warp] = ss;
            amax_s[warp] = amax;
        }
        bulk_consumer_sync();
        float sst = 0.f, am = 0.f;
#pragma unroll
        for (int w = 0; w < kBulkCW; ++w) {
            sst += ssq_s[w];
            am = fmaxf(am, amax_s[w]);
        }
        const float rs = p.norm_w ? 1.0f / sqrtf(sst / static_cast<float>(K) + p.eps) : 1.0f;
        int e = 0;
        if (am * rs > 0.f && isfinite(am * rs)) {
            int ex;
            frexpf(am * rs, &ex);  // am rs = f 2^ex, f in [0.5, 1): am rs 2^(26 - ex) < 2^26
            e = min(max(26 - ex, -120), 120);
        }
        const float sc = rs * ldexpf(1.0f, e);
        if (threadIdx.x == 0) oscale_s = ldexp(1.0, -e);
        for (int it = threadIdx.x; it < items; it += kBulkConsumers) {
            float4* slot = reinterpret_cast<float4*>(xs + static_cast<size_t>(it) * 64);
            uint32_t dw[4][4] = {};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 a = slot[q];
                const float v[4] = {a.x * sc, a.y * sc, a.z * sc, a.w * sc};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    int X = __float2int_rn(v[i]);
#pragma unroll
                    for (int dg = 0; dg < 3; ++dg) {
                        const int d = ((X + 64) & 127) - 64;
                        dw[dg][q] |= (static_cast<uint32_t>(d) & 0xFFu) << (8 * i);
                        X = (X - d) >> 7;
                    }
                    dw[3][q] |= (static_cast<uint32_t>(X) & 0xFFu) << (8 * i);
                }
            }
            uint4* out = reinterpret_cast<uint4*>(slot);
#pragma unroll
            for (int dg = 0; dg < 4; ++dg) out[dg] = make_uint4(dw[dg][0], dw[dg][1], dw[dg][2], dw[dg][3]);
        }
        bulk_consumer_sync();
    }

    // Epilogue of tile `tile` from the (row g, row g + 8) outputs; the lanes with t == 0 hold the real ones.
    // Rows (g, g + 8) of a tile and their scales; the reducer loads the scales when the tile starts so
    // the epilogue does not wait for them.
    auto tile_rows2 = [&](int tile, int& r0, int& r1, bool& v0, bool& v1) {
        r0 = swiglu ? tile * 8 + g : tile * 16 + g;
        r1 = swiglu ? r0 + half_n : r0 + 8;
        v0 = swiglu ? r0 < half_n : r0 < N;
        v1 = swiglu ? v0 : r1 < N;
    };
    const __half* sc = static_cast<const __half*>(p.scales);
    auto epilogue = [&](int tile, float y0, float y1) {
        int r0, r1;
        bool v0, v1;
        tile_rows2(tile, r0, r1, v0, v1);
        const bool live = t == 0;
        if (p.epi == EPI_ARGMAX) {
            unsigned long long key = 0;
            if (live && v0) key = argmax_key(epilogue_store(p, r0, 0, y0, false), r0 + p.argmax_base);
            if (live && v1) key = max(key, argmax_key(epilogue_store(p, r1, 0, y1, false), r1 + p.argmax_base));
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
            if (lane == 0 && key) atomicMax(p.argmax, key);
        } else if (live) {
            if (swiglu) {
                if (v0) epilogue_store(p, r0, 0, silu(y0) * y1);
            } else {
                if (v0) epilogue_store(p, r0, 0, y0);
                if (v1) epilogue_store(p, r1, 0, y1);
            }
        }
    };
    // A tile two CTAs share: publish this CTA's part (the exact x 2^e-scaled sums as doubles, 32 floats
    // per part); the second to arrive adds the other's (exact: both are integers times the same 2^-e,
    // below 2^53) and finishes.
    auto fixup = [&](int tile, int slot, double d0, double d1, float s0, float s1) {
        double* mine = reinterpret_cast<double*>(p.part) + (static_cast<long long>(tile) * 2 + slot) * 16;
        if (t == 0) {
            mine[g] = d0;
            mine[g + 8] = d1;
        }
        __threadfence();
        __syncwarp();
        unsigned old = 0;
        if (lane == 0) old = atomicAdd(p.counters + tile, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == 0) return;
        __threadfence();
        const double* other = reinterpret_cast<const double*>(p.part) + (static_cast<long long>(tile) * 2 + (slot ^ 1)) * 16;
        if (t == 0) {
            d0 += __ldcg(other + g);
            d1 += __ldcg(other + g + 8);
        }
        if (lane == 0) p.counters[tile] = 0u;
        epilogue(tile, static_cast<float>(d0 * s0), static_cast<float>(d1 * s1));
    };

    // Digit dg of x for this lane's 16 k of a piece: columns g < 4 of the B fragment, zero above.
    const char* xcol = g < 4 ? xs + t * 64 + g * 16 : nullptr;
    float sc0 = 0.f, sc1 = 0.f;  // the row scales of the tile this warp reduces next
    int acc[4] = {0, 0, 0, 0}, acc2[4] = {0, 0, 0, 0};
    int seg_first = 0;  // first unit of the current tile in this CTA's range
    int j = 0;          // tiles finished by this CTA (reducer rotation, red[] buffer parity)
    for (int u = u_begin, i = 0; u < u_end; ++u, ++i) {
        const int s = i % stages;
        const int tile = u / ug, uj = u - tile * ug;
        const bool first = i == 0 || uj == 0;
        const bool last = u + 1 == u_end || uj == ug - 1;
        // This warp's pieces of the unit (a unit of nblk blocks has nblk * ppb pieces).
        const int npu = blocked ? min(G, nb - uj * G) * ppb : npieces;
        const int p0 = warp * npu / kBulkCW, p1 = (warp + 1) * npu / kBulkCW;
        const bool reducer = warp == kBulkCW - 1 - (j & (kBulkCW - 1));
        if (first) {
            seg_first = uj;
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] = acc2[e] = 0;
            if (reducer) {
                int r0, r1;
                bool v0, v1;
                tile_rows2(tile, r0, r1, v0, v1);
                sc0 = v0 ? __half2float(sc[r0]) : 0.f;
                sc1 = v1 ? __half2float(sc[r1]) : 0.f;
            }
        }
        // Units issued before an abort are still waited for (their copies land in this CTA's memory).
        const bool skip = *reinterpret_cast<volatile int*>(&abort_s) && i >= *reinterpret_cast<volatile int*>(&issued_s);
        if (!skip && !bulk_wait(&full[s], (i / stages) & 1) && lane == 0) {
            if (error) atomicExch(error, 1);
            atomicMin(&issued_s, i);
            __threadfence_block();
            atomicExch(&abort_s, 1);
        }
        const char* st = ring + s * stage_bytes + t * 16;
        const int xpiece0 = uj * G * ppb;  // this unit's first piece in the staged activations
        // Rows g and g + 8 of piece `piece`: blocked, block piece / 8 of the stage (kWeightBlock = 512 =
        // 8 pieces), row r of the block; row-major, the stage is the tile with rows K apart.
        const char* wg0 = st + static_cast<size_t>(g) * kb;
        const char* wg1 = st + static_cast<size_t>(g + 8) * kb;
        for (int piece = p0; piece < p1; ++piece) {
            const size_t off = blocked ? static_cast<size_t>(piece >> 3) * (16 * kWeightBlock) + (piece & 7) * PE
                                       : static_cast<size_t>(piece) * PE;
            const uint4 w0 = *reinterpret_cast<const uint4*>(wg0 + off);
            const uint4 w1 = *reinterpret_cast<const uint4*>(wg1 + off);
            const uint4 b = xcol ? *reinterpret_cast<const uint4*>(xcol + static_cast<size_t>(xpiece0 + piece) * 256)
                                 : make_uint4(0, 0, 0, 0);
            // k [16 t, 16 t + 8) and [16 t + 8, 16 t + 16) of the piece; two accumulators: independent chains.
            mma_s8_16832(acc, w0.x, w1.x, w0.y, w1.y, b.x, b.y);
            mma_s8_16832(acc2, w0.z, w1.z, w0.w, w1.w, b.z, b.w);
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bulk_smem_u32(&empty[s])) : "memory");
        if (!last) continue;
        red[j & 1][warp][lane] = make_int4(acc[0] + acc2[0], acc[1] + acc2[1], acc[2] + acc2[2], acc[3] + acc2[3]);
        bulk_consumer_sync();
        // Tile j's partials are complete; its reducer sums them (exactly, in int32) while the other warps go
        // on (the next write to red[j & 1] comes after the next barrier, which the reducer reaches only
        // when done), then joins the four digit columns: lane t holds columns 2t, 2t + 1 of rows g, g + 8.
        if (reducer) {
            int c[4] = {0, 0, 0, 0};
#pragma unroll
            for (int w = 0; w < kBulkCW; ++w) {
                const int4 q = red[j & 1][w][lane];
                c[0] += q.x, c[1] += q.y, c[2] += q.z, c[3] += q.w;
            }
            const long long lo0 = c[0] + 128LL * c[1], lo1 = c[2] + 128LL * c[3];  // t = 0: digits 0, 1; t = 1: 2, 3
            const long long hi0 = __shfl_down_sync(0xffffffffu, lo0, 1);
            const long long hi1 = __shfl_down_sync(0xffffffffu, lo1, 1);
            const double d0 = static_cast<double>(lo0 + 16384LL * hi0) * oscale_s;
            const double d1 = static_cast<double>(lo1 + 16384LL * hi1) * oscale_s;
            if constexpr (!blocked) epilogue(tile, static_cast<float>(d0 * sc0), static_cast<float>(d1 * sc1));
            else if (seg_first == 0 && uj == ug - 1)
                epilogue(tile, static_cast<float>(d0 * sc0), static_cast<float>(d1 * sc1));
            else fixup(tile, seg_first == 0 ? 0 : 1, d0, d1, sc0, sc1);
        }
        ++j;
    }
}

// ---------------------------------------------------------------------------------------------
// K-split one-row GEMV over blocked int8 weights (q/k/v, o_proj, down at batch 1).
//
// CTA (k block kb, tile group tg) multiplies the 512 k of block kb of every 16-row tile of its group:
// the (tile, kb) blocks are 8 KB contiguous each in the blocked layout, four per stage by bulk copy.
// The activation row is read once for the RMS norm and its largest value (every CTA forms the same
// e), but only the CTA's own 512 values become int8 digits, so no CTA stages the whole row. The weights
// feed mma.sync m16n8k32 s8 as loaded (as in gemv_bulk_kernel); warp w takes pieces 2 (w % 4), +1 of
// block w / 4 of each stage, joins its digit columns to one exact int64 per row and adds it to the
// row's int64 sum with one atomic: integer addition is exact, so the result does not depend on the
// order the CTAs arrive in. (Adding a block's four warps in shared memory first, one atomic per row,
// measured slower: the atomics are not what bounds the kernel.) The last CTA of a group to finish (a counter per group) turns the group's
// sums into outputs -- times 2^-e and the row scale in f64, one rounding -- runs the store / bias /
// residual / SwiGLU epilogue, and leaves the sums and the counter zero for the next launch.
// ---------------------------------------------------------------------------------------------
constexpr int kKsCW = 16;
constexpr int kKsThreads = kKsCW * 32 + 32;  // consumers + 1 producer warp
constexpr int kKsMaxStages = 6;
constexpr int kKsBlockBytes = 16 * kWeightBlock;  // one (tile, k block) block
constexpr int kKsStageBytes = 4 * kKsBlockBytes;

// This CTA's slice of [base, base + bytes) as L2 prefetches of at most 32 KB (16-byte multiples).
__device__ __forceinline__ void l2_prefetch_slice(const void* base, long long bytes) {
    if (!base || bytes < 16 || (reinterpret_cast<uintptr_t>(base) & 15)) return;
    const long long G = gridDim.x, c = blockIdx.x;
    const long long b0 = (bytes * c / G) & ~15LL;
    const long long b1 = c + 1 == G ? (bytes & ~15LL) : ((bytes * (c + 1) / G) & ~15LL);
    for (long long o = b0; o < b1; o += 32768) {
        const uint32_t n = static_cast<uint32_t>(b1 - o < 32768 ? b1 - o : 32768);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const char*>(base) + o), "r"(n)
                     : "memory");
    }
}

__global__ void __launch_bounds__(kKsThreads, 1) gemv_ksplit_kernel(const GemvParams p, int stages, int groups,
                                                                  int* error) {
    extern __shared__ char ks_smem[];
    constexpr int PE = 64;
    __shared__ float ssq_s[kKsCW], amax_s[kKsCW];
    __shared__ double oscale_s;
    // After a timed-out wait the rest of the launch only drains: units from issued_s on were never
    // copied and are not waited for; earlier ones still are (their copies land in this CTA's memory).
    __shared__ int abort_s, issued_s, last_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int N = p.N, K = p.K, nb = K / kWeightBlock;
    // SwiGLU: the groups split the gate tiles, and a group's list is its gate tiles then the matching up
    // tiles (N / 2 rows further), so its last CTA holds both sums of every output.
    const bool swiglu = p.epi == EPI_SWIGLU;
    const int half_tiles = (N >> 1) >> 4;
    const int ntiles = swiglu ? half_tiles : N >> 4;
    const int kbi = blockIdx.x % nb, tg = blockIdx.x / nb;
    const int t_begin = static_cast<int>(static_cast<long long>(ntiles) * tg / groups);
    const int t_end = static_cast<int>(static_cast<long long>(ntiles) * (tg + 1) / groups);
    const int nt = t_end - t_begin;
    const int nlist = swiglu ? 2 * nt : nt;
    auto tile_of = [&](int j) { return swiglu && j >= nt ? half_tiles + t_begin + (j - nt) : t_begin + j; };
    const int nunits = (nlist + 3) / 4;  // stages of up to four tiles
    char* const base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(ks_smem) + 1023) & ~uintptr_t(1023));
    char* xs = base;            // 512 k as digits: item (piece, t) at (piece * 4 + t) * 64, digit dg at + dg * 16
    char* ring = base + 2048;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(stages) * kKsStageBytes);
    uint64_t* empty = full + kKsMaxStages;
    const char* W = static_cast<const char*>(p.w);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bulk_smem_u32(&full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bulk_smem_u32(&empty[s])), "r"(kKsCW)
                         : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        abort_s = 0;
        issued_s = INT_MAX;
    }
    __syncthreads();

    if (warp == kKsCW) {
        // Producer: the blocks of four tiles per stage (weights never depend on the previous kernel).
        if (lane == 0) {
            for (int u = 0; u < nunits; ++u) {
                const int s = u % stages;
                if (u >= stages && !bulk_wait(&empty[s], ((u / stages) & 1) ^ 1)) {
                    if (error) atomicExch(error, 1);
                    atomicMin(&issued_s, u);
                    __threadfence_block();
                    atomicExch(&abort_s, 1);
                    break;
                }
                const int nblk = min(4, nlist - 4 * u);
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bulk_smem_u32(&full[s])),
                             "r"(nblk * kKsBlockBytes)
                             : "memory");
                for (int b = 0; b < nblk; ++b)
                    bulk_copy(ring + static_cast<size_t>(s) * kKsStageBytes + b * kKsBlockBytes,
                              W + (static_cast<long long>(tile_of(4 * u + b)) * nb + kbi) * kKsBlockBytes, kKsBlockBytes,
                              &full[s]);
                // Once the first stages are on their way, the later projection's weights go to L2.
                if (u + 1 == min(stages, nunits)) {
                    l2_prefetch_slice(p.l2pf[0], p.l2pf_bytes[0]);
                    l2_prefetch_slice(p.l2pf[1], p.l2pf_bytes[1]);
                }
            }
        }
        return;
    }

    pdl_wait();
    pdl_launch_dependents();
    // The row's sum of squares and largest magnitude (after the RMS-norm weight), over all of K.
    {
        const float* xf = static_cast<const float*>(p.x);
        float ss = 0.f, am = 0.f;
        // Eight 16-byte loads in flight per thread (one L2 round trip per eight, not per load).
        constexpr int kStep = 4 * kKsCW * 32;
        for (int k0 = 4 * threadIdx.x; k0 < K; k0 += 8 * kStep) {
            float4 a[8], w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int k = k0 + j * kStep;
                a[j] = k < K ? *reinterpret_cast<const float4*>(xf + k) : make_float4(0.f, 0.f, 0.f, 0.f);
                w[j] = (p.norm_w && k < K) ? *reinterpret_cast<const float4*>(p.norm_w + k) : make_float4(1.f, 1.f, 1.f, 1.f);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                ss = fmaf(a[j].x, a[j].x, fmaf(a[j].y, a[j].y, fmaf(a[j].z, a[j].z, fmaf(a[j].w, a[j].w, ss))));
                const float4 b = make_float4(a[j].x * w[j].x, a[j].y * w[j].y, a[j].z * w[j].z, a[j].w * w[j].w);
                am = fmaxf(am, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
            }
        }
        ss = warp_sum(ss);
        am = warp_max(am);
        if (lane == 0) {
            ssq_s[warp] = ss;
            amax_s[warp] = am;
        }
        bulk_consumer_sync();
        float sst = 0.f, amt = 0.f;
#pragma unroll
        for (int w = 0; w < kKsCW; ++w) {
            sst += ssq_s[w];
            amt = fmaxf(amt, amax_s[w]);
        }
        const float rs = p.norm_w ? 1.0f / sqrtf(sst / static_cast<float>(K) + p.eps) : 1.0f;
        int e = 0;
        if (amt * rs > 0.f && isfinite(amt * rs)) {
            int ex;
            frexpf(amt * rs, &ex);
            e = min(max(26 - ex, -120), 120);
        }
        const float sc = rs * ldexpf(1.0f, e);
        if (threadIdx.x == 0) oscale_s = ldexp(1.0, -e);
        // Digits of this CTA's 512 k: item i = (piece i / 4, lane i % 4) holds x[kb 512 + 16 i, + 16).
        if (threadIdx.x < 32) {
            const int k0 = kbi * kWeightBlock + 16 * threadIdx.x;
            uint32_t dw[4][4] = {};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float4 a = *reinterpret_cast<const float4*>(xf + k0 + 4 * q);
                if (p.norm_w) {
                    const float4 w = *reinterpret_cast<const float4*>(p.norm_w + k0 + 4 * q);
                    a.x *= w.x, a.y *= w.y, a.z *= w.z, a.w *= w.w;
                }
                const float v[4] = {a.x * sc, a.y * sc, a.z * sc, a.w * sc};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    int X = __float2int_rn(v[i]);
#pragma unroll
                    for (int dg = 0; dg < 3; ++dg) {
                        const int d = ((X + 64) & 127) - 64;
                        dw[dg][q] |= (static_cast<uint32_t>(d) & 0xFFu) << (8 * i);
                        X = (X - d) >> 7;
                    }
                    dw[3][q] |= (static_cast<uint32_t>(X) & 0xFFu) << (8 * i);
                }
            }
            uint4* out = reinterpret_cast<uint4*>(xs + threadIdx.x * 64);
#pragma unroll
            for (int dg = 0; dg < 4; ++dg) out[dg] = make_uint4(dw[dg][0], dw[dg][1], dw[dg][2], dw[dg][3]);
        }
        bulk_consumer_sync();
    }
    // This warp's block of each stage and its two pieces; their B fragments serve every tile.
    const int blk = warp >> 2, pc0 = (warp & 3) * 2;
    uint4 bx0 = make_uint4(0, 0, 0, 0), bx1 = make_uint4(0, 0, 0, 0);
    if (g < 4) {
        bx0 = *reinterpret_cast<const uint4*>(xs + (pc0 * 4 + t) * 64 + g * 16);
        bx1 = *reinterpret_cast<const uint4*>(xs + ((pc0 + 1) * 4 + t) * 64 + g * 16);
    }
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(p.acc);
    for (int u = 0; u < nunits; ++u) {
        const int s = u % stages;
        const bool skip = *reinterpret_cast<volatile int*>(&abort_s) && u >= *reinterpret_cast<volatile int*>(&issued_s);
        if (!skip && !bulk_wait(&full[s], (u / stages) & 1) && lane == 0) {
            if (error) atomicExch(error, 1);
            atomicMin(&issued_s, u);
            __threadfence_block();
            atomicExch(&abort_s, 1);
        }
        if (4 * u + blk < nlist) {
            const int tile = tile_of(4 * u + blk);
            const char* blkp = ring + static_cast<size_t>(s) * kKsStageBytes + blk * kKsBlockBytes + t * 16;
            const uint4 a0 = *reinterpret_cast<const uint4*>(blkp + g * kWeightBlock + pc0 * PE);
            const uint4 a1 = *reinterpret_cast<const uint4*>(blkp + (g + 8) * kWeightBlock + pc0 * PE);
            const uint4 c0 = *reinterpret_cast<const uint4*>(blkp + g * kWeightBlock + (pc0 + 1) * PE);
            const uint4 c1 = *reinterpret_cast<const uint4*>(blkp + (g + 8) * kWeightBlock + (pc0 + 1) * PE);
            int accA[4] = {0, 0, 0, 0}, accB[4] = {0, 0, 0, 0};
            mma_s8_16832(accA, a0.x, a1.x, a0.y, a1.y, bx0.x, bx0.y);
            mma_s8_16832(accB, a0.z, a1.z, a0.w, a1.w, bx0.z, bx0.w);
            mma_s8_16832(accA, c0.x, c1.x, c0.y, c1.y, bx1.x, bx1.y);
            mma_s8_16832(accB, c0.z, c1.z, c0.w, c1.w, bx1.z, bx1.w);
            const long long lo0 = (accA[0] + accB[0]) + 128LL * (accA[1] + accB[1]);
            const long long lo1 = (accA[2] + accB[2]) + 128LL * (accA[3] + accB[3]);
            const long long hi0 = __shfl_down_sync(0xffffffffu, lo0, 1);
            const long long hi1 = __shfl_down_sync(0xffffffffu, lo1, 1);
            if (t == 0) {
                atomicAdd(acc + tile * 16 + g, static_cast<unsigned long long>(lo0 + 16384LL * hi0));
                atomicAdd(acc + tile * 16 + g + 8, static_cast<unsigned long long>(lo1 + 16384LL * hi1));
            }
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bulk_smem_u32(&empty[s])) : "memory");
    }
    // The last CTA of the group to get here finishes the group's rows.
    __threadfence();
    bulk_consumer_sync();
    if (threadIdx.x == 0) last_s = atomicAdd(p.counters + tg, 1u) == static_cast<unsigned>(nb - 1);
    bulk_consumer_sync();
    if (!last_s) return;
    __threadfence();
    const __half* sc = static_cast<const __half*>(p.scales);
    auto row_out = [&](int r) {
        const long long D = static_cast<long long>(atomicExch(acc + r, 0ull));
        return static_cast<float>(static_cast<double>(D) * oscale_s * static_cast<double>(__half2float(sc[r])));
    };
    for (int r = t_begin * 16 + threadIdx.x; r < t_end * 16; r += kKsCW * 32) {
        if (swiglu) {
            const float yg = row_out(r), yu = row_out((N >> 1) + r);
            epilogue_store(p, r, 0, silu(yg) * yu);
        } else {
            epilogue_store(p, r, 0, row_out(r));
        }
    }
    if (threadIdx.x == 0) p.counters[tg] = 0u;
}

// Unit size of the one-row bulk GEMV, in k blocks (0 = the kernel does not apply): row-major weights
// take whole 16-row tiles when there are at least 8 tiles per SM (returns 1); blocked weights take the
// largest group of G <= 4 blocks that still gives every SM >= 6 units (smaller units balance the SMs,
// larger ones stream faster), keeps >= 3 stages in shared memory and every CTA's range at least
// units-per-tile - 1 long (a tile then spans at most two CTAs).
int bulk_group(const GemvParams& p, int sm_count) {
    const int ntiles = p.epi == EPI_SWIGLU ? (p.N / 2 + 7) / 8 : (p.N + 15) / 16;
    if (p.kb <= 0) return ntiles >= 8 * sm_count && bulk_stages(p.K, p.K, true) >= 2 ? 1 : 0;
    if (p.epi == EPI_SWIGLU || p.N % 16 != 0 || p.K % p.kb != 0 || p.kb != kWeightBlock) return 0;
    if (!p.part || !p.counters || p.counter_count < ntiles) return 0;
    const int nb = p.K / p.kb;
    // Short rows (q/k/v and o_proj at K = 3584: 7 blocks) stay on the register GEMV unless
    // l0b_set_gemv_bulk_short_rows(1); long ones (down at K = 18944: 37 blocks) take the bulk GEMV.
    if (nb < 16 && !g_gemv_bulk_short) return 0;
    for (int G = 4; G >= 1; --G) {
        const int ug = (nb + G - 1) / G;
        const long long units = static_cast<long long>(ntiles) * ug;
        if (bulk_stages(p.K, G * p.kb, false) < 3 || units / sm_count < ug - 1) continue;
        if (units >= 6LL * sm_count || G == 1) return G;
    }
    return 0;
}

// One activation row, int8 with one scale per row, 16-byte aligned, and a split (above) that applies.
bool bulk_applies(int w_dtype, const GemvParams& p, int sm_count) {
    if (!g_gemv_mma || !g_gemv_bulk || w_dtype != L0B_I8 || p.M != 1 || p.nseg < 1) return false;
    if (p.group < p.K || p.K % 64 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.w) % 16 != 0 || (p.x_dtype == L0B_F32 && (reinterpret_cast<uintptr_t>(p.x) & 15)))
        return false;
    if (p.norm_w && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)) return false;
    return bulk_group(p, sm_count) > 0;
}

l0b_status launch_bulk(l0b_device* dev, cudaStream_t stream, int sm_count, GemvParams p) {
    static bool configured = false;
    if (!configured) {
        for (const void* f : {reinterpret_cast<const void*>(gemv_bulk_kernel<true>),
                              reinterpret_cast<const void*>(gemv_bulk_kernel<false>)}) {
            cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkSmemBudget);
            if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        }
        configured = true;
    }
    p.ugroup = bulk_group(p, sm_count);
    const int UK = p.kb > 0 ? p.ugroup * p.kb : p.K;  // k per stage
    const int stages = bulk_stages(p.K, UK, p.kb <= 0);
    const size_t smem = bulk_smem_bytes(p.K, stages, UK);
    int* err = dev ? dev->error_flag : nullptr;
    if (p.kb > 0)
        return launch_on(dev, stream, gemv_bulk_kernel<true>, dim3(sm_count), dim3(kBulkThreads), smem, p, stages, err);
    return launch_on(dev, stream, gemv_bulk_kernel<false>, dim3(sm_count), dim3(kBulkThreads), smem, p, stages, err);
}

// Tile groups of the k-split GEMV (0 = it does not apply): blocked int8 with one scale per row, one
// activation row, a store / residual epilogue, f32 x and norm weight 16-byte aligned, at most one CTA per
// SM: groups = SMs / k blocks (every CTA one k block of one group).
int ksplit_groups(const GemvParams& p, int sm_count) {
    if (!g_gemv_ksplit || !g_gemv_mma || p.kb != kWeightBlock || p.M != 1 || !p.acc || p.acc_count < p.N) return 0;
    if (p.epi != EPI_STORE && p.epi != EPI_ACCUM && p.epi != EPI_SWIGLU) return 0;
    if (p.group < p.K || p.N % 16 != 0 || p.K % kWeightBlock != 0 || p.x_dtype != L0B_F32) return 0;
    if (p.epi == EPI_SWIGLU && (p.N / 2) % 16 != 0) return 0;
    if ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.w)) & 15) return 0;
    if (p.norm_w && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)) return 0;
    const int nb = p.K / kWeightBlock;
    if (nb > sm_count) return 0;
    const int ntiles = p.epi == EPI_SWIGLU ? p.N / 32 : p.N / 16;  // SwiGLU: gate tiles
    int groups = sm_count / nb;
    if (groups > ntiles) groups = ntiles;
    if (!p.counters || groups > p.counter_count) return 0;
    return groups;
}

l0b_status launch_ksplit(l0b_device* dev, cudaStream_t stream, int sm_count, const GemvParams& p, int groups) {
    (void)sm_count;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemv_ksplit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kBulkSmemBudget);
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        configured = true;
    }
    const int nb = p.K / kWeightBlock;
    int stages = g_ksplit_stages;
    while (stages > 2 && 1024 + 2048 + static_cast<size_t>(stages) * kKsStageBytes + 2 * kKsMaxStages * 8 >
                             static_cast<size_t>(kBulkSmemBudget))
        --stages;
    const size_t smem = 1024 + 2048 + static_cast<size_t>(stages) * kKsStageBytes + 2 * kKsMaxStages * 8;
    int* err = dev ? dev->error_flag : nullptr;
    return launch_on(dev, stream, gemv_ksplit_kernel, dim3(nb * groups), dim3(kKsThreads), smem, p, stages, groups, err);
}

// Resident CTAs per SM for (kernel, dynamic smem), cached: the persistent grid is SMs x this.
int resident_ctas(const void* func, size_t smem) {
    struct Entry {
        const void* func;
        size_t smem;
        int n;
    };
    static Entry cache[128];
    static int used = 0;
    for (int i = 0; i < used; ++i)
        if (cache[i].func == func && cache[i].smem == smem) return cache[i].n;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, kThreads, smem) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 1;
    }
    if (used < 128) cache[used++] = {func, smem, n};
    return n;
}

template <typename WT, int MR>
l0b_status launch_vec(l0b_device* dev, cudaStream_t stream, int sm_count, const GemvParams& p) {
    constexpr int RPW = 2;
    auto kernel = gemv_nk_kernel<WT, MR, RPW>;
    const size_t smem = static_cast<size_t>(MR) * p.kt * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        configured = true;
    }
    const int units = p.epi == EPI_SWIGLU ? p.N / 2 : p.N;
    const int per_cta = p.epi == EPI_SWIGLU ? kWarps * (RPW / 2) : kWarps * RPW;
    const int nblocks = (units + per_cta - 1) / per_cta;
    const int cap = sm_count * resident_ctas(reinterpret_cast<const void*>(kernel), smem);
    const int grid = nblocks < cap ? nblocks : cap;
    return launch_on(dev, stream, kernel, dim3(grid), dim3(kThreads), smem, p);
}

// Split count S (cluster size) for the tensor-core kernel: the smallest of 1, 2, 4, 8 whose K slice of
// hi/lo activations fits the shared-memory budget (100 KB keeps two CTAs per SM); 0 = does not fit.
// With sm_count > 0, S then doubles (up to g_gemv_fill_split) while the 16-row tiles alone would leave
// SMs idle and each slice keeps at least 2048 k: a 1280-row projection over K = 8192 becomes 160 CTAs
// of half rows instead of 80 CTAs of whole rows.
template <typename WT>
int mma_splits(const GemvParams& p, int rows, int sm_count = 0) {
    const long long npieces = p.K / MmaPiece<WT>::kK;
    int s = 0;
    for (int c = 1; c <= 8 && !s; c *= 2) {
        const long long slice = (npieces + c - 1) / c * MmaPiece<WT>::kK;  // largest slice, in k
        if (4ll * rows * slice <= 100 * 1024) s = c;
    }
    if (!s) {
        const long long slice8 = (npieces + 7) / 8 * MmaPiece<WT>::kK;
        return 4ll * rows * slice8 <= 200 * 1024 ? 8 : 0;
    }
    if (sm_count > 0) {
        const bool swiglu = p.epi == EPI_SWIGLU;
        const long long ntiles = ((swiglu ? p.N / 2 : p.N) + (swiglu ? 7 : 15)) / (swiglu ? 8 : 16);
        while (2 * s <= g_gemv_fill_split && ntiles * s < sm_count && npieces / (2 * s) * MmaPiece<WT>::kK >= 2048)
            s *= 2;
    }
    return s;
}

template <typename WT, int NG>
l0b_status launch_mma(l0b_device* dev, cudaStream_t stream, int sm_count, const GemvParams& p, int S) {
    auto kernel = gemv_mma_kernel<WT, NG>;
    const long long npieces = p.K / MmaPiece<WT>::kK;
    const size_t smem = 4ull * p.M * ((npieces + S - 1) / S) * MmaPiece<WT>::kK;  // largest slice
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        configured = true;
    }
    const bool swiglu = p.epi == EPI_SWIGLU;
    const int units = swiglu ? p.N / 2 : p.N;
    const int ntiles = (units + (swiglu ? 7 : 15)) / (swiglu ? 8 : 16);
    int cap = sm_count * resident_ctas(reinterpret_cast<const void*>(kernel), smem) / S;
    if (p.epi == EPI_PEER_SUM && cap > kPeerSumCtas) cap = kPeerSumCtas;
    const dim3 grid(ntiles < cap ? ntiles : (cap > 0 ? cap : 1), S);
    if (dev) return dev->launch_cluster(kernel, grid, dim3(kThreads), smem, S, p);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
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
    if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
    add_launches(1);
    return L0B_OK;
}

// The tensor-core kernel takes 16-bit weights and per-row-scaled int8, K in whole pieces (64 / 32 k),
// and up to 8 activation rows per pass, split over a cluster of up to 8 CTAs along K when the
// activations of one CTA would not fit its shared memory. Returns the split count, 0 = does not apply.
template <typename WT>
int mma_applies(const GemvParams& p, int rows, int sm_count = 0) {
    if constexpr (sizeof(WT) > 2) {
        return 0;
    } else {
        if (!(g_gemv_mma && p.K % MmaPiece<WT>::kK == 0 && reinterpret_cast<uintptr_t>(p.w) % 16 == 0 &&
              (sizeof(WT) != 1 || p.group >= p.K) && rows <= 8))
            return 0;
        return mma_splits<WT>(p, rows, sm_count);
    }
}

template <typename WT>
l0b_status launch_typed(l0b_device* dev, cudaStream_t stream, int sm_count, GemvParams p) {
    constexpr int VEC = 16 / sizeof(WT);
    constexpr int CH = 32 * VEC;
    const bool vec_ok = (p.K % VEC == 0) && (reinterpret_cast<uintptr_t>(p.w) % 16 == 0) &&
                        (sizeof(WT) != 1 || (p.group % 16 == 0 && p.K % p.group == 0));
    const int M = p.M;
    const bool psum = p.epi == EPI_PEER_SUM;
    if constexpr (sizeof(WT) == 1) {
        if (const int groups = ksplit_groups(p, sm_count)) return launch_ksplit(dev, stream, sm_count, p, groups);
        if (!psum && bulk_applies(L0B_I8, p, sm_count)) return launch_bulk(dev, stream, sm_count, p);
    }
    if (psum) {
        L0B_REQUIRE(p.peer && p.nseg == 1 && p.out_dtype == L0B_F32 && p.seg[0].out, L0B_ERR_ARGUMENT,
                    "the peer-sum epilogue needs the communicator's mailboxes and one f32 output");
        L0B_REQUIRE(static_cast<long long>(p.N) * (M < 8 ? M : 8) <= kPeerSumSlotElems, L0B_ERR_OUT_OF_RANGE,
                    "peer-sum partials of %d x %d floats exceed the mailbox slot", M < 8 ? M : 8, p.N);
    }
    L0B_REQUIRE(p.kb == 0 || p.kb == kWeightBlock, L0B_ERR_ARGUMENT, "blocked layout with %d k per block", p.kb);
    if (p.kb > 0) {
        // Blocked weights are read by the tensor-core kernels only (the fp32-FMA kernel has no blocked
        // addressing): refuse rather than read the bytes in the wrong order.
        GemvParams t8 = p;
        t8.M = M < 8 ? M : 8;
        int ok = 0;
        if constexpr (sizeof(WT) == 1) ok = mma_applies<WT>(t8, t8.M);
        L0B_REQUIRE(ok > 0, L0B_ERR_UNSUPPORTED,
                    "int8 weights in the blocked layout need the tensor-core GEMV (N=%d K=%d M=%d)", p.N, p.K, M);
    }
    for (int m0 = 0; m0 < M;) {
        GemvParams q = p;
        // Passes of up to 8 rows. (Sixteen-row passes on four B-column groups fit shared memory only
        // as 4-way split-K at K = 3584, where the per-tile cluster barrier dominates: measured slower than
        // two 8-row passes, so the dispatcher does not form them.)
        const int mr = M - m0 < 8 ? M - m0 : 8;
        int splits = 0;
        if constexpr (sizeof(WT) <= 2) {
            GemvParams t8 = p;
            t8.M = mr;
            splits = mma_applies<WT>(t8, mr, sm_count);
        }
        q.M = mr;
        q.x = static_cast<const char*>(p.x) + static_cast<size_t>(m0) * p.x_ld * dtype_size((l0b_dtype)p.x_dtype);
        for (int s = 0; s < q.nseg; ++s) {
            if (!q.seg[s].out) continue;
            const size_t es = (p.epi == EPI_ACCUM) ? 4 : dtype_size((l0b_dtype)p.out_dtype);
            q.seg[s].out = static_cast<char*>(q.seg[s].out) + static_cast<size_t>(m0) * q.seg[s].ld * es;
        }
        if (q.argmax) q.argmax += m0;
        m0 += mr;
        if constexpr (sizeof(WT) <= 2) {
            if (splits) {
                if (mr <= 4) L0B_TRY((launch_mma<WT, 1>(dev, stream, sm_count, q, splits)));
                else L0B_TRY((launch_mma<WT, 2>(dev, stream, sm_count, q, splits)));
                continue;
            }
        }
        L0B_REQUIRE(!psum, L0B_ERR_UNSUPPORTED, "the peer-sum epilogue runs on the tensor-core GEMV only");
        if (!vec_ok) {
            const long long outs = (p.epi == EPI_SWIGLU ? p.N / 2 : p.N) * static_cast<long long>(mr);
            const int grid = static_cast<int>((outs + kWarps - 1) / kWarps);
            L0B_TRY(launch_on(dev, stream, gemv_nk_scalar_kernel<WT>, dim3(grid), dim3(kThreads), 0, q));
            continue;
        }
        // Shared-memory tile of x: the whole row when it fits (~100 KB), else multiples of a chunk.
        const int mpad = mr <= 1 ? 1 : mr <= 2 ? 2 : mr <= 4 ? 4 : 8;
        const int kpad = (p.K + CH - 1) / CH * CH;
        const int budget = 100 * 1024 / (4 * mpad);
        q.kt = kpad <= budget ? kpad : (budget / CH) * CH;
        switch (mpad) {
            case 1: L0B_TRY((launch_vec<WT, 1>(dev, stream, sm_count, q))); break;
            case 2: L0B_TRY((launch_vec<WT, 2>(dev, stream, sm_count, q))); break;
            case 4: L0B_TRY((launch_vec<WT, 4>(dev, stream, sm_count, q))); break;
            default: L0B_TRY((launch_vec<WT, 8>(dev, stream, sm_count, q))); break;
        }
    }
    return L0B_OK;
}

l0b_status gemv_dispatch(l0b_device* dev, cudaStream_t stream, int sm_count, int w_dtype, GemvParams p) {
    L0B_REQUIRE(p.N > 0 && p.K > 0 && p.M > 0, L0B_ERR_OUT_OF_RANGE, "GEMV shape M=%d N=%d K=%d", p.M, p.N, p.K);
    L0B_REQUIRE(p.epi != EPI_SWIGLU || p.N % 2 == 0, L0B_ERR_ARGUMENT, "SwiGLU-fused GEMV needs an even row count");
    L0B_REQUIRE(p.nseg >= 1 && p.nseg <= 4, L0B_ERR_ARGUMENT, "1..4 output segments");
    switch (w_dtype) {
        case L0B_I8:
            L0B_REQUIRE(p.scales && p.group > 0 && p.K % p.group == 0, L0B_ERR_ARGUMENT,
                        "int8 weights need scales and a group dividing K (group %d, K %d)", p.group, p.K);
            return launch_typed<int8_t>(dev, stream, sm_count, p);
        case L0B_F16: return launch_typed<__half>(dev, stream, sm_count, p);
        case L0B_BF16: return launch_typed<__nv_bfloat16>(dev, stream, sm_count, p);
        case L0B_F32: return launch_typed<float>(dev, stream, sm_count, p);
        default: return fail(L0B_ERR_UNSUPPORTED, "weight dtype %d is not supported", w_dtype);
    }
}

// ---------------------------------------------------------------------------------------------
// Reference layout W [K, N]: y[m, n] = sum_k x[m, k] * W[k, n]. A CTA owns 64 columns (16 threads
// x 4 columns, one 8/16-byte load per row) and splits K over 16 thread rows; partial sums are
// reduced through shared memory. Used by the reference-surface Gemv ops only.
// ---------------------------------------------------------------------------------------------
template <typename WT>
__global__ void __launch_bounds__(256) gemv_kn_kernel(int M, int N, int K, const float* __restrict__ x,
                                                      const WT* __restrict__ w, float* __restrict__ y) {
    __shared__ float red[16][65];
    pdl_wait();
    const int tc = threadIdx.x & 15, tr = threadIdx.x >> 4;
    const int n0 = blockIdx.x * 64 + tc * 4;
    const int m = blockIdx.y;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = tr; k < K; k += 16) {
        const float xv = x[static_cast<long long>(m) * K + k];
        const WT* row = w + static_cast<long long>(k) * N;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (n0 + c < N) {
                float wv;
                if constexpr (sizeof(WT) == 2) wv = __half2float(row[n0 + c]);
                else wv = row[n0 + c];
                a[c] = fmaf(xv, wv, a[c]);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) red[tr][tc * 4 + c] = a[c];
    __syncthreads();
    if (threadIdx.x < 64) {
        float s = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) s += red[r][threadIdx.x];
        const int n = blockIdx.x * 64 + threadIdx.x;
        if (n < N) y[static_cast<long long>(m) * N + n] = s;
    }
}

__global__ void __launch_bounds__(256) gemm_f32_kernel(int M, int N, int K, const float* __restrict__ A,
                                                       const float* __restrict__ B, float* __restrict__ C) {
    __shared__ float As[16][17], Bs[16][17];
    pdl_wait();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
    float acc = 0.f;
    for (int k0 = 0; k0 < K; k0 += 16) {
        As[ty][tx] = (row < M && k0 + tx < K) ? A[static_cast<long long>(row) * K + k0 + tx] : 0.f;
        Bs[ty][tx] = (k0 + ty < K && col < N) ? B[static_cast<long long>(k0 + ty) * N + col] : 0.f;
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) acc = fmaf(As[ty][kk], Bs[kk][tx], acc);
        __syncthreads();
    }
    if (row < M && col < N) C[static_cast<long long>(row) * N + col] = acc;
}

}  // namespace

bool gemv_takes_ksplit(int w_dtype, const GemvParams& p, int sm_count) {
    return w_dtype == L0B_I8 && ksplit_groups(p, sm_count) > 0;
}

bool gemv_peer_sum_applies(int w_dtype, const GemvParams& p) {
    if (!p.peer || p.nseg != 1 || p.out_dtype != L0B_F32 || !p.seg[0].out || p.M < 1) return false;
    if (static_cast<long long>(p.N) * (p.M < 8 ? p.M : 8) > kPeerSumSlotElems) return false;
    GemvParams t8 = p;
    t8.M = p.M < 8 ? p.M : 8;
    switch (w_dtype) {
        case L0B_I8: return mma_applies<int8_t>(t8, t8.M) > 0;
        case L0B_F16: return mma_applies<__half>(t8, t8.M) > 0;
        case L0B_BF16: return mma_applies<__nv_bfloat16>(t8, t8.M) > 0;
        default: return false;
    }
}

void gemv_set_tensor_cores(bool on) { g_gemv_mma = on; }
void gemv_set_bulk(bool on) { g_gemv_bulk = on; }
void gemv_set_bulk_short_rows(bool on) { g_gemv_bulk_short = on; }
void gemv_set_ksplit(bool on) { g_gemv_ksplit = on; }
void gemv_set_bulk_stages(int s) { g_bulk_max_stages = s < 0 ? 0 : s; }
int gemv_l2_prefetch_mb() { return g_l2_prefetch_mb; }
void gemv_set_l2_prefetch_mb(int mb) { g_l2_prefetch_mb = mb < 0 ? 0 : mb; }
void gemv_set_ksplit_stages(int s) { g_ksplit_stages = s < 2 ? 2 : (s > kKsMaxStages ? kKsMaxStages : s); }
void gemv_set_fill_split(int s) { g_gemv_fill_split = s <= 1 ? 1 : (s >= 8 ? 8 : (s >= 4 ? 4 : 2)); }

namespace {
bool g_weight_blocking = true;  // l0b_set_weight_blocking
}  // namespace

bool weight_blocking() { return g_weight_blocking; }
void set_weight_blocking(bool on) { g_weight_blocking = on; }

l0b_status gemv_nk_launch(l0b_device* dev, int w_dtype, GemvParams p) {
    return gemv_dispatch(dev, dev->stream, dev->sm_count, w_dtype, p);
}

l0b_status gemv_nk_launch_stream(cudaStream_t stream, int sm_count, int w_dtype, GemvParams p) {
    return gemv_dispatch(nullptr, stream, sm_count, w_dtype, p);
}

l0b_status gemv_kn_launch(l0b_device* dev, int w_dtype, int m, int n, int k, const float* x, const void* w,
                          float* y) {
    dim3 grid((n + 63) / 64, m);
    if (w_dtype == L0B_F16)
        return dev->launch(gemv_kn_kernel<__half>, grid, dim3(256), 0, m, n, k, x, static_cast<const __half*>(w), y);
    return dev->launch(gemv_kn_kernel<float>, grid, dim3(256), 0, m, n, k, x, static_cast<const float*>(w), y);
}

l0b_status gemm_f32_launch(l0b_device* dev, int m, int n, int k, const float* a, const float* b, float* c) {
    dim3 grid((n + 15) / 16, (m + 15) / 16);
    return dev->launch(gemm_f32_kernel, grid, dim3(256), 0, m, n, k, a, b, c);
}

}  // namespace l0b
