// Tensor-core GEMM for prefill and batched decode on sm_100a: tcgen05.mma with the accumulator in
// tensor memory, both operands staged by TMA into 128-byte-swizzled shared memory.
//
// "Swap-AB" orientation: the 128-row MMA M dimension runs over weight rows and the MMA N dimension
// (BN = 32, 64, 128 or 256) over activation rows, so one CTA computes D[128 weight rows, BN] =
// W_tile X_tile^T into BN fp32 TMEM columns. Warp 0 / lane 0 issues the TMA loads (W tile [128 x 64] and
// X tile [BN x 64] per stage, a ring of 4-8 stages filling ~100 KB, two CTAs per SM, for BN <= 64, or
// ~196 KB above), warp 1 / lane 0 issues four K=16 MMAs per stage and releases the stage with
// tcgen05.commit, and all four warps run the epilogue from TMEM (warp w owns TMEM lanes 32w..32w+31 =
// weight rows), storing token-major fp32 rows with coalesced 128-byte writes. The SwiGLU variant loads
// 64 gate rows and the 64 matching up rows into one tile and pairs them in the epilogue.
//
// f32 activations enter as hi / lo pairs of 16-bit rows (the lo row the rounding residual of the hi),
// so one tile's BN columns hold BN / 2 tokens twice and the epilogue adds the pair: about 22 bits (f16)
// or 16 bits (bf16) of each activation for one pass over K.
//
// Few tiles (decode batches, narrow projections) would leave most SMs idle, so K is split S ways across
// CTAs (blockIdx.z): each split writes its partial tile to global scratch, and the last split of a tile
// to arrive (an atomic counter per tile, no waiting) sums the S partials in split order — deterministic
// — runs the epilogue and re-arms the counter.
//
// int8 weights (one scale per weight row) run on the integer tensor-core MMA (kind::i8, s8 x s8 -> s32)
// straight from TMA: no conversion pass. Their f32 activations enter as four balanced base-128 int8
// digits per token (x * 2^s = d0 + 128 d1 + 128^2 d2 + 128^3 d3, |x * 2^s| < 2^26: ~27 bits of each
// token's largest value), four accumulator columns per token summed exactly in the epilogue, then times
// 2^-s and the row's scale. The integer sums are exact (|sum| < 2^31 for K < 2^17).
//
// Every mbarrier wait is bounded (~2 s); a timeout sets the device error flag and the CTA exits after
// releasing its tensor memory. No TMA multicast is used.
#include <cuda.h>

#include <cstring>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"

namespace l0b {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 128;
constexpr long long kWaitCycles = 4000000000LL;

struct TcParams {
    CUtensorMap wmap;  // W [N, K] 16-bit (int8: bytes, no swizzle), box {64, 128} (SwiGLU: {64, 64})
    CUtensorMap xmap;  // X row stride K, box {64 (int8: 128), BN}: [M, K], paired hi / lo, or int8 digits
    int M, N, K, epi, ld, half_n;
    float* out;
    const float* bias;
    int* error;
    int mode;              // x rows per token: 0 one, 1 hi / lo pair (BN / 2 tokens), 2 four int8 digits (BN / 4)
    const float* rscale;   // per-token result scale or null
    const __half* wscale;  // int8: f16 scale per weight row
    float* part;           // split-K partial tiles (gridDim.z > 1)
    unsigned* counters;    // split-K tile counters, zero at rest
    unsigned long long* argmax;  // EPI_ARGMAX: per-token keys (atomicMax), index = row + argmax_base
    int argmax_base;
    int wkb;  // > 0: wmap is the 4-D map of the blocked int8 layout {kb, 16, K / kb, N / 16}
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}

// Bounded wait for the phase with the given parity to complete; false after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    const long long t0 = clock64();
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(b)), "r"(parity)
            : "memory");
        if (done) return true;
        if (clock64() - t0 > kWaitCycles) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// The weight tile [rows row0 .. + box rows, k0 .. + 128 bytes): row-major 2-D map, or the blocked
// layout's 4-D map (the box {128 bytes, 16 rows, 1 block, rows / 16 tiles} lands in shared memory in the
// same row order, 128 bytes per row, as the 2-D box).
__device__ __forceinline__ void tma_load_w(void* dst, const TcParams& p, uint64_t* bar, int k0, int row0) {
    if (p.wkb > 0) tma_load_4d(dst, &p.wmap, bar, k0 % p.wkb, 0, k0 / p.wkb, row0 >> 4);
    else tma_load_2d(dst, &p.wmap, bar, k0, row0);
}

// UMMA shared-memory descriptor of a K-major tile with 128-byte swizzle: rows of 128 bytes, 8-row
// atoms 1024 bytes apart (stride byte offset), version 1 (sm_100), layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
    const uint32_t a = smem_u32(p);
    return static_cast<uint64_t>((a >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum)
        : "memory");
}

__device__ __forceinline__ void tc_mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory plan of one instantiation: an A tile [128 rows x 128 bytes] and a B tile [BN x 128 bytes]
// per stage (64 k of 16-bit values or 128 k of int8), stages filling ~100 KB (two CTAs per SM) for
// BN <= 64, ~196 KB (one CTA per SM) above, at most 8.
template <int BN, int FMT>
struct TcCfg {
    static constexpr bool kQ8 = FMT == 2;
    static constexpr int KB = kQ8 ? 128 : kBK;  // k per stage (128-byte rows)
    static constexpr int A_BYTES = kBM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TARGET = BN <= 64 ? 100 * 1024 : 196 * 1024;
    static constexpr int CTAS_PER_SM = BN <= 64 ? 2 : 1;
    static constexpr int STAGES_FIT = TARGET / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr size_t SMEM = 1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 256;
    static_assert(STAGES >= 3, "three or more stages");
};

// FMT: 0 = f16, 1 = bf16 (kind::f16, f32 accumulators), 2 = int8 weights and digits (kind::i8, s32).
template <int BN, int FMT>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
    using Cfg = TcCfg<BN, FMT>;
    constexpr bool kQ8 = Cfg::kQ8;
    constexpr int ST = Cfg::STAGES, KB = Cfg::KB;
    constexpr int A_BYTES = Cfg::A_BYTES, B_BYTES = Cfg::B_BYTES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int last_split;
    __shared__ unsigned long long amax_keys[4][16];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + ST * A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + ST * B_BYTES);
    uint64_t* empty = full + ST;
    uint64_t* accum = empty + ST;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tb = p.mode == 2 ? BN / 4 : p.mode == 1 ? BN / 2 : BN;  // tokens per tile
    const int t0 = blockIdx.x * tb;
    const int xrow0 = blockIdx.x * BN;         // first x row of this token tile
    const int wt = blockIdx.y;
    const int z = blockIdx.z, S = gridDim.z;
    const bool swiglu = p.epi == EPI_SWIGLU;
    const int nk = (p.K + KB - 1) / KB;
    const int kb0 = z * nk / S;
    const int nst = (z + 1) * nk / S - kb0;    // >= 1: the host keeps S <= nk

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.wmap)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.xmap)) : "memory");
    }

    pdl_wait();
    pdl_launch_dependents();

    bool ok = true;
    if (warp == 0 && lane == 0) {
        // TMA producer.
        for (int i = 0; i < nst; ++i) {
            const int s = i % ST;
            const uint32_t ph = (i / ST) & 1;
            if (i >= ST && !mbar_wait(&empty[s], ph ^ 1)) {
                ok = false;
                break;
            }
            mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
            const int k0 = (kb0 + i) * KB;
            if (swiglu) {
                tma_load_w(sA + s * A_BYTES, p, &full[s], k0, wt * 64);
                tma_load_w(sA + s * A_BYTES + A_BYTES / 2, p, &full[s], k0, p.half_n + wt * 64);
            } else {
                tma_load_w(sA + s * A_BYTES, p, &full[s], k0, wt * kBM);
            }
            tma_load_2d(sB + s * B_BYTES, &p.xmap, &full[s], k0, xrow0);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer: D[128, BN] (+)= A[128, 32 bytes] B[BN, 32 bytes]^T (k = 16 values of 16 bits, or
        // 32 of int8), four per stage.
        constexpr uint32_t idesc = kQ8 ? ((2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                          (static_cast<uint32_t>(kBM >> 4) << 24))
                                       : ((1u << 4) | (static_cast<uint32_t>(FMT) << 7) |
                                          (static_cast<uint32_t>(FMT) << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
                                          (static_cast<uint32_t>(kBM >> 4) << 24));
        for (int i = 0; i < nst; ++i) {
            const int s = i % ST;
            const uint32_t ph = (i / ST) & 1;
            if (!mbar_wait(&full[s], ph)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint64_t da = smem_desc(sA + s * A_BYTES), db = smem_desc(sB + s * B_BYTES);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if constexpr (kQ8) tc_mma_i8(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
                else tc_mma(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
            }
            tc_commit(&empty[s]);
        }
        tc_commit(accum);
    }
    __syncwarp();

    // Epilogue: all warps. Thread (warp, lane) owns TMEM lane rl = weight row `row` of the tile.
    const bool acc_ok = mbar_wait(accum, 0);
    __syncwarp();
    tc_fence_after();
    const int rl = warp * 32 + lane;
    const int row = swiglu ? (warp < 2 ? 0 : p.half_n - 64) + wt * 64 + rl : wt * kBM + rl;
    const float wsc = (kQ8 && row < p.N) ? __half2float(p.wscale[row]) : 1.f;
    const uint32_t tl = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float* xchg = reinterpret_cast<float*>(sA);  // SwiGLU: up rows handed from warps 2-3 to warps 0-1
    // Accumulator columns c0..c0+15 of this lane: the token's hi column plus (paired) its lo column,
    // or its four digit columns (s32, exact) combined in f64 and rounded once.
    auto load_acc = [&](int c0, float (&v)[16]) {
        tmem_ld16(tl + c0, v);
        if (kQ8) {
            double acc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = static_cast<double>(__float_as_int(v[j]));
#pragma unroll
            for (int dg = 1; dg < 4; ++dg) {
                float u[16];
                tmem_ld16(tl + dg * (BN / 4) + c0, u);
                const double w = static_cast<double>(1 << (7 * dg));
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[j] += w * static_cast<double>(__float_as_int(u[j]));
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = static_cast<float>(acc[j]);
        } else if (p.mode == 1) {
            float u[16];
            tmem_ld16(tl + BN / 2 + c0, u);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += u[j];
        }
    };
    // Scales, bias and the epilogue of tokens t0 + c0 .. t0 + c0 + 15 (uniform across the CTA).
    auto finish = [&](int c0, float (&v)[16]) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int t = t0 + c0 + j;
            v[j] *= wsc * ((p.rscale && t < p.M) ? p.rscale[t] : 1.f);
        }
        if (p.epi == EPI_ARGMAX) {
            // Logits (when stored) and one atomicMax per token per CTA: the largest of the tile's rows.
            const bool live = acc_ok && row < p.N;
            const float b = (live && p.bias) ? p.bias[row] : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = t0 + c0 + j;
                unsigned long long key = 0;
                if (live && t < p.M) {
                    if (p.out) p.out[static_cast<long long>(t) * p.ld + row] = v[j] + b;
                    key = argmax_key(v[j] + b, row + p.argmax_base);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                    key = other > key ? other : key;
                }
                if (lane == 0) amax_keys[warp][j] = key;
            }
            __syncthreads();
            if (threadIdx.x < 16) {
                unsigned long long key = amax_keys[0][threadIdx.x];
#pragma unroll
                for (int w = 1; w < 4; ++w) key = amax_keys[w][threadIdx.x] > key ? amax_keys[w][threadIdx.x] : key;
                if (key && t0 + c0 + static_cast<int>(threadIdx.x) < p.M)
                    atomicMax(p.argmax + t0 + c0 + threadIdx.x, key);
            }
            __syncthreads();
        } else if (!swiglu) {
            if (acc_ok && row < p.N) {
                const float b = p.bias ? p.bias[row] : 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + c0 + j;
                    if (t < p.M) {
                        float* o = p.out + static_cast<long long>(t) * p.ld + row;
                        if (p.epi == EPI_ACCUM) *o += v[j] + b;
                        else *o = v[j] + b;
                    }
                }
            }
        } else {
            __syncthreads();
            if (warp >= 2) {
#pragma unroll
                for (int j = 0; j < 16; ++j) xchg[((warp - 2) * 32 + lane) * 17 + j] = v[j];
            }
            __syncthreads();
            if (warp < 2) {
                const int i = wt * 64 + rl;
                if (acc_ok && i < p.half_n) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int t = t0 + c0 + j;
                        if (t < p.M)
                            p.out[static_cast<long long>(t) * p.ld + i] = silu(v[j]) * xchg[(warp * 32 + lane) * 17 + j];
                    }
                }
            }
        }
    };
    if (S == 1) {
        for (int c0 = 0; c0 < tb; c0 += 16) {
            float v[16];
            load_acc(c0, v);
            finish(c0, v);
        }
    } else {
        // Split-K: partial tile [tb columns][128 rows] of split z; the last split to arrive sums the
        // splits in order 0..S-1 (deterministic) and finishes; it also re-arms the tile's counter.
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        float* base = p.part + static_cast<size_t>(tile) * S * tb * kBM;
        for (int c0 = 0; c0 < tb; c0 += 16) {
            float v[16];
            load_acc(c0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) base[(static_cast<size_t>(z) * tb + c0 + j) * kBM + rl] = v[j];
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned prev = atomicAdd(&p.counters[tile], 1u);
            last_split = prev == static_cast<unsigned>(S - 1);
            if (last_split) p.counters[tile] = 0;
        }
        __syncthreads();
        if (last_split) {
            __threadfence();
            for (int c0 = 0; c0 < tb; c0 += 16) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0.f;
                // Four splits' loads in flight at a time; the sum still runs in split order.
                for (int z0 = 0; z0 < S; z0 += 4) {
                    float q[4][16];
#pragma unroll
                    for (int dz = 0; dz < 4; ++dz) {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            q[dz][j] = z0 + dz < S ? __ldcg(&base[(static_cast<size_t>(z0 + dz) * tb + c0 + j) * kBM + rl])
                                                   : 0.f;
                    }
#pragma unroll
                    for (int dz = 0; dz < 4; ++dz) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] += q[dz][j];
                    }
                }
                finish(c0, v);
            }
        }
    }
    if ((!ok || !acc_ok) && p.error) atomicExch(p.error, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
}

__global__ void __launch_bounds__(256) cast_rows_kernel(const float* x, long long ld_x, const float* norm_w, float eps,
                                                        void* out16, int dtype, int K) {
    __shared__ float red[32];
    pdl_wait();
    const float* xr = x + blockIdx.x * ld_x;
    float rstd = 1.f;
    if (norm_w) {
        float ss = 0.f;
        for (int k = threadIdx.x; k < K; k += blockDim.x) ss += xr[k] * xr[k];
        ss = block_sum(ss, red);
        rstd = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
    }
    const long long base = static_cast<long long>(blockIdx.x) * K;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = xr[k];
        if (norm_w) v = (v * rstd) * norm_w[k];
        store_from_float(out16, dtype, base + k, v);
    }
}

// One block per token: RMS norm (optional) and the row maximum, then the hi / lo pair, written to rows
// (t / tb) * bn + t % tb (hi) and that + tb (lo) of the paired layout, row stride K.
__global__ void __launch_bounds__(256) cast_rows_split_kernel(const float* x, long long ld_x, const float* norm_w,
                                                              float eps, void* out16, float* rscale, int dtype, int K,
                                                              int bn, int tb) {
    __shared__ float red[32];
    __shared__ float mx[32];
    pdl_wait();
    const float* xr = x + blockIdx.x * ld_x;
    float ss = 0.f, am = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = xr[k];
        ss += v * v;
        am = fmaxf(am, fabsf(norm_w ? v * norm_w[k] : v));
    }
    const float rstd = norm_w ? 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(K) + eps) : 1.0f;
    am = warp_max(am);
    if ((threadIdx.x & 31) == 0) mx[threadIdx.x >> 5] = am;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? mx[threadIdx.x] : 0.f;
        t = warp_max(t);
        if (threadIdx.x == 0) mx[0] = t;
    }
    __syncthreads();
    const float top = mx[0] * rstd;
    int e = 0;
    if (dtype == L0B_F16 && top > 0.f && isfinite(top)) {
        int ex;
        frexpf(top, &ex);
        e = min(max(14 - ex, -100), 100);
    }
    const float sc = rstd * ldexpf(1.0f, e);
    if (threadIdx.x == 0) rscale[blockIdx.x] = ldexpf(1.0f, -e);
    const int t = blockIdx.x;
    const long long hi_row = static_cast<long long>(t / tb) * bn + t % tb;
    const long long hbase = hi_row * K, lbase = (hi_row + tb) * K;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = (norm_w ? xr[k] * norm_w[k] : xr[k]) * sc;
        const float hi = dtype == L0B_F16 ? __half2float(__float2half_rn(v)) : __bfloat162float(__float2bfloat16_rn(v));
        store_from_float(out16, dtype, hbase + k, hi);
        store_from_float(out16, dtype, lbase + k, v - hi);
    }
}

// Register-resident variant of cast_rows_split_kernel for K % 4 == 0 and K <= 4 * VPT * blockDim.x:
// every thread loads its VPT float4 of the row at once (one read of x, all loads in flight), and the
// hi / lo halves are written from registers, four 16-bit values per store.
template <int VPT>
__global__ void __launch_bounds__(512) cast_rows_split_reg_kernel(const float* x, long long ld_x, const float* norm_w,
                                                                  float eps, void* out16, float* rscale, int dtype,
                                                                  int K, int bn, int tb) {
    __shared__ float red[32];
    __shared__ float mx[32];
    pdl_wait();
    const int t = blockIdx.x;
    const int K4 = K >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + t * ld_x);
    const float4* nw = reinterpret_cast<const float4*>(norm_w);
    float4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        v[i] = k4 < K4 ? xr[k4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.f, am = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        if (norm_w && k4 < K4) {
            const float4 w = nw[k4];
            v[i].x *= w.x;
            v[i].y *= w.y;
            v[i].z *= w.z;
            v[i].w *= w.w;
        }
        am = fmaxf(am, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
    const float rstd = norm_w ? 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(K) + eps) : 1.0f;
    am = warp_max(am);
    if ((threadIdx.x & 31) == 0) mx[threadIdx.x >> 5] = am;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < (blockDim.x >> 5) ? mx[threadIdx.x] : 0.f;
        m = warp_max(m);
        if (threadIdx.x == 0) mx[0] = m;
    }
    __syncthreads();
    const float top = mx[0] * rstd;
    int e = 0;
    if (dtype == L0B_F16 && top > 0.f && isfinite(top)) {
        int ex;
        frexpf(top, &ex);
        e = min(max(14 - ex, -100), 100);
    }
    const float sc = rstd * ldexpf(1.0f, e);
    if (threadIdx.x == 0) rscale[t] = ldexpf(1.0f, -e);
    const long long hi_row = static_cast<long long>(t / tb) * bn + t % tb;
    uint2* hrow = reinterpret_cast<uint2*>(static_cast<uint16_t*>(out16) + hi_row * K);
    uint2* lrow = reinterpret_cast<uint2*>(static_cast<uint16_t*>(out16) + (hi_row + tb) * K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        if (k4 < K4) {
            const float a0 = v[i].x * sc, a1 = v[i].y * sc, a2 = v[i].z * sc, a3 = v[i].w * sc;
            uint2 h, l;
            if (dtype == L0B_F16) {
                const __half2 h01 = __floats2half2_rn(a0, a1), h23 = __floats2half2_rn(a2, a3);
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                const __half2 l01 = __floats2half2_rn(a0 - f01.x, a1 - f01.y), l23 = __floats2half2_rn(a2 - f23.x, a3 - f23.y);
                h = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
                l = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
            } else {
                const __nv_bfloat162 h01 = __floats2bfloat162_rn(a0, a1), h23 = __floats2bfloat162_rn(a2, a3);
                const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
                const __nv_bfloat162 l01 = __floats2bfloat162_rn(a0 - f01.x, a1 - f01.y),
                                     l23 = __floats2bfloat162_rn(a2 - f23.x, a3 - f23.y);
                h = make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
                l = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
            }
            hrow[k4] = h;
            lrow[k4] = l;
        }
    }
}

// Four balanced base-128 digits of a scaled activation: X = rint(v) (|X| < 2^26) = d0 + 128 d1 + 128^2 d2
// + 128^3 d3 with d0..d2 in [-64, 64); packed into byte `lane` of each digit's word.
__device__ __forceinline__ void digits4(float v, int lane, uint32_t (&w)[4]) {
    int X = __float2int_rn(v);
#pragma unroll
    for (int dg = 0; dg < 3; ++dg) {
        const int d = ((X + 64) & 127) - 64;
        w[dg] |= (static_cast<uint32_t>(d) & 0xFFu) << (8 * lane);
        X = (X - d) >> 7;
    }
    w[3] |= (static_cast<uint32_t>(X) & 0xFFu) << (8 * lane);
}

// Per token: RMS norm (optional) and the row maximum, then int8 digits of x * 2^s with the largest |x|
// * 2^s just below 2^26, to rows (t / tb) * bn + dg * tb + t % tb (digit dg) of the digit layout; rscale =
// 2^-s. Register-resident: each thread holds VPT float4 of the row (K % 4 == 0, K <= 4 * VPT * threads).
template <int VPT>
__global__ void __launch_bounds__(512) cast_rows_digits_kernel(const float* x, long long ld_x, const float* norm_w,
                                                               float eps, uint8_t* out8, float* rscale, int K, int bn,
                                                               int tb) {
    __shared__ float red[32];
    __shared__ float mx[32];
    pdl_wait();
    const int t = blockIdx.x;
    const int K4 = K >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + t * ld_x);
    const float4* nw = reinterpret_cast<const float4*>(norm_w);
    float4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        v[i] = k4 < K4 ? xr[k4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float ss = 0.f, am = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        if (norm_w && k4 < K4) {
            const float4 w = nw[k4];
            v[i].x *= w.x;
            v[i].y *= w.y;
            v[i].z *= w.z;
            v[i].w *= w.w;
        }
        am = fmaxf(am, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
    const float rstd = norm_w ? 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(K) + eps) : 1.0f;
    am = warp_max(am);
    if ((threadIdx.x & 31) == 0) mx[threadIdx.x >> 5] = am;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < (blockDim.x >> 5) ? mx[threadIdx.x] : 0.f;
        m = warp_max(m);
        if (threadIdx.x == 0) mx[0] = m;
    }
    __syncthreads();
    const float top = mx[0] * rstd;
    int e = 0;
    if (top > 0.f && isfinite(top)) {
        int ex;
        frexpf(top, &ex);  // top = f 2^ex, f in [0.5, 1): top 2^(26 - ex) < 2^26
        e = min(max(26 - ex, -120), 120);
    }
    const float sc = rstd * ldexpf(1.0f, e);
    if (threadIdx.x == 0) rscale[t] = ldexpf(1.0f, -e);
    const long long row0 = static_cast<long long>(t / tb) * bn + t % tb;
    uint32_t* rows[4];
#pragma unroll
    for (int dg = 0; dg < 4; ++dg) rows[dg] = reinterpret_cast<uint32_t*>(out8 + (row0 + dg * tb) * K);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int k4 = threadIdx.x + i * blockDim.x;
        if (k4 < K4) {
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            digits4(v[i].x * sc, 0, w);
            digits4(v[i].y * sc, 1, w);
            digits4(v[i].z * sc, 2, w);
            digits4(v[i].w * sc, 3, w);
#pragma unroll
            for (int dg = 0; dg < 4; ++dg) rows[dg][k4] = w[dg];
        }
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// Row-major [rows, K] matrix with the 128-byte swizzle, box {128 bytes of k, box_rows}: 64 values of 16
// bits or 128 of int8.
l0b_status make_map(CUtensorMap* map, const void* base, int dtype, long long rows, long long K, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    L0B_REQUIRE(fn, L0B_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const long long esize = dtype == L0B_I8 ? 1 : 2;
    L0B_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0 && (K * esize) % 16 == 0, L0B_ERR_ARGUMENT,
                "TMA needs 16-byte aligned rows (K * element size %% 16 == 0)");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K * esize)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType type = dtype == L0B_I8     ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                     : dtype == L0B_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    L0B_REQUIRE(r == CUDA_SUCCESS, L0B_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return L0B_OK;
}

// int8 weights in the blocked layout [N / 16][K / kb][16][kb]: a 4-D map {kb, 16, K / kb, N / 16} with the
// 128-byte swizzle and box {128, 16, 1, box_rows / 16}.
l0b_status make_map_blocked(CUtensorMap* map, const void* base, long long rows, long long K, int kb, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    L0B_REQUIRE(fn, L0B_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    L0B_REQUIRE(reinterpret_cast<uintptr_t>(base) % 16 == 0 && rows % 16 == 0 && K % kb == 0 && kb % 128 == 0 &&
                    box_rows % 16 == 0,
                L0B_ERR_ARGUMENT, "blocked weight map: rows %lld, K %lld, kb %d", rows, K, kb);
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kb), 16, static_cast<cuuint64_t>(K / kb),
                                static_cast<cuuint64_t>(rows / 16)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kb), static_cast<cuuint64_t>(16) * kb,
                                   static_cast<cuuint64_t>(16) * K};
    const cuuint32_t box[4] = {128, 16, 1, static_cast<cuuint32_t>(box_rows / 16)};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    L0B_REQUIRE(r == CUDA_SUCCESS, L0B_ERR_CUDA, "cuTensorMapEncodeTiled (blocked) failed (%d)", static_cast<int>(r));
    return L0B_OK;
}

template <int BN, int FMT>
l0b_status launch_bn(l0b_device* d, const TcParams& p, const TcPlan& plan) {
    auto kernel = tc_gemm_kernel<BN, FMT>;
    constexpr size_t smem = TcCfg<BN, FMT>::SMEM;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return fail(L0B_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
        configured = true;
    }
    return d->launch(kernel, dim3(plan.tiles_x, plan.tiles_y, plan.S), dim3(kThreads), smem, p);
}

template <int FMT>
l0b_status launch_fmt(l0b_device* d, const TcParams& p, const TcPlan& plan) {
    switch (plan.bn) {
        case 32: return launch_bn<32, FMT>(d, p, plan);
        case 64: return launch_bn<64, FMT>(d, p, plan);
        case 128: return launch_bn<128, FMT>(d, p, plan);
        default: return launch_bn<256, FMT>(d, p, plan);
    }
}

}  // namespace

bool tc_gemm_supported(int wdtype, int M, int N, int K, int epi) {
    if (wdtype != L0B_F16 && wdtype != L0B_BF16 && wdtype != L0B_I8) return false;
    if (M < 1 || N < 1 || K < 64 || K % (wdtype == L0B_I8 ? 16 : 8) != 0) return false;
    if (epi == EPI_SWIGLU && (N % 2 != 0 || (N / 2) % 64 != 0)) return false;
    return epi == EPI_STORE || epi == EPI_ACCUM || epi == EPI_SWIGLU || epi == EPI_ARGMAX;
}

size_t tc_gemm_part_floats(int sm_count) { return static_cast<size_t>(2) * sm_count * 128 * kBM; }

namespace {
int g_max_splits = 16;  // upper bound on the K split (l0b_tc_set_max_splits)
}

void tc_gemm_set_max_splits(int s) { g_max_splits = s < 1 ? 16 : (s > 16 ? 16 : s); }

// Token columns: the smallest BN in {32, 64, 128, 256} that holds the tile's columns (hi and lo when
// paired). Weight tiles: 128 rows (SwiGLU: 64 gate + 64 up). K splits: when the tiles fill fewer than the
// resident slots (two CTAs per SM at BN <= 64), split K so tiles x S comes close to the slots, each
// split keeping two or more K blocks of 64 and the partial tiles within the scratch bound.
TcPlan tc_gemm_plan(int M, int N, int K, int epi, bool pair, int wdtype, int sm_count) {
    TcPlan pl;
    const bool q8 = wdtype == L0B_I8;  // int8 weights: four digit columns per token, BN >= 64
    const int cols = q8 ? 4 * M : pair ? 2 * M : M;
    pl.bn = (cols <= 32 && !q8) ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : 256;
    pl.tb = q8 ? pl.bn / 4 : pair ? pl.bn / 2 : pl.bn;
    pl.tiles_x = (M + pl.tb - 1) / pl.tb;
    pl.tiles_y = epi == EPI_SWIGLU ? (N / 2) / 64 : (N + kBM - 1) / kBM;
    const long long tiles = static_cast<long long>(pl.tiles_x) * pl.tiles_y;
    const int slots = sm_count * (pl.bn <= 64 ? 2 : 1);
    const int nk = (K + (q8 ? 127 : kBK - 1)) / (q8 ? 128 : kBK);
    int S = tiles >= slots ? 1 : static_cast<int>(slots / tiles);
    if (S > nk / 2) S = nk / 2;
    if (S > g_max_splits) S = g_max_splits;
    if (S < 1) S = 1;
    while (S > 1 && (tiles * S * pl.tb * kBM > static_cast<long long>(tc_gemm_part_floats(sm_count)) ||
                     tiles > kTcCounters))
        --S;
    pl.S = S;
    pl.part_floats = S > 1 ? static_cast<size_t>(tiles) * S * pl.tb * kBM : 0;
    pl.counters = S > 1 ? static_cast<int>(tiles) : 0;
    return pl;
}

l0b_status tc_gemm_launch(l0b_device* d, const TcGemmArgs& a) {
    L0B_REQUIRE(tc_gemm_supported(a.wdtype, a.M, a.N, a.K, a.epi), L0B_ERR_UNSUPPORTED,
                "tensor-core GEMM does not take M=%d N=%d K=%d epi=%d dtype=%d", a.M, a.N, a.K, a.epi, a.wdtype);
    TcPlan plan = tc_gemm_plan(a.M, a.N, a.K, a.epi, a.split != 0, a.wdtype, d->sm_count);
    if (plan.S > 1 && (!a.part || !a.counters || a.part_floats < plan.part_floats || a.counter_count < plan.counters)) {
        plan.S = 1;  // no scratch for the split: one CTA per tile
        plan.part_floats = 0;
        plan.counters = 0;
    }
    TcParams p;
    std::memset(&p, 0, sizeof(p));
    const bool swiglu = a.epi == EPI_SWIGLU;
    const bool q8 = a.wdtype == L0B_I8;
    L0B_REQUIRE(!q8 || a.wscale, L0B_ERR_ARGUMENT, "int8 weights need their row scales");
    if (q8 && a.kb > 0) {
        // SwiGLU loads 64 gate and 64 up rows per tile (four 16-row tiles of the blocked layout each).
        L0B_REQUIRE(!swiglu || (a.N / 2) % 64 == 0, L0B_ERR_UNSUPPORTED,
                    "blocked [gate; up] needs half the rows (%d) to be a multiple of 64", a.N / 2);
        L0B_TRY(make_map_blocked(&p.wmap, a.w, a.N, a.K, a.kb, swiglu ? 64 : kBM));
        p.wkb = a.kb;
    } else {
        L0B_TRY(make_map(&p.wmap, a.w, a.wdtype, a.N, a.K, swiglu ? 64 : kBM));
    }
    const long long xrows = (a.split || q8) ? tc_pair_rows(plan) : a.M;
    L0B_TRY(make_map(&p.xmap, a.x16, a.wdtype, xrows, a.K, plan.bn));
    p.wscale = static_cast<const __half*>(a.wscale);
    p.mode = q8 ? 2 : a.split ? 1 : 0;
    p.rscale = a.rscale;
    L0B_REQUIRE(a.epi != EPI_ARGMAX || a.argmax, L0B_ERR_ARGUMENT, "the argmax epilogue needs its key array");
    p.argmax = a.argmax;
    p.argmax_base = a.argmax_base;
    p.part = plan.S > 1 ? a.part : nullptr;
    p.counters = plan.S > 1 ? a.counters : nullptr;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.epi = a.epi;
    p.ld = a.ld;
    p.half_n = a.N / 2;
    p.out = a.out;
    p.bias = a.bias;
    p.error = d->error_flag;
    if (q8) return launch_fmt<2>(d, p, plan);
    if (a.wdtype == L0B_BF16) return launch_fmt<1>(d, p, plan);
    return launch_fmt<0>(d, p, plan);
}

l0b_status cast_rows_launch(l0b_device* d, const float* x, long long ld_x, const float* norm_w, float eps, void* out16,
                            int dtype, int M, int K) {
    return d->launch(cast_rows_kernel, dim3(M), dim3(256), 0, x, ld_x, norm_w, eps, out16, dtype, K);
}

l0b_status cast_rows_split_launch(l0b_device* d, const float* x, long long ld_x, const float* norm_w, float eps,
                                  void* out16, float* rscale, int dtype, int M, int K, const TcPlan& plan) {
    const bool vec = K % 4 == 0 && ld_x % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                     (!norm_w || reinterpret_cast<uintptr_t>(norm_w) % 16 == 0) &&
                     reinterpret_cast<uintptr_t>(out16) % 8 == 0;
    if (dtype == L0B_I8) {
        L0B_REQUIRE(vec && K <= 4 * 10 * 512, L0B_ERR_UNSUPPORTED,
                    "int8 digits need 16-byte aligned f32 rows with K %% 4 == 0 and K <= 20480");
        uint8_t* o = static_cast<uint8_t*>(out16);
        if (K <= 4 * 4 * 256)
            return d->launch(cast_rows_digits_kernel<4>, dim3(M), dim3(256), 0, x, ld_x, norm_w, eps, o, rscale, K,
                             plan.bn, plan.tb);
        return d->launch(cast_rows_digits_kernel<10>, dim3(M), dim3(512), 0, x, ld_x, norm_w, eps, o, rscale, K,
                         plan.bn, plan.tb);
    }
    if (vec && K <= 4 * 4 * 256)
        return d->launch(cast_rows_split_reg_kernel<4>, dim3(M), dim3(256), 0, x, ld_x, norm_w, eps, out16, rscale,
                         dtype, K, plan.bn, plan.tb);
    if (vec && K <= 4 * 10 * 512)
        return d->launch(cast_rows_split_reg_kernel<10>, dim3(M), dim3(512), 0, x, ld_x, norm_w, eps, out16, rscale,
                         dtype, K, plan.bn, plan.tb);
    return d->launch(cast_rows_split_kernel, dim3(M), dim3(256), 0, x, ld_x, norm_w, eps, out16, rscale, dtype, K,
                     plan.bn, plan.tb);
}

}  // namespace l0b
