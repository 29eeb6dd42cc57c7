// Device-side helpers shared by the kernels of libl0b200 (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "runtime.h"

namespace l0b {

constexpr float kNegInf = -__builtin_huge_valf();

// Programmatic dependent launch. Every kernel calls pdl_wait() before it touches memory that an
// earlier kernel writes (and before it exits), so completion stays transitive along the stream.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// L2 prefetch of a contiguous byte range (16-byte aligned start, size a multiple of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Streaming 128-bit load of data read once (weights): no L1 allocation.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Packed fp32 pair arithmetic (Blackwell f32x2): one instruction for two lanes of math.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Exact int8 -> fp32 for the four signed bytes of a word, two at a time.
// Byte b is biased to u = b ^ 0x80 (0..255) and placed in the mantissa of 2^23: the float
// 0x4B0000uu equals 8388608 + u exactly, and subtracting 8388608 + 128 recovers b exactly.
__device__ __forceinline__ void dequant_i8x4(uint32_t w, float2& lo, float2& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    float2 a, b;
    a.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440));
    a.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441));
    b.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442));
    b.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443));
    lo = fadd2(a, bias);
    hi = fadd2(b, bias);
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
}
// bf16 -> fp32 is a shift: the bf16 bits are the high half of the fp32 bits.
__device__ __forceinline__ float2 bf162_bits_to_float2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

template <typename T> struct DT;
template <> struct DT<float> { static constexpr l0b_dtype id = L0B_F32; };
template <> struct DT<__half> { static constexpr l0b_dtype id = L0B_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr l0b_dtype id = L0B_BF16; };
template <> struct DT<int8_t> { static constexpr l0b_dtype id = L0B_I8; };

// Scalar load/store with a run-time dtype (f32 / f16 / bf16).
__device__ __forceinline__ float load_as_float(const void* p, int dtype, long long i) {
    switch (dtype) {
        case L0B_F16: return __half2float(static_cast<const __half*>(p)[i]);
        case L0B_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
        default: return static_cast<const float*>(p)[i];
    }
}
__device__ __forceinline__ void store_from_float(void* p, int dtype, long long i, float v) {
    switch (dtype) {
        case L0B_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
        case L0B_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
        default: static_cast<float*>(p)[i] = v; break;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` holds >= 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
    t = warp_sum(t);
    return t;
}

// Ordered key for argmax with atomicMax: larger value wins, ties go to the lower index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(0x7FFFFFFF - idx);
}
__device__ __forceinline__ int argmax_key_index(unsigned long long key) {
    return 0x7FFFFFFF - static_cast<int>(key & 0xFFFFFFFFu);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

}  // namespace l0b
