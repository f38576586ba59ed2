// Shared device helpers for the decoder token loop kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wsp {

constexpr int kThreads = 256;  // every kernel of the step runs 8 warps
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kUnchosen = 0xFFFFFFFFu;  // Argmax.h:40 unchosenIndex

// Storage types for the 16-bit weights, activations and KV caches.
template <typename T> struct Half16;
template <> struct Half16<__half> {
    static __device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_float(float v) { return __float2half_rn(v); }
    static __device__ __forceinline__ float2 pair_to_float2(uint32_t bits) {
        __half2 h = *reinterpret_cast<__half2*>(&bits);
        return __half22float2(h);
    }
    // a in the low half, b in the high half (an MMA fragment's element order).
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <> struct Half16<__nv_bfloat16> {
    static __device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_float(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ float2 pair_to_float2(uint32_t bits) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&bits);
        return __bfloat1622float2(h);
    }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// A pair of fp32 values as two 16-bit pairs, hi + lo, whose sum carries
// about twice the 16-bit precision: the operand of two tensor-core products
// that together act as one with a wider operand.
template <typename T>
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
    const float ha = Half16<T>::to_float(Half16<T>::from_float(a));
    const float hb = Half16<T>::to_float(Half16<T>::from_float(b));
    hi = Half16<T>::pack2(a, b);
    lo = Half16<T>::pack2(a - ha, b - hb);
}

// The position of 16-byte piece p (0..15) of cross key row j in memory and
// in shared memory: the 8 key pieces and the 8 value pieces each rotate by
// j % 8, so eight consecutive keys' same piece fall in eight bank groups.
__host__ __device__ __forceinline__ int cross_piece(int p, int j) { return (p & 8) | ((p ^ j) & 7); }

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

// Block-wide sum / max over kThreads threads through `scratch` (>= kWarps floats).
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total += scratch[w];
    return total;
}

__device__ __forceinline__ float block_max(float v, float* scratch) {
    v = warp_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float best = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) best = fmaxf(best, scratch[w]);
    return best;
}

// The candidate order of Argmax.h:25-35: the larger value wins; on equal
// values the lower index; the unchosen sentinel loses to any chosen index.
__device__ __forceinline__ bool candidate_better(float v, uint32_t i, float bv, uint32_t bi) {
    if (i == kUnchosen) return false;
    if (bi == kUnchosen) return true;
    return v > bv || (v == bv && i < bi);
}

// Exact-erf GELU (Linear.h:222 / Gelu.h:12-18).
__device__ __forceinline__ float gelu_exact(float x) {
    return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
}

// m16n8k16 tensor-core product, fp32 accumulate, on 16-bit operands.
template <typename T>
__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, const uint32_t* b);

template <>
__device__ __forceinline__ void mma_16816<__half>(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float* c, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// 16-byte global load that bypasses L1 allocation (weights are streamed once).
__device__ __forceinline__ uint4 load_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 load_cached(const void* p) {
    return *reinterpret_cast<const uint4*>(p);
}

}  // namespace wsp
