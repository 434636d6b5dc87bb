// Shared device helpers: dtype loads/stores, reductions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/gdn_b200.h"

namespace gdn {

template <typename T> __device__ __forceinline__ float ld(const T* p, int64_t i);
template <> __device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}
template <> __device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }

template <typename T> __device__ __forceinline__ void st(T* p, int64_t i, float x);
template <> __device__ __forceinline__ void st<float>(float* p, int64_t i, float x) { p[i] = x; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float x) {
    p[i] = __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ void st<__half>(__half* p, int64_t i, float x) { p[i] = __float2half_rn(x); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Sequence bounds in the flattened token axis: cu_seqlens if given, else row n of a [B, T] batch.
__device__ __forceinline__ void seq_bounds(const int64_t* cu, int64_t T, int64_t n, int64_t& bos, int64_t& eos) {
    if (cu) {
        bos = cu[n];
        eos = cu[n + 1];
    } else {
        bos = n * T;
        eos = bos + T;
    }
}

constexpr float kL2Eps = 1e-12f;  // F.normalize's eps (gdn.py:177)

// PER consecutive elements of type TA at p + i (as floats), in the widest vector loads that PER elements
// allow; the address must be aligned to that width.
template <typename TA, int PER>
__device__ __forceinline__ void ldv(const void* p, int64_t i, float (&o)[PER]) {
    const TA* q = (const TA*)p + i;
    constexpr int BYTES = PER * (int)sizeof(TA);
    constexpr int CH = BYTES % 16 == 0 ? 16 : (BYTES % 8 == 0 ? 8 : (BYTES % 4 == 0 ? 4 : 0));
    if constexpr (CH == 0) {
#pragma unroll
        for (int e = 0; e < PER; ++e) o[e] = ld(q, e);
    } else {
        constexpr int EPC = CH / (int)sizeof(TA);  // elements per chunk
#pragma unroll
        for (int c = 0; c < PER / EPC; ++c) {
            alignas(16) TA h[EPC];
            if constexpr (CH == 16) *reinterpret_cast<uint4*>(h) = *reinterpret_cast<const uint4*>(q + c * EPC);
            else if constexpr (CH == 8) *reinterpret_cast<uint2*>(h) = *reinterpret_cast<const uint2*>(q + c * EPC);
            else *reinterpret_cast<uint32_t*>(h) = *reinterpret_cast<const uint32_t*>(q + c * EPC);
#pragma unroll
            for (int e = 0; e < EPC; ++e) o[c * EPC + e] = ld(h, e);
        }
    }
}
template <typename TA, int PER>
__device__ __forceinline__ void stv(void* p, int64_t i, const float (&v)[PER]) {
    TA* q = (TA*)p + i;
    constexpr int BYTES = PER * (int)sizeof(TA);
    constexpr int CH = BYTES % 16 == 0 ? 16 : (BYTES % 8 == 0 ? 8 : (BYTES % 4 == 0 ? 4 : 0));
    if constexpr (CH == 0) {
#pragma unroll
        for (int e = 0; e < PER; ++e) st(q, e, v[e]);
    } else {
        constexpr int EPC = CH / (int)sizeof(TA);
#pragma unroll
        for (int c = 0; c < PER / EPC; ++c) {
            alignas(16) TA h[EPC];
#pragma unroll
            for (int e = 0; e < EPC; ++e) st(h, e, v[c * EPC + e]);
            if constexpr (CH == 16) *reinterpret_cast<uint4*>(q + c * EPC) = *reinterpret_cast<const uint4*>(h);
            else if constexpr (CH == 8) *reinterpret_cast<uint2*>(q + c * EPC) = *reinterpret_cast<const uint2*>(h);
            else *reinterpret_cast<uint32_t*>(q + c * EPC) = *reinterpret_cast<const uint32_t*>(h);
        }
    }
}

// A gate value (g or beta) kept as loaded: fp32 as 32 bits, bf16/fp16 as 16 bits (no conversion, so the
// load does not stall the thread that issues it ahead of use); gate_f converts it when it is used.
__device__ __forceinline__ uint32_t ld_gate_raw(const void* p, int dtype, int64_t i) {
    uint32_t r;
    if (dtype == GDN_FP32) r = ((const uint32_t*)p)[i];
    else r = ((const uint16_t*)p)[i];
    return r;
}
__device__ __forceinline__ float gate_f(uint32_t r, int dtype) {
    if (dtype == GDN_FP32) return __uint_as_float(r);
    if (dtype == GDN_BF16) return __uint_as_float(r << 16);
    return __half2float(__ushort_as_half((unsigned short)r));
}

// N elements of type TA kept as loaded (not widened to fp32), so that many rows can be in flight in few
// registers; load() uses the widest vector N elements allow (the address must be aligned to it).
template <typename TA, int N>
struct RawVec {
    static constexpr int BYTES = N * (int)sizeof(TA);
    static constexpr int CH = BYTES % 16 == 0 ? 16 : (BYTES % 8 == 0 ? 8 : (BYTES % 4 == 0 ? 4 : 2));
    using Chunk = typename std::conditional<CH == 16, uint4,
                  typename std::conditional<CH == 8, uint2,
                  typename std::conditional<CH == 4, uint32_t, uint16_t>::type>::type>::type;
    union {
        Chunk c[BYTES / CH];
        TA h[N];
    };
    __device__ __forceinline__ void load(const void* p, int64_t i) {
        const Chunk* q = reinterpret_cast<const Chunk*>((const TA*)p + i);
#pragma unroll
        for (int k = 0; k < BYTES / CH; ++k) c[k] = q[k];
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int k = 0; k < BYTES / CH; ++k) c[k] = Chunk{};
    }
    __device__ __forceinline__ float get(int e) const { return ld(h, e); }
};

}  // namespace gdn

// Dispatch a dtype code to a C++ type.
#define GDN_DISPATCH_DTYPE(code, TYPE, ...)                  \
    switch (code) {                                          \
        case GDN_BF16: { using TYPE = __nv_bfloat16; __VA_ARGS__; } break; \
        case GDN_FP16: { using TYPE = __half; __VA_ARGS__; } break;        \
        case GDN_FP32: { using TYPE = float; __VA_ARGS__; } break;         \
        default: return GDN_ERR_DTYPE;                       \
    }
