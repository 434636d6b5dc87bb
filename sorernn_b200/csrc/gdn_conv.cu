// Short causal depthwise convolution with SiLU, the q/k/v prologue of the GDN layer
// (sore/model/conv.py:6-23 causal_conv1d_varlen, or FLA's causal_conv1d at sore/model/gdn.py:199-207):
//   z[t, c] = sum_{j < K} w[c, K-1-j] x[t-j, c]   over taps t-j inside t's document,   y = silu(z)
// Documents: rows of a [B, T, C] batch, or the cu_seqlens spans of a packed B == 1 batch (a tap before
// the document start contributes nothing, as the reference's masked_fill does).
// Backward, with dz = dy silu'(z) recomputed from x:
//   dx[t, c] = sum_{j < K} w[c, K-1-j] dz[t+j, c]   over t+j inside t's document,
//   dw[c, K-1-j] = sum_t x[t-j, c] dz[t, c]          (fp32, reduced per block, then one atomic add each).
// One thread per (token, 8 consecutive channels): 16-byte rows for bf16/fp16, fp32 accumulation.
#include "common.cuh"
#include "kernels.h"

namespace gdn {

constexpr int kConvThreads = 256;

template <typename T> struct Vec8;
template <> struct Vec8<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[8]) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            o[2 * e] = f.x;
            o[2 * e + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};
template <> struct Vec8<__half> {
    static __device__ __forceinline__ void load(const __half* p, float (&o)[8]) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h[e]);
            o[2 * e] = f.x;
            o[2 * e + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void store(__half* p, const float (&v)[8]) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};
template <> struct Vec8<float> {
    static __device__ __forceinline__ void load(const float* p, float (&o)[8]) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
    static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
};

struct ConvArgs {
    const void *x, *w, *dy;
    void *y, *dx;
    float* dw;
    const int64_t* cu;  // [N + 1] or null
    int64_t B, T, C, N;
    int w_dtype, silu;
};

__device__ __forceinline__ float ld_w(const void* p, int dtype, int64_t i) {
    if (dtype == GDN_FP32) return ((const float*)p)[i];
    if (dtype == GDN_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    return __half2float(((const __half*)p)[i]);
}
__device__ __forceinline__ float sig(float x) { return 1.f / (1.f + expf(-x)); }

// [start, end) of the document holding flattened token t
__device__ __forceinline__ void doc_span(const ConvArgs& a, int64_t t, int64_t& s, int64_t& e) {
    if (!a.cu) {
        s = (t / a.T) * a.T;
        e = s + a.T;
        return;
    }
    int64_t lo = 0, hi = a.N;  // largest n with cu[n] <= t
    while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (a.cu[mid] <= t) lo = mid;
        else hi = mid;
    }
    s = a.cu[lo];
    e = a.cu[lo + 1];
}

template <typename TA, int K>
__global__ void __launch_bounds__(kConvThreads) conv_fwd_kernel(const ConvArgs a) {
    const int64_t groups = a.C / 8, total = a.B * a.T * groups;
    for (int64_t i = blockIdx.x * (int64_t)kConvThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kConvThreads) {
        const int64_t t = i / groups, c0 = (i % groups) * 8;
        int64_t s, e;
        doc_span(a, t, s, e);
        float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < K; ++j) {
            if (t - j < s) break;
            float xv[8];
            Vec8<TA>::load((const TA*)a.x + (t - j) * a.C + c0, xv);
#pragma unroll
            for (int q = 0; q < 8; ++q) z[q] = fmaf(ld_w(a.w, a.w_dtype, (c0 + q) * K + (K - 1 - j)), xv[q], z[q]);
        }
        if (a.silu) {
#pragma unroll
            for (int q = 0; q < 8; ++q) z[q] *= sig(z[q]);
        }
        Vec8<TA>::store((TA*)a.y + t * a.C + c0, z);
    }
}

template <typename TA, int K>
__global__ void __launch_bounds__(kConvThreads) conv_bwd_kernel(const ConvArgs a) {
    extern __shared__ float s_dw[];  // [C][K] block partials
    for (int64_t i = threadIdx.x; i < a.C * K; i += kConvThreads) s_dw[i] = 0.f;
    __syncthreads();
    const int64_t groups = a.C / 8, total = a.B * a.T * groups;
    for (int64_t i = blockIdx.x * (int64_t)kConvThreads + threadIdx.x; i < total; i += (int64_t)gridDim.x * kConvThreads) {
        const int64_t t = i / groups, c0 = (i % groups) * 8;
        int64_t s, e;
        doc_span(a, t, s, e);
        float w[8][K];
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
            for (int j = 0; j < K; ++j) w[q][j] = ld_w(a.w, a.w_dtype, (c0 + q) * K + j);
        // x rows t-K+1 .. t+K-1 (inside the document), zero outside
        float xr[2 * K - 1][8];
#pragma unroll
        for (int r = 0; r < 2 * K - 1; ++r) {
            const int64_t tt = t - (K - 1) + r;
            if (tt >= s && tt < e) {
                Vec8<TA>::load((const TA*)a.x + tt * a.C + c0, xr[r]);
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) xr[r][q] = 0.f;
            }
        }
        float dx[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < K; ++j) {  // dz at t + j
            const int64_t tj = t + j;
            if (tj >= e) break;
            float dyv[8], dz[8];
            Vec8<TA>::load((const TA*)a.dy + tj * a.C + c0, dyv);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float z = 0.f;
#pragma unroll
                for (int i2 = 0; i2 < K; ++i2) z = fmaf(w[q][K - 1 - i2], xr[K - 1 + j - i2][q], z);
                if (a.silu) {
                    const float sg = sig(z);
                    dz[q] = dyv[q] * sg * (1.f + z * (1.f - sg));
                } else {
                    dz[q] = dyv[q];
                }
                dx[q] = fmaf(w[q][K - 1 - j], dz[q], dx[q]);
            }
            if (j == 0) {  // this thread owns dz[t]: its weight-gradient terms
#pragma unroll
                for (int q = 0; q < 8; ++q)
#pragma unroll
                    for (int i2 = 0; i2 < K; ++i2) atomicAdd(&s_dw[(c0 + q) * K + (K - 1 - i2)], xr[K - 1 - i2][q] * dz[q]);
            }
        }
        Vec8<TA>::store((TA*)a.dx + t * a.C + c0, dx);
    }
    __syncthreads();
    for (int64_t i = threadIdx.x; i < a.C * K; i += kConvThreads)
        if (s_dw[i] != 0.f) atomicAdd(&a.dw[i], s_dw[i]);
}

static unsigned conv_grid(int64_t work) {
    const int64_t blocks = (work + kConvThreads - 1) / kConvThreads;
    return (unsigned)(blocks < 148 * 8 ? (blocks > 0 ? blocks : 1) : 148 * 8);
}

template <typename TA>
static int conv_launch(const ConvArgs& a, int K, bool bwd, cudaStream_t s) {
    const unsigned grid = conv_grid(a.B * a.T * (a.C / 8));
    const size_t smem = bwd ? (size_t)a.C * K * sizeof(float) : 0;
    if (bwd && smem > 48 * 1024) {
        auto set = [&](const void* f) { return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); };
        if ((K == 1 && set((const void*)conv_bwd_kernel<TA, 1>) != cudaSuccess) ||
            (K == 2 && set((const void*)conv_bwd_kernel<TA, 2>) != cudaSuccess) ||
            (K == 3 && set((const void*)conv_bwd_kernel<TA, 3>) != cudaSuccess) ||
            (K == 4 && set((const void*)conv_bwd_kernel<TA, 4>) != cudaSuccess))
            return GDN_ERR_LAUNCH;
    }
#define CONV_CASE(KK)                                                                  \
    case KK:                                                                           \
        if (bwd) conv_bwd_kernel<TA, KK><<<grid, kConvThreads, smem, s>>>(a);          \
        else conv_fwd_kernel<TA, KK><<<grid, kConvThreads, 0, s>>>(a);                 \
        break;
    switch (K) {
        CONV_CASE(1)
        CONV_CASE(2)
        CONV_CASE(3)
        CONV_CASE(4)
        default: return GDN_ERR_SHAPE;
    }
#undef CONV_CASE
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn

using namespace gdn;

static int conv_check(int64_t B, int64_t T, int64_t C, int64_t K, int32_t act_dtype, int32_t w_dtype,
                      const int64_t* cu, int64_t N) {
    if (B < 0 || T < 0 || C <= 0 || C % 8 || K < 1 || K > 4 || C * K > 16384) return GDN_ERR_SHAPE;
    if (cu && (B != 1 || N < 1)) return GDN_ERR_SHAPE;
    if ((act_dtype != GDN_BF16 && act_dtype != GDN_FP16 && act_dtype != GDN_FP32) ||
        (w_dtype != GDN_BF16 && w_dtype != GDN_FP16 && w_dtype != GDN_FP32))
        return GDN_ERR_DTYPE;
    return GDN_OK;
}

extern "C" int gdn_causal_conv1d_fwd(int64_t B, int64_t T, int64_t C, int64_t K, const void* x, int32_t act_dtype,
                                     const void* weight, int32_t w_dtype, const int64_t* cu_seqlens, int64_t N,
                                     int32_t silu, void* y, gdn_stream_t stream) {
    int st = conv_check(B, T, C, K, act_dtype, w_dtype, cu_seqlens, N);
    if (st != GDN_OK) return st;
    if (!x || !weight || !y) return GDN_ERR_ARGUMENT;
    if (((uintptr_t)x | (uintptr_t)y) % 16) return GDN_ERR_ALIGN;
    if (B * T == 0) return GDN_OK;
    ConvArgs a{};
    a.x = x; a.w = weight; a.y = y; a.cu = cu_seqlens; a.B = B; a.T = T; a.C = C; a.N = N;
    a.w_dtype = w_dtype; a.silu = silu;
    cudaStream_t s = (cudaStream_t)stream;
    GDN_DISPATCH_DTYPE(act_dtype, TA, return conv_launch<TA>(a, (int)K, false, s);)
    return GDN_ERR_DTYPE;
}

extern "C" int gdn_causal_conv1d_bwd(int64_t B, int64_t T, int64_t C, int64_t K, const void* x, int32_t act_dtype,
                                     const void* weight, int32_t w_dtype, const int64_t* cu_seqlens, int64_t N,
                                     int32_t silu, const void* dy, void* dx, float* dweight, gdn_stream_t stream) {
    int st = conv_check(B, T, C, K, act_dtype, w_dtype, cu_seqlens, N);
    if (st != GDN_OK) return st;
    if (!x || !weight || !dy || !dx || !dweight) return GDN_ERR_ARGUMENT;
    if (((uintptr_t)x | (uintptr_t)dy | (uintptr_t)dx) % 16) return GDN_ERR_ALIGN;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(dweight, 0, C * K * sizeof(float), s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (B * T == 0) return GDN_OK;
    ConvArgs a{};
    a.x = x; a.w = weight; a.dy = dy; a.dx = dx; a.dw = dweight; a.cu = cu_seqlens; a.B = B; a.T = T; a.C = C;
    a.N = N; a.w_dtype = w_dtype; a.silu = silu;
    GDN_DISPATCH_DTYPE(act_dtype, TA, return conv_launch<TA>(a, (int)K, true, s);)
    return GDN_ERR_DTYPE;
}
