// Short causal depthwise convolution with SiLU, the q/k/v prologue of the GDN layer
// (sore/model/conv.py:6-23 causal_conv1d_varlen, or FLA's causal_conv1d at sore/model/gdn.py:199-207):
//   z[t, c] = sum_{j < K} w[c, K-1-j] x[t-j, c]   over taps t-j inside t's document,   y = silu(z)
// Documents: rows of a [B, T, C] batch, or the cu_seqlens spans of a packed B == 1 batch (a tap before
// the document start contributes nothing, as the reference's masked_fill does).
// Backward, with dz = dy silu'(z) recomputed from x:
//   dx[t, c] = sum_{j < K} w[c, K-1-j] dz[t+j, c]   over t+j inside t's document,
//   dw[c, K-1-j] = sum_t x[t-j, c] dz[t, c]          (fp32, reduced per block, then one atomic add each).
// One thread per (tile of 32 consecutive tokens, 8 channels forward / 4 backward): a sliding window over
// the taps, vector row loads, fp32 accumulation, weights and weight gradients in registers.
#include "common.cuh"
#include "kernels.h"

namespace gdn {

constexpr int kConvThreads = 256;

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

constexpr int kConvTile = 32;  // consecutive tokens per thread (a sliding window over the taps)

// Thread (token tile, group of CW channels): the C / CW threads of a tile are consecutive, so a warp's row
// loads are contiguous. Window rows before the document start read as zero. The next row is prefetched
// one token ahead.
template <typename TA, int K, int CW>
__global__ void __launch_bounds__(kConvThreads) conv_fwd_kernel(const ConvArgs a) {
    const int64_t groups = a.C / CW, BT = a.B * a.T, tiles = (BT + kConvTile - 1) / kConvTile;
    for (int64_t i = blockIdx.x * (int64_t)kConvThreads + threadIdx.x; i < tiles * groups;
         i += (int64_t)gridDim.x * kConvThreads) {
        const int64_t c0 = (i % groups) * CW, t0 = (i / groups) * kConvTile;
        const int64_t t1 = t0 + kConvTile < BT ? t0 + kConvTile : BT;
        float w[CW][K];
#pragma unroll
        for (int q = 0; q < CW; ++q)
#pragma unroll
            for (int j = 0; j < K; ++j) w[q][j] = ld_w(a.w, a.w_dtype, (c0 + q) * K + j);
        int64_t s, e;
        doc_span(a, t0, s, e);
        float win[K][CW];  // win[j] = x[t - j]
#pragma unroll
        for (int j = 1; j < K; ++j) {
            if (t0 - j >= s) ldv<TA, CW>(a.x, (t0 - j) * a.C + c0, win[j]);
            else {
#pragma unroll
                for (int q = 0; q < CW; ++q) win[j][q] = 0.f;
            }
        }
        float nxt[CW];
        ldv<TA, CW>(a.x, t0 * a.C + c0, nxt);
        for (int64_t t = t0; t < t1; ++t) {
            if (t >= e) {  // the next document starts here: no taps before it
                doc_span(a, t, s, e);
#pragma unroll
                for (int j = 1; j < K; ++j)
#pragma unroll
                    for (int q = 0; q < CW; ++q) win[j][q] = 0.f;
            }
#pragma unroll
            for (int q = 0; q < CW; ++q) win[0][q] = nxt[q];
            if (t + 1 < t1) ldv<TA, CW>(a.x, (t + 1) * a.C + c0, nxt);
            float z[CW];
#pragma unroll
            for (int q = 0; q < CW; ++q) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < K; ++j) acc = fmaf(w[q][K - 1 - j], win[j][q], acc);
                z[q] = a.silu ? acc * sig(acc) : acc;
            }
            stv<TA, CW>(a.y, t * a.C + c0, z);
#pragma unroll
            for (int j = K - 1; j >= 1; --j)
#pragma unroll
                for (int q = 0; q < CW; ++q) win[j][q] = win[j - 1][q];
        }
    }
}

// Backward over the same tiles: a window of x rows [t-K+1, t+K-1] and of dz rows [t, t+K-1] slides
// forward (the rows entering at t+K-1 are prefetched a token ahead); dw stays in registers for the tile.
template <typename TA, int K, int CW>
__global__ void __launch_bounds__(kConvThreads, 2) conv_bwd_kernel(const ConvArgs a) {
    extern __shared__ float s_dw[];  // [C][K] block partials
    for (int64_t i = threadIdx.x; i < a.C * K; i += kConvThreads) s_dw[i] = 0.f;
    __syncthreads();
    const int64_t groups = a.C / CW, BT = a.B * a.T, tiles = (BT + kConvTile - 1) / kConvTile;
    for (int64_t i = blockIdx.x * (int64_t)kConvThreads + threadIdx.x; i < tiles * groups;
         i += (int64_t)gridDim.x * kConvThreads) {
        const int64_t c0 = (i % groups) * CW, t0 = (i / groups) * kConvTile;
        const int64_t t1 = t0 + kConvTile < BT ? t0 + kConvTile : BT;
        float w[CW][K], dw[CW][K];
#pragma unroll
        for (int q = 0; q < CW; ++q)
#pragma unroll
            for (int j = 0; j < K; ++j) {
                w[q][j] = ld_w(a.w, a.w_dtype, (c0 + q) * K + j);
                dw[q][j] = 0.f;
            }
        int64_t s = 0, e = 0;
        float xw[2 * K - 1][CW];  // xw[r] = x[t - (K-1) + r]
        float dzw[K][CW];         // dzw[j] = dz[t + j]
        float px[CW], pdy[CW];    // raw rows t + K (prefetch for the next slide)
        // dz at token u (inside [s, e)) from dy[u] and the x window rows ending at u (xw index base..base+K-1)
        auto make_dz = [&](int64_t u, int base, const float (&dyv)[CW], float (&out)[CW]) {
#pragma unroll
            for (int q = 0; q < CW; ++q) {
                float z = 0.f;
#pragma unroll
                for (int i2 = 0; i2 < K; ++i2) z = fmaf(w[q][K - 1 - i2], xw[base + K - 1 - i2][q], z);
                float d = dyv[q];
                if (a.silu) {
                    const float sg = sig(z);
                    d *= sg * (1.f + z * (1.f - sg));
                }
                out[q] = u < e ? d : 0.f;
            }
        };
        bool fresh = true;
        for (int64_t t = t0; t < t1; ++t) {
            if (fresh || t >= e) {  // (re)build both windows at t: first token of the tile or of a document
                doc_span(a, t, s, e);
#pragma unroll
                for (int r = 0; r < 2 * K - 1; ++r) {
                    const int64_t u = t - (K - 1) + r;
                    if (u >= s && u < e) ldv<TA, CW>(a.x, u * a.C + c0, xw[r]);
                    else {
#pragma unroll
                        for (int q = 0; q < CW; ++q) xw[r][q] = 0.f;
                    }
                }
#pragma unroll
                for (int j = 0; j < K; ++j) {
                    float dyv[CW];
                    if (t + j < e) ldv<TA, CW>(a.dy, (t + j) * a.C + c0, dyv);
                    else {
#pragma unroll
                        for (int q = 0; q < CW; ++q) dyv[q] = 0.f;
                    }
                    make_dz(t + j, j, dyv, dzw[j]);
                }
                fresh = false;
            } else {  // slide by one token: x row and dz at t+K-1 enter from the prefetch
                const int64_t u = t + K - 1;
#pragma unroll
                for (int r = 0; r < 2 * K - 2; ++r)
#pragma unroll
                    for (int q = 0; q < CW; ++q) xw[r][q] = xw[r + 1][q];
#pragma unroll
                for (int q = 0; q < CW; ++q) xw[2 * K - 2][q] = u < e ? px[q] : 0.f;
#pragma unroll
                for (int j = 0; j < K - 1; ++j)
#pragma unroll
                    for (int q = 0; q < CW; ++q) dzw[j][q] = dzw[j + 1][q];
                make_dz(u, K - 1, pdy, dzw[K - 1]);
            }
            if (t + K < BT && t + 1 < t1) {  // rows entering at the next step
                ldv<TA, CW>(a.x, (t + K) * a.C + c0, px);
                ldv<TA, CW>(a.dy, (t + K) * a.C + c0, pdy);
            }
            float dx[CW];
#pragma unroll
            for (int q = 0; q < CW; ++q) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < K; ++j) acc = fmaf(w[q][K - 1 - j], dzw[j][q], acc);
                dx[q] = acc;
#pragma unroll
                for (int i2 = 0; i2 < K; ++i2) dw[q][K - 1 - i2] = fmaf(xw[K - 1 - i2][q], dzw[0][q], dw[q][K - 1 - i2]);
            }
            stv<TA, CW>(a.dx, t * a.C + c0, dx);
        }
#pragma unroll
        for (int q = 0; q < CW; ++q)
#pragma unroll
            for (int j = 0; j < K; ++j) atomicAdd(&s_dw[(c0 + q) * K + j], dw[q][j]);
    }
    __syncthreads();
    for (int64_t i = threadIdx.x; i < a.C * K; i += kConvThreads)
        if (s_dw[i] != 0.f) atomicAdd(&a.dw[i], s_dw[i]);
}

constexpr int kConvFwdCW = 8, kConvBwdCW = 4;

static unsigned conv_grid(int64_t work) {
    const int64_t blocks = (work + kConvThreads - 1) / kConvThreads;
    return (unsigned)(blocks < 148 * 8 ? (blocks > 0 ? blocks : 1) : 148 * 8);
}

template <typename TA>
static int conv_launch(const ConvArgs& a, int K, bool bwd, cudaStream_t s) {
    const int cw = bwd ? kConvBwdCW : kConvFwdCW;
    const unsigned grid = conv_grid((a.B * a.T + kConvTile - 1) / kConvTile * (a.C / cw));
    const size_t smem = bwd ? (size_t)a.C * K * sizeof(float) : 0;
    if (bwd && smem > 48 * 1024) {
        auto set = [&](const void* f) { return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); };
        if ((K == 1 && set((const void*)conv_bwd_kernel<TA, 1, kConvBwdCW>) != cudaSuccess) ||
            (K == 2 && set((const void*)conv_bwd_kernel<TA, 2, kConvBwdCW>) != cudaSuccess) ||
            (K == 3 && set((const void*)conv_bwd_kernel<TA, 3, kConvBwdCW>) != cudaSuccess) ||
            (K == 4 && set((const void*)conv_bwd_kernel<TA, 4, kConvBwdCW>) != cudaSuccess))
            return GDN_ERR_LAUNCH;
    }
#define CONV_CASE(KK)                                                                       \
    case KK:                                                                                \
        if (bwd) conv_bwd_kernel<TA, KK, kConvBwdCW><<<grid, kConvThreads, smem, s>>>(a);   \
        else conv_fwd_kernel<TA, KK, kConvFwdCW><<<grid, kConvThreads, 0, s>>>(a);          \
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
