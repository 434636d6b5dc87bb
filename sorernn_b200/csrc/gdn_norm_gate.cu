// The GDN layer's output step, RMSNorm(o) * silu(gate) in one pass (sore/model/gdn.py:180-188: FLA's
// rms_norm_gated with activation "swish", no bias, the o_norm weight and eps; the unfused path is
// o_norm(o) * F.silu(gate) with RMSNorm of sore/model/layers.py:15-18). Per row of D features, in fp32
// with one rounding to the output dtype:
//   r = rsqrt(mean(x^2) + eps),  n = x r,  y = n w silu(g)
// Backward, with s = silu(g), a = n w:
//   dg = dy a s'(g),  s'(g) = sigmoid(g) (1 + g (1 - sigmoid(g)))
//   dn = dy s w,  dx = r (dn - n mean(dn n)),  dw = sum over rows of dy s n
// One warp per row; each lane holds D/32 consecutive features (D % 32 == 0, D <= 1024). dw is reduced
// per block in shared memory and added to global memory with one atomic add per feature per block.
#include "common.cuh"
#include "kernels.h"

namespace gdn {

constexpr int kNgWarps = 8;
constexpr int kNgMaxPer = 32;  // features per lane: D <= 1024

__device__ __forceinline__ float ld_c(const void* p, int dtype, int64_t i) {
    if (dtype == GDN_FP32) return ((const float*)p)[i];
    if (dtype == GDN_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    return __half2float(((const __half*)p)[i]);
}
__device__ __forceinline__ void st_c(void* p, int dtype, int64_t i, float x) {
    if (dtype == GDN_FP32) ((float*)p)[i] = x;
    else if (dtype == GDN_BF16) ((__nv_bfloat16*)p)[i] = __float2bfloat16_rn(x);
    else ((__half*)p)[i] = __float2half_rn(x);
}
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }

struct NormGateArgs {
    const void *x, *g, *w, *dy;
    void *y, *dx, *dg;
    float* dw;
    int64_t rows;
    int D, act_dtype, w_dtype;
    float eps;
};

template <typename TA, int PER>
__global__ void __launch_bounds__(32 * kNgWarps) norm_gate_fwd_kernel(const NormGateArgs a) {
    const int lane = threadIdx.x & 31;
    float w[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) w[e] = ld_c(a.w, a.w_dtype, lane * PER + e);
    const int64_t warp0 = blockIdx.x * (int64_t)kNgWarps + (threadIdx.x >> 5);
    for (int64_t r = warp0; r < a.rows; r += (int64_t)gridDim.x * kNgWarps) {
        const int64_t base = r * a.D + lane * PER;
        float x[PER], g[PER], y[PER], ss = 0.f;
        ldv<TA, PER>(a.x, base, x);
        ldv<TA, PER>(a.g, base, g);
#pragma unroll
        for (int e = 0; e < PER; ++e) ss = fmaf(x[e], x[e], ss);
        const float rs = rsqrtf(warp_sum(ss) / a.D + a.eps);
#pragma unroll
        for (int e = 0; e < PER; ++e) y[e] = x[e] * rs * w[e] * g[e] * sigm(g[e]);
        stv<TA, PER>(a.y, base, y);
    }
}

template <typename TA, int PER>
__global__ void __launch_bounds__(32 * kNgWarps) norm_gate_bwd_kernel(const NormGateArgs a) {
    __shared__ float s_dw[1024];
    for (int i = threadIdx.x; i < a.D; i += 32 * kNgWarps) s_dw[i] = 0.f;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    float w[PER], dwp[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        w[e] = ld_c(a.w, a.w_dtype, lane * PER + e);
        dwp[e] = 0.f;
    }
    const int64_t warp0 = blockIdx.x * (int64_t)kNgWarps + (threadIdx.x >> 5);
    for (int64_t r = warp0; r < a.rows; r += (int64_t)gridDim.x * kNgWarps) {
        const int64_t base = r * a.D + lane * PER;
        float x[PER], g[PER], dy[PER], dn[PER], dg[PER], dx[PER], ss = 0.f;
        ldv<TA, PER>(a.x, base, x);
        ldv<TA, PER>(a.g, base, g);
        ldv<TA, PER>(a.dy, base, dy);
#pragma unroll
        for (int e = 0; e < PER; ++e) ss = fmaf(x[e], x[e], ss);
        const float rs = rsqrtf(warp_sum(ss) / a.D + a.eps);
        float c = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            const float sg = sigm(g[e]), sv = g[e] * sg, n = x[e] * rs;
            dg[e] = dy[e] * n * w[e] * sg * (1.f + g[e] * (1.f - sg));
            dn[e] = dy[e] * sv * w[e];
            dwp[e] = fmaf(dy[e] * sv, n, dwp[e]);
            c = fmaf(dn[e], n, c);
        }
        c = warp_sum(c) / a.D;
#pragma unroll
        for (int e = 0; e < PER; ++e) dx[e] = rs * (dn[e] - x[e] * rs * c);
        stv<TA, PER>(a.dg, base, dg);
        stv<TA, PER>(a.dx, base, dx);
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) atomicAdd(&s_dw[lane * PER + e], dwp[e]);
    __syncthreads();
    for (int i = threadIdx.x; i < a.D; i += 32 * kNgWarps) atomicAdd(&a.dw[i], s_dw[i]);
}

static unsigned ng_grid(int64_t rows) {
    const int64_t blocks = (rows + kNgWarps - 1) / kNgWarps;
    return (unsigned)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

#define NG_DISPATCH_PER(TA, D, KERNEL, ...)                                     \
    switch ((D) / 32) {                                                         \
        case 1: KERNEL<TA, 1><<<__VA_ARGS__>>>(a); break;                       \
        case 2: KERNEL<TA, 2><<<__VA_ARGS__>>>(a); break;                       \
        case 4: KERNEL<TA, 4><<<__VA_ARGS__>>>(a); break;                       \
        case 8: KERNEL<TA, 8><<<__VA_ARGS__>>>(a); break;                       \
        case 16: KERNEL<TA, 16><<<__VA_ARGS__>>>(a); break;                     \
        case 32: KERNEL<TA, 32><<<__VA_ARGS__>>>(a); break;                     \
        default: return GDN_ERR_SHAPE;                                          \
    }

}  // namespace gdn

using namespace gdn;

static bool ng_dtype_ok(int32_t d) { return d == GDN_BF16 || d == GDN_FP16 || d == GDN_FP32; }

extern "C" int gdn_rms_norm_gated_fwd(int64_t rows, int64_t D, const void* x, const void* gate, int32_t act_dtype,
                                      const void* weight, int32_t w_dtype, float eps, void* y, gdn_stream_t stream) {
    if (rows < 0 || D <= 0 || D > 1024 || D % 32) return GDN_ERR_SHAPE;
    if (!ng_dtype_ok(act_dtype) || !ng_dtype_ok(w_dtype)) return GDN_ERR_DTYPE;
    if (!x || !gate || !weight || !y) return GDN_ERR_ARGUMENT;
    if (rows == 0) return GDN_OK;
    NormGateArgs a{};
    a.x = x; a.g = gate; a.w = weight; a.y = y;
    a.rows = rows; a.D = (int)D; a.act_dtype = act_dtype; a.w_dtype = w_dtype; a.eps = eps;
    GDN_DISPATCH_DTYPE(act_dtype, TA, NG_DISPATCH_PER(TA, D, norm_gate_fwd_kernel, ng_grid(rows), 32 * kNgWarps, 0, (cudaStream_t)stream))
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_rms_norm_gated_bwd(int64_t rows, int64_t D, const void* x, const void* gate, int32_t act_dtype,
                                      const void* weight, int32_t w_dtype, float eps, const void* dy, void* dx,
                                      void* dgate, float* dweight, gdn_stream_t stream) {
    if (rows < 0 || D <= 0 || D > 1024 || D % 32) return GDN_ERR_SHAPE;
    if (!ng_dtype_ok(act_dtype) || !ng_dtype_ok(w_dtype)) return GDN_ERR_DTYPE;
    if (!x || !gate || !weight || !dy || !dx || !dgate || !dweight) return GDN_ERR_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(dweight, 0, D * sizeof(float), s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (rows == 0) return GDN_OK;
    NormGateArgs a{};
    a.x = x; a.g = gate; a.w = weight; a.dy = dy; a.dx = dx; a.dg = dgate; a.dw = dweight;
    a.rows = rows; a.D = (int)D; a.act_dtype = act_dtype; a.w_dtype = w_dtype; a.eps = eps;
    GDN_DISPATCH_DTYPE(act_dtype, TA, NG_DISPATCH_PER(TA, D, norm_gate_bwd_kernel, ng_grid(rows), 32 * kNgWarps, 0, s))
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
