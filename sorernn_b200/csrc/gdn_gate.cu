// The gate and beta activations that soreRNN's GDN layer can leave to the mixer kernel
// (sore/model/gdn.py:157-162, use_gate_in_kernel / use_beta_sigmoid_in_kernel):
//   g    = -exp(A_log[h]) * softplus(a + dt_bias[h])   (fp32; the layer's _gate_and_beta, gdn.py:191-194)
//   beta = sigmoid(b)
// with softplus(x) = log(1 + e^x), and x itself above 20 (torch's F.softplus threshold). Backward:
//   da = dg * (-exp(A_log)) * sigmoid(x),  ddt_bias[h] = sum over tokens of da,  dA_log[h] = sum of dg * g,
//   db = dbeta * beta * (1 - beta).
// Elementwise over [tokens, HV] with the per-head sums reduced in shared memory, then one atomic add per
// head per block (the launchers zero dA_log and ddt_bias first).
#include "common.cuh"
#include "kernels.h"

namespace gdn {

__device__ __forceinline__ float ld_code(const void* p, int dtype, int64_t i) {
    if (dtype == GDN_FP32) return ((const float*)p)[i];
    if (dtype == GDN_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    return __half2float(((const __half*)p)[i]);
}
__device__ __forceinline__ void st_code(void* p, int dtype, int64_t i, float x) {
    if (dtype == GDN_FP32) ((float*)p)[i] = x;
    else if (dtype == GDN_BF16) ((__nv_bfloat16*)p)[i] = __float2bfloat16_rn(x);
    else ((__half*)p)[i] = __float2half_rn(x);
}
// log(1 + e^x) for x <= 20 (log1pf keeps full precision for very negative x), x above
__device__ __forceinline__ float softplus20(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

struct GateArgs {
    const void* a;
    const void* A_log;
    const void* dt_bias;  // may be null
    const float* dg;      // backward only
    float* g;             // forward output
    void* da;             // backward output (dtype of a)
    float *dA_log, *ddt_bias;
    int64_t n;  // tokens x HV
    int HV, a_dtype, p_dtype;
};

constexpr int kGateThreads = 256;
constexpr int kGateMaxHV = 1024;

__global__ void __launch_bounds__(kGateThreads) gate_fwd_kernel(const GateArgs a) {
    for (int64_t i = blockIdx.x * (int64_t)kGateThreads + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * kGateThreads) {
        const int h = (int)(i % a.HV);
        const float x = ld_code(a.a, a.a_dtype, i) + (a.dt_bias ? ld_code(a.dt_bias, a.p_dtype, h) : 0.f);
        a.g[i] = -expf(ld_code(a.A_log, a.p_dtype, h)) * softplus20(x);
    }
}

__global__ void __launch_bounds__(kGateThreads) gate_bwd_kernel(const GateArgs a) {
    __shared__ float s_dA[kGateMaxHV], s_db[kGateMaxHV];
    for (int h = threadIdx.x; h < a.HV; h += kGateThreads) s_dA[h] = s_db[h] = 0.f;
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)kGateThreads + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * kGateThreads) {
        const int h = (int)(i % a.HV);
        const float x = ld_code(a.a, a.a_dtype, i) + (a.dt_bias ? ld_code(a.dt_bias, a.p_dtype, h) : 0.f);
        const float ea = expf(ld_code(a.A_log, a.p_dtype, h));
        const float dg = a.dg[i];
        const float dx = -dg * ea * (x > 20.f ? 1.f : sigmoidf_(x));
        st_code(a.da, a.a_dtype, i, dx);
        atomicAdd(&s_dA[h], dg * (-ea * softplus20(x)));
        atomicAdd(&s_db[h], dx);
    }
    __syncthreads();
    for (int h = threadIdx.x; h < a.HV; h += kGateThreads) {
        if (s_dA[h] != 0.f) atomicAdd(&a.dA_log[h], s_dA[h]);
        if (a.ddt_bias && s_db[h] != 0.f) atomicAdd(&a.ddt_bias[h], s_db[h]);
    }
}

struct BetaArgs {
    const void* b;
    const float* dbeta;
    float* beta;
    void* db;
    int64_t n;
    int b_dtype;
};

__global__ void __launch_bounds__(kGateThreads) beta_fwd_kernel(const BetaArgs a) {
    for (int64_t i = blockIdx.x * (int64_t)kGateThreads + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * kGateThreads)
        a.beta[i] = sigmoidf_(ld_code(a.b, a.b_dtype, i));
}
__global__ void __launch_bounds__(kGateThreads) beta_bwd_kernel(const BetaArgs a) {
    for (int64_t i = blockIdx.x * (int64_t)kGateThreads + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * kGateThreads) {
        const float s = sigmoidf_(ld_code(a.b, a.b_dtype, i));
        st_code(a.db, a.b_dtype, i, a.dbeta[i] * s * (1.f - s));
    }
}

static unsigned grid_for(int64_t n) {
    const int64_t blocks = (n + kGateThreads - 1) / kGateThreads;
    return (unsigned)(blocks < 148 * 8 ? (blocks > 0 ? blocks : 1) : 148 * 8);
}

}  // namespace gdn

using namespace gdn;

static bool dtype_code_ok(int32_t d) { return d == GDN_BF16 || d == GDN_FP16 || d == GDN_FP32; }

extern "C" int gdn_gate_fwd(int64_t n_tokens, int64_t HV, const void* a, int32_t a_dtype, const void* A_log,
                            const void* dt_bias, int32_t param_dtype, float* g_out, gdn_stream_t stream) {
    if (n_tokens < 0 || HV <= 0 || HV > kGateMaxHV) return GDN_ERR_SHAPE;
    if (!dtype_code_ok(a_dtype) || !dtype_code_ok(param_dtype)) return GDN_ERR_DTYPE;
    if (!a || !A_log || !g_out) return GDN_ERR_ARGUMENT;
    GateArgs g{};
    g.a = a; g.A_log = A_log; g.dt_bias = dt_bias; g.g = g_out;
    g.n = n_tokens * HV; g.HV = (int)HV; g.a_dtype = a_dtype; g.p_dtype = param_dtype;
    if (g.n == 0) return GDN_OK;
    gate_fwd_kernel<<<grid_for(g.n), kGateThreads, 0, (cudaStream_t)stream>>>(g);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_gate_bwd(int64_t n_tokens, int64_t HV, const void* a, int32_t a_dtype, const void* A_log,
                            const void* dt_bias, int32_t param_dtype, const float* dg, void* da, float* dA_log,
                            float* ddt_bias, gdn_stream_t stream) {
    if (n_tokens < 0 || HV <= 0 || HV > kGateMaxHV) return GDN_ERR_SHAPE;
    if (!dtype_code_ok(a_dtype) || !dtype_code_ok(param_dtype)) return GDN_ERR_DTYPE;
    if (!a || !A_log || !dg || !da || !dA_log || (dt_bias && !ddt_bias)) return GDN_ERR_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(dA_log, 0, HV * sizeof(float), s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (ddt_bias && cudaMemsetAsync(ddt_bias, 0, HV * sizeof(float), s) != cudaSuccess) return GDN_ERR_LAUNCH;
    GateArgs g{};
    g.a = a; g.A_log = A_log; g.dt_bias = dt_bias; g.dg = dg; g.da = da; g.dA_log = dA_log;
    g.ddt_bias = dt_bias ? ddt_bias : nullptr;
    g.n = n_tokens * HV; g.HV = (int)HV; g.a_dtype = a_dtype; g.p_dtype = param_dtype;
    if (g.n == 0) return GDN_OK;
    gate_bwd_kernel<<<grid_for(g.n), kGateThreads, 0, s>>>(g);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_beta_sigmoid_fwd(int64_t n, const void* b, int32_t b_dtype, float* beta_out, gdn_stream_t stream) {
    if (n < 0) return GDN_ERR_SHAPE;
    if (!dtype_code_ok(b_dtype)) return GDN_ERR_DTYPE;
    if (!b || !beta_out) return GDN_ERR_ARGUMENT;
    if (n == 0) return GDN_OK;
    BetaArgs a{};
    a.b = b; a.beta = beta_out; a.n = n; a.b_dtype = b_dtype;
    beta_fwd_kernel<<<grid_for(n), kGateThreads, 0, (cudaStream_t)stream>>>(a);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_beta_sigmoid_bwd(int64_t n, const void* b, int32_t b_dtype, const float* dbeta, void* db,
                                    gdn_stream_t stream) {
    if (n < 0) return GDN_ERR_SHAPE;
    if (!dtype_code_ok(b_dtype)) return GDN_ERR_DTYPE;
    if (!b || !dbeta || !db) return GDN_ERR_ARGUMENT;
    if (n == 0) return GDN_OK;
    BetaArgs a{};
    a.b = b; a.dbeta = dbeta; a.db = db; a.n = n; a.b_dtype = b_dtype;
    beta_bwd_kernel<<<grid_for(n), kGateThreads, 0, (cudaStream_t)stream>>>(a);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
