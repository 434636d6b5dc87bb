// The GDN layer's output step, RMSNorm(o) * silu(gate) in one pass (sore/model/gdn.py:180-188: FLA's
// rms_norm_gated with activation "swish", no bias, the o_norm weight and eps; the unfused path is
// o_norm(o) * F.silu(gate) with RMSNorm of sore/model/layers.py:15-18). Per row of D features, in fp32
// with one rounding to the output dtype:
//   r = rsqrt(mean(x^2) + eps),  n = x r,  y = n w silu(g)
// Backward, with s = silu(g), a = n w:
//   dg = dy a s'(g),  s'(g) = sigmoid(g) (1 + g (1 - sigmoid(g)))
//   dn = dy s w,  dx = r (dn - n mean(dn n)),  dw = sum over rows of dy s n
// HBM-bound streaming: each block walks tiles of whole rows (8 KB of each input per tile), bulk-copied into
// a 4-stage shared-memory ring by one thread, so three tiles per block are in flight while the block computes
// the fourth (at config-1 sizes the fastest of 3-8 stages of 4-16 KB tiles: backward 127 -> 115 us against
// 3 stages). A row of D features is held by LPR = min(32, D / VEC) consecutive lanes, PER = D / LPR features
// each (VEC = the elements of 16 bytes: at D = 128 bf16, 16 lanes of 8 features). Outputs go straight from
// registers to global memory in 16-byte stores. dw is reduced across the lanes that share features, then
// per block in shared memory, then added to global memory with one atomic add per feature per block.
#include "bulk.cuh"
#include "common.cuh"
#include "kernels.h"

namespace gdn {

// Device error word of this file's kernels (a stage wait that gave up); read and cleared by
// read_clear_norm_gate_error().
static __device__ int g_norm_gate_err;

namespace ngs {
constexpr int NTHR = 256;
constexpr int STAGES = 4;
constexpr uint32_t TILE = 8192;  // bytes of one input per tile (whole rows)
}  // namespace ngs

__device__ __forceinline__ float ld_c(const void* p, int dtype, int64_t i) {
    if (dtype == GDN_FP32) return ((const float*)p)[i];
    if (dtype == GDN_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    return __half2float(((const __half*)p)[i]);
}
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

struct NormGateArgs {
    const void *x, *g, *w, *dy;
    void *y, *dx, *dg;
    float* dw;
    int64_t rows;
    int D, act_dtype, w_dtype;
    float eps;
};

template <int LPR>
__device__ __forceinline__ float group_sum(float x) {  // sum over the LPR lanes of this row
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// NT inputs staged per tile: x, g (forward) and dy (backward)
template <typename TA, int PER, int LPR, bool BWD>
__global__ void __launch_bounds__(ngs::NTHR) norm_gate_kernel(const NormGateArgs a) {
    using namespace ngs;
    constexpr int NT = BWD ? 3 : 2;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bar = (uint64_t*)(smem + STAGES * NT * TILE);
    float* s_dw = (float*)(smem + STAGES * NT * TILE + bulk::kBarBytes);  // [D], backward only
    const int tid = threadIdx.x, lane = tid & 31, f0 = (lane % LPR) * PER;
    const int rpass = NTHR / LPR;                    // rows one pass of the block covers
    const int row_in_pass = (tid >> 5) * (32 / LPR) + lane / LPR;
    const uint32_t rb = (uint32_t)a.D * sizeof(TA);  // bytes per row
    const int tr = (int)(TILE / rb);                 // rows per tile
    const int64_t tiles = (a.rows + tr - 1) / tr;
    const void* src[3] = {a.x, a.g, a.dy};

    auto issue = [&](int64_t tile, int s) {  // thread 0: the tile's rows of every input into stage s
        const int64_t r0 = tile * tr;
        const uint32_t bytes = (uint32_t)((a.rows - r0 < tr ? a.rows - r0 : tr) * rb);
        sm100::mbar_arrive_expect_tx(&bar[s], NT * bytes);
#pragma unroll
        for (int t = 0; t < NT; ++t)
            bulk::load(smem + (s * NT + t) * TILE, (const uint8_t*)src[t] + r0 * rb, bytes, &bar[s]);
    };

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) sm100::mbar_init(&bar[s], 1);
        sm100::fence_barrier_init();
    }
    if (BWD)
        for (int i = tid; i < a.D; i += NTHR) s_dw[i] = 0.f;
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < STAGES; ++s)
            if (blockIdx.x + (int64_t)s * gridDim.x < tiles) issue(blockIdx.x + (int64_t)s * gridDim.x, s);

    float w[PER], dwp[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        w[e] = ld_c(a.w, a.w_dtype, f0 + e);
        dwp[e] = 0.f;
    }
    bool ok = true;
    int it = 0;
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
        const int s = it % STAGES;
        ok = sm100::mbar_wait(&bar[s], (uint32_t)(it / STAGES) & 1u, &g_norm_gate_err, GDN_DEV_ERR_NORM_GATE,
                              ok ? (1u << 22) : 1u) && ok;
        const int64_t r0 = tile * tr;
        const int nr = (int)(a.rows - r0 < tr ? a.rows - r0 : tr);
        const uint8_t* st = smem + s * NT * TILE;
        for (int p = 0; p < tr; p += rpass) {  // every lane takes part in the row reductions
            const int rr = p + row_in_pass;
            const bool valid = rr < nr && ok;  // after a timed-out wait the stage holds nothing usable
            const int rs_ = valid ? rr : 0;  // rows past the tile's end read row 0 and store nothing
            float x[PER], g[PER];
            ldv<TA, PER>(st, (int64_t)rs_ * a.D + f0, x);
            ldv<TA, PER>(st + TILE, (int64_t)rs_ * a.D + f0, g);
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < PER; ++e) ss = fmaf(x[e], x[e], ss);
            const float rs = rsqrtf(group_sum<LPR>(ss) / a.D + a.eps);
            const int64_t go = (r0 + rr) * a.D + f0;
            if constexpr (!BWD) {
                float y[PER];
#pragma unroll
                for (int e = 0; e < PER; ++e) y[e] = x[e] * rs * w[e] * g[e] * sigm(g[e]);
                if (valid) stv<TA, PER>(a.y, go, y);
            } else {
                float dy[PER], dn[PER], dg[PER], dx[PER], c = 0.f;
                ldv<TA, PER>(st + 2 * TILE, (int64_t)rs_ * a.D + f0, dy);
#pragma unroll
                for (int e = 0; e < PER; ++e) {
                    const float sg = sigm(g[e]), sv = g[e] * sg, n = x[e] * rs;
                    dg[e] = dy[e] * n * w[e] * sg * (1.f + g[e] * (1.f - sg));
                    dn[e] = dy[e] * sv * w[e];
                    if (valid) dwp[e] = fmaf(dy[e] * sv, n, dwp[e]);
                    c = fmaf(dn[e], n, c);
                }
                c = group_sum<LPR>(c) / a.D;
#pragma unroll
                for (int e = 0; e < PER; ++e) dx[e] = rs * (dn[e] - x[e] * rs * c);
                if (valid) {
                    stv<TA, PER>(a.dg, go, dg);
                    stv<TA, PER>(a.dx, go, dx);
                }
            }
        }
        __syncthreads();  // every read of stage s is done: refill it
        if (tid == 0 && tile + (int64_t)STAGES * gridDim.x < tiles) issue(tile + (int64_t)STAGES * gridDim.x, s);
    }
    if constexpr (BWD) {
#pragma unroll
        for (int e = 0; e < PER; ++e) {  // lanes with equal lane % LPR hold the same features
#pragma unroll
            for (int o = LPR; o < 32; o <<= 1) dwp[e] += __shfl_xor_sync(0xffffffffu, dwp[e], o);
        }
        if (lane < LPR) {
#pragma unroll
            for (int e = 0; e < PER; ++e) atomicAdd(&s_dw[f0 + e], dwp[e]);
        }
        __syncthreads();
        for (int i = tid; i < a.D; i += NTHR) atomicAdd(&a.dw[i], s_dw[i]);
    }
}

// LPR = min(32, D / VEC) lanes per row, PER = D / LPR features per lane (D a power of two in [32, 1024])
template <typename TA, bool BWD>
static int ng_launch(const NormGateArgs& a, cudaStream_t s) {
    using namespace ngs;
    constexpr int VEC = 16 / (int)sizeof(TA);
    const int lpr = a.D / VEC < 32 ? a.D / VEC : 32;
    const size_t smem = (size_t)STAGES * (BWD ? 3 : 2) * TILE + bulk::kBarBytes + (BWD ? a.D * sizeof(float) : 0);
    const int64_t tr = TILE / (a.D * sizeof(TA));
    const int64_t tiles = (a.rows + tr - 1) / tr;
#define NG_CASE(LPR_, PER_)                                                                               \
    if (lpr == LPR_ && a.D / lpr == PER_) {                                                              \
        const void* k_ = (const void*)norm_gate_kernel<TA, PER_, LPR_, BWD>;                             \
        int per_sm = 0;                                                                                  \
        if (bulk::allow_smem(k_, smem) != cudaSuccess ||                                                 \
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, norm_gate_kernel<TA, PER_, LPR_, BWD>, \
                                                          NTHR, smem) != cudaSuccess || per_sm < 1)       \
            return GDN_ERR_LAUNCH;                                                                       \
        const int64_t cap = (int64_t)bulk::sm_count() * per_sm;                                          \
        const unsigned grid_ = (unsigned)(tiles < cap ? tiles : cap);                                    \
        norm_gate_kernel<TA, PER_, LPR_, BWD><<<grid_, NTHR, smem, s>>>(a);                              \
        return GDN_OK;                                                                                   \
    }
    if constexpr (VEC == 8) {
        NG_CASE(4, 8) NG_CASE(8, 8) NG_CASE(16, 8) NG_CASE(32, 8) NG_CASE(32, 16) NG_CASE(32, 32)
    } else {
        NG_CASE(8, 4) NG_CASE(16, 4) NG_CASE(32, 4) NG_CASE(32, 8) NG_CASE(32, 16) NG_CASE(32, 32)
    }
#undef NG_CASE
    return GDN_ERR_SHAPE;
}

int read_clear_norm_gate_error(cudaStream_t s, int* out) {
    static const int zero = 0;
    if (cudaMemcpyFromSymbolAsync(out, g_norm_gate_err, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_norm_gate_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    return GDN_OK;
}

}  // namespace gdn

using namespace gdn;

static bool ng_dtype_ok(int32_t d) { return d == GDN_BF16 || d == GDN_FP16 || d == GDN_FP32; }

extern "C" int gdn_rms_norm_gated_fwd(int64_t rows, int64_t D, const void* x, const void* gate, int32_t act_dtype,
                                      const void* weight, int32_t w_dtype, float eps, void* y, gdn_stream_t stream) {
    if (rows < 0 || D <= 0 || D > 1024 || D % 32) return GDN_ERR_SHAPE;
    if (!ng_dtype_ok(act_dtype) || !ng_dtype_ok(w_dtype)) return GDN_ERR_DTYPE;
    if (!x || !gate || !weight || !y) return GDN_ERR_ARGUMENT;
    if (((uintptr_t)x | (uintptr_t)gate | (uintptr_t)y) % 16) return GDN_ERR_ALIGN;
    if (rows == 0) return GDN_OK;
    NormGateArgs a{};
    a.x = x; a.g = gate; a.w = weight; a.y = y;
    a.rows = rows; a.D = (int)D; a.act_dtype = act_dtype; a.w_dtype = w_dtype; a.eps = eps;
    int st = GDN_ERR_DTYPE;
    GDN_DISPATCH_DTYPE(act_dtype, TA, st = (ng_launch<TA, false>(a, (cudaStream_t)stream)))
    if (st != GDN_OK) return st;
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_rms_norm_gated_bwd(int64_t rows, int64_t D, const void* x, const void* gate, int32_t act_dtype,
                                      const void* weight, int32_t w_dtype, float eps, const void* dy, void* dx,
                                      void* dgate, float* dweight, gdn_stream_t stream) {
    if (rows < 0 || D <= 0 || D > 1024 || D % 32) return GDN_ERR_SHAPE;
    if (!ng_dtype_ok(act_dtype) || !ng_dtype_ok(w_dtype)) return GDN_ERR_DTYPE;
    if (!x || !gate || !weight || !dy || !dx || !dgate || !dweight) return GDN_ERR_ARGUMENT;
    if (((uintptr_t)x | (uintptr_t)gate | (uintptr_t)dy | (uintptr_t)dx | (uintptr_t)dgate) % 16) return GDN_ERR_ALIGN;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(dweight, 0, D * sizeof(float), s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (rows == 0) return GDN_OK;
    NormGateArgs a{};
    a.x = x; a.g = gate; a.w = weight; a.dy = dy; a.dx = dx; a.dg = dgate; a.dw = dweight;
    a.rows = rows; a.D = (int)D; a.act_dtype = act_dtype; a.w_dtype = w_dtype; a.eps = eps;
    int st = GDN_ERR_DTYPE;
    GDN_DISPATCH_DTYPE(act_dtype, TA, st = (ng_launch<TA, true>(a, s)))
    if (st != GDN_OK) return st;
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}
