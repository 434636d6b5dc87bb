// Short causal depthwise convolution with SiLU, the q/k/v prologue of the GDN layer
// (sore/model/conv.py:6-23 causal_conv1d_varlen, or FLA's causal_conv1d at sore/model/gdn.py:199-207):
//   z[t, c] = sum_{j < K} w[c, K-1-j] x[t-j, c]   over taps t-j inside t's document,   y = silu(z)
// Documents: rows of a [B, T, C] batch, or the cu_seqlens spans of a packed B == 1 batch (a tap before
// the document start contributes nothing, as the reference's masked_fill does).
// Backward, with dz = dy silu'(z) recomputed from x:
//   dx[t, c] = sum_{j < K} w[c, K-1-j] dz[t+j, c]   over t+j inside t's document,
//   dw[c, K-1-j] = sum_t x[t-j, c] dz[t, c]          (fp32 per thread over its range, one atomic add per block).
// HBM-bound streaming: rows are bulk-copied into a shared-memory ring and each thread slides a window over
// the taps for its 16-byte channel group (conv_kernel below); fp32 accumulation, weights and weight
// gradients in registers.
#include <type_traits>

#include "bulk.cuh"
#include "common.cuh"
#include "kernels.h"

namespace gdn {

// Device error word of this file's kernels (a stage wait that gave up); read and cleared by
// read_clear_conv_error().
static __device__ int g_conv_err;

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
// The sigmoid for activations of type TA. 16-bit activations: sigmoid(x) = (1 + tanh(x / 2)) / 2 with the
// hardware tanh approximation (tanh.approx.f32, one MUFU operation, relative error ~2^-11, below the 16-bit
// rounding of y and dx), half the MUFU work of 1 / (1 + exp(-x)); fp32 activations keep the latter.
template <typename TA>
__device__ __forceinline__ float sig(float x) {
    if constexpr (std::is_same<TA, float>::value) {
        return __fdividef(1.f, 1.f + __expf(-x));
    } else {
        float t;
        asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * x));
        return fmaf(0.5f, t, 0.5f);
    }
}

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

namespace cvs {
// One 512-thread block per SM with two 96 KB stages, a stage holding TT rows of the slab of every staged
// input (24 rows forward, 12 backward: multiples of the 4-row unroll). At config-1 sizes this measured
// fastest of 2-3 stages of 32-112 KB with 4-, 8- or 16-byte channel groups (fwd 58 -> 51 us, bwd 113 ->
// 107 us against three stages of 32 KB / 64 KB with 16- / 8-byte groups).
constexpr int STAGES = 2;
constexpr uint32_t STAGE_BYTES = 98304;
constexpr uint32_t SLAB_BYTES = 4096;    // bytes of a row one block covers
constexpr int GROUP_BYTES = 8;  // bytes of a row one thread covers
}  // namespace cvs

// Block = (slab of channels, contiguous range [tb, te) of the flattened token axis). The block streams the
// rows u of its range, plus the K-1 rows before it (and, backward, the K-1 after it), through a STAGES-deep
// ring: tile i of TT rows lands in stage i % STAGES by bulk copies (one per input when the slab is the whole
// row, else one per row, issued by warp 0). Each thread owns one 8-byte channel group of the slab and slides
// a window over the rows in order:
//   forward:  x window [u-K+1, u] -> y[u] for u in [tb, te)
//   backward: x window -> z[u], dz[u] for u in [tb, te+K-1); dz window [t, t+K-1] -> dx[t], t = u-K+1 in
//             [tb, te); dw += x[u-j] dz[u] for u in [tb, te), kept in registers and added once per block.
// Window rows from before the current document are zero, and dz rows past the document end of t are masked.
// __maxnreg__(128): 512 threads per block fit the register file; under __launch_bounds__(512) ptxas chose 64
// registers and spills for the K = 3 kernels
template <typename TA, int K, bool BWD>
__global__ void __maxnreg__(128) conv_kernel(const ConvArgs a, int64_t range_len, int nslabs) {
    using namespace cvs;
    constexpr int VEC = GROUP_BYTES / (int)sizeof(TA);  // channels per thread
    constexpr int MAX_GROUPS = SLAB_BYTES / GROUP_BYTES;
    constexpr int NTN = BWD ? 2 : 1;                              // staged inputs: x (and dy)
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bar = (uint64_t*)(smem + STAGES * STAGE_BYTES);
    const int tid = threadIdx.x;
    const int64_t BT = a.B * a.T;
    const int slab = blockIdx.x % nslabs;
    const int64_t c_begin = (int64_t)slab * MAX_GROUPS * VEC;
    const int64_t cs = (a.C - c_begin < MAX_GROUPS * VEC) ? a.C - c_begin : MAX_GROUPS * VEC;  // slab width
    const uint32_t rbs = (uint32_t)(cs * sizeof(TA));                                       // slab row bytes
    const int64_t rstride = a.C * (int64_t)sizeof(TA);                                      // global row bytes
    const uint32_t per_t = STAGE_BYTES / NTN;
    const int TT = (int)(per_t / rbs) < 64 ? (int)(per_t / rbs) : 64;  // rows per tile
    const int64_t tb = (blockIdx.x / nslabs) * range_len;
    const int64_t te = tb + range_len < BT ? tb + range_len : BT;
    if (tb >= te) return;
    const int64_t u_lo = tb - (K - 1) > 0 ? tb - (K - 1) : 0;
    const int64_t u_end = BWD ? te + (K - 1) : te;  // rows the window passes (past BT: zero)
    const int64_t u_hi = u_end < BT ? u_end : BT;   // rows that exist
    const int64_t ntiles = (u_hi - u_lo + TT - 1) / TT;
    const void* src[2] = {a.x, a.dy};

    auto issue = [&](int64_t tile, int s) {  // warp 0: rows [u0, u0 + n) of every staged input into stage s
        const int64_t u0 = u_lo + tile * TT;
        const int n = (int)(u_hi - u0 < TT ? u_hi - u0 : TT);
        if ((tid & 31) == 0) sm100::mbar_arrive_expect_tx(&bar[s], NTN * n * rbs);
        __syncwarp();
#pragma unroll
        for (int t = 0; t < NTN; ++t) {
            uint8_t* dst = smem + s * STAGE_BYTES + t * per_t;
            const uint8_t* g = (const uint8_t*)src[t] + u0 * rstride + c_begin * (int64_t)sizeof(TA);
            if (cs == a.C) {  // whole rows: one contiguous copy
                if ((tid & 31) == 0) bulk::load(dst, g, n * rbs, &bar[s]);
            } else {
                for (int r = tid & 31; r < n; r += 32) bulk::load(dst + r * rbs, g + r * rstride, rbs, &bar[s]);
            }
        }
    };

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) sm100::mbar_init(&bar[s], 1);
        sm100::fence_barrier_init();
    }
    __syncthreads();
    if (tid < 32)
        for (int s = 0; s < STAGES && s < ntiles; ++s) issue(s, s);

    const bool active = (int64_t)tid * VEC < cs;
    const int64_t c0 = c_begin + (int64_t)tid * VEC;
    float w[VEC][K], dw[VEC][K];
#pragma unroll
    for (int q = 0; q < VEC; ++q)
#pragma unroll
        for (int j = 0; j < K; ++j) {
            w[q][j] = active ? ld_w(a.w, a.w_dtype, (c0 + q) * K + j) : 0.f;
            dw[q][j] = 0.f;
        }
    float xw[K][VEC];   // xw[j] = x[u - j] (zero before the document start)
    float dzw[K][VEC];  // dzw[j] = dz[u - K + 1 + j] (backward)
    int64_t ew[K];      // document end of the token of dzw[j]
#pragma unroll
    for (int j = 0; j < K; ++j) {
        ew[j] = 0;
#pragma unroll
        for (int q = 0; q < VEC; ++q) xw[j][q] = dzw[j][q] = 0.f;
    }
    int64_t s_doc, e_doc;
    doc_span(a, u_lo, s_doc, e_doc);

    bool ok = true;  // false once a stage wait timed out: from then on this thread stores nothing
    // one row u of the current document through the window; `have`: the row exists (u < BT), else zero.
    // No branches besides the predicated stores, so the unrolled rows of a document segment interleave.
    auto row = [&](int64_t u, const TA* xrow, const TA* dyrow, bool have) {
#pragma unroll
        for (int j = K - 1; j >= 1; --j)
#pragma unroll
            for (int q = 0; q < VEC; ++q) xw[j][q] = xw[j - 1][q];
        if (have) ldv<TA, VEC>(xrow, 0, xw[0]);
        else {
#pragma unroll
            for (int q = 0; q < VEC; ++q) xw[0][q] = 0.f;
        }
        // 16-bit activations: the K-tap sums run on channel pairs as packed fp32 FMAs (__ffma2_rn, fmaf's
        // rounding in each lane), half the FMA instructions of these issue-bound rows. fp32 activations keep
        // scalar FMAs, as ptxas spills their paired form.
        constexpr bool PAIRS = sizeof(TA) == 2;
        if constexpr (!BWD) {
            float y[VEC];
            if constexpr (PAIRS) {
#pragma unroll
                for (int q = 0; q < VEC; q += 2) {
                    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < K; ++j) {
                        const float2 wj = make_float2(w[q][K - 1 - j], w[q + 1][K - 1 - j]);
                        acc = __ffma2_rn(wj, make_float2(xw[j][q], xw[j][q + 1]), acc);
                    }
                    y[q] = a.silu ? acc.x * sig<TA>(acc.x) : acc.x;
                    y[q + 1] = a.silu ? acc.y * sig<TA>(acc.y) : acc.y;
                }
            } else {
#pragma unroll
                for (int q = 0; q < VEC; ++q) {
                    float acc = 0.f;
#pragma unroll
                    for (int j = 0; j < K; ++j) acc = fmaf(w[q][K - 1 - j], xw[j][q], acc);
                    y[q] = a.silu ? acc * sig<TA>(acc) : acc;
                }
            }
            if (active && ok && u >= tb) stv<TA, VEC>(a.y, u * a.C + c0, y);
        } else {
            float dyv[VEC];
            if (have) ldv<TA, VEC>(dyrow, 0, dyv);
            else {
#pragma unroll
                for (int q = 0; q < VEC; ++q) dyv[q] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < K - 1; ++j) {
                ew[j] = ew[j + 1];
#pragma unroll
                for (int q = 0; q < VEC; ++q) dzw[j][q] = dzw[j + 1][q];
            }
            const bool acc_dw = u < te && ok;  // rows past the range feed dx only
            if constexpr (PAIRS) {
#pragma unroll
                for (int q = 0; q < VEC; q += 2) {
                    float2 z = make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < K; ++j) {
                        const float2 wj = make_float2(w[q][K - 1 - j], w[q + 1][K - 1 - j]);
                        z = __ffma2_rn(wj, make_float2(xw[j][q], xw[j][q + 1]), z);
                    }
                    float d0 = dyv[q], d1 = dyv[q + 1];
                    if (a.silu) {
                        const float s0 = sig<TA>(z.x), s1 = sig<TA>(z.y);
                        d0 *= s0 * (1.f + z.x * (1.f - s0));
                        d1 *= s1 * (1.f + z.y * (1.f - s1));
                    }
                    const float2 dd = acc_dw ? make_float2(d0, d1) : make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < K; ++j) {
                        const float2 dwj = make_float2(dw[q][K - 1 - j], dw[q + 1][K - 1 - j]);
                        const float2 r = __ffma2_rn(make_float2(xw[j][q], xw[j][q + 1]), dd, dwj);
                        dw[q][K - 1 - j] = r.x;
                        dw[q + 1][K - 1 - j] = r.y;
                    }
                    dzw[K - 1][q] = d0;
                    dzw[K - 1][q + 1] = d1;
                }
            } else {
#pragma unroll
                for (int q = 0; q < VEC; ++q) {
                    float z = 0.f;
#pragma unroll
                    for (int j = 0; j < K; ++j) z = fmaf(w[q][K - 1 - j], xw[j][q], z);
                    float d = dyv[q];
                    if (a.silu) {
                        const float sg = sig<TA>(z);
                        d *= sg * (1.f + z * (1.f - sg));
                    }
                    const float dd = acc_dw ? d : 0.f;
#pragma unroll
                    for (int j = 0; j < K; ++j) dw[q][K - 1 - j] = fmaf(xw[j][q], dd, dw[q][K - 1 - j]);
                    dzw[K - 1][q] = d;
                }
            }
            ew[K - 1] = have ? e_doc : 0;
            const int64_t t = u - (K - 1);  // < te, as u < te + K - 1
            float dx[VEC];
            if constexpr (PAIRS) {
#pragma unroll
                for (int q = 0; q < VEC; q += 2) {
                    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < K; ++j) {
                        const bool in = t + j < ew[0];
                        const float2 wj = in ? make_float2(w[q][K - 1 - j], w[q + 1][K - 1 - j]) : make_float2(0.f, 0.f);
                        acc = __ffma2_rn(wj, make_float2(dzw[j][q], dzw[j][q + 1]), acc);
                    }
                    dx[q] = acc.x;
                    dx[q + 1] = acc.y;
                }
            } else {
#pragma unroll
                for (int q = 0; q < VEC; ++q) {
                    float acc = 0.f;
#pragma unroll
                    for (int j = 0; j < K; ++j) acc = fmaf(t + j < ew[0] ? w[q][K - 1 - j] : 0.f, dzw[j][q], acc);
                    dx[q] = acc;
                }
            }
            if (active && ok && t >= tb) stv<TA, VEC>(a.dx, t * a.C + c0, dx);
        }
    };

    for (int64_t tile = 0; tile < ntiles; ++tile) {
        const int s = (int)(tile % STAGES);
        ok = sm100::mbar_wait(&bar[s], (uint32_t)(tile / STAGES) & 1u, &g_conv_err, GDN_DEV_ERR_CONV,
                              ok ? (1u << 22) : 1u) && ok;
        const int64_t u0 = u_lo + tile * TT;
        const int n = (int)(u_hi - u0 < TT ? u_hi - u0 : TT);
        // inactive threads (past a narrow slab's last group) read the group-0 column and store nothing
        const uint8_t* st = smem + s * STAGE_BYTES + (active ? (uint32_t)tid * GROUP_BYTES : 0u);
        int r = 0;
        while (r < n) {
            if (u0 + r >= e_doc) {  // a new document starts here: no taps before it
                doc_span(a, u0 + r, s_doc, e_doc);
#pragma unroll
                for (int j = 0; j < K; ++j)
#pragma unroll
                    for (int q = 0; q < VEC; ++q) xw[j][q] = 0.f;
            }
            const int r_end = (int)(e_doc - u0 < n ? e_doc - u0 : n);  // rows of this document in the tile
            if constexpr (BWD) {
                for (; r < r_end && u0 + r < tb; ++r) {  // rows before the range only fill the x window
#pragma unroll
                    for (int j = K - 1; j >= 1; --j)
#pragma unroll
                        for (int q = 0; q < VEC; ++q) xw[j][q] = xw[j - 1][q];
                    ldv<TA, VEC>((const TA*)(st + r * rbs), 0, xw[0]);
                }
            }
#pragma unroll 4
            for (; r < r_end; ++r) row(u0 + r, (const TA*)(st + r * rbs), (const TA*)(st + per_t + r * rbs), true);
        }
        __syncthreads();  // every read of stage s is done: refill it
        if (tid < 32 && tile + STAGES < ntiles) issue(tile + STAGES, s);
    }
    for (int64_t u = u_hi; u < u_end; ++u) row(u, nullptr, nullptr, false);  // backward: rows past BT
    if constexpr (BWD) {
        if (active) {
#pragma unroll
            for (int q = 0; q < VEC; ++q) {
                if constexpr (K == 4) {
                    atomicAdd(reinterpret_cast<float4*>(a.dw + (c0 + q) * K),
                              make_float4(dw[q][0], dw[q][1], dw[q][2], dw[q][3]));
                } else {
#pragma unroll
                    for (int j = 0; j < K; ++j) atomicAdd(&a.dw[(c0 + q) * K + j], dw[q][j]);
                }
            }
        }
    }
}

template <typename TA>
static int conv_launch(const ConvArgs& a, int K, bool bwd, cudaStream_t s) {
    using namespace cvs;
    const int VEC = GROUP_BYTES / (int)sizeof(TA);
    const int MAX_GROUPS = (int)SLAB_BYTES / GROUP_BYTES;
    const int64_t BT = a.B * a.T;
    const int nslabs = (int)((a.C + MAX_GROUPS * VEC - 1) / (MAX_GROUPS * VEC));
    const int64_t g0 = (a.C < MAX_GROUPS * VEC ? a.C : MAX_GROUPS * VEC) / VEC;  // groups of the widest slab
    const int nthr = (int)((g0 + 31) / 32 * 32);
    const size_t smem = (size_t)STAGES * STAGE_BYTES + bulk::kBarBytes;
    const void* k = nullptr;
    switch (K * 2 + (bwd ? 1 : 0)) {
        case 2: k = (const void*)conv_kernel<TA, 1, false>; break;
        case 3: k = (const void*)conv_kernel<TA, 1, true>; break;
        case 4: k = (const void*)conv_kernel<TA, 2, false>; break;
        case 5: k = (const void*)conv_kernel<TA, 2, true>; break;
        case 6: k = (const void*)conv_kernel<TA, 3, false>; break;
        case 7: k = (const void*)conv_kernel<TA, 3, true>; break;
        case 8: k = (const void*)conv_kernel<TA, 4, false>; break;
        case 9: k = (const void*)conv_kernel<TA, 4, true>; break;
        default: return GDN_ERR_SHAPE;
    }
    int per_sm = 0;
    if (bulk::allow_smem(k, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, nthr, smem) != cudaSuccess || per_sm < 1)
        return GDN_ERR_LAUNCH;
    // ranges per slab: fill every SM's resident blocks, no range shorter than 16 tokens
    int64_t nranges = ((int64_t)bulk::sm_count() * per_sm + nslabs - 1) / nslabs;
    if (nranges > (BT + 15) / 16) nranges = (BT + 15) / 16;
    if (nranges < 1) nranges = 1;
    const int64_t range_len = (BT + nranges - 1) / nranges;
    nranges = (BT + range_len - 1) / range_len;
    void* args[] = {(void*)&a, (void*)&range_len, (void*)&nslabs};
    if (cudaLaunchKernel(k, dim3((unsigned)(nranges * nslabs)), dim3(nthr), args, smem, s) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    count_launch();
    return GDN_OK;
}

int read_clear_conv_error(cudaStream_t s, int* out) {
    static const int zero = 0;
    if (cudaMemcpyFromSymbolAsync(out, g_conv_err, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_conv_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    return GDN_OK;
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
    if (((uintptr_t)x | (uintptr_t)dy | (uintptr_t)dx | (uintptr_t)dweight) % 16) return GDN_ERR_ALIGN;
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(dweight, 0, C * K * sizeof(float), s) != cudaSuccess) return GDN_ERR_LAUNCH;
    if (B * T == 0) return GDN_OK;
    ConvArgs a{};
    a.x = x; a.w = weight; a.dy = dy; a.dx = dx; a.dw = dweight; a.cu = cu_seqlens; a.B = B; a.T = T; a.C = C;
    a.N = N; a.w_dtype = w_dtype; a.silu = silu;
    GDN_DISPATCH_DTYPE(act_dtype, TA, return conv_launch<TA>(a, (int)K, true, s);)
    return GDN_ERR_DTYPE;
}
