// Single-token decode step for DK = DV = 128 on sm_100a: a persistent, bulk-copy (TMA) pipelined stream
// over the fp32 states.
//
// The step (soreRNN sore/model/gdn_ref.py:17-22 for one token) is, per (sequence, value head) with
// gamma = exp(g), qn = q/|q|, kn = k/|k| (when the L2 norm is on):
//   S' = gamma S;  delta = beta (v - S'^T kn);  S_new = S' + kn delta^T;  o = scale S_new^T qn
// and o is formed from the same pass over S' as o = scale (S'^T qn + delta (qn . kn)). Every value column
// is independent, and the whole step reads and writes each state once: 2 x 64 KiB of HBM traffic per
// head against ~1 KiB of activations, so the kernel is a copy-speed stream.
//
// One CTA per SM walks heads h = blockIdx.x, + gridDim.x, ... through three 64 KiB shared-memory stages:
// while head h is updated in shared memory, head h+1's state is arriving (bulk copy, mbarrier) and head
// h-1's new state is leaving (bulk store, bulk-group). 256 threads: thread (rg = warp, c = lane) holds
// the float4 of columns 4c..4c+3 for rows rg + 8 r (r < 16); a warp's row access is one contiguous
// 512-byte shared-memory line; the column sums over rows go through shared memory across the 8 warps.
#include "common.cuh"
#include "kernels.h"
#include "launch.h"
#include "sm100.cuh"

namespace gdn {
using namespace sm100;

// Device error word of the decode kernel (a stage wait that gave up); read and cleared by
// read_clear_decode_error().
static __device__ int g_decode_err;

namespace dec {
constexpr int NTHR = 256;
constexpr int STAGES = 3;
constexpr uint32_t STATE_BYTES = 128 * 128 * 4;
constexpr uint32_t ACT_BYTES = 512;  // q, k, v rows: 128 elements of up to 4 bytes each
constexpr uint32_t STAGE_BYTES = STATE_BYTES + 3 * ACT_BYTES;
constexpr uint32_t OFF_RED = STAGES * STAGE_BYTES;  // [2][8][128] fp32 partial column sums
constexpr uint32_t OFF_BAR = OFF_RED + 2 * 8 * 128 * 4;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 64 + 128;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
}  // namespace dec

struct DecodeArgs {
    const void *q, *k, *v, *g, *beta;
    void* o;
    float* state;
    int64_t heads;  // N * HV
    int H, HV, g_dtype, beta_dtype, l2norm;
    float scale;
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"((uint64_t)dst),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most one bulk group (the newest) still reading shared memory
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <typename TA>
__global__ void __launch_bounds__(dec::NTHR, 1) decode_tma_kernel(const __grid_constant__ DecodeArgs a) {
    using namespace dec;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    float* red = (float*)(sm + OFF_RED);
    uint64_t* bar = (uint64_t*)(sm + OFF_BAR);
    const int tid = threadIdx.x, rg = tid >> 5, c = tid & 31;
    constexpr uint32_t ROW = 128 * sizeof(TA);

    auto issue = [&](int64_t h, int s) {  // thread 0: state + q, k, v of head h into stage s
        const int64_t n = h / a.HV;
        const int hv = (int)(h % a.HV), hq = hv / (a.HV / a.H);
        uint8_t* st = sm + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&bar[s], STATE_BYTES + 3 * ROW);
        bulk_g2s(st, a.state + h * 16384, STATE_BYTES, &bar[s]);
        bulk_g2s(st + STATE_BYTES, (const uint8_t*)a.q + (n * a.H + hq) * ROW, ROW, &bar[s]);
        bulk_g2s(st + STATE_BYTES + ACT_BYTES, (const uint8_t*)a.k + (n * a.H + hq) * ROW, ROW, &bar[s]);
        bulk_g2s(st + STATE_BYTES + 2 * ACT_BYTES, (const uint8_t*)a.v + h * ROW, ROW, &bar[s]);
    };

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int64_t h0 = blockIdx.x, stride = gridDim.x;
    if (tid == 0) {
        if (h0 < a.heads) issue(h0, 0);
        if (h0 + stride < a.heads) issue(h0 + stride, 1);
    }
    // gates of the current head, loaded one head ahead (their latency hides behind a whole head)
    uint32_t g_nx = 0u, b_nx = 0u;  // kept as loaded bits (no stall at the load); converted at use
    if (h0 < a.heads) {
        g_nx = ld_gate_raw(a.g, a.g_dtype, h0);
        b_nx = ld_gate_raw(a.beta, a.beta_dtype, h0);
    }
    bool ok = true;
    int it = 0;
    for (int64_t h = h0; h < a.heads; h += stride, ++it) {
        const int s = it % STAGES;
        const float gam = __expf(gate_f(g_nx, a.g_dtype)), bt = gate_f(b_nx, a.beta_dtype);
        if (h + stride < a.heads) {
            g_nx = ld_gate_raw(a.g, a.g_dtype, h + stride);
            b_nx = ld_gate_raw(a.beta, a.beta_dtype, h + stride);
        }
        ok = mbar_wait(&bar[s], (uint32_t)(it / STAGES) & 1u, &g_decode_err, GDN_DEV_ERR_DECODE,
                       ok ? (1u << 22) : 1u) && ok;
        float* S = (float*)(sm + s * STAGE_BYTES);
        const TA* qs = (const TA*)(sm + s * STAGE_BYTES + STATE_BYTES);
        const TA* ks = (const TA*)(sm + s * STAGE_BYTES + STATE_BYTES + ACT_BYTES);
        const TA* vs = (const TA*)(sm + s * STAGE_BYTES + STATE_BYTES + 2 * ACT_BYTES);

        // norms and q.k: every warp reduces the 128-element rows itself (no extra barrier)
        float nq = 0.f, nk = 0.f, qk = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float x = ld(qs, c + 32 * e), y = ld(ks, c + 32 * e);
            nq = fmaf(x, x, nq);
            nk = fmaf(y, y, nk);
            qk = fmaf(x, y, qk);
        }
        nq = warp_sum(nq);
        nk = warp_sum(nk);
        qk = warp_sum(qk);
        float iq = 1.f, ik = 1.f;
        if (a.l2norm) {
            iq = 1.f / fmaxf(sqrtf(nq), kL2Eps);
            ik = 1.f / fmaxf(sqrtf(nk), kL2Eps);
        }

        // pass over S: S' = gamma S (kept in registers), partial S'^T kn and S'^T qn over this thread's rows
        float4 sv[16];
        float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int i = rg + 8 * r;
            float4 x = *reinterpret_cast<const float4*>(S + i * 128 + 4 * c);
            x.x *= gam; x.y *= gam; x.z *= gam; x.w *= gam;
            sv[r] = x;
            const float ki = ld(ks, i) * ik, qi = ld(qs, i) * iq;
            pk.x = fmaf(x.x, ki, pk.x); pk.y = fmaf(x.y, ki, pk.y); pk.z = fmaf(x.z, ki, pk.z); pk.w = fmaf(x.w, ki, pk.w);
            pq.x = fmaf(x.x, qi, pq.x); pq.y = fmaf(x.y, qi, pq.y); pq.z = fmaf(x.z, qi, pq.z); pq.w = fmaf(x.w, qi, pq.w);
        }
        *reinterpret_cast<float4*>(red + rg * 128 + 4 * c) = pk;
        *reinterpret_cast<float4*>(red + 1024 + rg * 128 + 4 * c) = pq;
        // every thread learns whether all waits so far succeeded: after a timeout the stage holds no valid
        // state, so neither o nor the state is written from then on (the resident state keeps its old value)
        ok = __syncthreads_and(ok) != 0;
        float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sq = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const float4 x = *reinterpret_cast<const float4*>(red + w * 128 + 4 * c);
            const float4 y = *reinterpret_cast<const float4*>(red + 1024 + w * 128 + 4 * c);
            sk.x += x.x; sk.y += x.y; sk.z += x.z; sk.w += x.w;
            sq.x += y.x; sq.y += y.y; sq.z += y.z; sq.w += y.w;
        }
        float dl[4];
        dl[0] = bt * (ld(vs, 4 * c + 0) - sk.x);
        dl[1] = bt * (ld(vs, 4 * c + 1) - sk.y);
        dl[2] = bt * (ld(vs, 4 * c + 2) - sk.z);
        dl[3] = bt * (ld(vs, 4 * c + 3) - sk.w);
        if (rg == 0 && ok) {  // o = scale (S'^T qn + delta (qn . kn))
            const float kq = qk * iq * ik;
            TA* o = (TA*)a.o + h * 128 + 4 * c;
            st(o, 0, a.scale * fmaf(dl[0], kq, sq.x));
            st(o, 1, a.scale * fmaf(dl[1], kq, sq.y));
            st(o, 2, a.scale * fmaf(dl[2], kq, sq.z));
            st(o, 3, a.scale * fmaf(dl[3], kq, sq.w));
        }
        // S_new = S' + kn delta^T, back into the stage for the bulk store
        if (ok) {
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const int i = rg + 8 * r;
                const float ki = ld(ks, i) * ik;
                float4 x = sv[r];
                x.x = fmaf(ki, dl[0], x.x); x.y = fmaf(ki, dl[1], x.y); x.z = fmaf(ki, dl[2], x.z); x.w = fmaf(ki, dl[3], x.w);
                *reinterpret_cast<float4*>(S + i * 128 + 4 * c) = x;
            }
        }
        fence_async_smem();
        __syncthreads();  // also: every read of red is done before the next head writes it
        if (tid == 0) {
            if (ok) bulk_s2g(a.state + h * 16384, S, STATE_BYTES);
            bulk_commit();  // an empty group after a timeout keeps the group count of the refill schedule
            if (h + 2 * stride < a.heads) {
                bulk_wait_read_1();  // stage (it + 2) % 3 held head h - stride, whose store has now read it
                issue(h + 2 * stride, (it + 2) % STAGES);
            }
        }
    }
    if (tid == 0) bulk_wait_all();
}

bool decode_tma_supported(int64_t DK, int64_t DV, const void* q, const void* k, const void* v, const float* state) {
    return DK == 128 && DV == 128 && ((uintptr_t)q % 16) == 0 && ((uintptr_t)k % 16) == 0 &&
           ((uintptr_t)v % 16) == 0 && ((uintptr_t)state % 16) == 0;
}

int decode_tma(const void* q, const void* k, const void* v, const void* g, const void* beta, float* state, void* o,
               int64_t N, int64_t H, int64_t HV, float scale, int act_dtype, int g_dtype, int beta_dtype, int l2norm,
               cudaStream_t s) {
    using namespace dec;
    DecodeArgs a{};
    a.q = q; a.k = k; a.v = v; a.g = g; a.beta = beta; a.o = o; a.state = state;
    a.heads = N * HV;
    a.H = (int)H; a.HV = (int)HV; a.g_dtype = g_dtype; a.beta_dtype = beta_dtype; a.l2norm = l2norm;
    a.scale = scale;
    if (a.heads == 0) return GDN_OK;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    const unsigned grid = (unsigned)(a.heads < sms ? a.heads : sms);
    GDN_DISPATCH_DTYPE(act_dtype, TA,
        if (smem_optin((const void*)decode_tma_kernel<TA>, SMEM_BYTES) != cudaSuccess) return GDN_ERR_LAUNCH;
        decode_tma_kernel<TA><<<grid, NTHR, SMEM_BYTES, s>>>(a);)
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int read_clear_decode_error(cudaStream_t s, int* out) {
    static const int zero = 0;
    if (cudaMemcpyFromSymbolAsync(out, g_decode_err, sizeof(int), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemcpyToSymbolAsync(g_decode_err, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s) != cudaSuccess)
        return GDN_ERR_LAUNCH;
    return GDN_OK;
}

}  // namespace gdn
