// Chunked gated-delta-rule forward on sm_100a: tcgen05 (UMMA) tile contractions, TMA-fed shared memory,
// fp32 state resident in tensor memory (TMEM) for the whole sequence.
//
// One CTA (256 threads) per (sequence, value head) walks the sequence in chunks of C = 64 tokens.
// With Gamma = in-chunk inclusive cumsum of g, E_ij = exp(Gamma_i - Gamma_j), and S0 the state at the
// chunk start (the algebra checked against the per-token recurrence in tests/test_chunk_algebra.py):
//   A   = strict_lower(diag(beta) K K^T . E)             T = (I + A)^-1   (fp32, blocked 16x16 solve)
//   W   = T diag(beta e^Gamma) K        U = T diag(beta) V        Delta = U - W S0
//   O   = scale e^Gamma Q S0 + P Delta,  P = scale lower_incl(Q K^T . E)
//   S1  = e^Gamma_C S0 + (diag(e^(Gamma_C - Gamma)) K)^T Delta
// Every GEMM is issued as an M = 128 UMMA with the feature dimension (d = 128) on the TMEM lanes:
//   MMA1  D1[128x64]  = [Q;K] K^T              (rows 0-63: Q K^T, rows 64-127: K K^T)
//   MMA2  W^T[dk x i] = K^T (T diag(beta e^G))^T            MMA3  U^T[dv x i] = V^T (T diag(beta))^T
//   MMA4  U^T        += S0^T (-W)^T   -> Delta^T          MMA5  O^T = S0^T (scale e^G Q)^T
//   MMA6  O^T        += Delta^T P^T                       MMA7  S^T += (Delta^T diag(e^(G_C-G))) K
// S^T (fp32, 128 TMEM columns) is never written to HBM except as checkpoints for the backward
// (every ckpt_every chunks) and the final state.
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.h"

namespace gdn {
using namespace sm100;

namespace cf {
constexpr int NTHR = 256;
// shared memory carve (bytes from a 1024-aligned base)
constexpr uint32_t OFF_QK = 0;                 // 2 stages x 32 KB: per d-block kb: [Q 8 KB | K 8 KB]
constexpr uint32_t OFF_V = 65536;              // 2 stages x 16 KB: [kb][V 8 KB]
constexpr uint32_t OFF_S = 98304;              // S0^T bf16 [dv][dk] K-major, 2 dk-blocks x 16 KB
constexpr uint32_t OFF_W = 131072;             // -W bf16 [i][d] K-major, 2 d-blocks x 8 KB
constexpr uint32_t OFF_D = 147456;             // Delta^T bf16 [dv][j], 16 KB
constexpr uint32_t OFF_DD = 163840;            // Delta^T diag(exp(G_C - G_j)), 16 KB
constexpr uint32_t OFF_TB = 180224;            // T diag(beta e^G) bf16 [i][j], 8 KB
constexpr uint32_t OFF_TV = 188416;            // T diag(beta) bf16 [i][j], 8 KB
constexpr uint32_t OFF_P = 196608;             // P bf16 [i][j], 8 KB
constexpr uint32_t OFF_A = 204800;             // A -> T in place, fp32 [64][AST]
constexpr int AST = 68;                        // padded fp32 row stride (conflict-free float4 rows)
constexpr uint32_t OFF_Y = OFF_A + 64 * AST * 4;   // Y blocks, fp32 3 x 16 x 16
constexpr uint32_t OFF_VEC = OFF_Y + 3 * 256 * 4;  // G, e^G, beta, e^(G_C-G), misc: 5 x 64 fp32
constexpr uint32_t OFF_BAR = OFF_VEC + 5 * 64 * 4;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 64 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// TMEM columns
constexpr uint32_t T_D1 = 0, T_W = 64, T_U = 128, T_O = 192, T_S = 256, T_COLS = 512;
constexpr uint32_t TX_QKV = 6 * 8192, TX_QK = 4 * 8192;
}  // namespace cf

struct ChunkFwdArgs {
    CUtensorMap tq, tk, tv;
    const void* g;
    const void* beta;
    void* o;
    const float* h0;
    float* ht;
    float* ckpt;
    const int64_t* cu;
    int* err;
    int64_t T;
    int N, H, HV, g_dtype, beta_dtype;
    float scale;
    int l2norm, zero_v, o_mode, h0_identity, ht_accumulate, ckpt_every;
};

__device__ __forceinline__ float ld_any2(const void* p, int dtype, int64_t i) {
    if (dtype == GDN_FP32) return ((const float*)p)[i];
    if (dtype == GDN_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    return __half2float(((const __half*)p)[i]);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 8 consecutive fp32 -> one 16-byte chunk of bf16 at smem byte address `dst`
__device__ __forceinline__ void st_chunk8(uint8_t* dst, const float* v) {
    uint4 u;
    u.x = pack_bf16(v[0], v[1]);
    u.y = pack_bf16(v[2], v[3]);
    u.z = pack_bf16(v[4], v[5]);
    u.w = pack_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(dst) = u;
}

__device__ __forceinline__ void block_sync_tc() {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

__device__ __forceinline__ bool wait_mma(uint64_t* bar, uint32_t& phase, int* err, int code) {
    const bool ok = mbar_wait(bar, phase, err, code);
    phase ^= 1u;
    tc_fence_after();
    return ok;
}

__global__ void __launch_bounds__(cf::NTHR, 1) chunk_fwd_kernel(const __grid_constant__ ChunkFwdArgs a) {
    using namespace cf;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* Am = (float*)(sm + OFF_A);
    float* Yb = (float*)(sm + OFF_Y);
    float* vG = (float*)(sm + OFF_VEC);
    float* vEG = vG + 64;
    float* vB = vG + 128;
    float* vX = vG + 192;
    float* vMisc = vG + 256;
    uint64_t* bar_tma = (uint64_t*)(sm + OFF_BAR);
    uint64_t* bar_mma = bar_tma + 2;
    uint32_t* tmem_slot = (uint32_t*)(bar_tma + 3);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lg = warp & 3, chh = warp >> 2;  // TMEM lane group, column half
    const int row = 32 * lg + lane;            // accumulator row (TMEM lane) of this thread
    const int n = blockIdx.x / a.HV, hv = blockIdx.x % a.HV, hq = hv / (a.HV / a.H);
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t len = eos - bos;
    const int nchunks = (int)((len + 63) / 64);

    // checkpoint slot of this sequence's first checkpoint
    int64_t ck_base = 0;
    if (a.ckpt) {
        const int K = a.ckpt_every;
        if (!a.cu) {
            ck_base = (int64_t)n * (((a.T + 63) / 64 + K - 1) / K);
        } else {
            int64_t part = 0;
            for (int m = tid; m < n; m += NTHR) {
                const int64_t lm = a.cu[m + 1] - a.cu[m];
                part += (((lm + 63) / 64) + K - 1) / K;
            }
            for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (lane == 0) ((int64_t*)Yb)[warp] = part;
            __syncthreads();
            for (int w = 0; w < NTHR / 32; ++w) ck_base += ((int64_t*)Yb)[w];
            __syncthreads();
        }
    }

    if (tid == 0) {
        mbar_init(&bar_tma[0], 1);
        mbar_init(&bar_tma[1], 1);
        mbar_init(bar_mma, 1);
        fence_barrier_init();
        prefetch_tmap(&a.tq);
        prefetch_tmap(&a.tk);
        if (!a.zero_v) prefetch_tmap(&a.tv);
    }
    if (warp == 0) tmem_alloc(tmem_slot, T_COLS);
    if (a.zero_v) {
        for (int e = tid; e < 2 * 16384 / 16; e += NTHR) ((uint4*)(sm + OFF_V))[e] = make_uint4(0, 0, 0, 0);
    }
    block_sync_tc();
    const uint32_t tm = *tmem_slot;
    const uint32_t tD1 = tm + T_D1, tW = tm + T_W, tU = tm + T_U, tO = tm + T_O, tS = tm + T_S;
    const uint32_t lane_base = (uint32_t)(32 * lg) << 16;
    uint32_t mma_phase = 0;
    bool ok = true;

    // initial state -> TMEM: thread (row = dv, half chh) holds S^T[dv][dk] for dk in [64 chh, 64 chh + 64)
    {
        const float* h0 = a.h0 ? a.h0 + ((int64_t)n * a.HV + hv) * 16384 : nullptr;
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int dk = 64 * chh + c0 + i;
                v[i] = a.h0_identity ? (dk == row ? 1.f : 0.f) : (h0 ? h0[dk * 128 + row] : 0.f);
            }
            tmem_st16(tS + lane_base + 64 * chh + c0, v);
        }
        tmem_wait_st();
    }

    auto issue_tma = [&](int c, int s) {
        const int tok0 = (int)(bos + 64 * c);
        uint8_t* sQK = sm + OFF_QK + s * 32768;
        uint8_t* sV = sm + OFF_V + s * 16384;
        mbar_arrive_expect_tx(&bar_tma[s], a.zero_v ? TX_QK : TX_QKV);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
            tma_load_3d(sQK + kb * 16384, &a.tq, &bar_tma[s], kb * 64, hq, tok0);
            tma_load_3d(sQK + kb * 16384 + 8192, &a.tk, &bar_tma[s], kb * 64, hq, tok0);
            if (!a.zero_v) tma_load_3d(sV + kb * 8192, &a.tv, &bar_tma[s], kb * 64, hv, tok0);
        }
    };
    if (tid == 0 && nchunks > 0) issue_tma(0, 0);
    int tma_pending = nchunks > 0 ? 1 : 0;

    const uint32_t sbase = smem_u32(sm);
    for (int c = 0; c < nchunks && ok; ++c) {
        const int s = c & 1;
        const int64_t tok0 = bos + 64 * (int64_t)c;
        const int nv = (len - 64 * (int64_t)c) < 64 ? (int)(len - 64 * (int64_t)c) : 64;
        uint8_t* sQK = sm + OFF_QK + s * 32768;
        uint8_t* sV = sm + OFF_V + s * 16384;
        const uint32_t aQK = sbase + OFF_QK + s * 32768, aV = sbase + OFF_V + s * 16384;

        // (a) gates: Gamma = cumsum(g) inside the chunk, beta; padded rows carry g = 0, beta = 0
        if (tid < 64) {
            const bool in = tid < nv;
            const int64_t gi = (tok0 + tid) * a.HV + hv;
            float x = in ? ld_any2(a.g, a.g_dtype, gi) : 0.f;
            vB[tid] = in ? ld_any2(a.beta, a.beta_dtype, gi) : 0.f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            vG[tid] = x;
        }
        __syncthreads();
        if (tid >= 32 && tid < 64) vG[tid] += vG[31];
        __syncthreads();
        if (tid < 64) {
            vEG[tid] = __expf(vG[tid]);
            vX[tid] = __expf(vG[63] - vG[tid]);
        }
        if (tid == 64) vMisc[0] = __expf(vG[63]);

        // (b) this chunk's Q, K, V tiles; then prefetch the next chunk into the other stage
        ok = mbar_wait(&bar_tma[s], (uint32_t)(c >> 1) & 1u, a.err, 1);
        if (!ok) break;
        tma_pending = 0;
        if (tid == 0 && c + 1 < nchunks) {
            issue_tma(c + 1, s ^ 1);
        }
        if (c + 1 < nchunks) tma_pending = 1;

        // (c) L2-normalise q/k rows in place (2 threads per row); zero rows past the sequence end
        {
            const int r = tid >> 1, half = tid & 1, i = r & 63;
            uint8_t* rowp = sQK + half * 16384 + (r < 64 ? 0 : 8192) + i * 128;
            float x[64];
            float ss = 0.f;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const uint4 u = *reinterpret_cast<const uint4*>(rowp + ((cc ^ (i & 7)) << 4));
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(h[e]);
                    x[cc * 8 + 2 * e] = f.x;
                    x[cc * 8 + 2 * e + 1] = f.y;
                    ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
                }
            }
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            float inv = a.l2norm ? 1.f / fmaxf(sqrtf(ss), kL2Eps) : 1.f;
            if (i >= nv) inv = 0.f;
            if (a.l2norm || i >= nv) {
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    float y[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = x[cc * 8 + e] * inv;
                    st_chunk8(rowp + ((cc ^ (i & 7)) << 4), y);
                }
            }
            if (!a.zero_v && tid < 128 && (tid >> 1) >= nv) {
                const int vi = tid >> 1;
                uint8_t* vrow = sV + (tid & 1) * 8192 + vi * 128;
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) *reinterpret_cast<uint4*>(vrow + cc * 16) = make_uint4(0, 0, 0, 0);
            }
        }
        fence_async_smem();
        block_sync_tc();

        // (d) MMA1: D1 = [Q;K] K^T  (M=128, N=64, K=128)
        if (tid == 0) {
            const uint32_t id = idesc_bf16(128, 64, 0, 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                umma_bf16(tD1, desc_kmajor(aQK + kb * 16384 + ko), desc_kmajor(aQK + kb * 16384 + 8192 + ko), id,
                          ks > 0);
            }
            umma_commit(bar_mma);
        }

        // (e) meanwhile: S0 -> bf16 S0^T operand, TMEM state <- e^G_C S0, checkpoint
        {
            const float eGC = vMisc[0];
            const bool ck = a.ckpt && (c % a.ckpt_every == 0);
            float* ckp = ck ? a.ckpt + ((ck_base + c / a.ckpt_every) * a.HV + hv) * 16384 : nullptr;
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 16) {
                float v[16];
                tmem_ld16(tS + lane_base + 64 * chh + c0, v);
                tmem_wait_ld();
                uint8_t* dst = sm + OFF_S + chh * 16384;
                st_chunk8(dst + sw128_off(row, c0), v);
                st_chunk8(dst + sw128_off(row, c0 + 8), v + 8);
                if (ck) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) ckp[(64 * chh + c0 + i) * 128 + row] = v[i];
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] *= eGC;
                tmem_st16(tS + lane_base + 64 * chh + c0, v);
            }
            tmem_wait_st();
        }
        ok = wait_mma(bar_mma, mma_phase, a.err, 2);
        if (!ok) break;

        // (f) D1 -> P (bf16) for rows 0-63 and A (fp32) for rows 64-127
        {
            float v[32];
            tmem_ld16(tD1 + lane_base + 32 * chh, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tD1 + lane_base + 32 * chh + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
            if (lg < 2) {  // Q K^T row i
                const int i = row;
                const float gi = vG[i];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int jj = 32 * chh + j;
                    v[j] = (jj <= i) ? a.scale * v[j] * __expf(gi - vG[jj]) : 0.f;
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) st_chunk8(sm + OFF_P + sw128_off(i, 32 * chh + 8 * q), v + 8 * q);
            } else {  // K K^T row i
                const int i = row - 64;
                const float gi = vG[i], bi = vB[i];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int jj = 32 * chh + j;
                    v[j] = (jj < i) ? bi * v[j] * __expf(gi - vG[jj]) : 0.f;
                }
                float4* dst = reinterpret_cast<float4*>(Am + i * AST + 32 * chh);
#pragma unroll
                for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        }
        __syncthreads();

        // (g) T = (I + A)^-1 in place: 16x16 diagonal blocks by column-wise forward substitution ...
        {
            float x[16];
            const int b = tid >> 4, cidx = tid & 15;
            if (tid < 64) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float sacc = 0.f;
#pragma unroll
                    for (int j = 0; j < i; ++j) sacc = fmaf(Am[(16 * b + i) * AST + 16 * b + j], x[j], sacc);
                    x[i] = (i == cidx) ? 1.f : (i < cidx ? 0.f : -sacc);
                }
            }
            __syncthreads();
            if (tid < 64) {
#pragma unroll
                for (int i = 0; i < 16; ++i) Am[(16 * b + i) * AST + 16 * b + cidx] = x[i];
            }
            __syncthreads();
        }
        // ... then off-diagonal blocks by block rows: T_rs = -T_rr sum_{m=s}^{r-1} A_rm T_ms
#pragma unroll 1
        for (int r = 1; r < 4; ++r) {
            for (int e = tid; e < r * 256; e += NTHR) {
                const int s2 = e >> 8, i = (e >> 4) & 15, cc = e & 15;
                float y = 0.f;
                for (int m = s2; m < r; ++m) {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        y = fmaf(Am[(16 * r + i) * AST + 16 * m + jj], Am[(16 * m + jj) * AST + 16 * s2 + cc], y);
                }
                Yb[e] = y;
            }
            __syncthreads();
            for (int e = tid; e < r * 256; e += NTHR) {
                const int s2 = e >> 8, i = (e >> 4) & 15, cc = e & 15;
                float t = 0.f;
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                    t = fmaf(Am[(16 * r + i) * AST + 16 * r + jj], Yb[s2 * 256 + jj * 16 + cc], t);
                Am[(16 * r + i) * AST + 16 * s2 + cc] = -t;
            }
            __syncthreads();
        }

        // (h) TB = T diag(beta e^G), TV = T diag(beta)  (bf16, K-major [i][j])
        {
            const int i = tid >> 2, q = tid & 3;
            float tb[16], tv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int jj = 16 * q + j;
                const float t = Am[i * AST + jj];
                tv[j] = t * vB[jj];
                tb[j] = tv[j] * vEG[jj];
            }
            st_chunk8(sm + OFF_TB + sw128_off(i, 16 * q), tb);
            st_chunk8(sm + OFF_TB + sw128_off(i, 16 * q + 8), tb + 8);
            st_chunk8(sm + OFF_TV + sw128_off(i, 16 * q), tv);
            st_chunk8(sm + OFF_TV + sw128_off(i, 16 * q + 8), tv + 8);
        }
        fence_async_smem();
        block_sync_tc();

        // (i) MMA2: W^T = K^T TB^T ; MMA3: U^T = V^T TV^T   (M=128, N=64, K=64 tokens)
        if (tid == 0) {
            const uint32_t id = idesc_bf16(128, 64, 1, 0);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tW, desc_mnmajor(aQK + 8192 + ks * 2048, 16384), desc_kmajor(sbase + OFF_TB + ks * 32), id,
                          ks > 0);
                umma_bf16(tU, desc_mnmajor(aV + ks * 2048, 8192), desc_kmajor(sbase + OFF_TV + ks * 32), id, ks > 0);
            }
            umma_commit(bar_mma);
        }
        // meanwhile: Q <- scale e^Gamma_i Q (Q is no longer read by MMA2/MMA3)
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int e = tid + it * NTHR;
            const int i = e >> 4, cc = e & 15;
            uint8_t* p = sQK + (cc >> 3) * 16384 + i * 128 + (((cc & 7) ^ (i & 7)) << 4);
            uint4 u = *reinterpret_cast<uint4*>(p);
            const float f = a.scale * vEG[i];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                float2 z = __bfloat1622float2(h[k2]);
                h[k2] = __floats2bfloat162_rn(z.x * f, z.y * f);
            }
            *reinterpret_cast<uint4*>(p) = u;
        }
        ok = wait_mma(bar_mma, mma_phase, a.err, 3);
        if (!ok) break;

        // (j) W^T (TMEM, lane = d) -> -W bf16 [i][d] (K-major B operand of MMA4)
        {
            float v[32];
            tmem_ld16(tW + lane_base + 32 * chh, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tW + lane_base + 32 * chh + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
            const int d = row;
            uint8_t* dst = sm + OFF_W + (d >> 6) * 8192;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                *reinterpret_cast<__nv_bfloat16*>(dst + sw128_off(32 * chh + j, d & 63)) = __float2bfloat16_rn(-v[j]);
        }
        fence_async_smem();
        block_sync_tc();

        // (k) MMA4: U^T += S0^T (-W)^T  -> Delta^T ; MMA5: O^T = S0^T Qg^T   (K = dk = 128)
        if (tid == 0) {
            const uint32_t id = idesc_bf16(128, 64, 0, 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                const uint64_t ad = desc_kmajor(sbase + OFF_S + kb * 16384 + ko);
                umma_bf16(tU, ad, desc_kmajor(sbase + OFF_W + kb * 8192 + ko), id, 1);
                umma_bf16(tO, ad, desc_kmajor(aQK + kb * 16384 + ko), id, ks > 0);
            }
            umma_commit(bar_mma);
        }
        ok = wait_mma(bar_mma, mma_phase, a.err, 4);
        if (!ok) break;

        // (l) Delta^T (TMEM, lane = dv) -> bf16 Delta^T and Delta^T diag(exp(G_C - G)) (K-major A operands)
        {
            float v[32], w2[32];
            tmem_ld16(tU + lane_base + 32 * chh, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tU + lane_base + 32 * chh + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) w2[j] = v[j] * vX[32 * chh + j];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                st_chunk8(sm + OFF_D + sw128_off(row, 32 * chh + 8 * q), v + 8 * q);
                st_chunk8(sm + OFF_DD + sw128_off(row, 32 * chh + 8 * q), w2 + 8 * q);
            }
        }
        fence_async_smem();
        block_sync_tc();

        // (m) MMA6: O^T += Delta^T P^T (K = 64) ; MMA7: S^T += DeltaD^T K (N = 128, K = 64)
        if (tid == 0) {
            const uint32_t id6 = idesc_bf16(128, 64, 0, 0), id7 = idesc_bf16(128, 128, 0, 1);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tO, desc_kmajor(sbase + OFF_D + ks * 32), desc_kmajor(sbase + OFF_P + ks * 32), id6, 1);
                umma_bf16(tS, desc_kmajor(sbase + OFF_DD + ks * 32), desc_mnmajor(aQK + 8192 + ks * 2048, 16384), id7,
                          1);
            }
            umma_commit(bar_mma);
        }
        ok = wait_mma(bar_mma, mma_phase, a.err, 5);
        if (!ok) break;

        // (n) O^T (TMEM, lane = dv) -> o[token][hv][dv]
        if (a.o_mode != 2) {
            float v[32];
            tmem_ld16(tO + lane_base + 32 * chh, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tO + lane_base + 32 * chh + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
            __nv_bfloat16* o = (__nv_bfloat16*)a.o;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int i = 32 * chh + j;
                if (i < nv) {
                    const int64_t idx = ((tok0 + i) * a.HV + hv) * 128 + row;
                    float val = v[j];
                    if (a.o_mode == 1) val += __bfloat162float(o[idx]);
                    o[idx] = __float2bfloat16_rn(val);
                }
            }
        }
        block_sync_tc();
    }

    // final state
    if (ok && a.ht) {
        float* ht = a.ht + ((int64_t)n * a.HV + hv) * 16384;
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
            float v[16];
            tmem_ld16(tS + lane_base + 64 * chh + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float* p = ht + (64 * chh + c0 + i) * 128 + row;
                *p = a.ht_accumulate ? *p + v[i] : v[i];
            }
        }
    }
    if (!ok && tma_pending) {
        // a wait gave up: let the outstanding tile load land before the CTA's shared memory goes away
        mbar_wait(&bar_tma[0], 0, nullptr, 0, 1u << 20);
    }
    block_sync_tc();
    if (warp == 0) tmem_dealloc(tm, T_COLS);
}

bool chunk_fwd_supported(int64_t DK, int64_t DV, int act_dtype) {
    return DK == 128 && DV == 128 && act_dtype == GDN_BF16;
}

int chunk_fwd(const ChunkLaunch& L, cudaStream_t s) {
    using namespace cf;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(chunk_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
            cudaSuccess)
            return GDN_ERR_LAUNCH;
        attr_set = true;
    }
    ChunkFwdArgs a;
    memset(&a, 0, sizeof(a));
    const int64_t Ttot = L.B * L.T;
    if (!make_tmap_3d_sw128(&a.tq, L.q, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    if (!make_tmap_3d_sw128(&a.tk, L.k, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    if (!L.zero_v && !make_tmap_3d_sw128(&a.tv, L.v, 128, L.HV, Ttot, 128, L.HV * 128, 64)) return GDN_ERR_ALIGN;
    a.g = L.g;
    a.beta = L.beta;
    a.o = L.o;
    a.h0 = L.h0;
    a.ht = L.ht;
    a.ckpt = L.ckpt;
    a.cu = L.cu;
    a.err = L.err;
    a.T = L.T;
    a.N = (int)L.N;
    a.H = (int)L.H;
    a.HV = (int)L.HV;
    a.g_dtype = L.g_dtype;
    a.beta_dtype = L.beta_dtype;
    a.scale = L.scale;
    a.l2norm = L.l2norm;
    a.zero_v = L.zero_v;
    a.o_mode = L.o_mode;
    a.h0_identity = L.h0_identity;
    a.ht_accumulate = L.ht_accumulate;
    a.ckpt_every = L.ckpt_every;
    const unsigned grid = (unsigned)(L.N * L.HV);
    if (grid == 0) return GDN_OK;
    chunk_fwd_kernel<<<grid, NTHR, SMEM_BYTES, s>>>(a);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
