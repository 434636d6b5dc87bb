// Chunked gated-delta-rule forward on sm_100a: tcgen05 (UMMA) tile contractions, TMA-fed shared memory,
// fp32 state resident in tensor memory (TMEM) for the whole sequence.
//
// One CTA (512 threads) per (sequence, value head) walks the sequence in chunks of C = 64 tokens.
// With Gamma = in-chunk inclusive cumsum of g, E_ij = exp(Gamma_i - Gamma_j), S0 the state at the chunk
// start, and nq_i, nk_j the L2 norms of the raw q/k rows (1 when the norm is off), the chunk computes
// (algebra checked against the per-token recurrence in tests/test_chunk_algebra.py):
//   A   = strict_lower(diag(beta) (K K^T / nk nk^T) . E)    T = (I + A)^-1   (fp32 block doubling from
//         8x8 blocks on warps 0-7, beside the S0 read-out on warps 8-15; tri_inverse64 in chunk_common.cuh)
//   W   = T diag(beta e^Gamma / nk) K     U = T diag(beta) V     Delta = U - W S0
//   O_i = [ scale e^Gamma_i (S0^T q_i) + (P' Delta)_i ] / nq_i,   P' = scale lower_incl(Q K^T / nk^T . E)
//   S1  = e^Gamma_C S0 + K^T diag(e^(Gamma_C - Gamma) / nk) Delta
// The raw bf16 q/k tiles feed the tensor cores unmodified (the norms are applied in fp32), and Delta and
// P' are split into bf16 hi + lo parts, so the only bf16 roundings left are those of T, W, S0 (whose
// effect is below the output's own rounding) and the output itself.
// Every GEMM is an M = 128 UMMA with a 128-wide dimension on the TMEM lanes:
//   MMA1  D1[128x64] = [Q;K] K^T                 (rows 0-63: Q K^T, rows 64-127: K K^T)
//   MMA2  [W; -] = [TB; TV] K  (W rows on lanes 0-63)       MMA3  U^T = V^T TV^T,  TV = T diag(beta)
//         TB = T diag(beta e^G / nk)
//   MMA4  U^T += S0^T (-W)^T  -> Delta^T                   MMA5  [-; O1] = [-; Q] S0  (O rows on lanes 64-127,
//         issued right after S0's read-out, into TMEM columns 128-255)
//   MMA6  [-; O2] = [-; P'] Delta  (hi.hi + lo.hi + hi.lo) MMA7  S^T += Dd^T K,  Dd = diag(e^(G_C-G)/nk) Delta
// A 128-row A operand whose half is ignored always takes that half from an allocated tile below or above
// the real one (never past the end of shared memory).
// S^T (fp32, 128 TMEM columns) reaches HBM only as checkpoints for the backward (every ckpt_every
// chunks) and as the final state.
#include <cstring>

#include "chunk_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.h"
#include "sm100.cuh"
#include "tmap.h"

namespace gdn {
using namespace sm100;

namespace cf {
constexpr int NTHR = 512;  // 16 warps: 4 per TMEM lane quadrant, each owning 16 of 64 columns
// shared memory carve (bytes from a 1024-aligned base)
// Q/K: per d-block kb (24 KB apart): [K odd chunks 8 KB | Q 8 KB | K even chunks 8 KB], 64 rows x 128 B
// each. K is double-buffered, Q single-buffered; either way [Q;K] (even) or [K;Q] (odd) is one
// contiguous 128-row K-major operand for MMA1.
constexpr uint32_t OFF_QK = 0;
constexpr uint32_t QK_BLK = 24576;
constexpr uint32_t OFF_V = 49152;     // V, single stage, [kb][8 KB]
constexpr uint32_t OFF_S = 65536;     // S0^T hi bf16 [dv][dk] K-major, 2 dk-blocks x 16 KB
constexpr uint32_t OFF_SL = 98304;    // S0^T lo
constexpr uint32_t OFF_D = 131072;    // Delta^T hi bf16 [dv][j], 16 KB
constexpr uint32_t OFF_DL = 147456;   // Delta^T lo
constexpr uint32_t OFF_DD = 163840;   // Dd^T hi
constexpr uint32_t OFF_DDL = 180224;  // Dd^T lo
constexpr uint32_t OFF_TB = 196608;   // TB bf16 [i][j], 8 KB
constexpr uint32_t OFF_TV = 204800;   // TV bf16 [i][j], 8 KB
constexpr uint32_t OFF_P = 212992;    // P' hi bf16 [i][j], 8 KB
constexpr uint32_t OFF_PL = 221184;   // P' lo
constexpr uint32_t OFF_W = OFF_TB;    // -W bf16 [i][d] K-major, 2 d-blocks x 8 KB: reuses TB/TV once MMA2/3 ran
constexpr uint32_t OFF_VEC = 229376;  // G, e^G, beta, e^(G_C-G), 1/nq, 1/nk, misc: 7 x 64 fp32
constexpr uint32_t OFF_BAR = OFF_VEC + 7 * 64 * 4;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 64 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// The fp32 triangular-solve scratch lives in the Delta region, which is dead between MMA7 of one chunk
// and step (l) of the next.
constexpr int AST = 68;  // padded fp32 row stride (conflict-free float4 rows)
constexpr uint32_t OFF_A = OFF_D;
constexpr uint32_t OFF_Y = OFF_A + 64 * AST * 4;
static_assert(OFF_Y + 32 * kSolveYStride * 4 <= OFF_DD, "solve scratch overlaps live tiles");
// TMEM columns
// O2 (128 columns) reuses D1 + U once both are read; O1 has its own columns (it is computed early).
constexpr uint32_t T_D1 = 0, T_U = 64, T_O2 = 0, T_O1 = 128, T_S = 256, T_W = 384, T_COLS = 512;
constexpr uint32_t TX_QK = 4 * 8192, TX_V = 2 * 8192;
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
    uint8_t* s0_out;  // recompute mode: checkpoints are read, S0^T tiles written here (see ChunkLaunch)
};

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
// hi = bf16(v), lo = bf16(v - hi): two chunks whose sum carries ~16 significant bits
__device__ __forceinline__ void st_chunk8_split(uint8_t* hi, uint8_t* lo, const float* v) {
    float h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        h[e] = __bfloat162float(__float2bfloat16_rn(v[e]));
        l[e] = v[e] - h[e];
    }
    st_chunk8(hi, h);
    st_chunk8(lo, l);
}

// bulk (TMA) copy shared -> global, tracked by the issuing thread's bulk groups
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"((uint64_t)dst),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void block_sync_tc() {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

// Bounded waits never make threads leave the chunk loop (a divergent exit would strand the others at the
// next barrier): a timeout records an error code and every later wait of the CTA polls only once, so a
// broken launch still ends in bounded time.
__device__ __forceinline__ void wait_bar(uint64_t* bar, uint32_t parity, int* err, int code, bool& ok) {
    ok = mbar_wait(bar, parity, err, code, ok ? (1u << 22) : 1u) && ok;
}
__device__ __forceinline__ void wait_mma(uint64_t* bar, uint32_t& phase, int* err, int code, bool& ok) {
    wait_bar(bar, phase, err, code, ok);
    phase ^= 1u;
    tc_fence_after();
}

__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) {
    tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
    tmem_ld16(taddr + 16, *reinterpret_cast<float(*)[16]>(v + 16));
    tmem_wait_ld();
}
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
    tmem_ld16(taddr, v);
    tmem_wait_ld();
}
// o[j] = v[base + j] as float4 loads (base % 4 == 0): a warp-uniform float4 load costs about 2.4
// shared-memory cycles against 1.1 for each of four scalar loads.
template <int N>
__device__ __forceinline__ void vecN(const float* v, int base, float (&o)[N]) {
    const float4* p = reinterpret_cast<const float4*>(v + base);
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
        const float4 x = p[q];
        o[4 * q] = x.x;
        o[4 * q + 1] = x.y;
        o[4 * q + 2] = x.z;
        o[4 * q + 3] = x.w;
    }
}

// MODE 0: plain forward (o written, no transition-map flags); 1: recompute pass (records, no outputs);
// 2: the sequence-split passes (zero_v / h0_identity / o_mode 1 / ht_accumulate read at run time)
template <int MODE>
__global__ void __launch_bounds__(cf::NTHR, 1) chunk_fwd_kernel(const __grid_constant__ ChunkFwdArgs a) {
    const int o_mode = MODE == 0 ? 0 : (MODE == 1 ? 2 : a.o_mode);
    const bool zero_v = MODE == 2 && a.zero_v, h0_identity = MODE == 2 && a.h0_identity;
    const bool ht_accumulate = MODE == 2 && a.ht_accumulate;
    using namespace cf;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* Am = (float*)(sm + OFF_A);
    float* Yb = (float*)(sm + OFF_Y);
    float* vG = (float*)(sm + OFF_VEC);
    float* vEG = vG + 64;
    float* vB = vG + 128;
    float* vX = vG + 192;
    float* vNQ = vG + 256;  // 1/nq (0 on padded rows)
    float* vNK = vG + 320;  // 1/nk (0 on padded rows)
    float* vMisc = vG + 384;
    uint64_t* bar_k = (uint64_t*)(sm + OFF_BAR);  // [2]: K tile of even / odd chunks
    uint64_t* bar_q = bar_k + 2;
    uint64_t* bar_v = bar_k + 3;
    uint64_t* bar_mma = bar_k + 4;
    uint32_t* tmem_slot = (uint32_t*)(bar_k + 5);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lg = warp & 3, cq = warp >> 2;  // TMEM lane group, column quarter
    const int row = 32 * lg + lane;            // accumulator row (TMEM lane) of this thread
    const int n = blockIdx.x / a.HV, hv = blockIdx.x % a.HV, hq = hv / (a.HV / a.H);
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t len = eos - bos;
    const int nchunks_seq = (int)((len + 63) / 64);
    // recompute mode: this CTA covers chunks [c_begin, c_end) of its sequence, starting from a checkpoint
    constexpr bool recompute = MODE == 1;
    const int c_begin = recompute ? (int)blockIdx.y * a.ckpt_every : 0;
    if (c_begin >= nchunks_seq && c_begin > 0) return;
    const int nchunks = recompute ? min(nchunks_seq, c_begin + a.ckpt_every) : nchunks_seq;

    // first chunk of this sequence in the flattened chunk list (S0 tile slots in recompute mode)
    int64_t cbase = 0;
    if (recompute) {
        if (!a.cu) {
            cbase = (int64_t)n * ((a.T + 63) / 64);
        } else {
            int64_t part = 0;
            for (int m = tid; m < n; m += NTHR) part += (a.cu[m + 1] - a.cu[m] + 63) / 64;
            for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (lane == 0) ((int64_t*)Yb)[warp] = part;
            __syncthreads();
            for (int w = 0; w < NTHR / 32; ++w) cbase += ((int64_t*)Yb)[w];
            __syncthreads();
        }
    }

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
        mbar_init(&bar_k[0], 1);
        mbar_init(&bar_k[1], 1);
        mbar_init(bar_q, 1);
        mbar_init(bar_v, 1);
        mbar_init(bar_mma, 1);
        fence_barrier_init();
        prefetch_tmap(&a.tq);
        prefetch_tmap(&a.tk);
        if (!zero_v) prefetch_tmap(&a.tv);
    }
    if (warp == 0) tmem_alloc(tmem_slot, T_COLS);
    if (zero_v) {
        for (int e = tid; e < 16384 / 16; e += NTHR) ((uint4*)(sm + OFF_V))[e] = make_uint4(0, 0, 0, 0);
        fence_async_smem();
    }
    block_sync_tc();
    const uint32_t tm = *tmem_slot;
    const uint32_t tD1 = tm + T_D1, tW = tm + T_W, tU = tm + T_U, tO1 = tm + T_O1, tO2 = tm + T_O2, tS = tm + T_S;
    const uint32_t lane_base = (uint32_t)(32 * lg) << 16;
    uint32_t mma_phase = 0;
    bool ok = true;

    // initial state -> TMEM: thread (row = dv, quarter cq) holds S^T[dv][dk] for dk in [32 cq, 32 cq + 32)
    {
        const float* h0 = a.h0 ? a.h0 + ((int64_t)n * a.HV + hv) * 16384 : nullptr;
        if (recompute) h0 = a.ckpt + ((ck_base + blockIdx.y) * a.HV + hv) * 16384;
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int dk = 32 * cq + c0 + i;
                v[i] = (h0_identity && !recompute) ? (dk == row ? 1.f : 0.f) : (h0 ? h0[dk * 128 + row] : 0.f);
            }
            tmem_st16(tS + lane_base + 32 * cq + c0, v);
        }
        tmem_wait_st();
    }

    // K of chunk c goes to slot (c & 1): +16 KB (even) or +0 (odd) inside each d-block; Q to +8 KB
    // slots and mbarrier phases follow the CTA-local chunk count cl = c - c_begin
    auto issue_k = [&](int c, int s) {
        const int tok0 = (int)(bos + 64 * c);
        mbar_arrive_expect_tx(&bar_k[s], TX_QK / 2);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
            tma_load_3d(sm + OFF_QK + kb * QK_BLK + (s ? 0 : 16384), &a.tk, &bar_k[s], kb * 64, hq, tok0);
    };
    auto issue_q = [&](int c) {
        const int tok0 = (int)(bos + 64 * c);
        mbar_arrive_expect_tx(bar_q, TX_QK / 2);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) tma_load_3d(sm + OFF_QK + kb * QK_BLK + 8192, &a.tq, bar_q, kb * 64, hq, tok0);
    };
    auto issue_v = [&](int c) {
        const int tok0 = (int)(bos + 64 * c);
        mbar_arrive_expect_tx(bar_v, TX_V);
        tma_load_3d(sm + OFF_V, &a.tv, bar_v, 0, hv, tok0);
        tma_load_3d(sm + OFF_V + 8192, &a.tv, bar_v, 64, hv, tok0);
    };
    if (tid == 0 && nchunks > 0) {
        issue_k(c_begin, 0);
        if (!recompute) issue_q(c_begin);  // recompute mode forms no outputs: Q is never read
        if (!zero_v) issue_v(c_begin);
    }

    const uint32_t sbase = smem_u32(sm);
    uint32_t g_next = 0u, b_next = 0u;  // gates of the next chunk (threads 0-63), loaded one chunk ahead, raw
    if (tid < 64 && c_begin < nchunks) {
        const bool in = tid < len - 64 * (int64_t)c_begin;
        const int64_t gi = (bos + 64 * (int64_t)c_begin + tid) * a.HV + hv;
        if (in) {
            g_next = ld_gate_raw(a.g, a.g_dtype, gi);
            b_next = ld_gate_raw(a.beta, a.beta_dtype, gi);
        }
    }
    for (int c = c_begin; c < nchunks; ++c) {
        const int cl = c - c_begin;
        const int s = cl & 1;
        const int64_t tok0 = bos + 64 * (int64_t)c;
        const int nv = (len - 64 * (int64_t)c) < 64 ? (int)(len - 64 * (int64_t)c) : 64;
        const uint32_t kofs = s ? 0u : 16384u;              // K slot inside a d-block
        const uint32_t aBlk = sbase + OFF_QK, aV = sbase + OFF_V;
        const uint32_t aK = aBlk + kofs, aQ = aBlk + 8192;  // d-block 0 of K and Q
        const uint32_t aA1 = s ? aK : aQ;                   // MMA1's 128-row A: [Q;K] even, [K;Q] odd
        uint8_t* rec_g = recompute ? a.s0_out + ((cbase + c) * a.HV + hv) * kBwdRecordBytes : nullptr;

        // (a) gates: Gamma = cumsum(g) inside the chunk, beta; padded rows carry g = 0, beta = 0
        if (tid < 64) {
            float x = gate_f(g_next, a.g_dtype);
            vB[tid] = gate_f(b_next, a.beta_dtype);
            g_next = b_next = 0u;
            if (c + 1 < nchunks) {  // next chunk's gates: their latency hides behind this chunk
                const int64_t len1 = len - 64 * (int64_t)(c + 1);
                const int64_t gi = (tok0 + 64 + tid) * a.HV + hv;
                if (tid < len1) {
                    g_next = ld_gate_raw(a.g, a.g_dtype, gi);
                    b_next = ld_gate_raw(a.beta, a.beta_dtype, gi);
                }
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            vG[tid] = x;
        }

        // (b) this chunk's Q, K tiles; prefetch the next chunk's into the other stage
        wait_bar(&bar_k[s], (uint32_t)(cl >> 1) & 1u, a.err, 1, ok);
        if (!recompute) wait_bar(bar_q, (uint32_t)cl & 1u, a.err, 7, ok);
        if (tid == 0 && c + 1 < nchunks) issue_k(c + 1, s ^ 1);  // the other K slot: MMA7 of chunk c-1 is done

        // (c) MMA1: D1 = [Q;K] K^T (even chunks) or [K;Q] K^T (odd) on the raw tiles (M=128, N=64, K=128);
        //     in recompute mode the Q half of A is whatever the Q slot holds and its rows of D1 go unread
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id = idesc_bf16(128, 64, 0, 0);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                umma_bf16(tD1, desc_kmajor(aA1 + kb * QK_BLK + ko), desc_kmajor(aK + kb * QK_BLK + ko), id, ks > 0);
            }
            umma_commit(bar_mma);
        }
        __syncthreads();
        if (tid >= 32 && tid < 64) vG[tid] += vG[31];
        // (d) meanwhile: row norms of q and k (4 threads per row, 32 elements each; rows 0-63 are q, on warps
        //     0-7, skipped in recompute mode)
        if (!recompute || tid >= 256) {
            const int r = tid >> 2, part = tid & 3, i = r & 63;
            const uint8_t* rowp = sm + OFF_QK + (part >> 1) * QK_BLK + (r < 64 ? 8192 : kofs) + i * 128;
            float ss = 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                // chunk order rotated by (2 d-block + row parity): the 8 lanes of a quarter-warp read 8
                // distinct 16-byte bank groups (the sum is order-free)
                const int ch = (cc + 4 * (part & 1) + 2 * (part >> 1) + (r & 1)) & 7;
                const uint4 u = *reinterpret_cast<const uint4*>(rowp + ch * 16);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(h[e]);
                    ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
                }
            }
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            ss += __shfl_xor_sync(0xffffffffu, ss, 2);
            float inv = a.l2norm ? 1.f / fmaxf(sqrtf(ss), kL2Eps) : 1.f;
            if (i >= nv) inv = 0.f;
            if (part == 0) (r < 64 ? vNQ : vNK)[i] = inv;
        }
        __syncthreads();
        if (tid < 64) {
            vEG[tid] = __expf(vG[tid]);
            vX[tid] = __expf(vG[63] - vG[tid]) * vNK[tid];  // includes 1/nk: Dd = diag(e^(G_C-G)/nk) Delta
        }
        if (tid == 64) vMisc[0] = __expf(vG[63]);
        // recompute mode: the previous chunk's bulk stores must have read their tiles before (f) and (g)
        // overwrite them
        if (recompute && tid == 0) bulk_wait_read_all();
        __syncthreads();

        wait_mma(bar_mma, mma_phase, a.err, 2, ok);

        // (f) D1 -> P' (hi/lo bf16) for rows 0-63 and A (fp32) for rows 64-127
        {
            float v[16];
            ld16(tD1 + lane_base + 16 * cq, v);
            if ((lg < 2) == (s == 0)) {  // Q K^T row i (rows 0-63 on even chunks, 64-127 on odd)
              if (!recompute) {  // no outputs in recompute mode: OFF_P carries the backward's T tile instead
                const int i = row & 63;
                const float gi = vG[i];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int jj = 16 * cq + j;
                    v[j] = (jj <= i) ? a.scale * v[j] * vNK[jj] * __expf(gi - vG[jj]) : 0.f;
                }
#pragma unroll
                for (int q = 0; q < 2; ++q)
                    st_chunk8_split(sm + OFF_P + sw128_off(i, 16 * cq + 8 * q),
                                    sm + OFF_PL + sw128_off(i, 16 * cq + 8 * q), v + 8 * q);
              }
            } else {  // K K^T row i
                const int i = row & 63;
                const float gi = vG[i], bi = vB[i] * vNK[i];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int jj = 16 * cq + j;
                    v[j] = (jj < i) ? bi * v[j] * vNK[jj] * __expf(gi - vG[jj]) : 0.f;
                }
                float4* dst = reinterpret_cast<float4*>(Am + i * AST + 16 * cq);
#pragma unroll
                for (int q = 0; q < 4; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        }
        __syncthreads();

        // (g) T = (I + A)^-1 in place on warps 0-7, while warps 8-15 do
        // (e): S0 -> bf16 S0^T operand (hi/lo), TMEM state <- e^G_C S0, checkpoint or recompute tile
        if (warp < 8) {
            tri_inverse64<AST>(Am, Yb);
        } else if (warp >= 8) {
            const int half = (warp - 8) >> 2;  // dk columns 64 half .. 64 half + 63 = S0^T block `half`
            const float eGC = vMisc[0];
            const bool ck = a.ckpt && !recompute && (c % a.ckpt_every == 0);
            float* ckp = ck ? a.ckpt + ((ck_base + c / a.ckpt_every) * a.HV + hv) * 16384 : nullptr;
#pragma unroll 1
            for (int c0 = 0; c0 < 64; c0 += 16) {
                float v[16];
                tmem_ld16(tS + lane_base + 64 * half + c0, v);
                tmem_wait_ld();
                const uint32_t blk = half * 16384;
                const uint32_t o0 = blk + sw128_off(row, c0), o1 = blk + sw128_off(row, c0 + 8);
                st_chunk8_split(sm + OFF_S + o0, sm + OFF_SL + o0, v);
                st_chunk8_split(sm + OFF_S + o1, sm + OFF_SL + o1, v + 8);
                if (ck) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) ckp[(64 * half + c0 + i) * 128 + row] = v[i];
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] *= eGC;
                tmem_st16(tS + lane_base + 64 * half + c0, v);
            }
            tmem_wait_st();
            fence_async_smem();
        }
        __syncthreads();
        if (recompute && tid == 0) bulk_s2g(rec_g, sm + OFF_S, 32768);  // S0^T hi tile
        if (tid == 0 && o_mode != 2) {  // MMA5 as soon as S0^T is in place: [-; O1] = [-; Q] S0hi
            tc_fence_after();             // (O1 in the otherwise idle columns 128-255; waited on with MMA4)
            const uint32_t id5 = idesc_bf16(128, 128, 0, 0);
            const uint64_t dS_h = desc_kmajor(sbase + OFF_S);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                // A = [K odd slot (ignored); Q]: rows 64-127 are Q, so O1 lands on lanes 64-127
                umma_bf16(tO1, desc_kmajor(aQ - 8192 + kb * QK_BLK + ko), dS_h + ((kb * 16384 + ko) >> 4), id5,
                          ks > 0);
            }
        }

        // (h) TB = T diag(beta e^G / nk), TV = T diag(beta)  (bf16, K-major [i][j])
        {  // a quarter-warp covers rows i, i + 1 and four chunks of one 32-column half: its row loads and
           // vector loads hit distinct banks
            const int wl = tid & 31, qq = wl >> 3, sub = wl & 7;
            const int i = 4 * (tid >> 5) + 2 * (qq & 1) + (sub >> 2), c8 = 8 * ((sub & 3) + 4 * (qq >> 1));
            float tb[8], tv[8];
            const float4 t0 = *reinterpret_cast<const float4*>(Am + i * AST + c8);
            const float4 t1 = *reinterpret_cast<const float4*>(Am + i * AST + c8 + 4);
            const float t[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
            float b8[8], e8[8], n8[8];
            vecN(vB, c8, b8);
            vecN(vEG, c8, e8);
            vecN(vNK, c8, n8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                tv[j] = t[j] * b8[j];
                tb[j] = tv[j] * e8[j] * n8[j];
            }
            st_chunk8(sm + OFF_TB + sw128_off(i, c8), tb);
            st_chunk8(sm + OFF_TV + sw128_off(i, c8), tv);
            if (recompute)  // the backward's T operand tile, right after -W (P' is not formed in this mode)
                st_chunk8(sm + OFF_P + sw128_off(i, c8), t);
        }
        fence_async_smem();
        block_sync_tc();

        // (i) MMA2: W^T = K^T TB^T ; MMA3: U^T = V^T TV^T   (M=128, N=64, K=64 tokens)
        if (tid == 0) {
            if (!zero_v) wait_bar(bar_v, (uint32_t)cl & 1u, a.err, 6, ok);
            const uint32_t id = idesc_bf16(128, 64, 1, 0);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_bf16(tW, desc_kmajor(sbase + OFF_TB + ks * 32), desc_mnmajor(aK + ks * 2048, QK_BLK),
                          idesc_bf16(128, 128, 0, 1), ks > 0);
                umma_bf16(tU, desc_mnmajor(aV + ks * 2048, 8192), desc_kmajor(sbase + OFF_TV + ks * 32), id, ks > 0);
            }
            umma_commit(bar_mma);
        }
        wait_mma(bar_mma, mma_phase, a.err, 3, ok);
        // V is consumed: load the next chunk's V
        if (tid == 0 && !zero_v && c + 1 < nchunks) issue_v(c + 1);

        // (j) W (TMEM rows i = lanes 0-63, columns d) -> -W bf16 [i][d] (K-major B operand of MMA4);
        //     warp column quarter cq writes d = 32 cq .. 32 cq + 31 with 16-byte stores
        if (lg < 2) {
            float v[32];
            uint8_t* dst = sm + OFF_W + (cq >> 1) * 8192;
            ld32(tW + lane_base + 32 * cq, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = -v[e];
#pragma unroll
            for (int q = 0; q < 4; ++q) st_chunk8(dst + sw128_off(row, 32 * (cq & 1) + 8 * q), v + 8 * q);
        }
        fence_async_smem();
        block_sync_tc();
        if (recompute && tid == 0) bulk_s2g(rec_g + kBwdRecW, sm + OFF_W, 24576);  // -W | T (at OFF_P)

        // (k) MMA4: U^T += (S0hi + S0lo)^T (-W)^T -> Delta^T   (K = dk = 128); the commit also covers MMA5
        if (tid == 0) {
            const uint32_t id = idesc_bf16(128, 64, 0, 0);
            // base descriptors; the 14-bit start-address field (bytes >> 4) never carries for smem addresses
            const uint64_t dS_h = desc_kmajor(sbase + OFF_S), dS_l = desc_kmajor(sbase + OFF_SL);
            const uint64_t dW_ = desc_kmajor(sbase + OFF_W);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                const uint64_t ah = dS_h + ((kb * 16384 + ko) >> 4);
                const uint64_t al = dS_l + ((kb * 16384 + ko) >> 4);
                const uint64_t bw = dW_ + ((kb * 8192 + ko) >> 4);
                umma_bf16(tU, ah, bw, id, 1);
                umma_bf16(tU, al, bw, id, 1);
            }
            umma_commit(bar_mma);
        }
        wait_mma(bar_mma, mma_phase, a.err, 4, ok);
        // Q is consumed: load the next chunk's Q
        if (tid == 0 && !recompute && c + 1 < nchunks) issue_q(c + 1);

        // (l) Delta^T (TMEM, lane = dv) -> hi/lo bf16 Delta^T and Dd^T (K-major A operands)
        {
            float v[16], x16[16], w2[16];
            ld16(tU + lane_base + 16 * cq, v);
            vecN(vX, 16 * cq, x16);
#pragma unroll
            for (int j = 0; j < 16; ++j) w2[j] = v[j] * x16[j];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint32_t off = sw128_off(row, 16 * cq + 8 * q);
                st_chunk8_split(sm + OFF_DD + off, sm + OFF_DDL + off, w2 + 8 * q);
                if (!recompute) {
                    st_chunk8_split(sm + OFF_D + off, sm + OFF_DL + off, v + 8 * q);
                } else {  // the backward's Delta^T tile and Dd^T low part (relative to bf16(bf16(Delta) x)),
                          // staged where MMA6's operands would go (no outputs in this mode)
                    float lo[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float dh = __bfloat162float(__float2bfloat16_rn(v[8 * q + e]));
                        lo[e] = w2[8 * q + e] - __bfloat162float(__float2bfloat16_rn(dh * x16[8 * q + e]));
                    }
                    st_chunk8(sm + OFF_D + off, v + 8 * q);
                    st_chunk8(sm + OFF_DL + off, lo);
                }
            }
        }
        fence_async_smem();
        block_sync_tc();
        if (recompute && tid == 0) bulk_s2g(rec_g + kBwdRecDel, sm + OFF_D, 32768);  // Delta^T | Dd^T lo

        // (m) MMA6: O2^T = Delta^T P'^T (hi.hi + lo.hi + hi.lo) ; MMA7: S^T += Dd^T K (hi + lo), N = 128
        // [-; O2] = [-; P'] Delta: the 64 rows below each P' tile (TV for P' hi, P' hi for P' lo, both
        // allocated and finite) fill the ignored half, so O2 lands on lanes 64-127 like O1
        if (tid == 0) {
            const uint32_t id6 = idesc_bf16(128, 128, 0, 0), id7 = idesc_bf16(128, 128, 0, 1);
            const uint64_t dD_ = desc_kmajor(sbase + OFF_D), dDL_ = desc_kmajor(sbase + OFF_DL);
            const uint64_t dDD_ = desc_kmajor(sbase + OFF_DD), dDDL_ = desc_kmajor(sbase + OFF_DDL);
            const uint64_t dP_ = desc_kmajor(sbase + OFF_P - 8192), dPL_ = desc_kmajor(sbase + OFF_PL - 8192);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint64_t dh = dD_ + ks * 2, dl = dDL_ + ks * 2;  // +32 bytes per K step
                const uint64_t ph = dP_ + ks * 2, pl = dPL_ + ks * 2;
                if (o_mode != 2) {
                    umma_bf16(tO2, ph, dh, id6, ks > 0);
                    umma_bf16(tO2, pl, dh, id6, 1);
                    umma_bf16(tO2, ph, dl, id6, 1);
                }
                const uint64_t kd = desc_mnmajor(aK + ks * 2048, QK_BLK);
                umma_bf16(tS, dDD_ + ks * 2, kd, id7, 1);
                umma_bf16(tS, dDDL_ + ks * 2, kd, id7, 1);
            }
            umma_commit(bar_mma);
        }
        wait_mma(bar_mma, mma_phase, a.err, 5, ok);

        // (n) O = (scale e^G O1 + O2) / nq -> o[token][hv][dv]
        //     rows i on lanes 64-127: each thread writes 32 contiguous dv of one token (16-byte stores)
        if (o_mode != 2 && lg >= 2) {
            const int i = row - 64;
            const float f1 = a.scale * vEG[i] * vNQ[i], f2 = vNQ[i];
            __nv_bfloat16* orow = (__nv_bfloat16*)a.o + ((tok0 + i) * a.HV + hv) * 128 + 32 * cq;
            {
                float v1[32], v2[32];
                tmem_ld16(tO1 + lane_base + 32 * cq, *reinterpret_cast<float(*)[16]>(v1));
                tmem_ld16(tO1 + lane_base + 32 * cq + 16, *reinterpret_cast<float(*)[16]>(v1 + 16));
                tmem_ld16(tO2 + lane_base + 32 * cq, *reinterpret_cast<float(*)[16]>(v2));
                tmem_ld16(tO2 + lane_base + 32 * cq + 16, *reinterpret_cast<float(*)[16]>(v2 + 16));
                tmem_wait_ld();
                if (i < nv) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float y[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) y[e] = fmaf(f1, v1[8 * q + e], f2 * v2[8 * q + e]);
                        uint4* dst = reinterpret_cast<uint4*>(orow + 8 * q);
                        if (o_mode == 1) {
                            const uint4 old = *dst;
                            const __nv_bfloat162* ob = reinterpret_cast<const __nv_bfloat162*>(&old);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 z = __bfloat1622float2(ob[e]);
                                y[2 * e] += z.x;
                                y[2 * e + 1] += z.y;
                            }
                        }
                        uint4 u;
                        u.x = pack_bf16(y[0], y[1]);
                        u.y = pack_bf16(y[2], y[3]);
                        u.z = pack_bf16(y[4], y[5]);
                        u.w = pack_bf16(y[6], y[7]);
                        *dst = u;
                    }
                }
            }
        }
        block_sync_tc();
    }

    if (recompute && tid == 0) bulk_wait_all();  // the last chunk's record is in global memory

    // final state
    if (ok && a.ht) {
        float* ht = a.ht + ((int64_t)n * a.HV + hv) * 16384;
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 16) {
            float v[16];
            tmem_ld16(tS + lane_base + 32 * cq + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float* p = ht + (32 * cq + c0 + i) * 128 + row;
                *p = ht_accumulate ? *p + v[i] : v[i];
            }
        }
    }
    block_sync_tc();
    if (warp == 0) tmem_dealloc(tm, T_COLS);
}

bool chunk_fwd_supported(int64_t DK, int64_t DV, int act_dtype) {
    return DK == 128 && DV == 128 && act_dtype == GDN_BF16;
}

int chunk_fwd(const ChunkLaunch& L, cudaStream_t s) {
    using namespace cf;
    if (smem_optin((const void*)chunk_fwd_kernel<0>, SMEM_BYTES) != cudaSuccess ||
        smem_optin((const void*)chunk_fwd_kernel<1>, SMEM_BYTES) != cudaSuccess ||
        smem_optin((const void*)chunk_fwd_kernel<2>, SMEM_BYTES) != cudaSuccess)
        return GDN_ERR_LAUNCH;
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
    a.s0_out = (uint8_t*)L.s0_out;
    dim3 grid((unsigned)(L.N * L.HV), 1);
    if (L.s0_out) {
        if (!L.ckpt) return GDN_ERR_ARGUMENT;
        const int64_t maxlen = L.max_seqlen > 0 ? L.max_seqlen : (L.cu ? L.B * L.T : L.T);
        const int64_t segs = (((maxlen + 63) / 64) + L.ckpt_every - 1) / L.ckpt_every;
        grid.y = (unsigned)(segs > 0 ? segs : 1);
        a.ht = nullptr;
        a.o_mode = 2;
    }
    if (grid.x == 0) return GDN_OK;
    if (a.s0_out) chunk_fwd_kernel<1><<<grid, NTHR, SMEM_BYTES, s>>>(a);
    else if (a.o_mode == 0 && !a.zero_v && !a.h0_identity && !a.ht_accumulate)
        chunk_fwd_kernel<0><<<grid, NTHR, SMEM_BYTES, s>>>(a);
    else chunk_fwd_kernel<2><<<grid, NTHR, SMEM_BYTES, s>>>(a);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
