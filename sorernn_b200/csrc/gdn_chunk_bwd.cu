// Chunked gated-delta-rule backward on sm_100a (tcgen05 UMMA, TMA / bulk-copy fed, TMEM accumulators).
//
// One CTA (512 threads) per (sequence, value head) walks the chunks in reverse, carrying dS (the gradient
// of the state at the chunk end, fp32 in TMEM). The chunk-start states S0 are not saved by the forward:
// a segment-parallel pass of the forward kernel (chunk_fwd in recompute mode) rebuilds them from the
// forward's checkpoints and writes one record per (chunk, head) to the workspace: the bf16 operand tiles of
// S0^T, -W, T = (I + A)^-1, Delta^T and the low part of Dd^T (kBwdRecordBytes, kernels.h), so the
// triangular solve and the W, U, Delta products run once per chunk, in that pass; this kernel bulk-copies
// the record with the chunk's Q, K, dO tiles and recomputes only the Gram matrix D1 = [Q;K] K^T.
//
// With qn = q/nq, kn = k/nk (the raw bf16 tiles feed the tensor cores; norms are applied in fp32),
// Gamma = in-chunk cumsum(g), E_ij = exp(Gamma_i - Gamma_j), P, A from D1, and T, W, Delta from the
// record (the algebra of tests/test_chunk_algebra.py::chunked_backward):
//   dDelta = P^T dO + Kd dS                      Kd = kn e^(Gamma_C - Gamma)
//   dS0    = scale (qn e^Gamma)^T dO + e^Gamma_C dS - W^T dDelta
//   dP     = dO Delta^T,  dPs = lower_incl(dP . scale E)
//   dqn    = scale e^Gamma (dO S0^T) + dPs kn
//   dkn    = dPs^T qn + (Delta dS^T) e^(Gamma_C-Gamma) + beta e^Gamma dKb + (dG + dG^T) kn
//   dVb = T^T dDelta, dv = beta dVb;   dW = -dDelta S0^T, dKb = T^T dW
//   dA  = strict_lower(-Z T^T),  Z = dVb (beta V)^T + dKb (beta e^Gamma kn)^T
//   dbeta = dVb.v + e^Gamma dKb.kn + rowsum(dA . G E);   dG = dA . beta E
//   dGamma = rowsum-colsum(dA . A) + rowsum-colsum(dP . P) + scale e^Gamma qn.(S0 dO) + beta e^Gamma dKb.kn
//            - kn.dKst_j  (+ sum_j kn.dKst_j + e^Gamma_C <dS, S0> on the last row);  dg = reverse cumsum
//   dq = (dqn - qn (qn.dqn)) / nq,  dk likewise (chain rule through the L2 norm)
// MMAs are issued by two threads, 0 and 32, each committing its groups to its own mbarriers (thread 0:
// bar_mma; thread 32: bar_mma2, and bar_mma3 for its share of step 6's first group), so two issuers halve the
// issue time of the larger steps, and a phase waits only for the groups it reads. Issue loops are unrolled
// over hoisted descriptors (one N = 64 UMMA per ~50 cycles against ~100 rolled), except thread 0's in step 10,
// whose unrolled form spills registers (its issuers hold the dq operands live); thread 32's step-10 loop is
// unrolled (sweep 1.440 -> 1.429 ms at config 1). Products that accumulate into one TMEM region stay on one thread.
// Every GEMM is an M = 128 UMMA with a 128-wide dimension on the TMEM lanes. The three 64 x 64 x K
// products (dP, Z, dA) use a 128-row A operand of which one 64-row half is ignored; Z and dA put their
// rows on lanes 64-127, where the same threads also hold the K K^T rows of the recomputed Gram matrix.
// Operands are bf16 with the raw q/k tiles exact; the products that carry the state gradient's large
// dynamic range take a second bf16 "lo" operand (x - bf16(x)) for dS (in dS K^T and dS Dd^T), dDelta
// (in dDelta T, S0 dDelta^T and the dS update) and P'' (in dO^T P''^T), which keeps every gradient
// within the bf16 tolerance.
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "launch.h"
#include "sm100.cuh"
#include "tmap.h"

namespace gdn {
using namespace sm100;

namespace cb {
constexpr int NTHR = 512;  // 16 warps: 4 per TMEM lane quadrant, each owning 16 of 64 columns
// shared memory carve (bytes from a 1024-aligned base)
constexpr uint32_t OFF_QK = 0, QK_BLK = 16384;  // per d-block kb: [Q 8 KB | K 8 KB] (64 tokens x 128 B)
constexpr uint32_t OFF_V = 32768;                // [kb][8 KB]
constexpr uint32_t OFF_DO = 49152;               // [kb][8 KB]
constexpr uint32_t OFF_S0 = 65536;               // S0^T bf16 [dv][dk], 2 dk-blocks x 16 KB (workspace image)
constexpr uint32_t OFF_DS = 98304;               // dS^T bf16 [dv][dk]
constexpr uint32_t OFF_W = 131072;               // -W bf16 [j][dk], 2 d-blocks x 8 KB
constexpr uint32_t OFF_T = 147456;    // T bf16 [i][j]
constexpr uint32_t OFF_DEL = 155648;  // Delta^T bf16 [dv][j] -> Dd^T; later dG fp32 [64][64]
constexpr uint32_t OFF_DD = 172032;   // dDelta^T bf16 [dv][j]
constexpr uint32_t OFF_PS = 188416;   // P'' bf16 [i][j] -> dPs / nk_j
constexpr uint32_t OFF_PS2 = 196608;  // dPs / (nq_i nk_j) -> Z bf16 [j][m]
constexpr uint32_t OFF_A = 204800;    // 17 KB: the dDelta^T lo tile (OFF_DDL) in steps 7-8
constexpr int AST = 68;
constexpr int NVEC = 14;
constexpr uint32_t OFF_VEC = OFF_A + 64 * AST * 4;     // NVEC x 64 fp32
constexpr uint32_t OFF_RED = OFF_VEC + NVEC * 64 * 4;  // 4 reduction buffers of 4 x 64 fp32
constexpr uint32_t OFF_BAR = OFF_RED + 4 * 256 * 4;    // 2 mbarriers, TMEM slot, scalars
constexpr uint32_t SMEM_BYTES = OFF_BAR + 128 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
constexpr uint32_t OFF_DVB = OFF_S0;          // dVb^T bf16 [dv][j]   (S0 dead after step 8)
constexpr uint32_t OFF_DWT = OFF_S0 + 16384;  // dW^T bf16 [dk][i]
constexpr uint32_t OFF_DKB = OFF_DS;          // dKb^T bf16 [dk][j]   (dS tile dead after step 8)
constexpr uint32_t OFF_GS = OFF_DS + 16384;   // (dG + dG^T) / (nk nk) bf16 [j][m]
constexpr uint32_t OFF_DDL = OFF_A;  // dDelta^T lo bf16 [dv][j] (16 KB)
// TMEM columns (fp32, 128 lanes)
constexpr uint32_t T_S = 0, T_D1 = 128, C192 = 192, C256 = 256, C320 = 320, C384 = 384, C448 = 448, T_COLS = 512;
}  // namespace cb

struct ChunkBwdArgs {
    CUtensorMap tq, tk, tv, tdo;
    const void* g;
    const void* beta;
    const uint8_t* s0_tiles;  // per (chunk, head) kBwdRecordBytes records: S0^T, TB, TV, T tile images
    const float* dht;
    void* dq;  // bf16 [tok][H][128], or fp32 accumulators when accumulate_qk
    void* dk;
    void* dv;
    float* dg;
    float* dbeta;
    float* dh0;
    const int64_t* cu;
    int* err;
    int64_t T;
    int N, H, HV, g_dtype, beta_dtype;
    float scale;
    int l2norm, accumulate_qk;
    int state_grad_only;  // 1: only dS is carried (steps 1-8b) and dh0 written; no token gradients
};

__device__ __forceinline__ uint32_t pk_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void st8(uint8_t* dst, const float* v) {
    uint4 u;
    u.x = pk_bf16(v[0], v[1]);
    u.y = pk_bf16(v[2], v[3]);
    u.z = pk_bf16(v[4], v[5]);
    u.w = pk_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(dst) = u;
}
__device__ __forceinline__ float bfv(const uint8_t* base, uint32_t off) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(base + off));
}
// element (row r, col c) of a [rows][128] bf16 tile stored as two 64-column swizzled blocks `blk` bytes apart
__device__ __forceinline__ float tile128(const uint8_t* base, uint32_t blk, int r, int c) {
    return bfv(base, (uint32_t)(c >> 6) * blk + sw128_off(r, c & 63));
}
__device__ __forceinline__ void sync_tc() {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}
__device__ __forceinline__ void bwait(uint64_t* bar, uint32_t parity, int* err, int code, bool& ok) {
    ok = mbar_wait(bar, parity, err, code, ok ? (1u << 22) : 1u) && ok;
}
__device__ __forceinline__ void mwait(uint64_t* bar, uint32_t& phase, int* err, int code, bool& ok) {
    bwait(bar, phase, err, code, ok);
    phase ^= 1u;
    tc_fence_after();
}
__device__ __forceinline__ void ld32c(uint32_t taddr, float (&v)[32]) {
    tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(v));
    tmem_ld16(taddr + 16, *reinterpret_cast<float(*)[16]>(v + 16));
    tmem_wait_ld();
}
__device__ __forceinline__ void ld16c(uint32_t taddr, float (&v)[16]) {
    tmem_ld16(taddr, v);
    tmem_wait_ld();
}
__device__ __forceinline__ void ld16x2(uint32_t ta, float (&va)[16], uint32_t tb, float (&vb)[16]) {
    tmem_ld16(ta, va);
    tmem_ld16(tb, vb);
    tmem_wait_ld();
}
// L2 prefetches: a chunk's tiles and record are brought into L2 two chunks before their shared-memory loads
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((uint64_t)src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_tile_l2(const CUtensorMap* map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"((uint64_t)map), "r"(c0),
                 "r"(c1), "r"(c2)
                 : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// v[k] holds this thread's value for column 16*cq + k. Afterwards lane l holds the sum over the warp's
// 32 lanes of column 16*cq + (l & 15) (recursive halving over lane bits 3..0, then one exchange across
// the two half-warps: 16 shuffles for 16 columns).
__device__ __forceinline__ float warp_colsum16(float (&v)[16]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1) {
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int k = 0; k < off; ++k) {
            const float send = up ? v[k] : v[k + off];
            const float keep = up ? v[k + off] : v[k];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
}
// Column sums over all 128 TMEM lanes: every warp deposits its 16 column partials in red[lg][col];
// after a barrier colsum(red, col) is the total. Called by all 16 warps.
__device__ __forceinline__ void deposit_colsum(float (&v)[16], float* red, int lg, int cq) {
    const float s = warp_colsum16(v);
    if ((threadIdx.x & 31) < 16) red[lg * 64 + 16 * cq + (threadIdx.x & 15)] = s;
}
__device__ __forceinline__ float colsum(const float* red, int col) {
    return red[col] + red[64 + col] + red[128 + col] + red[192 + col];
}
// o[j] = v[base + j], j < 16, as four float4 loads (base % 4 == 0): a warp-uniform float4 load costs
// about 2.4 shared-memory cycles against 1.1 for each of four scalar loads.
__device__ __forceinline__ void vec16(const float* v, int base, float (&o)[16]) {
    const float4* p = reinterpret_cast<const float4*>(v + base);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 x = p[q];
        o[4 * q] = x.x;
        o[4 * q + 1] = x.y;
        o[4 * q + 2] = x.z;
        o[4 * q + 3] = x.w;
    }
}
__device__ __forceinline__ void vec8(const float* v, int base, float (&o)[8]) {
    const float4* p = reinterpret_cast<const float4*>(v + base);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const float4 x = p[q];
        o[4 * q] = x.x;
        o[4 * q + 1] = x.y;
        o[4 * q + 2] = x.z;
        o[4 * q + 3] = x.w;
    }
}

__global__ void __launch_bounds__(cb::NTHR, 1) chunk_bwd_kernel(const __grid_constant__ ChunkBwdArgs a) {
    using namespace cb;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* dGm = (float*)(sm + OFF_DEL);
    float* vG = (float*)(sm + OFF_VEC);
    float* vEG = vG + 64;
    float* vB = vG + 128;
    float* vX = vG + 192;   // e^(G_C - G) / nk
    float* vNQ = vG + 256;  // 1/nq (0 on padded rows)
    float* vNK = vG + 320;  // 1/nk (0 on padded rows)
    float* vDG = vG + 384;  // dGamma
    float* vDB = vG + 448;  // dbeta
    float* vR4 = vG + 512;  // kn_j . dKst_j
    float* vEN = vG + 576;   // e^G / nk
    float* vBEN = vG + 640;  // beta e^G / nk
    float* vQ1 = vG + 704;   // scale e^G_i
    float* vQ2 = vG + 768;   // dq norm term: (1/nq)^2 (scale e^G colsum(qn.S0dO) + colsum(qn.QB))
    float* vK3 = vG + 832;   // dk norm term: (1/nk)^2 colsum(k.u)
    float* red0 = (float*)(sm + OFF_RED);
    float* red1 = red0 + 256;
    float* red2 = red0 + 512;
    float* red3 = red0 + 768;
    uint64_t* bar_in = (uint64_t*)(sm + OFF_BAR);
    uint64_t* bar_mma = bar_in + 1;
    uint64_t* bar_v = bar_in + 2;  // V tile reloaded for Z1 (its region holds the Dd lo tile in steps 5-8)
    uint64_t* bar_mma2 = bar_in + 13;  // second MMA group of a step (after the scalars below)
    uint64_t* bar_mma3 = bar_in + 14;  // thread 32's share of step 6's first group
    uint32_t* tmem_slot = (uint32_t*)(bar_in + 3);
    float* scal = (float*)(bar_in + 4);  // [0] e^G_C, [1..16] <dS, S0> per warp

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lg = warp & 3, cq = warp >> 2;  // TMEM lane quadrant; column quarter
    const int row = 32 * lg + lane;  // TMEM lane of this thread
    const int n = blockIdx.x / a.HV, hv = blockIdx.x % a.HV, hq = hv / (a.HV / a.H);
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t len = eos - bos;
    const int nchunks = (int)((len + 63) / 64);

    // index of this sequence's first chunk in the flattened chunk list (S0 tile slots)
    int64_t cbase = 0;
    if (!a.cu) {
        cbase = (int64_t)n * ((a.T + 63) / 64);
    } else {
        int64_t part = 0;
        for (int m = tid; m < n; m += NTHR) part += (a.cu[m + 1] - a.cu[m] + 63) / 64;
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0) ((int64_t*)red0)[warp] = part;
        __syncthreads();
        for (int w = 0; w < NTHR / 32; ++w) cbase += ((int64_t*)red0)[w];
        __syncthreads();
    }

    if (tid == 0) {
        mbar_init(bar_in, 1);
        mbar_init(bar_mma, 1);
        mbar_init(bar_v, 1);
        mbar_init(bar_mma2, 1);
        mbar_init(bar_mma3, 1);
        fence_barrier_init();
        prefetch_tmap(&a.tq);
        prefetch_tmap(&a.tk);
        prefetch_tmap(&a.tv);
        prefetch_tmap(&a.tdo);
    }
    if (warp == 0) tmem_alloc(tmem_slot, T_COLS);
    sync_tc();
    const uint32_t tm = *tmem_slot;
    const uint32_t lb = (uint32_t)(32 * lg) << 16;
    const uint32_t tS = tm + T_S, tD1 = tm + T_D1;
    uint32_t mph = 0, mph2 = 0, mph3 = 0;
    bool ok = true;
    const uint32_t sb = smem_u32(sm);

    // dS^T <- dht^T (TMEM lane = dv, columns dk)
    {
        const float* dht = a.dht ? a.dht + ((int64_t)n * a.HV + hv) * 16384 : nullptr;
#pragma unroll 1
        for (int c0 = 0; c0 < 32; c0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = dht ? dht[(32 * cq + c0 + i) * 128 + row] : 0.f;
            tmem_st16(tS + lb + 32 * cq + c0, v);
        }
        tmem_wait_st();
    }

    // A chunk's inputs arrive on bar_in in two parts (one expect_tx for both): part A (Q, dO, and the record's
    // S0^T and Dd^T low part, where V goes later) as soon as the previous chunk's step-11 MMAs completed, the
    // last readers of those regions; part B (K, and the record's -W | T and Delta^T) at the chunk's end.
    auto issue_inputs_a = [&](int c) {
        const int tok0 = (int)(bos + 64 * c);
        mbar_arrive_expect_tx(bar_in, 6 * 8192 + 32768 + 24576 + 2 * 16384);
#pragma unroll 1
        for (int kb = 0; kb < 2; ++kb) {
            tma_load_3d(sm + OFF_QK + kb * QK_BLK, &a.tq, bar_in, kb * 64, hq, tok0);
            tma_load_3d(sm + OFF_DO + kb * 8192, &a.tdo, bar_in, kb * 64, hv, tok0);
        }
        const uint8_t* rec = a.s0_tiles + ((cbase + c) * a.HV + hv) * kBwdRecordBytes;
        bulk_load(sm + OFF_S0, rec, 32768, bar_in);
        bulk_load(sm + OFF_V, rec + kBwdRecDdl, 16384, bar_in);
    };
    auto issue_inputs_b = [&](int c) {
        const int tok0 = (int)(bos + 64 * c);
#pragma unroll 1
        for (int kb = 0; kb < 2; ++kb)
            tma_load_3d(sm + OFF_QK + kb * QK_BLK + 8192, &a.tk, bar_in, kb * 64, hq, tok0);
        const uint8_t* rec = a.s0_tiles + ((cbase + c) * a.HV + hv) * kBwdRecordBytes;
        bulk_load(sm + OFF_W, rec + kBwdRecW, 24576, bar_in);  // -W | T, contiguous here and there
        bulk_load(sm + OFF_DEL, rec + kBwdRecDel, 16384, bar_in);
    };
    auto prefetch_chunk = [&](int c) {  // every tile and the record chunk c reads, into L2
        const int tok0 = (int)(bos + 64 * c);
#pragma unroll 1
        for (int kb = 0; kb < 2; ++kb) {
            prefetch_tile_l2(&a.tq, kb * 64, hq, tok0);
            prefetch_tile_l2(&a.tk, kb * 64, hq, tok0);
            prefetch_tile_l2(&a.tdo, kb * 64, hv, tok0);
            prefetch_tile_l2(&a.tv, kb * 64, hv, tok0);
        }
        prefetch_l2(a.s0_tiles + ((cbase + c) * a.HV + hv) * kBwdRecordBytes, (uint32_t)kBwdRecordBytes);
    };
    if (tid == 0 && nchunks > 0) {
        issue_inputs_a(nchunks - 1);
        issue_inputs_b(nchunks - 1);
        if (nchunks > 1) prefetch_chunk(nchunks - 2);
    }
    uint32_t in_phase = 0, v_phase = 0;
    const uint32_t aQ = sb + OFF_QK, aK = sb + OFF_QK + 8192, aV = sb + OFF_V, aDO = sb + OFF_DO;

    uint32_t g_next = 0u, b_next = 0u;  // gates of the chunk processed next (threads 0-63), raw
    if (tid < 64 && nchunks > 0) {
        const int64_t t0 = bos + 64 * (int64_t)(nchunks - 1);
        const bool in = tid < len - 64 * (int64_t)(nchunks - 1);
        if (in) {
            g_next = ld_gate_raw(a.g, a.g_dtype, (t0 + tid) * a.HV + hv);
            b_next = ld_gate_raw(a.beta, a.beta_dtype, (t0 + tid) * a.HV + hv);
        }
    }
    for (int c = nchunks - 1; c >= 0; --c) {
        const int64_t tok0 = bos + 64 * (int64_t)c;
        const int nv = (len - 64 * (int64_t)c) < 64 ? (int)(len - 64 * (int64_t)c) : 64;
        if (tid == 0 && c >= 2) prefetch_chunk(c - 2);

        // ---- 1. gates; wait for this chunk's tiles ------------------------------------------------------
        if (tid < 64) {
            float x = gate_f(g_next, a.g_dtype);
            vB[tid] = gate_f(b_next, a.beta_dtype);
            if (c > 0) {  // gates of chunk c-1 (always 64 tokens): their latency hides behind this chunk
                const int64_t gi = (tok0 - 64 + tid) * a.HV + hv;
                g_next = ld_gate_raw(a.g, a.g_dtype, gi);
                b_next = ld_gate_raw(a.beta, a.beta_dtype, gi);
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            vG[tid] = x;
            vDG[tid] = 0.f;
            vDB[tid] = 0.f;
        }
        bwait(bar_in, in_phase, a.err, 11, ok);
        in_phase ^= 1u;

        // ---- 2. R1: D1 = [Q;K] K^T (rows 0-63 Q K^T, 64-127 K K^T; kept for the whole chunk) ----------
        if (tid == 0) {
            tc_fence_after();
            const uint32_t id = idesc_bf16(128, 64, 0, 0);
            const uint64_t dQ = desc_kmajor(aQ), dK = desc_kmajor(aK);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t o = (ks >> 2) * QK_BLK + (ks & 3) * 32;
                umma_bf16(tD1, desc_at(dQ, o), desc_at(dK, o), id, ks > 0);
            }
            umma_commit(bar_mma);
        }
        __syncthreads();
        if (tid >= 32 && tid < 64) vG[tid] += vG[31];
        {  // row norms (4 threads per row, 32 elements each; rows 0-63 q, 64-127 k)
            const int r = tid >> 2, part = tid & 3, i = r & 63;
            const uint8_t* rowp = sm + OFF_QK + (part >> 1) * QK_BLK + (r < 64 ? 0 : 8192) + i * 128;
            float ss = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                // chunk order rotated by (2 d-block + row parity): the 8 lanes of a quarter-warp read 8
                // distinct 16-byte bank groups (the sum is order-free)
                const int ch = (c + 4 * (part & 1) + 2 * (part >> 1) + (r & 1)) & 7;
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
            const float eg = __expf(vG[tid]);
            vEG[tid] = eg;
            vX[tid] = __expf(vG[63] - vG[tid]) * vNK[tid];
            vEN[tid] = eg * vNK[tid];
            vBEN[tid] = vB[tid] * eg * vNK[tid];
            vQ1[tid] = a.scale * eg;
        }
        if (tid == 64) scal[0] = __expf(vG[63]);
        __syncthreads();
        mwait(bar_mma, mph, a.err, 12, ok);

        // ---- 3. D1 rows 0-63 -> P'' (bf16 hi and lo); dS^T -> hi tile and <dS, S0>. T, -W, Delta^T and
        //         the Dd^T low part arrived with the inputs (the recompute pass built them for its own state
        //         update)
        if (lg < 2) {  // P''_ij = scale qn_i.kn_j E_ij (j <= i)
            float v[16];
            ld16c(tD1 + lb + 16 * cq, v);
            const int i = row;
            const float gi = vG[i], f = a.scale * vNQ[i];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int jj = 16 * cq + j;
                v[j] = (jj <= i) ? f * v[j] * vNK[jj] * __expf(gi - vG[jj]) : 0.f;
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {  // hi tile, and its lo part where dPs2 goes later (idle until step 7)
                float lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) lo[e] = v[8 * q + e] - __bfloat162float(__float2bfloat16_rn(v[8 * q + e]));
                st8(sm + OFF_PS + sw128_off(i, 16 * cq + 8 * q), v + 8 * q);
                st8(sm + OFF_PS2 + sw128_off(i, 16 * cq + 8 * q), lo);
            }
        }
        {  // dS^T -> bf16 hi tile and its lo part (dk block 0 at OFF_DD, 1 at OFF_A: both idle until step 7),
           // <dS, S0>
            float dss = 0.f;
            uint8_t* lo_blk = sm + ((cq >> 1) ? OFF_A : OFF_DD);
#pragma unroll 1
            for (int c0 = 0; c0 < 32; c0 += 16) {
                float v[16], lo[16];
                tmem_ld16(tS + lb + 32 * cq + c0, v);
                tmem_wait_ld();
                const uint32_t cb_ = 32 * (cq & 1) + c0;
                const uint32_t s0 = sw128_off(row, cb_), s1 = sw128_off(row, cb_ + 8);
                const uint32_t o0 = (cq >> 1) * 16384 + s0, o1 = (cq >> 1) * 16384 + s1;
                st8(sm + OFF_DS + o0, v);
                st8(sm + OFF_DS + o1, v + 8);
#pragma unroll
                for (int e = 0; e < 16; ++e) lo[e] = v[e] - __bfloat162float(__float2bfloat16_rn(v[e]));
                st8(lo_blk + s0, lo);
                st8(lo_blk + s1, lo + 8);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    dss = fmaf(v[e], bfv(sm + OFF_S0, o0 + 2 * e), dss);
                    dss = fmaf(v[8 + e], bfv(sm + OFF_S0, o1 + 2 * e), dss);
                }
            }
            dss = warp_sum(dss);
            if (lane == 0) scal[1 + warp] = dss;
        }
        fence_async_smem();
        sync_tc();

        // ---- 6. dO^T P''^T (320); dS^T K^T, hi and lo (384); dP = [dO;-] Delta^T (448); QA = S0 dO^T (192)
        if (tid == 0) {
            const uint32_t id_kk = idesc_bf16(128, 64, 0, 0);
            const uint64_t dDS = desc_kmajor(sb + OFF_DS), dK = desc_kmajor(aK);
            const uint64_t dLo0 = desc_kmajor(sb + OFF_DD), dLo1 = desc_kmajor(sb + OFF_A);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                umma_bf16(tm + C384, desc_at(dDS, kb * 16384 + ko), desc_at(dK, kb * QK_BLK + ko), id_kk, ks > 0);
                umma_bf16(tm + C384, desc_at(kb ? dLo1 : dLo0, ko), desc_at(dK, kb * QK_BLK + ko), id_kk,
                          1);  // dS lo . K
            }
            umma_commit(bar_mma);  // dDelta's two products: step 7 starts on them
        } else if (tid == 32) {  // a second issuing thread: its MMAs and commits are tracked apart from thread 0's
            const uint32_t id_km = idesc_bf16(128, 64, 0, 1), id_mk = idesc_bf16(128, 64, 1, 0);
            const uint32_t id_mm = idesc_bf16(128, 64, 1, 1);
            const uint64_t dDOm = desc_mnmajor(aDO, 8192), dPS = desc_mnmajor(sb + OFF_PS, 8192),
                           dPS2 = desc_mnmajor(sb + OFF_PS2, 8192);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {  // K = i: dDelta's first product
                umma_bf16(tm + C320, desc_at(dDOm, ks * 2048), desc_at(dPS, ks * 2048), id_mm, ks > 0);
                umma_bf16(tm + C320, desc_at(dDOm, ks * 2048), desc_at(dPS2, ks * 2048), id_mm, 1);
            }
            umma_commit(bar_mma3);
            if (!a.state_grad_only) {  // dP and QA feed only the token gradients
                const uint64_t dDOk = desc_kmajor(aDO), dDEL = desc_mnmajor(sb + OFF_DEL, 8192),
                               dS0 = desc_mnmajor(sb + OFF_S0, 16384);
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint32_t ok_ = (ks >> 2) * 8192 + (ks & 3) * 32;
                    umma_bf16(tm + C448, desc_at(dDOk, ok_), desc_at(dDEL, ks * 2048), id_km, ks > 0);
                    umma_bf16(tm + C192, desc_at(dS0, ks * 2048), desc_at(dDOk, ok_), id_mk, ks > 0);
                }
            }
            umma_commit(bar_mma2);  // dP and QA: run while step 7 forms dDelta (without them: no new MMAs)
        }
        // ---- 7. dDelta^T = (320) + (384) diag(vX) -> tile; r4; dP -> dPs tiles, X_P sums -------------------
        {
            float d1[16], d2[16], de[16], x16[16];
            vec16(vX, 16 * cq, x16);
            // Delta x (= Dd) to ~16 bits: bf16(bf16(Delta) x) from the Delta^T tile plus the Dd^T low part
            // (shared-memory operands only: formed while step 6's MMAs run)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t off = sw128_off(row, 16 * cq + 8 * h);
                const uint4 dh = *reinterpret_cast<const uint4*>(sm + OFF_DEL + off);
                const uint4 dl = *reinterpret_cast<const uint4*>(sm + OFF_V + off);
                const __nv_bfloat162* ph = reinterpret_cast<const __nv_bfloat162*>(&dh);
                const __nv_bfloat162* pl = reinterpret_cast<const __nv_bfloat162*>(&dl);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 fh = __bfloat1622float2(ph[e]), fl = __bfloat1622float2(pl[e]);
                    const int j = 8 * h + 2 * e;
                    de[j] = __bfloat162float(__float2bfloat16_rn(fh.x * x16[j])) + fl.x;
                    de[j + 1] = __bfloat162float(__float2bfloat16_rn(fh.y * x16[j + 1])) + fl.y;
                }
            }
            mwait(bar_mma, mph, a.err, 15, ok);
            mwait(bar_mma3, mph3, a.err, 27, ok);
            tmem_ld16(tm + C320 + lb + 16 * cq, d1);
            tmem_ld16(tm + C384 + lb + 16 * cq, d2);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                de[j] = de[j] * d2[j];  // kn_j . dKst_j partial over this lane (dv)
                d1[j] = fmaf(d2[j], x16[j], d1[j]);
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                float lo[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) lo[e] = d1[8 * q + e] - __bfloat162float(__float2bfloat16_rn(d1[8 * q + e]));
                st8(sm + OFF_DD + sw128_off(row, 16 * cq + 8 * q), d1 + 8 * q);
                st8(sm + OFF_DDL + sw128_off(row, 16 * cq + 8 * q), lo);
            }
            deposit_colsum(de, red0, lg, cq);
        }
        mwait(bar_mma2, mph2, a.err, 24, ok);
        if (!a.state_grad_only) {
            float v[16], p[16];
            ld16x2(tm + C448 + lb + 16 * cq, v, tD1 + lb + 16 * cq, p);
            if (lg < 2) {
                const int i = row;
                const float gi = vG[i], nq = vNQ[i];
                float d1v[16], d2v[16], rs = 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int jj = 16 * cq + j;
                    const bool m = jj <= i;
                    const float e = m ? __expf(gi - vG[jj]) : 0.f;
                    const float P = a.scale * p[j] * nq * vNK[jj] * e;
                    const float xp = m ? v[j] * P : 0.f;
                    rs += xp;
                    p[j] = xp;
                    const float dps = m ? v[j] * a.scale * e : 0.f;
                    d1v[j] = dps * vNK[jj];
                    d2v[j] = d1v[j] * nq;
                }
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    st8(sm + OFF_PS + sw128_off(i, 16 * cq + 8 * q), d1v + 8 * q);
                    st8(sm + OFF_PS2 + sw128_off(i, 16 * cq + 8 * q), d2v + 8 * q);
                }
                red2[cq * 64 + i] = rs;  // row i's four column-quarter partials, summed in fixed order below
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) p[j] = 0.f;
            }
            deposit_colsum(p, red1, lg, cq);
        }
        __syncthreads();
        if (tid < 64) {
            const float r4 = colsum(red0, tid);
            vR4[tid] = r4;
            vDG[tid] += colsum(red2, tid) - (colsum(red1, tid) + r4);
        }
        // dO <- dO scale e^G / nq in place (A operand of the dS update; the raw dO readers have finished)
#pragma unroll 1
        for (int it = 0; it < 1024 / NTHR; ++it) {
            const int e = tid + it * NTHR;
            const int i = e >> 4, cc = e & 15;
            uint8_t* pp = sm + OFF_DO + (cc >> 3) * 8192 + i * 128 + (((cc & 7) ^ (i & 7)) << 4);
            uint4 u = *reinterpret_cast<uint4*>(pp);
            const float f = a.scale * vEG[i] * vNQ[i];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                const float2 z = __bfloat1622float2(h[k2]);
                h[k2] = __floats2bfloat162_rn(z.x * f, z.y * f);
            }
            *reinterpret_cast<uint4*>(pp) = u;
        }
        if (!a.state_grad_only) {  // Delta^T -> Dd^T = Delta^T diag(vX) in place (thread owns row dv, 16 columns)
            float x16[16];
            vec16(vX, 16 * cq, x16);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint32_t off = sw128_off(row, 16 * cq + 8 * q);
                uint4 u = *reinterpret_cast<uint4*>(sm + OFF_DEL + off);
                __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
                for (int k2 = 0; k2 < 4; ++k2) {
                    const float2 z = __bfloat1622float2(h[k2]);
                    const int j = 8 * q + 2 * k2;
                    h[k2] = __floats2bfloat162_rn(z.x * x16[j], z.y * x16[j + 1]);
                }
                *reinterpret_cast<uint4*>(sm + OFF_DEL + off) = u;
            }
        }
        fence_async_smem();
        sync_tc();

        // ---- 8. dVb^T = dDelta^T T (256); S0 dDelta^T = -dW^T (320); QB = K^T dPs1^T (384);
        //         dK' = Q^T dPs2 + dS Dd^T (448). Thread 0 issues QB and dK', thread 32 dVb and -dW^T. All of it
        //         feeds only the token gradients: without them the chunk goes on to the dS update.
        if (a.state_grad_only) {
        } else if (tid == 0) {
            const uint32_t id_mm = idesc_bf16(128, 64, 1, 1);
            const uint64_t dQm = desc_mnmajor(aQ, QK_BLK), dPS2 = desc_mnmajor(sb + OFF_PS2, 8192);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)  // K = tokens
                umma_bf16(tm + C448, desc_at(dQm, ks * 2048), desc_at(dPS2, ks * 2048), id_mm, ks > 0);
            const uint64_t dDSm = desc_mnmajor(sb + OFF_DS, 16384), dDEL = desc_mnmajor(sb + OFF_DEL, 8192),
                           dVm = desc_mnmajor(sb + OFF_V, 8192);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {  // K = dv
                umma_bf16(tm + C448, desc_at(dDSm, ks * 2048), desc_at(dDEL, ks * 2048), id_mm, 1);
                umma_bf16(tm + C448, desc_at(dDSm, ks * 2048), desc_at(dVm, ks * 2048), id_mm, 1);  // dS hi . Dd lo
            }
            umma_commit(bar_mma);
        } else if (tid == 32) {
            const uint32_t id_km = idesc_bf16(128, 64, 0, 1), id_mm = idesc_bf16(128, 64, 1, 1);
            const uint32_t id_mk = idesc_bf16(128, 64, 1, 0);
            const uint64_t dKm = desc_mnmajor(aK, QK_BLK), dPSk = desc_kmajor(sb + OFF_PS), dDDk = desc_kmajor(sb + OFF_DD),
                           dDDLk = desc_kmajor(sb + OFF_DDL), dTm = desc_mnmajor(sb + OFF_T, 8192);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {  // K = tokens
                umma_bf16(tm + C384, desc_at(dKm, ks * 2048), desc_at(dPSk, ks * 32), id_mk, ks > 0);
                umma_bf16(tm + C256, desc_at(dDDk, ks * 32), desc_at(dTm, ks * 2048), id_km, ks > 0);
                umma_bf16(tm + C256, desc_at(dDDLk, ks * 32), desc_at(dTm, ks * 2048), id_km, 1);
            }
            const uint64_t dS0m = desc_mnmajor(sb + OFF_S0, 16384), dDDm = desc_mnmajor(sb + OFF_DD, 8192);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)  // K = dv
                umma_bf16(tm + C320, desc_at(dS0m, ks * 2048), desc_at(dDDm, ks * 2048), id_mm, ks > 0);
            umma_commit(bar_mma2);
        }
        if (!a.state_grad_only) {
            mwait(bar_mma, mph, a.err, 16, ok);
            mwait(bar_mma2, mph2, a.err, 25, ok);
        }
        if (tid == 0 && !a.state_grad_only) {  // the Dd lo tile is consumed: bring V back for Z1 (step 10)
            const int tok0i = (int)tok0;
            mbar_arrive_expect_tx(bar_v, 2 * 8192);
            tma_load_3d(sm + OFF_V, &a.tv, bar_v, 0, hv, tok0i);
            tma_load_3d(sm + OFF_V + 8192, &a.tv, bar_v, 64, hv, tok0i);
        }

        // ---- 8b. the dS tile's readers (B1b, hi part of dS Dd^T) are done: overwrite it with the lo part
        //          of dS and finish dS Dd^T; dS (TMEM) <- e^G_C dS + dOg^T Q + dDelta^T (-W). These MMAs
        //          complete before the step-10 commit, ahead of any write to the tiles they read.
        {
            const float eGC = scal[0];
#pragma unroll 1
            for (int c0 = 0; c0 < 32; c0 += 16) {
                float v[16], lo[16];
                tmem_ld16(tS + lb + 32 * cq + c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    lo[e] = v[e] - __bfloat162float(__float2bfloat16_rn(v[e]));
                    v[e] *= eGC;
                }
                const uint32_t blk = (cq >> 1) * 16384, cb_ = 32 * (cq & 1) + c0;
                st8(sm + OFF_DS + blk + sw128_off(row, cb_), lo);
                st8(sm + OFF_DS + blk + sw128_off(row, cb_ + 8), lo + 8);
                tmem_st16(tS + lb + 32 * cq + c0, v);
            }
            tmem_wait_st();
        }
        fence_async_smem();
        sync_tc();
        if (tid == 0 && !a.state_grad_only) {  // dK' (thread 0, after its other dK' products); dS update (thread 32)
            const uint32_t id_mm = idesc_bf16(128, 64, 1, 1);
            const uint64_t dDSm = desc_mnmajor(sb + OFF_DS, 16384), dDEL = desc_mnmajor(sb + OFF_DEL, 8192);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)  // K = dv
                umma_bf16(tm + C448, desc_at(dDSm, ks * 2048), desc_at(dDEL, ks * 2048), id_mm, 1);
        } else if (tid == 32) {
            const uint32_t id_mm128 = idesc_bf16(128, 128, 1, 1), id_km128 = idesc_bf16(128, 128, 0, 1);
            const uint64_t dDOm = desc_mnmajor(aDO, 8192), dQm = desc_mnmajor(aQ, QK_BLK), dDDk = desc_kmajor(sb + OFF_DD),
                           dDDLk = desc_kmajor(sb + OFF_DDL), dWm = desc_mnmajor(sb + OFF_W, 8192);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {  // K = tokens
                umma_bf16(tS, desc_at(dDOm, ks * 2048), desc_at(dQm, ks * 2048), id_mm128, 1);
                umma_bf16(tS, desc_at(dDDk, ks * 32), desc_at(dWm, ks * 2048), id_km128, 1);
                umma_bf16(tS, desc_at(dDDLk, ks * 32), desc_at(dWm, ks * 2048), id_km128, 1);
            }
        }

        if (a.state_grad_only) {  // the dS update lands; every reader of this chunk's tiles is done
            if (tid == 32) umma_commit(bar_mma2);
            mwait(bar_mma2, mph2, a.err, 28, ok);
            if (tid == 0 && c > 0) {
                issue_inputs_a(c - 1);
                issue_inputs_b(c - 1);
            }
            continue;
        }

        // ---- 9. dv, dVb tile, dVb.v; dW^T tile; qn.(S0 dO) and qn.QB -------------------------------------
        bwait(bar_v, v_phase, a.err, 21, ok);  // V is back (reloaded after step 8)
        v_phase ^= 1u;
        {
            float v[16], r2[16], w[16], b16[16];
            ld16x2(tm + C256 + lb + 16 * cq, v, tm + C320 + lb + 16 * cq, w);  // dVb^T[dv][j], -dW^T[dk][i]
            vec16(vB, 16 * cq, b16);
            // dv[token][hv][dv]: this thread's column, tokens 16 cq .. 16 cq + 15 (stride HV x 128)
            __nv_bfloat16* dvp = (__nv_bfloat16*)a.dv + ((tok0 + 16 * cq) * a.HV + hv) * 128 + row;
            const int64_t vstride = (int64_t)a.HV * 128;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int jj = 16 * cq + j;
                r2[j] = v[j] * tile128(sm + OFF_V, 8192, jj, row);
                if (jj < nv) dvp[j * vstride] = __float2bfloat16_rn(v[j] * b16[j]);
                w[j] = -w[j];
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                st8(sm + OFF_DVB + sw128_off(row, 16 * cq + 8 * q), v + 8 * q);
                st8(sm + OFF_DWT + sw128_off(row, 16 * cq + 8 * q), w + 8 * q);
            }
            deposit_colsum(r2, red0, lg, cq);
        }
        float qa[16], qb[16];  // dqn^T pieces [dk][i] for this thread's 16 tokens
        {
            ld16x2(tm + C192 + lb + 16 * cq, qa, tm + C384 + lb + 16 * cq, qb);
            float xa[16], xb[16], nq16[16];
            vec16(vNQ, 16 * cq, nq16);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = 16 * cq + j;
                const float qn = tile128(sm + OFF_QK, QK_BLK, i, row) * nq16[j];
                xa[j] = qn * qa[j];
                xb[j] = qn * qb[j];
            }
            deposit_colsum(xa, red1, lg, cq);
            deposit_colsum(xb, red2, lg, cq);
        }
        fence_async_smem();
        sync_tc();

        // ---- 10. dKb^T = dW^T T (192) ; Z1 = [-; dVb] V^T (256, rows j on lanes 64-127) ------------------
        if (tid == 0) {  // dKb (thread 0) and Z1 (thread 32); each commit also covers that thread's step-8b MMAs
            const uint32_t id_km = idesc_bf16(128, 64, 0, 1);
            const uint64_t dDWk = desc_kmajor(sb + OFF_DWT), dTm = desc_mnmajor(sb + OFF_T, 8192);
#pragma unroll 1
            for (int ks = 0; ks < 4; ++ks)
                umma_bf16(tm + C192, desc_at(dDWk, ks * 32), desc_at(dTm, ks * 2048), id_km, ks > 0);
            umma_commit(bar_mma);
        } else if (tid == 32) {
            const uint32_t id_mk = idesc_bf16(128, 64, 1, 0);
            const uint64_t dDVBm = desc_mnmajor(sb + OFF_DVB - 16384, 16384), dVk = desc_kmajor(aV);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                umma_bf16(tm + C256, desc_at(dDVBm, ks * 2048), desc_at(dVk, (ks >> 2) * 8192 + (ks & 3) * 32), id_mk,
                          ks > 0);
            umma_commit(bar_mma2);
        }
        if (tid < 64) {  // per-column terms of the dq epilogue; dGamma and dbeta contributions
            const float c1 = colsum(red1, tid);
            vQ2[tid] = vNQ[tid] * vNQ[tid] * fmaf(vQ1[tid], c1, colsum(red2, tid));
            vDG[tid] += vQ1[tid] * c1;      // rowsum(dO . O_inter)
            vDB[tid] += colsum(red0, tid);  // dVb . v
        }
        __syncthreads();
        {  // dq epilogue: dqn = scale e^G (dO S0^T) + dPs kn;  dq = dqn / nq - q_raw (qn . dqn) / nq^2
            float xs[16], s16[16], nq16[16], c16[16];
            vec16(vQ1, 16 * cq, s16);
            vec16(vNQ, 16 * cq, nq16);
            vec16(vQ2, 16 * cq, c16);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = 16 * cq + j;
                const float dqn = fmaf(s16[j], qa[j], qb[j]);
                xs[j] = a.l2norm ? fmaf(-tile128(sm + OFF_QK, QK_BLK, i, row), c16[j], dqn * nq16[j]) : dqn;
            }
            // dq[token][hq][dk]: this thread's column, tokens 16 cq .. (stride H x 128)
            const int64_t qidx = ((tok0 + 16 * cq) * a.H + hq) * 128 + row, qstride = (int64_t)a.H * 128;
            if (a.accumulate_qk) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (16 * cq + j < nv) atomicAdd((float*)a.dq + qidx + j * qstride, xs[j]);
            } else {
                __nv_bfloat16* dqp = (__nv_bfloat16*)a.dq + qidx;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (16 * cq + j < nv) dqp[j * qstride] = __float2bfloat16_rn(xs[j]);
            }
        }
        mwait(bar_mma, mph, a.err, 17, ok);
        mwait(bar_mma2, mph2, a.err, 26, ok);

        // ---- 11. dKb (kept in registers), dKb.kn, dKb tile ; Z2 = [-; dKb] K^T (320) -------------------
        float kbr[16];
        {
            ld16c(tm + C192 + lb + 16 * cq, kbr);  // dKb^T[dk][j]
            float r3[16], nk16[16];
            vec16(vNK, 16 * cq, nk16);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int jj = 16 * cq + j;
                r3[j] = kbr[j] * tile128(sm + OFF_QK + 8192, QK_BLK, jj, row) * nk16[j];
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) st8(sm + OFF_DKB + sw128_off(row, 16 * cq + 8 * q), kbr + 8 * q);
            deposit_colsum(r3, red0, lg, cq);
        }
        fence_async_smem();
        sync_tc();
        if (tid == 0) {
            const uint32_t id_mk = idesc_bf16(128, 64, 1, 0);
            const uint64_t dDKBm = desc_mnmajor(sb + OFF_DKB - 16384, 16384), dKk = desc_kmajor(aK);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
                umma_bf16(tm + C320, desc_at(dDKBm, ks * 2048), desc_at(dKk, (ks >> 2) * QK_BLK + (ks & 3) * 32), id_mk,
                          ks > 0);
            umma_commit(bar_mma);
        }
        if (tid < 64) {
            const float r3 = colsum(red0, tid);  // dKb_j . kn_j
            vDB[tid] += vEG[tid] * r3;
            vDG[tid] += vB[tid] * vEG[tid] * r3;
        }
        mwait(bar_mma, mph, a.err, 18, ok);
        if (tid == 0 && c > 0) issue_inputs_a(c - 1);  // Z2 was the last reader of the part-A regions

        // ---- 12. Z = beta_m (Z1 + e^G_m / nk_m Z2) -> bf16 [j][m] ; dA' = [-; Z] T^T (256) ---------------
        if (lg >= 2) {
            float z1[16], z2[16], b16[16], en16[16];
            ld16x2(tm + C256 + lb + 16 * cq, z1, tm + C320 + lb + 16 * cq, z2);
            vec16(vB, 16 * cq, b16);
            vec16(vEN, 16 * cq, en16);
            const int j = row - 64;
#pragma unroll
            for (int m = 0; m < 16; ++m) z1[m] = b16[m] * fmaf(en16[m], z2[m], z1[m]);
#pragma unroll
            for (int q = 0; q < 2; ++q) st8(sm + OFF_PS2 + sw128_off(j, 16 * cq + 8 * q), z1 + 8 * q);
        }
        fence_async_smem();
        sync_tc();
        if (tid == 0) {
            const uint32_t id = idesc_bf16(128, 64, 0, 0);
            const uint64_t dPSk = desc_kmajor(sb + OFF_PS), dTk = desc_kmajor(sb + OFF_T);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)  // A rows 0-63 = the dPs1 tile (ignored), 64-127 = Z
                umma_bf16(tm + C256, desc_at(dPSk, ks * 32), desc_at(dTk, ks * 32), id, ks > 0);
            umma_commit(bar_mma);
        }
        mwait(bar_mma, mph, a.err, 19, ok);
        {  // rows j on lanes 64-127: dA = -dA' (l < j); G E from the K K^T rows of D1
            float xa[16];
            if (lg >= 2) {
                float dap[16], kk[16], g16[16], nk16[16];
                ld16x2(tm + C256 + lb + 16 * cq, dap, tD1 + lb + 16 * cq, kk);
                vec16(vG, 16 * cq, g16);
                vec16(vNK, 16 * cq, nk16);
                const int j = row - 64;
                const float gj = vG[j], bj = vB[j], nkj = vNK[j];
                float sb_ = 0.f, sx = 0.f;
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const int l = 16 * cq + t;
                    const bool m = l < j;
                    const float e = m ? __expf(gj - g16[t]) : 0.f;
                    const float ge = kk[t] * nkj * nk16[t] * e;
                    const float dA = m ? -dap[t] : 0.f;
                    sb_ = fmaf(dA, ge, sb_);
                    xa[t] = dA * bj * ge;
                    sx += xa[t];
                    dGm[j * 64 + (l ^ (j & 31))] = dA * bj * e;  // column swizzled by the row: conflict-free
                }
                red2[cq * 64 + j] = sb_;  // partials per column quarter, summed in fixed order below
                red3[cq * 64 + j] = sx;
            } else {
#pragma unroll
                for (int t = 0; t < 16; ++t) xa[t] = 0.f;
            }
            deposit_colsum(xa, red1, lg, cq);
        }
        __syncthreads();
        if (tid < 64) {
            vDB[tid] += colsum(red2, tid);
            vDG[tid] += colsum(red3, tid) - colsum(red1, tid);
        }
        {  // Gs = (dG + dG^T) / (nk nk)  bf16 [j][m]
            const int j = tid >> 3, c8 = 8 * (tid & 7);
            float gs[8], nk8[8];
            vec8(vNK, c8, nk8);
            const float nkj = vNK[j];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int m = c8 + t;
                gs[t] = (dGm[j * 64 + (m ^ (j & 31))] + dGm[m * 64 + (j ^ (m & 31))]) * nkj * nk8[t];
            }
            st8(sm + OFF_GS + sw128_off(j, c8), gs);
        }
        fence_async_smem();
        sync_tc();

        // ---- 13. dK' += K^T Gs (448) ----------------------------------------------------------------
        if (tid == 0) {
            const uint32_t id_mk = idesc_bf16(128, 64, 1, 0);
            const uint64_t dKm = desc_mnmajor(aK, QK_BLK), dGSk = desc_kmajor(sb + OFF_GS);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) umma_bf16(tm + C448, desc_at(dKm, ks * 2048), desc_at(dGSk, ks * 32), id_mk, 1);
            umma_commit(bar_mma);
        }
        float kr[16], w16[16];  // step 14's shared-memory operands, loaded while the MMAs run
#pragma unroll
        for (int j = 0; j < 16; ++j) kr[j] = tile128(sm + OFF_QK + 8192, QK_BLK, 16 * cq + j, row);
        vec16(vBEN, 16 * cq, w16);
        mwait(bar_mma, mph, a.err, 20, ok);

        // ---- 14. dk = u - kn (kn.u), u = dK' + beta e^G / nk dKb ; dg, dbeta ---------------------------------
        {
            float u[16], xk[16];
            ld16c(tm + C448 + lb + 16 * cq, u);
#pragma unroll
            for (int j = 0; j < 16; ++j) u[j] = fmaf(w16[j], kbr[j], u[j]);
            vec16(vNK, 16 * cq, w16);
#pragma unroll
            for (int j = 0; j < 16; ++j) xk[j] = kr[j] * w16[j] * u[j];
            deposit_colsum(xk, red3, lg, cq);
            __syncthreads();
            if (tid < 64) vK3[tid] = vNK[tid] * colsum(red3, tid);  // (1/nk) (kn . u)
            __syncthreads();
            vec16(vK3, 16 * cq, w16);
            // dk[token][hq][dk]: this thread's column, tokens 16 cq .. (stride H x 128)
            const int64_t kidx = ((tok0 + 16 * cq) * a.H + hq) * 128 + row, kstride = (int64_t)a.H * 128;
#pragma unroll
            for (int j = 0; j < 16; ++j) u[j] = a.l2norm ? fmaf(-kr[j], w16[j], u[j]) : u[j];
            if (a.accumulate_qk) {
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (16 * cq + j < nv) atomicAdd((float*)a.dk + kidx + j * kstride, u[j]);
            } else {
                __nv_bfloat16* dkp = (__nv_bfloat16*)a.dk + kidx;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (16 * cq + j < nv) dkp[j * kstride] = __float2bfloat16_rn(u[j]);
            }
        }
        if (tid < 32) {  // last row: + sum_j kn.dKst_j + e^G_C <dS, S0>
            float s = vR4[tid] + vR4[tid + 32];
            s = warp_sum(s);
            float d = (tid < 16) ? scal[1 + tid] : 0.f;
            d = warp_sum(d);
            if (tid == 0) vDG[63] += s + scal[0] * d;
        }
        __syncthreads();
        if (tid < 64) {  // dg = reverse cumsum of dGamma
            float x = vDG[tid];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_down_sync(0xffffffffu, x, o);
                if (lane + o < 32) x += y;
            }
            red0[tid] = x;
        }
        __syncthreads();
        if (tid < 64 && tid < nv) {
            const float x = red0[tid] + (tid < 32 ? red0[32] : 0.f);
            a.dg[(tok0 + tid) * a.HV + hv] = x;
            a.dbeta[(tok0 + tid) * a.HV + hv] = vDB[tid];
        }
        sync_tc();
        if (tid == 0 && c > 0) issue_inputs_b(c - 1);
    }

    if (ok && a.dh0) {
        float* dh0 = a.dh0 + ((int64_t)n * a.HV + hv) * 16384;
#pragma unroll 1
        for (int c0 = 0; c0 < 32; c0 += 16) {
            float v[16];
            tmem_ld16(tS + lb + 32 * cq + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) dh0[(32 * cq + c0 + i) * 128 + row] = v[i];
        }
    }
    sync_tc();
    if (warp == 0) tmem_dealloc(tm, T_COLS);
}

template <typename TO>
__global__ void qk_convert_kernel(const float* __restrict__ src, TO* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

bool chunk_bwd_supported(int64_t DK, int64_t DV, int act_dtype) {
    return DK == 128 && DV == 128 && act_dtype == GDN_BF16;
}

size_t chunk_saved_bytes(int64_t B, int64_t T, int64_t N, int64_t HV, bool varlen) {
    const int64_t chunks = varlen ? (B * T + 63 * N) / 64 + N : N * ((T + 63) / 64);
    return (size_t)chunks * HV * kBwdRecordBytes;
}

size_t chunk_bwd_workspace(int64_t B, int64_t T, int64_t N, int64_t H, int64_t HV, bool varlen, bool saved) {
    // the records of the recompute pass, unless the forward saved them
    size_t bytes = saved ? 0 : chunk_saved_bytes(B, T, N, HV, varlen);
    if (HV > H) bytes += (size_t)B * T * H * 128 * 4 * 2;  // fp32 dq/dk accumulators (grouped value heads)
    return bytes;
}

int chunk_bwd(const ChunkBwdLaunch& L, cudaStream_t s) {
    using namespace cb;
    if (smem_optin((const void*)chunk_bwd_kernel, SMEM_BYTES) != cudaSuccess) return GDN_ERR_LAUNCH;
    // 1. rebuild every chunk-start state from the checkpoints (segment-parallel forward, no outputs), unless
    //    the forward saved the records
    const uint8_t* records = (const uint8_t*)L.saved_rec;
    uint8_t* scratch = (uint8_t*)L.ws;
    if (!records) {
        ChunkLaunch R{};
        R.q = L.q; R.k = L.k; R.v = L.v; R.g = L.g; R.beta = L.beta; R.o = nullptr;
        R.h0 = L.h0; R.ht = nullptr; R.ckpt = const_cast<float*>(L.ckpt); R.cu = L.cu; R.err = L.err;
        R.B = L.B; R.T = L.T; R.N = L.N; R.H = L.H; R.HV = L.HV; R.scale = L.scale;
        R.g_dtype = L.g_dtype; R.beta_dtype = L.beta_dtype; R.l2norm = L.l2norm; R.o_mode = 2;
        R.ckpt_every = L.ckpt_every;
        R.s0_out = L.ws;
        R.max_seqlen = L.max_seqlen;
        int st = chunk_fwd(R, s);
        if (st != GDN_OK) return st;
        records = (const uint8_t*)L.ws;
        scratch += chunk_saved_bytes(L.B, L.T, L.N, L.HV, L.cu != nullptr);
    }

    // 2. reverse sweep
    ChunkBwdArgs a;
    memset(&a, 0, sizeof(a));
    const int64_t Ttot = L.B * L.T;
    if (!make_tmap_3d_sw128(&a.tq, L.q, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    if (!make_tmap_3d_sw128(&a.tk, L.k, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    if (!make_tmap_3d_sw128(&a.tv, L.v, 128, L.HV, Ttot, 128, L.HV * 128, 64)) return GDN_ERR_ALIGN;
    if (!make_tmap_3d_sw128(&a.tdo, L.dout, 128, L.HV, Ttot, 128, L.HV * 128, 64)) return GDN_ERR_ALIGN;
    const bool acc = L.HV > L.H && !L.state_grad_only;
    float* acc_q = acc ? (float*)scratch : nullptr;
    float* acc_k = acc ? acc_q + Ttot * L.H * 128 : nullptr;
    if (acc && cudaMemsetAsync(acc_q, 0, (size_t)Ttot * L.H * 128 * 4 * 2, s) != cudaSuccess) return GDN_ERR_LAUNCH;
    a.g = L.g;
    a.beta = L.beta;
    a.s0_tiles = records;
    a.dht = L.dht;
    a.dq = acc ? (void*)acc_q : L.dq;
    a.dk = acc ? (void*)acc_k : L.dk;
    a.dv = L.dv;
    a.dg = L.dg;
    a.dbeta = L.dbeta;
    a.dh0 = L.dh0;
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
    a.accumulate_qk = acc ? 1 : 0;
    a.state_grad_only = L.state_grad_only;
    const unsigned grid = (unsigned)(L.N * L.HV);
    if (grid > 0) {
        chunk_bwd_kernel<<<grid, NTHR, SMEM_BYTES, s>>>(a);
        count_launch();
    }
    if (acc) {
        const int64_t nqk = Ttot * L.H * 128;
        const int64_t want = (nqk + 255) / 256;
        const unsigned blocks = (unsigned)(want < 148 * 16 ? want : 148 * 16);
        qk_convert_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(acc_q, (__nv_bfloat16*)L.dq, nqk);
        qk_convert_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(acc_k, (__nv_bfloat16*)L.dk, nqk);
        count_launch(2);
    }
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
