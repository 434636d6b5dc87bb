// Chunked gated-delta-rule forward split in two launches on sm_100a: a chunk-parallel prep pass and a lean
// per-(sequence, head) state pass.
//
// Notation (the algebra of tests/test_chunk_algebra.py, the same as gdn_chunk_fwd.cu): Gamma = in-chunk
// cumsum of g, E_ij = exp(Gamma_i - Gamma_j), nq_i, nk_j the inverse L2 norms of the raw q/k rows (1 without
// the norm, 0 on rows past the sequence end), S0 the state at the chunk start, S^T its transpose [dv][dk].
//   A  = strict_lower(diag(beta) (K K^T . nk nk^T) . E)       T = (I + A)^-1
//   W  = T diag(beta e^Gamma nk) K      U = T diag(beta) V      Delta = U - W S0
//   O_i = nq_i [ (Qg S0)_i + (P Delta)_i ],   Qg = diag(scale e^Gamma) Q,   P_ij = scale (q_i . k_j) nk_j E_ij
//         (j <= i)
//   S1 = e^Gamma_C S0 + K^T diag(e^(Gamma_C - Gamma) nk) Delta
// Everything except Delta, O and S1 is independent of the state, so chunk_prep_kernel computes it for all
// (chunk, head) pairs at once (8,192 CTAs of 256 threads at B8 T4096 H16, four per SM: Gram matrix, norms,
// gates, P, the triangular solve, W) and hands it to the state pass as one record per (chunk, head) in the
// workspace (kFwdRecordBytes, kernels.h): the bf16 operand tiles Qg, -W, TV = T diag(beta), P hi and lo as
// shared-memory images in the 128-byte-swizzled layout, staged in shared memory and written by bulk copies,
// and the vectors e^(Gamma_C - Gamma) nk, nq, e^Gamma_C.
// chunk_state_kernel runs one CTA per (sequence, value head) that keeps S^T (fp32) in tensor memory. Per
// chunk, 16 warps turn S into the S0^T hi/lo operand tiles (and scale the TMEM state by e^Gamma_C), then
//   Delta^T = V^T TV^T + S0hi^T (-W)^T  [+ S0lo^T (-W)^T in a second accumulator]     (M = dv = 128, N = 64)
//   O      = [Qg; -] (S0hi + S0lo)                                                   (rows 0-63 used)
// 16 warps turn Delta^T (all 128 TMEM lanes) into the Delta^T and Dd^T = Delta^T diag(e^(Gamma_C - Gamma) nk)
// hi/lo tiles, and
//   S^T += Dd^T K (hi + lo)        O += P Delta (hi.hi + lo.hi + hi.lo)
// Two extra warps only issue the loads and MMAs (unrolled, one N = 64 UMMA per ~50 cycles from a thread): warp 16
// the state chain, warp 17 the output products and the loads they read, so issue overlaps the data phases;
// four warps emit chunk c-1's outputs while the Delta^T products of chunk c run, and every chunk's operands
// are prefetched into L2 two chunks ahead. The raw bf16 q, k, v tiles feed the tensor cores unmodified;
// Qg is the one operand rounded from a scaled q.
// Saved-record mode (ChunkLaunch::bwd_rec set): the two passes also write the backward sweep's record of every
// (chunk, head) (kBwdRecordBytes, kernels.h) from what they already hold: the prep pass -W (bulk copies of its
// staged tile) and T (16-byte stores from registers), the state pass S0^T, Delta^T and the low part of Dd^T:
// its hi/lo splits round the hi part to nearest, so those staged operand tiles are the record's tiles as they
// are, and thread 0 bulk-copies them out after each phase's barrier. The backward then skips its recompute
// pass.
#include <cstring>

#include "chunk_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "launch.h"
#include "sm100.cuh"
#include "tmap.h"

namespace gdn {
using namespace sm100;

namespace split {

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint4 pack8(const float* v) {
    return make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
}
// hi = bf16(v), lo = bf16(v - hi): the pair carries ~16 significant bits
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
    float h[8], l[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        h[e] = __bfloat162float(__float2bfloat16_rn(v[e]));
        l[e] = v[e] - h[e];
    }
    hi = pack8(h);
    lo = pack8(l);
}
__device__ __forceinline__ void sync_tc() {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}
// bounded waits (see gdn_chunk_fwd.cu): after a timeout every later wait polls once and the CTA runs out
__device__ __forceinline__ void wait_bar(uint64_t* bar, uint32_t parity, int* err, int code, bool& ok) {
    ok = mbar_wait(bar, parity, err, code, ok ? (1u << 22) : 1u) && ok;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// bulk (TMA engine) copy shared -> global in this thread's bulk group; wait until the group's reads are done
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"((uint64_t)dst), "r"(smem_u32(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// L2 prefetches: a chunk's operands are brought into L2 two chunks before its shared-memory loads
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"((uint64_t)src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_tile_l2(const CUtensorMap* map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"((uint64_t)map), "r"(c0),
                 "r"(c1), "r"(c2)
                 : "memory");
}
template <int N>
__device__ __forceinline__ void vload(const float* v, int base, float (&o)[N]) {
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

}  // namespace split

// ================================================================================================
// chunk_prep_kernel: one CTA (256 threads) per (chunk, sequence, value head)
// ================================================================================================
namespace cp {
constexpr int NTHR = 256;
constexpr uint32_t OFF_QK = 0;       // per d-block kb (16 KB apart): [Q 8 KB | K 8 KB], 64 rows x 128 B
constexpr uint32_t OFF_A = 32768;    // fp32 A / T, 64 x AST
constexpr int AST = 68;
constexpr uint32_t OFF_Y = OFF_A + 64 * AST * 4;       // solve scratch
constexpr uint32_t OFF_TB = OFF_A;                     // after the solve: TB bf16 [i][j] 8 KB, then TV: [TB; TV]
                                                       // is MMA2's A (T is read into registers first)
constexpr uint32_t OFF_VEC = OFF_Y + 32 * kSolveYStride * 4;  // G, EG, B, NQ, NK: 5 x 64 fp32
constexpr uint32_t OFF_BAR = OFF_VEC + 5 * 256;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 64 + 1024;   // four CTAs per SM
constexpr uint32_t T_COLS = 128;                       // D1 in columns 0-63, then W in 0-127
static_assert(SMEM_BYTES + 1024 <= 233472 / 4, "four CTAs per SM");
}  // namespace cp

struct ChunkPrepArgs {
    CUtensorMap tq, tk;
    const void* g;
    const void* beta;
    const int64_t* cu;
    const int64_t* cbase;  // varlen: first flattened chunk of each sequence (NULL: n * ceil(T / 64))
    uint8_t* rec;          // kFwdRecordBytes per (flattened chunk, value head)
    uint8_t* rec_bwd;      // NULL, or the backward's kBwdRecordBytes records: -W and T are written here too
    int* err;
    int64_t T;
    int H, HV, g_dtype, beta_dtype, l2norm;
    float scale;
};

__global__ void __launch_bounds__(cp::NTHR, 4) chunk_prep_kernel(const __grid_constant__ ChunkPrepArgs a) {
    using namespace cp;
    using namespace split;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    float* Am = (float*)(sm + OFF_A);
    float* Yb = (float*)(sm + OFF_Y);
    float* vG = (float*)(sm + OFF_VEC);
    float* vEG = vG + 64;
    float* vB = vG + 128;
    float* vNQ = vG + 192;
    float* vNK = vG + 256;
    uint64_t* bar_in = (uint64_t*)(sm + OFF_BAR);
    uint64_t* bar_mma = bar_in + 1;
    uint32_t* tmem_slot = (uint32_t*)(bar_in + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int lg = warp & 3, hf = warp >> 2;  // TMEM lane quadrant, column half
    const int row = 32 * lg + lane;
    const int c = blockIdx.x;
    const int n = blockIdx.y / a.HV, hv = blockIdx.y % a.HV, hq = hv / (a.HV / a.H);
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t len = eos - bos;
    if (64 * (int64_t)c >= len) return;
    const int nv = (len - 64 * (int64_t)c) < 64 ? (int)(len - 64 * (int64_t)c) : 64;
    const int64_t tok0 = bos + 64 * (int64_t)c;
    const int64_t cb = a.cbase ? a.cbase[n] : (int64_t)n * ((a.T + 63) / 64);
    uint8_t* rec = a.rec + ((cb + c) * a.HV + hv) * kFwdRecordBytes;

    if (tid == 0) {
        mbar_init(bar_in, 1);
        mbar_init(bar_mma, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(bar_in, 4 * 8192);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
            tma_load_3d(sm + OFF_QK + kb * 16384, &a.tq, bar_in, kb * 64, hq, (int)tok0);
            tma_load_3d(sm + OFF_QK + kb * 16384 + 8192, &a.tk, bar_in, kb * 64, hq, (int)tok0);
        }
    }
    if (warp == 0) tmem_alloc(tmem_slot, T_COLS);
    sync_tc();
    const uint32_t tm = *tmem_slot;
    const uint32_t lb = (uint32_t)(32 * lg) << 16;
    const uint32_t sb = smem_u32(sm);
    bool ok = true;
    // gates: Gamma = inclusive cumsum of g in the chunk; rows past the sequence end carry g = 0, beta = 0
    if (tid < 64) {
        float x = 0.f, bt = 0.f;
        if (tid < nv) {
            const int64_t gi = (tok0 + tid) * a.HV + hv;
            x = gate_f(ld_gate_raw(a.g, a.g_dtype, gi), a.g_dtype);
            bt = gate_f(ld_gate_raw(a.beta, a.beta_dtype, gi), a.beta_dtype);
        }
        vB[tid] = bt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        vG[tid] = x;
    }
    wait_bar(bar_in, 0, a.err, 41, ok);
    // MMA1: D1 = [Q; K] K^T on the raw tiles (M = 128, N = 64, K = 128)
    if (tid == 0) {
        tc_fence_after();
        const uint32_t id = idesc_bf16(128, 64, 0, 0);
        const uint64_t dA = desc_kmajor(sb + OFF_QK), dB = desc_kmajor(sb + OFF_QK + 8192);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const uint32_t o = (ks >> 2) * 16384 + (ks & 3) * 32;
            umma_bf16(tm, desc_at(dA, o), desc_at(dB, o), id, ks > 0);
        }
        umma_commit(bar_mma);
    }
    __syncthreads();
    if (tid >= 32 && tid < 64) vG[tid] += vG[31];
    {  // inverse row norms: 2 threads per row (one d-block each); rows 0-63 q, 64-127 k
        const int r = tid >> 1, kb = tid & 1, i = r & 63;
        const uint8_t* rowp = sm + OFF_QK + kb * 16384 + (r < 64 ? 0 : 8192) + i * 128;
        float ss = 0.f;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const uint4 u = *reinterpret_cast<const uint4*>(rowp + ((cc + 4 * kb) & 7) * 16);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(h[e]);
                ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
            }
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        float inv = a.l2norm ? 1.f / fmaxf(sqrtf(ss), kL2Eps) : 1.f;
        if (i >= nv) inv = 0.f;
        if (kb == 0) (r < 64 ? vNQ : vNK)[i] = inv;
    }
    __syncthreads();
    if (tid < 64) {  // record vectors: vX = e^(G_C - G) nk, nq, e^G_C
        vEG[tid] = __expf(vG[tid]);
        float* rv = (float*)(rec + kFwdRecVec);
        rv[tid] = __expf(vG[63] - vG[tid]) * vNK[tid];
        rv[64 + tid] = vNQ[tid];
        if (tid == 0) rv[128] = __expf(vG[63]);
    }
    __syncthreads();
    wait_bar(bar_mma, 0, a.err, 42, ok);
    tc_fence_after();
    // Qg = diag(scale e^G) Q (raw q rows), in place in the Q tile (MMA1 has read it), then one bulk store per
    // d-block: 16-byte chunks keep the tile's swizzled layout, each scaled by its row's factor
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int e = tid + 256 * it, i = e >> 4, kb = (e >> 3) & 1, ch = e & 7;
        uint4* pc = reinterpret_cast<uint4*>(sm + OFF_QK + kb * 16384 + i * 128 + ch * 16);
        const uint4 u = *pc;
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
        const float f = a.scale * vEG[i];
        float y[8];
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
            const float2 z = __bfloat1622float2(h[k2]);
            y[2 * k2] = z.x * f;
            y[2 * k2 + 1] = z.y * f;
        }
        *pc = pack8(y);
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
        bulk_s2g(rec + kFwdRecQg, sm + OFF_QK, 8192);
        bulk_s2g(rec + kFwdRecQg + 8192, sm + OFF_QK + 16384, 8192);
        bulk_commit();
    }
    // D1 rows 0-63 -> P hi/lo (staged in the Q slots once Qg has left), rows 64-127 -> A (fp32, shared memory)
    {
        float v[32];
        tmem_ld16(tm + lb + 32 * hf, *reinterpret_cast<float(*)[16]>(v));
        tmem_ld16(tm + lb + 32 * hf + 16, *reinterpret_cast<float(*)[16]>(v + 16));
        tmem_wait_ld();
        const int i = row & 63;
        const float gi = vG[i];
        // rows 32 lg' .. (lg' = lg & 1) against columns 32 hf ..: the block above the diagonal is all zero
        const bool zero_blk = hf > (lg & 1);
        if (lg < 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int jj = 32 * hf + j;
                v[j] = (!zero_blk && jj <= i) ? a.scale * v[j] * vNK[jj] * __expf(gi - vG[jj]) : 0.f;
            }
        } else {
            const float bi = vB[i] * vNK[i];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int jj = 32 * hf + j;
                v[j] = (!zero_blk && jj < i) ? bi * v[j] * vNK[jj] * __expf(gi - vG[jj]) : 0.f;
            }
            float4* dst = reinterpret_cast<float4*>(Am + i * AST + 32 * hf);
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        if (tid == 0) bulk_wait_read();  // the Qg stores have read the Q slots
        __syncthreads();
        if (lg < 2) {  // P hi into the d-block-0 Q slot, P lo into the d-block-1 Q slot
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 hi, lo;
                split8(v + 8 * q, hi, lo);
                const uint32_t off = sw128_off(i, 32 * hf + 8 * q);
                *reinterpret_cast<uint4*>(sm + OFF_QK + off) = hi;
                *reinterpret_cast<uint4*>(sm + OFF_QK + 16384 + off) = lo;
            }
        }
        fence_async_smem();
        __syncthreads();
        if (tid == 0) {
            bulk_s2g(rec + kFwdRecP, sm + OFF_QK, 8192);
            bulk_s2g(rec + kFwdRecP + 8192, sm + OFF_QK + 16384, 8192);
            bulk_commit();
        }
    }
    sync_tc();
    // T = (I + A)^-1 in place (all 8 warps)
    tri_inverse64<AST>(Am, Yb);
    __syncthreads();
    // TB = T diag(beta e^G nk), TV = T diag(beta): bf16 K-major [i][j] tiles in shared memory (MMA2's A, over
    // the T region: every thread reads its T elements first); TV also to the record
    float tr[2][8];
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int wl = tid & 31, qq = wl >> 3, sub = wl & 7;
        const int i = 32 * it + 4 * warp + 2 * (qq & 1) + (sub >> 2), c8 = 8 * ((sub & 3) + 4 * (qq >> 1));
        const float4 t0 = *reinterpret_cast<const float4*>(Am + i * AST + c8);
        const float4 t1 = *reinterpret_cast<const float4*>(Am + i * AST + c8 + 4);
        tr[it][0] = t0.x; tr[it][1] = t0.y; tr[it][2] = t0.z; tr[it][3] = t0.w;
        tr[it][4] = t1.x; tr[it][5] = t1.y; tr[it][6] = t1.z; tr[it][7] = t1.w;
    }
    __syncthreads();
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int wl = tid & 31, qq = wl >> 3, sub = wl & 7;
        const int i = 32 * it + 4 * warp + 2 * (qq & 1) + (sub >> 2), c8 = 8 * ((sub & 3) + 4 * (qq >> 1));
        const float* t = tr[it];
        float b8[8], e8[8], n8[8], tb[8], tv[8];
        vload(vB, c8, b8);
        vload(vEG, c8, e8);
        vload(vNK, c8, n8);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            tv[j] = t[j] * b8[j];
            tb[j] = tv[j] * e8[j] * n8[j];
        }
        const uint32_t off = sw128_off(i, c8);
        *reinterpret_cast<uint4*>(sm + OFF_TB + off) = pack8(tb);
        *reinterpret_cast<uint4*>(sm + OFF_TB + 8192 + off) = pack8(tv);
        if (a.rec_bwd)  // the backward's T tile (same image layout), straight from registers
            *reinterpret_cast<uint4*>(a.rec_bwd + ((cb + c) * a.HV + hv) * kBwdRecordBytes + kBwdRecT + off) =
                pack8(t);
    }
    fence_async_smem();
    sync_tc();
    if (tid == 0) {
        bulk_s2g(rec + kFwdRecTV, sm + OFF_TB + 8192, 8192);
        bulk_commit();
    }
    // MMA2: [W; TV K] = [TB; TV] K  (M = 128, N = 128 = dk, K = 64 tokens); W rows on lanes 0-63
    if (tid == 0) {
        const uint32_t id = idesc_bf16(128, 128, 0, 1);
        const uint64_t dTB = desc_kmajor(sb + OFF_TB), dK = desc_mnmajor(sb + OFF_QK + 8192, 16384);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) umma_bf16(tm, desc_at(dTB, ks * 32), desc_at(dK, ks * 2048), id, ks > 0);
        umma_commit(bar_mma);
    }
    wait_bar(bar_mma, 1, a.err, 43, ok);
    tc_fence_after();
    // -W (bf16, K-major [i][dk]) staged in the Q slots (the P stores have read them), then bulk-stored:
    // warps of lanes 0-63, 64 columns (one d-block) each
    if (tid == 0) bulk_wait_read();
    __syncthreads();
    if (lg < 2) {
        uint8_t* dst = sm + OFF_QK + hf * 16384;
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // two halves of 32 columns (the register cap of four CTAs per SM)
            float v[32];
            tmem_ld16(tm + lb + 64 * hf + 32 * h, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tm + lb + 64 * hf + 32 * h + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = -v[e];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                *reinterpret_cast<uint4*>(dst + sw128_off(row, 32 * h + 8 * q)) = pack8(v + 8 * q);
        }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
        bulk_s2g(rec + kFwdRecW, sm + OFF_QK, 8192);
        bulk_s2g(rec + kFwdRecW + 8192, sm + OFF_QK + 16384, 8192);
        if (a.rec_bwd) {  // -W for the backward's record too
            uint8_t* rb = a.rec_bwd + ((cb + c) * a.HV + hv) * kBwdRecordBytes + kBwdRecW;
            bulk_s2g(rb, sm + OFF_QK, 8192);
            bulk_s2g(rb + 8192, sm + OFF_QK + 16384, 8192);
        }
        bulk_commit();
        bulk_wait_all();  // the records are in global memory before the CTA ends
    }
    sync_tc();
    if (warp == 0) tmem_dealloc(tm, T_COLS);
}

// ================================================================================================
// chunk_state_kernel: one CTA per (sequence, value head), chunks in order. Warps 0-15 move data between
// tensor memory and operand tiles; warps 16 and 17 only issue loads and MMAs (one thread issues an N = 64
// tcgen05.mma about every 50 cycles), so that issue overlaps the other warps' work: warp 16 the state chain (the
// Delta^T products with S0 hi, the state update), warp 17 the rest (the Delta^T products with S0 lo into a
// second accumulator, the output products) and the loads those read.
// ================================================================================================
namespace cs {
constexpr int NWORK = 512;              // warps 0-15: TMEM lane quadrant w % 4, column quarter w / 4
constexpr int NTHR = NWORK + 64;        // + warps 16, 17: load and MMA issue
constexpr uint32_t OFF_W = 0;           // -W bf16 [i][dk], two 8 KB d-blocks: G1's B (N = 64 tokens)
constexpr uint32_t OFF_PH = 16384;      // P hi [i][j]; [P hi; P lo] and [P lo; Z] are the 128-row A operands
constexpr uint32_t OFF_PL = 24576;      //   of the output products (rows 0-63 used)
constexpr uint32_t OFF_Z = 32768;       // zeros
constexpr uint32_t OFF_TV = 40960;      // TV [i][j]: B of U^T = V^T TV^T
constexpr uint32_t OFF_V = 49152;       // V [token][dv], 2 x 8 KB
constexpr uint32_t OFF_K = 65536;       // K [token][dk], 2 x 8 KB
constexpr uint32_t OFF_S0 = 81920;      // S0^T hi [dv][dk], 2 dk-blocks x 16 KB (A of G1, B of the output MMA)
// per d-block kb (24 KB apart): [Qg_kb 8 KB | S0^T lo block kb 16 KB]: [Qg; S0lo rows] is the output MMA's A
constexpr uint32_t OFF_QL = 114688;
constexpr uint32_t QL_BLK = 24576;
constexpr uint32_t OFF_DH = 163840;     // Delta^T hi [dv][j] (128 rows x 128 B)
constexpr uint32_t OFF_DL = 180224;
constexpr uint32_t OFF_DDH = 196608;    // Dd^T = Delta^T diag(e^(G_C - G) nk), hi
constexpr uint32_t OFF_DDL = 212992;
constexpr uint32_t OFF_VEC = 229376;    // record vectors, two buffers
constexpr uint32_t OFF_BAR = OFF_VEC + 2 * kFwdRecVecBytes;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 128 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
// TMEM columns: S^T [dv][dk], Delta^T [dv][j] (the S0 hi part, and the S0 lo part: 64 each), two output
// accumulators (rows 0-63 used)
constexpr uint32_t T_S = 0, T_DT = 128, T_DT2 = 192, T_O = 256, T_COLS = 512;
constexpr uint32_t TX_L1 = 2 * 8192 + 8192 + 2 * 8192;  // -W, TV, V
constexpr uint32_t TX_LB = 2 * 8192 + kFwdRecVecBytes;  // Qg, vectors
}  // namespace cs

struct ChunkStateArgs {
    CUtensorMap tk, tv;
    const uint8_t* rec;
    const int64_t* cbase;
    uint8_t* rec_bwd;  // NULL, or the backward's records: S0^T, Delta^T and the low part of Dd^T are written here
    void* o;           // NULL: no outputs (the output products and stores are skipped; the final state is kept)
    const float* h0;
    float* ht;
    float* ckpt;
    const int64_t* cu;
    int* err;
    int64_t T;
    int HV, H, ckpt_every;
    int zero_v;       // 1: v = 0 (no U term, V not loaded): the state evolves by its homogeneous part only
    int h0_identity;  // 1: the state starts as the identity (dk = dv): the final state is the transition map
};

// (a0, a1) -> hi = bf16x2(a0, a1) rounded to nearest, lo = bf16x2(a - hi); hf0, hf1 = hi as floats
__device__ __forceinline__ void split2_rn(float a0, float a1, uint32_t& hi, uint32_t& lo, float& hf0, float& hf1) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    hf0 = __uint_as_float(hi << 16);
    hf1 = __uint_as_float(hi & 0xffff0000u);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a0 - hf0, a1 - hf1);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
// 8 values: hi/lo words as above, hf = hi as floats
__device__ __forceinline__ void split8_rn(const float* v, uint4& hi, uint4& lo, float* hf) {
    split2_rn(v[0], v[1], hi.x, lo.x, hf[0], hf[1]);
    split2_rn(v[2], v[3], hi.y, lo.y, hf[2], hf[3]);
    split2_rn(v[4], v[5], hi.z, lo.z, hf[4], hf[5]);
    split2_rn(v[6], v[7], hi.w, lo.w, hf[6], hf[7]);
}

__global__ void __launch_bounds__(cs::NTHR, 1) chunk_state_kernel(const __grid_constant__ ChunkStateArgs a) {
    using namespace cs;
    using namespace split;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bar = (uint64_t*)(sm + OFF_BAR);
    uint64_t* bar_l1 = bar;      // -W, TV, V of a chunk
    uint64_t* bar_l2 = bar + 1;  // K
    uint64_t* bar_l3 = bar + 2;  // P hi/lo
    uint64_t* bar_g = bar + 3;   // Delta^T products done
    uint64_t* bar_q = bar + 4;   // Qg S0 done
    uint64_t* bar_s = bar + 5;   // state update done
    uint64_t* bar_o = bar + 6;   // P Delta done
    uint64_t* bar_g2 = bar + 7;  // Delta^T product with S0 lo done
    uint64_t* bar_lb = bar + 8;  // Qg and vectors of a chunk
    uint64_t* bar_od = bar + 9;  // the output step of a chunk has read its vector buffer (4 warps arrive)
    uint32_t* tmem_slot = (uint32_t*)(bar + 10);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool issuer = tid == NWORK;        // warp 16, lane 0: the state chain
    const bool issuer2 = tid == NWORK + 32;  // warp 17, lane 0: the rest
    const int lg = warp & 3, cq = (warp >> 2) & 3;
    const int row = 32 * lg + lane;
    const int n = blockIdx.x / a.HV, hv = blockIdx.x % a.HV, hq = hv / (a.HV / a.H);
    int64_t bos, eos;
    seq_bounds(a.cu, a.T, n, bos, eos);
    const int64_t len = eos - bos;
    const int nchunks = (int)((len + 63) / 64);
    const int64_t cb = a.cbase ? a.cbase[n] : (int64_t)n * ((a.T + 63) / 64);

    // checkpoint slot of this sequence's first checkpoint
    int64_t ck_base = 0;
    if (a.ckpt) {
        const int K = a.ckpt_every;
        if (!a.cu) {
            ck_base = (int64_t)n * (((a.T + 63) / 64 + K - 1) / K);
        } else {
            int64_t part = 0;
            for (int m = tid; m < n; m += NTHR) part += (((a.cu[m + 1] - a.cu[m] + 63) / 64) + K - 1) / K;
            for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            int64_t* red = (int64_t*)(sm + OFF_DH);
            if (lane == 0) red[warp] = part;
            __syncthreads();
            for (int w = 0; w < NTHR / 32; ++w) ck_base += red[w];
            __syncthreads();
        }
    }

    if (issuer) {
        for (int i = 0; i < 9; ++i) mbar_init(&bar[i], 1);
        mbar_init(bar_od, 4);
        fence_barrier_init();
        prefetch_tmap(&a.tk);
        prefetch_tmap(&a.tv);
    }
    if (warp == 0) tmem_alloc(tmem_slot, T_COLS);
    for (int e = tid; e < 8192 / 16; e += NTHR) ((uint4*)(sm + OFF_Z))[e] = make_uint4(0, 0, 0, 0);
    fence_async_smem();
    sync_tc();
    const uint32_t tm = *tmem_slot;
    const uint32_t tS = tm + T_S, tDT = tm + T_DT, tDT2 = tm + T_DT2;
    const uint32_t lb = (uint32_t)(32 * lg) << 16;
    const uint32_t sb = smem_u32(sm);
    bool ok = true;

    // initial state -> TMEM: thread (row = dv, quarter cq) holds S^T[dv][dk] for dk in [32 cq, 32 cq + 32)
    if (!issuer && tid < NWORK) {
        const float* h0 = a.h0 ? a.h0 + ((int64_t)n * a.HV + hv) * 16384 : nullptr;
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
                v[i] = h0 ? h0[(32 * cq + c0 + i) * 128 + row] : (a.h0_identity && 32 * cq + c0 + i == row ? 1.f : 0.f);
            tmem_st16(tS + lb + 32 * cq + c0, v);
        }
        tmem_wait_st();
    }

    auto recp = [&](int c) { return a.rec + ((cb + c) * a.HV + hv) * kFwdRecordBytes; };
    // saved-record mode: thread 0 bulk-copies the staged tiles into the backward's record of each chunk
    const bool rec_copier = a.rec_bwd != nullptr && tid == 0;
    auto recb = [&](int c) { return a.rec_bwd + ((cb + c) * a.HV + hv) * kBwdRecordBytes; };
    // -W, TV, V of chunk c (bar_l1; issued once the Delta^T products of chunk c-1 have read them) and Qg and
    // the vectors (bar_lb; once the output product of chunk c-1 has read Qg and the output step of chunk c-2
    // has read that vector buffer)
    auto issue_l1_a = [&](int c) {
        const int tok0 = (int)(bos + 64 * c);
        const uint8_t* r = recp(c);
        mbar_arrive_expect_tx(bar_l1, a.zero_v ? TX_L1 - 2 * 8192 : TX_L1);
        bulk_g2s(sm + OFF_W, r + kFwdRecW, 16384, bar_l1);
        bulk_g2s(sm + OFF_TV, r + kFwdRecTV, 8192, bar_l1);
        if (!a.zero_v) {
#pragma unroll
            for (int kb = 0; kb < 2; ++kb) tma_load_3d(sm + OFF_V + kb * 8192, &a.tv, bar_l1, kb * 64, hv, tok0);
        }
    };
    auto issue_l1_b = [&](int c) {
        const uint8_t* r = recp(c);
        mbar_arrive_expect_tx(bar_lb, TX_LB);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) bulk_g2s(sm + OFF_QL + kb * QL_BLK, r + kFwdRecQg + kb * 8192, 8192, bar_lb);
        bulk_g2s(sm + OFF_VEC + (c & 1) * kFwdRecVecBytes, r + kFwdRecVec, kFwdRecVecBytes, bar_lb);
    };
    auto issue_l2 = [&](int c) {  // K of chunk c
        const int tok0 = (int)(bos + 64 * c);
        mbar_arrive_expect_tx(bar_l2, 2 * 8192);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) tma_load_3d(sm + OFF_K + kb * 8192, &a.tk, bar_l2, kb * 64, hq, tok0);
    };
    auto issue_l3 = [&](int c) {  // P hi | lo of chunk c (contiguous in the record and here)
        mbar_arrive_expect_tx(bar_l3, 16384);
        bulk_g2s(sm + OFF_PH, recp(c) + kFwdRecP, 16384, bar_l3);
    };
    auto prefetch_chunk = [&](int c) {  // everything chunk c reads from global memory, into L2
        const int tok0 = (int)(bos + 64 * c);
        prefetch_l2(recp(c), (uint32_t)kFwdRecordBytes);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
            prefetch_tile_l2(&a.tk, kb * 64, hq, tok0);
            if (!a.zero_v) prefetch_tile_l2(&a.tv, kb * 64, hv, tok0);
        }
    };
    // output step of chunk c on warps 8, 9, 12, 13 (lanes 0-63, 64 columns each): o = nq (Qg S0 + P Delta)
    auto output_step = [&](int c) {
        const int i = row;
        const float* vec = (const float*)(sm + OFF_VEC + (c & 1) * kFwdRecVecBytes);
        const float f = vec[64 + i];
        const int nv = (len - 64 * (int64_t)c) < 64 ? (int)(len - 64 * (int64_t)c) : 64;
        const uint32_t tO = tm + T_O + (uint32_t)(c & 1) * 128 + lb + 64 * ((warp >> 2) & 1);
        __nv_bfloat16* orow = (__nv_bfloat16*)a.o + ((bos + 64 * (int64_t)c + i) * a.HV + hv) * 128 +
                              64 * ((warp >> 2) & 1);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float v[32];
            tmem_ld16(tO + 32 * h, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tO + 32 * h + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
            if (i < nv) {
#pragma unroll
                for (int e = 0; e < 32; ++e) v[e] *= f;
                uint4* dst = reinterpret_cast<uint4*>(orow + 32 * h);
#pragma unroll
                for (int q = 0; q < 4; ++q) dst[q] = pack8(v + 8 * q);
            }
        }
    };
    const bool out_warp = warp >= 8 && warp < 16 && lg < 2;  // warps 8, 9, 12, 13
    // without outputs warp 17 issues no output products but keeps committing bar_q / bar_o (a commit with no new
    // MMAs arrives once the thread's earlier ones are done), so every wait below keeps its meaning
    const bool outs = a.o != nullptr;

    if (issuer && nchunks > 0) {
        issue_l1_a(0);
        issue_l1_b(0);
        issue_l2(0);
        if (outs) issue_l3(0);
        if (nchunks > 1) prefetch_chunk(1);
    }

    for (int c = 0; c < nchunks; ++c) {
        const uint32_t par = (uint32_t)c & 1u;
        const float* vec = (const float*)(sm + OFF_VEC + par * kFwdRecVecBytes);
        // A. this chunk's Qg and vectors; the previous chunk's state update and output product have landed
        wait_bar(bar_lb, par, a.err, 51, ok);
        if (c > 0) {
            wait_bar(bar_s, par ^ 1u, a.err, 52, ok);
            wait_bar(bar_q, par ^ 1u, a.err, 53, ok);
            tc_fence_after();
        }
        if (issuer) {
            if (c > 0) issue_l2(c);  // the state update of chunk c-1 has read K
            if (c + 2 < nchunks) prefetch_chunk(c + 2);
        }
        // B. S^T -> S0^T hi/lo operand tiles (hi = bf16(S0), round to nearest: the backward record's S0^T
        //    tile as it is); TMEM state <- e^G_C S0; checkpoint
        if (tid < NWORK) {
            const float eGC = vec[128];
            const bool ck = a.ckpt && (c % a.ckpt_every == 0);
            float* ckp = ck ? a.ckpt + ((ck_base + c / a.ckpt_every) * a.HV + hv) * 16384 : nullptr;
            float v[32];
            tmem_ld16(tS + lb + 32 * cq, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(tS + lb + 32 * cq + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
            if (ck) {
#pragma unroll
                for (int i = 0; i < 32; ++i) ckp[(32 * cq + i) * 128 + row] = v[i];
            }
            const uint32_t kb = (uint32_t)(cq >> 1);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint4 hi, lo;
                float hf[8];
                split8_rn(v + 8 * q, hi, lo, hf);
                const uint32_t off = sw128_off(row, 32 * (cq & 1) + 8 * q);
                *reinterpret_cast<uint4*>(sm + OFF_S0 + kb * 16384 + off) = hi;
                *reinterpret_cast<uint4*>(sm + OFF_QL + kb * QL_BLK + 8192 + off) = lo;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= eGC;
            tmem_st16(tS + lb + 32 * cq, *reinterpret_cast<float(*)[16]>(v));
            tmem_st16(tS + lb + 32 * cq + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_st();
        }
        // saved-record mode: thread 0 copies tiles into the backward record with bulk copies; the copy of the
        // previous chunk's Delta^T / Dd^T low tiles has read them before anyone passes this barrier towards D
        if (rec_copier && c > 0) bulk_wait_read();
        fence_async_smem();
        sync_tc();
        if (rec_copier) {  // S0^T hi (= the record's bf16 S0^T), 32 KB contiguous here and there
            bulk_s2g(recb(c), sm + OFF_S0, 32768);
            bulk_commit();
        }
        // C. warp 16: Delta^T = V^T TV^T + S0hi^T (-W)^T -> bar_g; warp 17: Delta2^T = S0lo^T (-W)^T -> bar_g2,
        //    O = [Qg; -] (S0hi + S0lo) -> bar_q, then this chunk's P and the next chunk's Qg and vectors.
        //    Warps 8, 9, 12, 13 meanwhile emit the previous chunk's outputs.
        if (issuer) {
            wait_bar(bar_l1, par, a.err, 66, ok);
            const uint32_t idU = idesc_bf16(128, 64, 1, 0), idD = idesc_bf16(128, 64, 0, 0);
            if (!a.zero_v) {
                const uint64_t dV = desc_mnmajor(sb + OFF_V, 8192), dTV = desc_kmajor(sb + OFF_TV);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) umma_bf16(tDT, desc_at(dV, ks * 2048), desc_at(dTV, ks * 32), idU, ks > 0);
            }
            const uint64_t dS0 = desc_kmajor(sb + OFF_S0), dW = desc_kmajor(sb + OFF_W);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                umma_bf16(tDT, desc_at(dS0, kb * 16384 + ko), desc_at(dW, kb * 8192 + ko), idD, !a.zero_v || ks > 0);
            }
            umma_commit(bar_g);
        } else if (issuer2) {
            wait_bar(bar_l1, par, a.err, 67, ok);
            const uint32_t idD = idesc_bf16(128, 64, 0, 0), idO = idesc_bf16(128, 128, 0, 0);
            const uint64_t dSL = desc_kmajor(sb + OFF_QL + 8192), dW = desc_kmajor(sb + OFF_W);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                umma_bf16(tDT2, desc_at(dSL, kb * QL_BLK + ko), desc_at(dW, kb * 8192 + ko), idD, ks > 0);
            }
            umma_commit(bar_g2);
            const uint32_t tO = tm + T_O + par * 128;
            if (outs) {
                const uint64_t dQg = desc_kmajor(sb + OFF_QL), dHi = desc_kmajor(sb + OFF_S0),
                               dLo = desc_kmajor(sb + OFF_QL + 8192);
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // Qg (S0hi + S0lo)
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint32_t kb = ks >> 2, ko = (ks & 3) * 32;
                        const uint64_t s0 = h ? desc_at(dLo, kb * QL_BLK + ko) : desc_at(dHi, kb * 16384 + ko);
                        umma_bf16(tO, desc_at(dQg, kb * QL_BLK + ko), s0, idO, h > 0 || ks > 0);
                    }
                }
            }
            umma_commit(bar_q);
            if (c > 0 && outs) {
                wait_bar(bar_o, par ^ 1u, a.err, 54, ok);  // the P tiles of chunk c-1 have been read
                issue_l3(c);
            }
            if (c + 1 < nchunks) {  // Qg of chunk c read by the output product, vectors of c-1 by the output step
                wait_bar(bar_q, par, a.err, 61, ok);
                if (c > 0) wait_bar(bar_od, par ^ 1u, a.err, 68, ok);
                issue_l1_b(c + 1);
            }
        } else if (out_warp && c > 0) {
            wait_bar(bar_o, par ^ 1u, a.err, 56, ok);
            tc_fence_after();
            if (outs) output_step(c - 1);
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_od);
        }
        // D. Delta^T (TMEM, lanes = dv) -> Delta^T and Dd^T hi/lo tiles (all 16 warps, 16 tokens each)
        if (tid < NWORK) {
            if (c > 0) wait_bar(bar_o, par ^ 1u, a.err, 57, ok);  // the previous P Delta has read the tiles
            wait_bar(bar_g, par, a.err, 58, ok);
            wait_bar(bar_g2, par, a.err, 65, ok);
            tc_fence_after();
            float v[16], v2[16], x[16];
            tmem_ld16(tDT + lb + 16 * cq, v);
            tmem_ld16(tDT2 + lb + 16 * cq, v2);
            vload(vec, 16 * cq, x);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] += v2[e];
            // Delta hi = bf16(Delta), lo = Delta - hi; Dd = Delta x as hi = bf16(hi x), lo = Dd - that hi: the hi
            // tile and the Dd^T lo tile are the backward record's Delta^T and Dd^T low part as they are
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                uint4 hi, lo, dhi, dlo;
                float hf[8], hx[8], dhf[8];
                split8_rn(v + 8 * q, hi, lo, hf);
#pragma unroll
                for (int e = 0; e < 8; ++e) hx[e] = hf[e] * x[8 * q + e];
                split8_rn(hx, dhi, dlo, dhf);  // dhi = bf16(hi x); dlo below is taken against the exact Delta x
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                    const __nv_bfloat162 l = __floats2bfloat162_rn(v[8 * q + e] * x[8 * q + e] - dhf[e],
                                                                   v[8 * q + e + 1] * x[8 * q + e + 1] - dhf[e + 1]);
                    (&dlo.x)[e / 2] = *reinterpret_cast<const uint32_t*>(&l);
                }
                const uint32_t off = sw128_off(row, 16 * cq + 8 * q);
                *reinterpret_cast<uint4*>(sm + OFF_DH + off) = hi;
                *reinterpret_cast<uint4*>(sm + OFF_DL + off) = lo;
                *reinterpret_cast<uint4*>(sm + OFF_DDH + off) = dhi;
                *reinterpret_cast<uint4*>(sm + OFF_DDL + off) = dlo;
            }
        }
        if (rec_copier) bulk_wait_read();  // the S0^T copy has read its tiles before the next chunk's B
        fence_async_smem();
        sync_tc();
        if (rec_copier) {  // Delta^T hi and the Dd^T low part into the record
            bulk_s2g(recb(c) + kBwdRecDel, sm + OFF_DH, 16384);
            bulk_s2g(recb(c) + kBwdRecDdl, sm + OFF_DDL, 16384);
            bulk_commit();
        }
        // E. warp 16: S^T += Dd^T K (hi + lo) -> bar_s; warp 17: the next chunk's Qg and vectors, then
        //    O += P Delta (hi.hi + lo.hi + hi.lo) -> bar_o
        if (issuer) {
            wait_bar(bar_l2, par, a.err, 59, ok);
            tc_fence_after();
            const uint32_t idS = idesc_bf16(128, 128, 0, 1);
            const uint64_t dK = desc_mnmajor(sb + OFF_K, 8192);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint64_t dd = desc_kmajor(sb + (h ? OFF_DDL : OFF_DDH));
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) umma_bf16(tS, desc_at(dd, ks * 32), desc_at(dK, ks * 2048), idS, 1);
            }
            umma_commit(bar_s);
            if (c + 1 < nchunks) issue_l1_a(c + 1);  // the Delta^T products (bar_g, bar_g2 waited) read -W, TV, V
        } else if (issuer2) {
            if (outs) {
                wait_bar(bar_l3, par, a.err, 60, ok);
                tc_fence_after();
                const uint32_t idO = idesc_bf16(128, 128, 0, 0);
                const uint32_t tO = tm + T_O + par * 128;
                const uint64_t dDH = desc_kmajor(sb + OFF_DH), dDL = desc_kmajor(sb + OFF_DL),
                               dPH = desc_kmajor(sb + OFF_PH), dPL = desc_kmajor(sb + OFF_PL);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t dh = desc_at(dDH, ks * 32), dl = desc_at(dDL, ks * 32);
                    umma_bf16(tO, desc_at(dPH, ks * 32), dh, idO, 1);
                    umma_bf16(tO, desc_at(dPL, ks * 32), dh, idO, 1);
                    umma_bf16(tO, desc_at(dPH, ks * 32), dl, idO, 1);
                }
            }
            umma_commit(bar_o);
        }
    }
    // the last chunk's outputs and the final state
    if (nchunks > 0) {
        const uint32_t par = (uint32_t)(nchunks - 1) & 1u;
        wait_bar(bar_o, par, a.err, 62, ok);
        wait_bar(bar_s, par, a.err, 63, ok);
        tc_fence_after();
        if (out_warp && outs) output_step(nchunks - 1);
    }
    if (ok && a.ht && tid < NWORK) {
        float* ht = a.ht + ((int64_t)n * a.HV + hv) * 16384;
        float v[32];
        tmem_ld16(tS + lb + 32 * cq, *reinterpret_cast<float(*)[16]>(v));
        tmem_ld16(tS + lb + 32 * cq + 16, *reinterpret_cast<float(*)[16]>(v + 16));
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) ht[(32 * cq + i) * 128 + row] = v[i];
    }
    if (rec_copier) bulk_wait_all();  // the last records are in global memory before the CTA ends
    sync_tc();
    if (warp == 0) tmem_dealloc(tm, T_COLS);
}

// First flattened chunk of every sequence: exclusive scan of ceil(len_n / 64) over cu_seqlens (one CTA);
// cbase[N] = the total.
__global__ void __launch_bounds__(1024) chunk_base_kernel(const int64_t* __restrict__ cu, int64_t N,
                                                          int64_t* __restrict__ cbase) {
    __shared__ int64_t wsum[32];
    __shared__ int64_t carry;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < N; base += 1024) {
        const int64_t n = base + tid;
        const int64_t x = n < N ? (cu[n + 1] - cu[n] + 63) / 64 : 0;
        int64_t s = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane == 31) wsum[warp] = s;
        __syncthreads();
        if (warp == 0) {
            int64_t w = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += y;
            }
            wsum[lane] = w;
        }
        __syncthreads();
        const int64_t incl = s + (warp > 0 ? wsum[warp - 1] : 0) + carry;
        if (n < N) cbase[n] = incl - x;
        __syncthreads();
        if (tid == 1023) carry = incl;
        __syncthreads();
    }
    if (tid == 0) cbase[N] = carry;
}

// Zero the backward-record slots past the last sequence's chunks (the record buffer is sized for the worst
// split of the packed tokens): the saved buffer is then the same bytes on every call with these inputs.
__global__ void record_tail_zero_kernel(uint8_t* __restrict__ rec, const int64_t* __restrict__ total_chunks,
                                        int64_t HV, int64_t capacity_chunks) {
    const int64_t begin = total_chunks[0] * HV * (int64_t)(kBwdRecordBytes / 16);
    const int64_t end = capacity_chunks * HV * (int64_t)(kBwdRecordBytes / 16);
    uint4* p = reinterpret_cast<uint4*>(rec);
    for (int64_t i = begin + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < end;
         i += (int64_t)gridDim.x * blockDim.x)
        p[i] = make_uint4(0, 0, 0, 0);
}

size_t chunk_fwd_split_workspace(int64_t B, int64_t T, int64_t N, int64_t HV, bool varlen) {
    const int64_t chunks = varlen ? (B * T + 63 * N) / 64 + N : N * ((T + 63) / 64);
    size_t bytes = (size_t)chunks * HV * kFwdRecordBytes;
    if (varlen) bytes += ((size_t)(N + 1) * 8 + 255) / 256 * 256;
    return bytes;
}

// Workspace layout of chunk_fwd_split: varlen: cbase [N + 1] (256-byte aligned), then the records.
static void split_ws(const ChunkLaunch& L, void* ws, uint8_t*& rec, int64_t*& cbase) {
    rec = (uint8_t*)ws;
    cbase = nullptr;
    if (L.cu) {
        cbase = (int64_t*)ws;
        rec = (uint8_t*)ws + ((size_t)(L.N + 1) * 8 + 255) / 256 * 256;
    }
}

int chunk_prep_pass(const ChunkLaunch& L, void* ws, cudaStream_t s) {
    if (L.N * L.HV == 0) return GDN_OK;
    if (smem_optin((const void*)chunk_prep_kernel, (int)cp::SMEM_BYTES) != cudaSuccess) return GDN_ERR_LAUNCH;
    const int64_t Ttot = L.B * L.T;
    uint8_t* rec;
    int64_t* cbase;
    split_ws(L, ws, rec, cbase);
    if (L.cu) {
        chunk_base_kernel<<<1, 1024, 0, s>>>(L.cu, L.N, cbase);
        count_launch();
        if (L.bwd_rec) {
            const int64_t capacity = (Ttot + 63 * L.N) / 64 + L.N;  // chunk_saved_bytes' chunk count
            record_tail_zero_kernel<<<148, 256, 0, s>>>((uint8_t*)L.bwd_rec, cbase + L.N, L.HV, capacity);
            count_launch();
        }
    }
    ChunkPrepArgs p;
    memset(&p, 0, sizeof(p));
    if (!make_tmap_3d_sw128(&p.tq, L.q, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    if (!make_tmap_3d_sw128(&p.tk, L.k, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    p.g = L.g;
    p.beta = L.beta;
    p.cu = L.cu;
    p.cbase = cbase;
    p.rec = rec;
    p.rec_bwd = (uint8_t*)L.bwd_rec;
    p.err = L.err;
    p.T = L.T;
    p.H = (int)L.H;
    p.HV = (int)L.HV;
    p.g_dtype = L.g_dtype;
    p.beta_dtype = L.beta_dtype;
    p.l2norm = L.l2norm;
    p.scale = L.scale;
    const int64_t maxlen = L.max_seqlen > 0 ? L.max_seqlen : (L.cu ? Ttot : L.T);
    const int64_t maxchunks = (maxlen + 63) / 64;
    if (maxchunks > 0) {
        chunk_prep_kernel<<<dim3((unsigned)maxchunks, (unsigned)(L.N * L.HV)), cp::NTHR, cp::SMEM_BYTES, s>>>(p);
        count_launch();
    }
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int chunk_state_pass(const ChunkLaunch& L, void* ws, cudaStream_t s) {
    if (L.N * L.HV == 0) return GDN_OK;
    if (smem_optin((const void*)chunk_state_kernel, (int)cs::SMEM_BYTES) != cudaSuccess) return GDN_ERR_LAUNCH;
    const int64_t Ttot = L.B * L.T;
    uint8_t* rec;
    int64_t* cbase;
    split_ws(L, ws, rec, cbase);
    ChunkStateArgs a;
    memset(&a, 0, sizeof(a));
    if (!make_tmap_3d_sw128(&a.tk, L.k, 128, L.H, Ttot, 128, L.H * 128, 64)) return GDN_ERR_ALIGN;
    if (!make_tmap_3d_sw128(&a.tv, L.v, 128, L.HV, Ttot, 128, L.HV * 128, 64)) return GDN_ERR_ALIGN;
    a.rec = rec;
    a.cbase = cbase;
    a.rec_bwd = (uint8_t*)L.bwd_rec;
    a.o = L.o;
    a.h0 = L.h0;
    a.ht = L.ht;
    a.ckpt = L.ckpt;
    a.cu = L.cu;
    a.err = L.err;
    a.T = L.T;
    a.HV = (int)L.HV;
    a.H = (int)L.H;
    a.ckpt_every = L.ckpt_every;
    a.zero_v = L.zero_v;
    a.h0_identity = L.h0_identity;
    chunk_state_kernel<<<(unsigned)(L.N * L.HV), cs::NTHR, cs::SMEM_BYTES, s>>>(a);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

int chunk_fwd_split(const ChunkLaunch& L, void* ws, cudaStream_t s) {
    const int st = chunk_prep_pass(L, ws, s);
    return st != GDN_OK ? st : chunk_state_pass(L, ws, s);
}

}  // namespace gdn
