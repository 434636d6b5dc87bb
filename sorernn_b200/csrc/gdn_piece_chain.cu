// Joining the pieces of sequences cut for training on pieces (sorernn_b200/pieces.py): the chain of affine
// maps along each sequence's pieces, forward (the state entering every piece) and reverse (the gradient of
// every piece's end state).
//
// Piece p of sequence n maps the state entering it to the state leaving it, S_out = M_p S_in + C_p (M_p is
// dk x dk, C_p the piece's final state from its own start, dk x dv; the gated delta rule of gdn_ref.py:18-21 is
// linear in (S, v)), and the backward maps the gradient leaving it to the one entering, dS_in = M_p^T dS_out
// + R_p. Both chains are serial in p but independent across (sequence, head) and across the dv columns, so
// one CTA per (sequence, head, 16-column block) walks the pieces with fp32 FMAs on the CUDA cores: 128 CTAs at
// 16 (sequence, head) pairs, the case the pieces are for. The column block of the running value stays in
// shared memory; each step's map (64 KB, shared through L2 by the 8 CTAs of a (sequence, head)) is staged
// into shared memory by 16-byte cp.async copies one step ahead, so the L2 latency hides behind the previous
// step's FMAs.
#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace gdn {

namespace pc {
constexpr int NTHR = 256;  // thread t: row t / 2 of the running value, columns 8 (t % 2) .. + 7 of the block
constexpr int D = 128;
constexpr int BLK = 16;   // columns per CTA
constexpr int LDM = 132;  // padded row stride of a staged map: a quarter-warp's 16-byte reads of 8 rows hit
                          // 8 distinct bank groups, and a warp's reads of one column are consecutive words
constexpr int SMEM_BYTES = (2 * D * LDM + D * BLK) * 4;  // two map buffers + the running value
}  // namespace pc

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(pc::NTHR) piece_chain_kernel(const float* __restrict__ maps,
                                                                const float* __restrict__ terms,
                                                                const float* __restrict__ start, float* __restrict__ out,
                                                                float* __restrict__ final_state, int P, int HV,
                                                                int reverse) {
    using namespace pc;
    extern __shared__ __align__(16) float sm_chain[];
    float* Ms = sm_chain;                // [2][D][LDM]: the maps of this step and the next, staged by cp.async
    float* Y = sm_chain + 2 * D * LDM;  // running value, [k][16 columns]
    const int nh = blockIdx.x, cb = blockIdx.y, n = nh / HV, h = nh % HV;
    const int tid = threadIdx.x, i = tid >> 1, c0 = 8 * (tid & 1);
    const int64_t mat = (int64_t)D * D;
    // element (row r, column cb * BLK + c) of the [D, D] block of piece p
    auto at = [&](int p, int r, int c) -> int64_t {
        return (((int64_t)n * P + p) * HV + h) * mat + (int64_t)r * D + cb * BLK + c;
    };
    // step s (1 .. P-1) writes piece p and applies the map of piece m
    auto piece_of = [&](int s) { return reverse ? P - 1 - s : s; };
    auto map_of = [&](int s) { return reverse ? P - s : s; };
    auto stage = [&](int s) {  // the whole map of step s into buffer s & 1
        const float* src = maps + (((int64_t)n * P + map_of(s)) * HV + h) * mat;
        float* dst = Ms + (s & 1) * D * LDM;
        for (int e = tid; e < D * D / 4; e += NTHR) {
            const int r = e >> 5, c4 = e & 31;
            cp_async16(dst + r * LDM + 4 * c4, src + (int64_t)r * D + 4 * c4);
        }
        cp_async_commit();
    };
    const int64_t start_off = ((int64_t)n * HV + h) * mat + (int64_t)i * D + cb * BLK + c0;
    if (P > 1) stage(1);
    float y[8];
    if (!reverse) {  // Y = C_0; out[0] = start
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            y[e] = terms[at(0, i, c0 + e)];
            out[at(0, i, c0 + e)] = start ? start[start_off + e] : 0.f;
        }
    } else {  // Z = start; out[P - 1] = Z
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            y[e] = start ? start[start_off + e] : 0.f;
            out[at(P - 1, i, c0 + e)] = y[e];
        }
    }
    for (int s = 1; s < P; ++s) {
        const int p = piece_of(s), m = map_of(s);
        if (!reverse) {
#pragma unroll
            for (int e = 0; e < 8; ++e) out[at(p, i, c0 + e)] = y[e];
        }
        __syncthreads();  // the previous step's readers of Y and of buffer (s + 1) & 1 are done
        const bool more = s + 1 < P;
        if (more) stage(s + 1);
#pragma unroll
        for (int e = 0; e < 8; ++e) Y[i * BLK + c0 + e] = y[e];
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = terms[at(m, i, c0 + e)];
        if (more) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();
        const float* Mb = Ms + (s & 1) * D * LDM;
        if (!reverse) {  // acc += M[i][k] Y[k][:]: row i of M, 16 bytes at a time
            const float* row = Mb + i * LDM;
#pragma unroll 4
            for (int k4 = 0; k4 < D / 4; ++k4) {
                const float4 a = *reinterpret_cast<const float4*>(row + 4 * k4);
                const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 y0 = *reinterpret_cast<const float4*>(&Y[(4 * k4 + q) * BLK + c0]);
                    const float4 y1 = *reinterpret_cast<const float4*>(&Y[(4 * k4 + q) * BLK + c0 + 4]);
                    acc[0] = fmaf(av[q], y0.x, acc[0]);
                    acc[1] = fmaf(av[q], y0.y, acc[1]);
                    acc[2] = fmaf(av[q], y0.z, acc[2]);
                    acc[3] = fmaf(av[q], y0.w, acc[3]);
                    acc[4] = fmaf(av[q], y1.x, acc[4]);
                    acc[5] = fmaf(av[q], y1.y, acc[5]);
                    acc[6] = fmaf(av[q], y1.z, acc[6]);
                    acc[7] = fmaf(av[q], y1.w, acc[7]);
                }
            }
        } else {  // acc += M[k][i] Y[k][:] (M^T): column i of M
#pragma unroll 8
            for (int k = 0; k < D; ++k) {
                const float a = Mb[k * LDM + i];
                const float4 y0 = *reinterpret_cast<const float4*>(&Y[k * BLK + c0]);
                const float4 y1 = *reinterpret_cast<const float4*>(&Y[k * BLK + c0 + 4]);
                acc[0] = fmaf(a, y0.x, acc[0]);
                acc[1] = fmaf(a, y0.y, acc[1]);
                acc[2] = fmaf(a, y0.z, acc[2]);
                acc[3] = fmaf(a, y0.w, acc[3]);
                acc[4] = fmaf(a, y1.x, acc[4]);
                acc[5] = fmaf(a, y1.y, acc[5]);
                acc[6] = fmaf(a, y1.z, acc[6]);
                acc[7] = fmaf(a, y1.w, acc[7]);
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = acc[e];
        if (reverse) {
#pragma unroll
            for (int e = 0; e < 8; ++e) out[at(p, i, c0 + e)] = y[e];
        }
    }
    if (!reverse && final_state) {
#pragma unroll
        for (int e = 0; e < 8; ++e) final_state[start_off + e] = y[e];
    }
}

int piece_chain(int64_t n_seq, int64_t pieces, int64_t HV, const float* maps, const float* terms, const float* start,
                float* out, float* final_state, int reverse, cudaStream_t s) {
    if (n_seq * HV == 0 || pieces == 0) return GDN_OK;
    if (smem_optin((const void*)piece_chain_kernel, pc::SMEM_BYTES) != cudaSuccess) return GDN_ERR_LAUNCH;
    piece_chain_kernel<<<dim3((unsigned)(n_seq * HV), pc::D / pc::BLK), pc::NTHR, pc::SMEM_BYTES, s>>>(
        maps, terms, start, out, final_state, (int)pieces, (int)HV, reverse);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
