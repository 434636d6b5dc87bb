// Joining the pieces of sequences cut for training on pieces (sorernn_b200/pieces.py): the chain of affine
// maps along each sequence's pieces, forward (the state entering every piece) and reverse (the gradient of
// every piece's end state).
//
// Piece p of sequence n maps the state entering it to the state leaving it, S_out = M_p S_in + C_p (M_p is
// dk x dk, C_p the piece's final state from its own start, dk x dv; the gated delta rule of gdn_ref.py:18-21 is
// linear in (S, v)), and the backward maps the gradient leaving it to the one entering, dS_in = M_p^T dS_out
// + R_p. Both chains are serial in p but independent across (sequence, head) and across the dv columns, so
// one CTA per (sequence, head, 16-column block) walks the pieces with fp32 FMAs on the CUDA cores: 128 CTAs at
// 16 (sequence, head) pairs, the case the pieces are for. Each thread keeps a 4 x 4 block of the running value,
// so the products are bound by shared-memory reads at 16 FMAs per read rather than 8 or fewer. The column
// block of the running value stays in shared memory; each step's map (64 KB, shared through L2 by the 8 CTAs
// of a (sequence, head)) is staged into shared memory by 16-byte cp.async copies one step ahead, so the L2
// latency hides behind the previous step's FMAs.
#include "common.cuh"
#include "kernels.h"
#include "launch.h"

namespace gdn {

namespace pc {
// thread t: rows rg + 32 r (rg = t / 4, r = 0..3) and columns 4 (t % 4) .. + 3 of the CTA's 16-column block,
// so every shared-memory read of a k step serves 16 FMAs: the running value's rows are read once per thread
// as 16 bytes, and a warp's map reads (8 rows 1 apart, or one row 16 bytes at a time) hit distinct banks
constexpr int NTHR = 128;
constexpr int D = 128;
constexpr int BLK = 16;   // columns per CTA
constexpr int LDM = 132;  // padded row stride of a staged map: 8 consecutive rows' 16-byte chunks at one k hit
                          // 8 distinct bank groups
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
                                                                int mode) {
    using namespace pc;
    const bool reverse = mode == 1;
    const bool product = mode == 2;  // the terms of pieces 1 .. P-1 are zero: final = M_{P-1} .. M_1 terms[0]
    extern __shared__ __align__(16) float sm_chain[];
    float* Ms = sm_chain;                // [2][D][LDM]: the maps of this step and the next, staged by cp.async
    float* Y = sm_chain + 2 * D * LDM;  // running value, [k][16 columns]
    const int nh = blockIdx.x, cb = blockIdx.y, n = nh / HV, h = nh % HV;
    const int tid = threadIdx.x, rg = tid >> 2, c0 = 4 * (tid & 3);
    const int64_t mat = (int64_t)D * D;
    // this thread's 4 columns of row rg + 32 r of the [D, D] block of piece p (sequence n, head h)
    auto at = [&](int p, int r) -> int64_t {
        return (((int64_t)n * P + p) * HV + h) * mat + (int64_t)(rg + 32 * r) * D + cb * BLK + c0;
    };
    auto at0 = [&](int r) -> int64_t {  // the same in a [n_seq, HV, D, D] state
        return ((int64_t)n * HV + h) * mat + (int64_t)(rg + 32 * r) * D + cb * BLK + c0;
    };
    auto ld4 = [](const float* p) { return *reinterpret_cast<const float4*>(p); };
    auto st4 = [](float* p, const float4& v) { *reinterpret_cast<float4*>(p) = v; };
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
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (P > 1) stage(1);
    float4 y[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        if (!reverse) {  // Y = C_0; out[0] = start
            y[r] = ld4(terms + at(0, r));
            if (out) st4(out + at(0, r), start ? ld4(start + at0(r)) : zero4);
        } else {  // Z = start; out[P - 1] = Z
            y[r] = start ? ld4(start + at0(r)) : zero4;
            st4(out + at(P - 1, r), y[r]);
        }
    }
    for (int s = 1; s < P; ++s) {
        const int p = piece_of(s), m = map_of(s);
        if (!reverse && out) {
#pragma unroll
            for (int r = 0; r < 4; ++r) st4(out + at(p, r), y[r]);
        }
        __syncthreads();  // the previous step's readers of Y and of buffer (s + 1) & 1 are done
        const bool more = s + 1 < P;
        if (more) stage(s + 1);
        float acc[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            st4(&Y[(rg + 32 * r) * BLK + c0], y[r]);
            const float4 t = product ? zero4 : ld4(terms + at(m, r));
            acc[r][0] = t.x;
            acc[r][1] = t.y;
            acc[r][2] = t.z;
            acc[r][3] = t.w;
        }
        if (more) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();
        const float* Mb = Ms + (s & 1) * D * LDM;
        if (!reverse) {  // acc[r] += M[rg + 32 r][k] Y[k][:], four k per 16-byte map read
#pragma unroll 2
            for (int k4 = 0; k4 < D / 4; ++k4) {
                float4 a[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) a[r] = ld4(Mb + (rg + 32 * r) * LDM + 4 * k4);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 yk = ld4(&Y[(4 * k4 + q) * BLK + c0]);
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float av = q == 0 ? a[r].x : q == 1 ? a[r].y : q == 2 ? a[r].z : a[r].w;
                        acc[r][0] = fmaf(av, yk.x, acc[r][0]);
                        acc[r][1] = fmaf(av, yk.y, acc[r][1]);
                        acc[r][2] = fmaf(av, yk.z, acc[r][2]);
                        acc[r][3] = fmaf(av, yk.w, acc[r][3]);
                    }
                }
            }
        } else {  // acc[r] += M[k][rg + 32 r] Y[k][:] (M^T)
#pragma unroll 4
            for (int k = 0; k < D; ++k) {
                const float4 yk = ld4(&Y[k * BLK + c0]);
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float av = Mb[k * LDM + rg + 32 * r];
                    acc[r][0] = fmaf(av, yk.x, acc[r][0]);
                    acc[r][1] = fmaf(av, yk.y, acc[r][1]);
                    acc[r][2] = fmaf(av, yk.z, acc[r][2]);
                    acc[r][3] = fmaf(av, yk.w, acc[r][3]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) y[r] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        if (reverse) {
#pragma unroll
            for (int r = 0; r < 4; ++r) st4(out + at(p, r), y[r]);
        }
    }
    if (!reverse && final_state) {
#pragma unroll
        for (int r = 0; r < 4; ++r) st4(final_state + at0(r), y[r]);
    }
}

int piece_chain(int64_t n_seq, int64_t pieces, int64_t HV, const float* maps, const float* terms, const float* start,
                float* out, float* final_state, int mode, cudaStream_t s) {
    if (n_seq * HV == 0 || pieces == 0) return GDN_OK;
    if (smem_optin((const void*)piece_chain_kernel, pc::SMEM_BYTES) != cudaSuccess) return GDN_ERR_LAUNCH;
    piece_chain_kernel<<<dim3((unsigned)(n_seq * HV), pc::D / pc::BLK), pc::NTHR, pc::SMEM_BYTES, s>>>(
        maps, terms, start, out, final_state, (int)pieces, (int)HV, mode);
    count_launch();
    return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

}  // namespace gdn
