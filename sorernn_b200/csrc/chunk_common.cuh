// Device helpers shared by the chunked forward and backward kernels.
#pragma once
#include "common.cuh"

namespace gdn {

// T = (I + A)^-1 for a strictly lower-triangular 64 x 64 fp32 matrix A stored in shared memory with row
// stride `ST` floats (ST % 4 == 0; the upper triangle holds zeros), in place; `Y` is 32 x 32 fp32
// scratch. Only threads 0-63 compute; with GROUP64 the caller is those 64 threads alone (warps 0-1,
// synchronised by named barrier 1, so the other warps can work meanwhile), otherwise every thread of the
// CTA calls it (CTA barriers). Block doubling:
//  1. the four 16 x 16 diagonal blocks by column-wise forward substitution (one thread per column);
//  2. merge 16-blocks into 32-blocks, both pairs at once: for L = [[T0, 0], [A10, T1]]^-1 the lower-left
//     block is -T1 (A10 T0): two 16 x 16 x 16 products;
//  3. merge the two 32-blocks the same way: two 32 x 32 x 32 products.
// Every product runs over the full block width (the zeros above the diagonals make that exact), so the
// dependent chains are 16 + 16 + 32 + 32 multiply-adds after the substitution.
template <bool GROUP64>
__device__ __forceinline__ void solve_sync() {
    if constexpr (GROUP64) asm volatile("bar.sync 1, 64;" ::: "memory");
    else __syncthreads();
}
template <int ST, bool GROUP64 = false>
__device__ __forceinline__ void tri_inverse64(float* Am, float* Y) {
    const int tid = threadIdx.x;
    {
        float x[16];
        const int b = tid >> 4, cidx = tid & 15;
        if (tid < 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float sacc = 0.f;
#pragma unroll
                for (int j = 0; j < i; ++j) sacc = fmaf(Am[(16 * b + i) * ST + 16 * b + j], x[j], sacc);
                x[i] = (i == cidx) ? 1.f : (i < cidx ? 0.f : -sacc);
            }
        }
        solve_sync<GROUP64>();
        if (tid < 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) Am[(16 * b + i) * ST + 16 * b + cidx] = x[i];
        }
        solve_sync<GROUP64>();
    }
    // The merge products are bound by shared-memory bandwidth (bytes delivered to threads), not by their
    // dependent chains, so each thread computes a register block (2 x 4 or 4 x 4 outputs) from float4 loads
    // and reuses every loaded value 4 or 2 times. Block rows are interleaved (row = base + 8 r) so the
    // float4 loads of a warp's rows fall in distinct banks.
    {  // 16-blocks -> 32-blocks: pair p (warp p) covers rows/columns 32p .. 32p + 31; rows {i, i + 8}
        const int p = (tid >> 5) & 1, i = (tid >> 2) & 7, c4 = 4 * (tid & 3);
        const int r0 = 32 * p + 16, c0 = 32 * p;  // lower-left block origin
        if (tid < 64) {
            float acc[2][4] = {};
#pragma unroll
            for (int kq = 0; kq < 16; kq += 4) {
                float av[2][4];
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const float4 a4 = *reinterpret_cast<const float4*>(&Am[(r0 + i + 8 * r) * ST + c0 + kq]);
                    av[r][0] = a4.x; av[r][1] = a4.y; av[r][2] = a4.z; av[r][3] = a4.w;
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 t = *reinterpret_cast<const float4*>(&Am[(c0 + kq + kk) * ST + c0 + c4]);
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        acc[r][0] = fmaf(av[r][kk], t.x, acc[r][0]);
                        acc[r][1] = fmaf(av[r][kk], t.y, acc[r][1]);
                        acc[r][2] = fmaf(av[r][kk], t.z, acc[r][2]);
                        acc[r][3] = fmaf(av[r][kk], t.w, acc[r][3]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < 2; ++r)
                *reinterpret_cast<float4*>(&Y[p * 256 + (i + 8 * r) * 16 + c4]) =
                    make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        }
        solve_sync<GROUP64>();
        if (tid < 64) {
            float acc[2][4] = {};
#pragma unroll
            for (int kq = 0; kq < 16; kq += 4) {
                float av[2][4];
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const float4 a4 = *reinterpret_cast<const float4*>(&Am[(r0 + i + 8 * r) * ST + r0 + kq]);
                    av[r][0] = a4.x; av[r][1] = a4.y; av[r][2] = a4.z; av[r][3] = a4.w;
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 yv = *reinterpret_cast<const float4*>(&Y[p * 256 + (kq + kk) * 16 + c4]);
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        acc[r][0] = fmaf(av[r][kk], yv.x, acc[r][0]);
                        acc[r][1] = fmaf(av[r][kk], yv.y, acc[r][1]);
                        acc[r][2] = fmaf(av[r][kk], yv.z, acc[r][2]);
                        acc[r][3] = fmaf(av[r][kk], yv.w, acc[r][3]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < 2; ++r)
                *reinterpret_cast<float4*>(&Am[(r0 + i + 8 * r) * ST + c0 + c4]) =
                    make_float4(-acc[r][0], -acc[r][1], -acc[r][2], -acc[r][3]);
        }
        solve_sync<GROUP64>();
    }
    {  // 32-blocks -> 64: rows 32-63, columns 0-31; 64 threads, rows {i, i + 8, i + 16, i + 24} x 4 columns
        const int i = (tid >> 3) & 7, c4 = 4 * (tid & 7);
        if (tid < 64) {
            float acc[4][4] = {};
#pragma unroll 2
            for (int kq = 0; kq < 32; kq += 4) {
                float av[4][4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float4 a4 = *reinterpret_cast<const float4*>(&Am[(32 + i + 8 * r) * ST + kq]);
                    av[r][0] = a4.x; av[r][1] = a4.y; av[r][2] = a4.z; av[r][3] = a4.w;
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 t = *reinterpret_cast<const float4*>(&Am[(kq + kk) * ST + c4]);
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        acc[r][0] = fmaf(av[r][kk], t.x, acc[r][0]);
                        acc[r][1] = fmaf(av[r][kk], t.y, acc[r][1]);
                        acc[r][2] = fmaf(av[r][kk], t.z, acc[r][2]);
                        acc[r][3] = fmaf(av[r][kk], t.w, acc[r][3]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
                *reinterpret_cast<float4*>(&Y[(i + 8 * r) * 32 + c4]) =
                    make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        }
        solve_sync<GROUP64>();
        if (tid < 64) {
            float acc[4][4] = {};
#pragma unroll 2
            for (int kq = 0; kq < 32; kq += 4) {
                float av[4][4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float4 a4 = *reinterpret_cast<const float4*>(&Am[(32 + i + 8 * r) * ST + 32 + kq]);
                    av[r][0] = a4.x; av[r][1] = a4.y; av[r][2] = a4.z; av[r][3] = a4.w;
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 yv = *reinterpret_cast<const float4*>(&Y[(kq + kk) * 32 + c4]);
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        acc[r][0] = fmaf(av[r][kk], yv.x, acc[r][0]);
                        acc[r][1] = fmaf(av[r][kk], yv.y, acc[r][1]);
                        acc[r][2] = fmaf(av[r][kk], yv.z, acc[r][2]);
                        acc[r][3] = fmaf(av[r][kk], yv.w, acc[r][3]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
                *reinterpret_cast<float4*>(&Am[(32 + i + 8 * r) * ST + c4]) =
                    make_float4(-acc[r][0], -acc[r][1], -acc[r][2], -acc[r][3]);
        }
        solve_sync<GROUP64>();
    }
}

}  // namespace gdn
