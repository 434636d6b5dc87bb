// Device helpers shared by the chunked forward and backward kernels.
#pragma once
#include "common.cuh"

namespace gdn {

// T = (I + A)^-1 for a strictly lower-triangular 64 x 64 fp32 matrix A stored in shared memory with row
// stride `ST` floats (ST % 4 == 0), in place; `Y` is 3 x 16 x 16 fp32 scratch. Called by all 256 threads
// of the CTA (contains barriers). Blocked by 16 x 16 tiles:
//  1. diagonal blocks by column-wise forward substitution (one thread per column of a block);
//  2. block rows r = 1..3: Y_s = sum_{m=s}^{r-1} A_rm T_ms, then T_rs = -T_rr Y_s, every thread computing
//     a 1 x 4 strip with float4 shared-memory loads.
template <int ST>
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
        __syncthreads();
        if (tid < 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) Am[(16 * b + i) * ST + 16 * b + cidx] = x[i];
        }
        __syncthreads();
    }
#pragma unroll 1
    for (int r = 1; r < 4; ++r) {
        // strips: (s < r, row i, column group c4) -> r * 64 strips
        const int s = tid >> 6, i = (tid >> 2) & 15, c4 = (tid & 3) * 4;
        if (s < r) {
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int m = 0; m < 3; ++m) {
                if (m >= s && m < r) {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const float a = Am[(16 * r + i) * ST + 16 * m + jj];
                        const float4 t = *reinterpret_cast<const float4*>(&Am[(16 * m + jj) * ST + 16 * s + c4]);
                        y.x = fmaf(a, t.x, y.x);
                        y.y = fmaf(a, t.y, y.y);
                        y.z = fmaf(a, t.z, y.z);
                        y.w = fmaf(a, t.w, y.w);
                    }
                }
            }
            *reinterpret_cast<float4*>(&Y[s * 256 + i * 16 + c4]) = y;
        }
        __syncthreads();
        if (s < r) {
            float4 t4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                if (jj <= i) {
                    const float a = Am[(16 * r + i) * ST + 16 * r + jj];
                    const float4 y = *reinterpret_cast<const float4*>(&Y[s * 256 + jj * 16 + c4]);
                    t4.x = fmaf(a, y.x, t4.x);
                    t4.y = fmaf(a, y.y, t4.y);
                    t4.z = fmaf(a, y.z, t4.z);
                    t4.w = fmaf(a, y.w, t4.w);
                }
            }
            *reinterpret_cast<float4*>(&Am[(16 * r + i) * ST + 16 * s + c4]) =
                make_float4(-t4.x, -t4.y, -t4.z, -t4.w);
        }
        __syncthreads();
    }
}

}  // namespace gdn
