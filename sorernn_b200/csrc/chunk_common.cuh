// Device helpers shared by the chunked forward and backward kernels.
#pragma once
#include "common.cuh"

namespace gdn {

// ---- warp-level bf16 MMA on fp32 data, split into bf16 hi + lo operands ----------------------------
// x = hi + lo with hi = bf16(x), lo = bf16(x - hi) represents x to about 2^-17; a product taken as
// hi*hi + hi*lo + lo*hi (fp32 accumulation) is accurate to about 2^-16 of its terms.
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - __low2float(h), x1 - __high2float(h));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
__device__ __forceinline__ void mma_m16n8k16_bf16(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// d += A B over 16 k for one warp's 16 x 8 output tile: A (r, k) at a[r * lda + k], B (k, n) at
// b[k * ldb + n], both fp32 in shared memory (lda even). Fragment layout of m16n8k16 (lane = 4 g + t):
// A registers (g, 2t..2t+1), (g+8, 2t..), (g, 2t+8..), (g+8, 2t+8..); B registers (2t..2t+1, g),
// (2t+8.., g); accumulator (g, 2t..2t+1), (g+8, 2t..2t+1).
// the hi*hi term accumulates in d, the two cross terms in e (independent chains); the result is d + e
__device__ __forceinline__ void mma_split_k16(float (&d)[4], float (&e)[4], const float* a, int lda, const float* b,
                                              int ldb) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    uint32_t ah[4], al[4], bh[2], bl[2];
    float2 x;
    x = *reinterpret_cast<const float2*>(a + g * lda + 2 * t);
    split_bf16x2(x.x, x.y, ah[0], al[0]);
    x = *reinterpret_cast<const float2*>(a + (g + 8) * lda + 2 * t);
    split_bf16x2(x.x, x.y, ah[1], al[1]);
    x = *reinterpret_cast<const float2*>(a + g * lda + 2 * t + 8);
    split_bf16x2(x.x, x.y, ah[2], al[2]);
    x = *reinterpret_cast<const float2*>(a + (g + 8) * lda + 2 * t + 8);
    split_bf16x2(x.x, x.y, ah[3], al[3]);
    split_bf16x2(b[(2 * t) * ldb + g], b[(2 * t + 1) * ldb + g], bh[0], bl[0]);
    split_bf16x2(b[(2 * t + 8) * ldb + g], b[(2 * t + 9) * ldb + g], bh[1], bl[1]);
    mma_m16n8k16_bf16(d, ah, bh);
    mma_m16n8k16_bf16(e, ah, bl);
    mma_m16n8k16_bf16(e, al, bh);
}
// store a warp's 16 x 8 accumulator tile (times `sign`) at c[r * ldc + n] (ldc even)
__device__ __forceinline__ void store_tile16x8(float* c, int ldc, const float (&d)[4], const float (&e)[4],
                                               float sign) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    *reinterpret_cast<float2*>(c + g * ldc + 2 * t) = make_float2(sign * (d[0] + e[0]), sign * (d[1] + e[1]));
    *reinterpret_cast<float2*>(c + (g + 8) * ldc + 2 * t) = make_float2(sign * (d[2] + e[2]), sign * (d[3] + e[3]));
}

// T = (I + A)^-1 for a strictly lower-triangular 64 x 64 fp32 matrix A stored in shared memory with row
// stride `ST` floats (ST % 4 == 0; the upper triangle holds zeros), in place; `Y` is 32 x 36 fp32
// scratch. Called by warps 0-7 alone (256 threads, synchronised by named barrier 1), so the other warps
// of the CTA can work meanwhile. Block doubling: for L = [[T0, 0], [A10, T1]] with T0, T1 the inverses of
// the diagonal blocks, the lower-left block of L^-1 is -T1 (A10 T0):
//  1. the eight 8 x 8 diagonal blocks by column-wise forward substitution (threads 0-63, one column each);
//  2. 8-blocks -> 16-blocks, all four at once: two 8 x 8 x 8 products (fp32 FMA, one output per thread);
//  3. 16-blocks -> 32-blocks, both pairs at once: two 16 x 16 x 16 products on the tensor cores (warps
//     0-3, one 16 x 8 tile each; bf16 hi/lo splits);
//  4. 32-blocks -> 64: two 32 x 32 x 32 products on the tensor cores (warps 0-7, one 16 x 8 tile each).
// Every product runs over the full block width (the zeros above the diagonals make that exact). The
// tensor-core merges carry about 2^-16 relative error, far below the bf16 rounding T's consumers apply.
__device__ __forceinline__ void solve_sync256() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
constexpr int kSolveYStride = 36;  // Y row stride: conflict-free B-operand loads

template <int ST>
__device__ __forceinline__ void tri_inverse64(float* Am, float* Y) {
    const int tid = threadIdx.x, warp = tid >> 5;
    constexpr int LY = kSolveYStride;
    {  // 1. 8 x 8 diagonal blocks
        const int R = 8 * (tid >> 3), c = tid & 7;
        float x[8];
        if (tid < 64) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float sacc = 0.f;
#pragma unroll
                for (int j = 0; j < i; ++j) sacc = fmaf(Am[(R + i) * ST + R + j], x[j], sacc);
                x[i] = (i == c) ? 1.f : (i < c ? 0.f : -sacc);
            }
        }
        solve_sync256();
        if (tid < 64) {
#pragma unroll
            for (int i = 0; i < 8; ++i) Am[(R + i) * ST + R + c] = x[i];
        }
        solve_sync256();
    }
    {  // 2. 8 -> 16: block q (rows/columns 16q .. 16q + 15), output (r, c) of its 8 x 8 lower-left block
        const int q = tid >> 6, r = (tid >> 3) & 7, c = tid & 7, B0 = 16 * q;
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fmaf(Am[(B0 + 8 + r) * ST + B0 + k], Am[(B0 + k) * ST + B0 + c], acc);
        Y[q * 64 + r * 8 + c] = acc;
        solve_sync256();
        acc = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fmaf(Am[(B0 + 8 + r) * ST + B0 + 8 + k], Y[q * 64 + k * 8 + c], acc);
        Am[(B0 + 8 + r) * ST + B0 + c] = -acc;
        solve_sync256();
    }
    {  // 3. 16 -> 32: warp w < 4 takes pair p = w / 2 (rows/columns 32p .. 32p + 31), output columns 8 (w & 1) ..
        const int p = warp >> 1, n0 = 8 * (warp & 1), B0 = 32 * p;
        float* Yp = Y + p * 16 * LY;
        float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};
        if (warp < 4) {
            mma_split_k16(d, e, Am + (B0 + 16) * ST + B0, ST, Am + B0 * ST + B0 + n0, ST);  // A10 T0
            store_tile16x8(Yp + n0, LY, d, e, 1.f);
        }
        solve_sync256();
        if (warp < 4) {
            d[0] = d[1] = d[2] = d[3] = e[0] = e[1] = e[2] = e[3] = 0.f;
            mma_split_k16(d, e, Am + (B0 + 16) * ST + B0 + 16, ST, Yp + n0, LY);  // T1 (A10 T0)
            store_tile16x8(Am + (B0 + 16) * ST + B0 + n0, ST, d, e, -1.f);
        }
        solve_sync256();
    }
    {  // 4. 32 -> 64: warp w takes rows 32 + 16 (w >> 2) .., output columns 8 (w & 3) .. of the lower-left block
        const int m0 = 16 * (warp >> 2), n0 = 8 * (warp & 3);
        float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 32; ks += 16)
            mma_split_k16(d, e, Am + (32 + m0) * ST + ks, ST, Am + ks * ST + n0, ST);  // A10 T0
        store_tile16x8(Y + m0 * LY + n0, LY, d, e, 1.f);
        solve_sync256();
        d[0] = d[1] = d[2] = d[3] = e[0] = e[1] = e[2] = e[3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 32; ks += 16)
            mma_split_k16(d, e, Am + (32 + m0) * ST + 32 + ks, ST, Y + ks * LY + n0, LY);  // T1 (A10 T0)
        store_tile16x8(Am + (32 + m0) * ST + n0, ST, d, e, -1.f);
        solve_sync256();
    }
}

}  // namespace gdn
