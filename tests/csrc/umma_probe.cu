// Test-only probes of the sm_100a building blocks used by the chunk kernels (built into
// tests/_build/libumma_probe.so by tests/csrc/build_probe.py; never part of the product library):
//   * umma_probe: one CTA computes D[128 x N] = A[128 x K] * B[N x K]^T with tcgen05.mma from shared-memory
//     operands in every major-ness combination (K-major / MN-major), accumulator read back with tcgen05.ld;
//   * tma_probe: one 128-byte-swizzled TMA tile load, de-swizzled by the layout formula the kernels use;
//   * wait_timeout_probe: the kernels' bounded mbarrier wait on a barrier nothing arrives on: it must give
//     up after its poll limit, record the error code and return (no trap, no hang), leaving the context
//     usable.
#include <cuda_bf16.h>

#include "../../sorernn_b200/csrc/sm100.cuh"
#include "../../sorernn_b200/csrc/tmap.h"

using namespace gdn::sm100;

__global__ void __launch_bounds__(128) umma_probe_kernel(const __nv_bfloat16* A, const __nv_bfloat16* B, float* D,
                                                         int N, int K, int a_mn, int b_mn, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;              // 128 x K bf16 = 32 KB max
    uint8_t* sB = smem + 128 * 256;  // N x K bf16
    __shared__ uint64_t bar;
    __shared__ uint32_t tbase;
    const int tid = threadIdx.x;
    // fill A
    for (int e = tid; e < 128 * K; e += 128) {
        const int m = e / K, k = e % K;
        uint32_t off = a_mn ? (uint32_t)(m >> 6) * K * 128 + sw128_off(k, m & 63)
                            : (uint32_t)(k >> 6) * 128 * 128 + sw128_off(m, k & 63);
        *(__nv_bfloat16*)(sA + off) = A[e];
    }
    for (int e = tid; e < N * K; e += 128) {
        const int n = e / K, k = e % K;
        uint32_t off = b_mn ? (uint32_t)(n >> 6) * K * 128 + sw128_off(k, n & 63)
                            : (uint32_t)(k >> 6) * N * 128 + sw128_off(n, k & 63);
        *(__nv_bfloat16*)(sB + off) = B[e];
    }
    fence_async_smem();
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    if (tid < 32) tmem_alloc(&tbase, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t d = tbase;
    if (tid == 0) {
        const uint32_t idesc = idesc_bf16(128, N, a_mn, b_mn);
        for (int ks = 0; ks < K / 16; ++ks) {
            uint64_t ad, bd;
            if (a_mn) ad = desc_mnmajor(smem_u32(sA) + ks * 2048, K * 128);
            else ad = desc_kmajor(smem_u32(sA) + (ks >> 2) * 128 * 128 + (ks & 3) * 32);
            if (b_mn) bd = desc_mnmajor(smem_u32(sB) + ks * 2048, K * 128);
            else bd = desc_kmajor(smem_u32(sB) + (ks >> 2) * N * 128 + (ks & 3) * 32);
            umma_bf16(d, ad, bd, idesc, ks > 0);
        }
        umma_commit(&bar);
    }
    __syncwarp();
    mbar_wait(&bar, 0, err, 1);
    tc_fence_after();
    const int w = tid >> 5, l = tid & 31;
    for (int c0 = 0; c0 < N; c0 += 16) {
        float v[16];
        tmem_ld16(tmem_addr(d, 32 * w, c0), v);
        tmem_wait_ld();
        for (int i = 0; i < 16; ++i) D[(32 * w + l) * N + c0 + i] = v[i];
    }
    tc_fence_before();
    __syncthreads();
    if (tid < 32) tmem_dealloc(d, 128);
}

__global__ void tma_probe_kernel(const __grid_constant__ CUtensorMap map, int c0, int c1, int c2, __nv_bfloat16* out,
                                 int* err) {
    __shared__ __align__(1024) uint8_t tile[64 * 128];
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, 64 * 128);
        tma_load_3d(tile, &map, &bar, c0, c1, c2);
    }
    mbar_wait(&bar, 0, err, 2);
    for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
        const int r = e / 64, c = e % 64;
        out[e] = *(const __nv_bfloat16*)(tile + sw128_off(r, c));
    }
}

extern "C" int umma_probe(const void* A, const void* B, float* D, int N, int K, int a_mn, int b_mn, int* err,
                          cudaStream_t s) {
    const int smem = 128 * 256 + 128 * 256 + 1024;
    cudaFuncSetAttribute(umma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    umma_probe_kernel<<<1, 128, smem, s>>>((const __nv_bfloat16*)A, (const __nv_bfloat16*)B, D, N, K, a_mn, b_mn,
                                           err);
    return (int)cudaGetLastError();
}

// src: [T][H][128] bf16. Loads the 64-token x 64-column box at (col0 = half*64, head h, token t0).
extern "C" int tma_probe(const void* src, long T, long H, int t0, int h, int half, void* out, int* err,
                         cudaStream_t s) {
    CUtensorMap m;
    if (!gdn::make_tmap_3d_sw128(&m, src, 128, H, T, 128, H * 128, 64)) return -1;
    tma_probe_kernel<<<1, 128, 0, s>>>(m, half * 64, h, t0, (__nv_bfloat16*)out, err);
    return (int)cudaGetLastError();
}

// One CTA: thread 0 inits an mbarrier expecting one arrival that never comes and waits on it with the
// kernels' bounded wait (mbar_wait) and `limit` polls; every thread then waits on the same barrier
// once more with limit 1 (the kernels' "already failed" mode). out[0] = 1 if the first wait reported
// success, out[1] = number of threads whose second wait reported success; *err receives the code.
__global__ void wait_timeout_probe_kernel(int* err, int* out, unsigned limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) out[0] = mbar_wait(&bar, 0, err, 77, limit) ? 1 : 0;
    __syncthreads();
    const bool ok2 = mbar_wait(&bar, 0, err, 78, 1u);
    if (ok2) atomicAdd(&out[1], 1);
}

extern "C" int wait_timeout_probe(int* err, int* out, unsigned limit, cudaStream_t s) {
    wait_timeout_probe_kernel<<<1, 64, 0, s>>>(err, out, limit);
    return (int)cudaGetLastError();
}
