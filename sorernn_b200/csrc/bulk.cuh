// Bulk (TMA engine) copies between global and shared memory without tensor maps, and the staging ring the
// streaming kernels (output norm-gate, causal conv) build on: one thread issues a tile's row copies onto a
// stage's mbarrier with the byte count expected, every thread waits for the stage's phase, and the stage is
// refilled only after a block barrier marks every read of it done.
#pragma once
#include "sm100.cuh"

namespace gdn {
namespace bulk {

// global -> shared, completion counted in bytes on `bar`; both addresses 16-byte aligned, bytes % 16 == 0
__device__ __forceinline__ void load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sm100::smem_u32(dst)),
                 "l"((uint64_t)src), "r"(bytes), "r"(sm100::smem_u32(bar))
                 : "memory");
}

// Largest stage count the per-block shared memory allows, and the dynamic shared memory of a launch.
constexpr uint32_t kBarBytes = 64;  // room for up to 8 stage mbarriers

inline cudaError_t allow_smem(const void* kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

inline int sm_count() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            sms = 148;
    }
    return sms;
}

}  // namespace bulk
}  // namespace gdn
