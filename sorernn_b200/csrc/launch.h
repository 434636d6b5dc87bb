// Host-side launch helpers shared by the kernel files.
#pragma once
#include <cuda_runtime.h>

#include <mutex>
#include <tuple>
#include <vector>

namespace gdn {

// Opts `kernel` in to `bytes` of dynamic shared memory on the current device. The attribute is a
// per-device property of the function, so the opt-in is remembered per (kernel, device); the table is
// guarded by a mutex, so host threads launching on several devices may call this concurrently.
inline cudaError_t smem_optin(const void* kernel, int bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::vector<std::tuple<const void*, int, int>> done;  // (kernel, device, bytes)
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& t : done)
        if (std::get<0>(t) == kernel && std::get<1>(t) == dev && std::get<2>(t) >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.emplace_back(kernel, dev, bytes);
    return e;
}

// Number of SMs of the current device.
inline int device_sm_count() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 148;
    return sms;
}

}  // namespace gdn
