// gdn_chunk_bwd_noalloc: the backward entry point for callers that cannot allocate device memory.
//
// gdn_chunk_bwd needs a caller-provided workspace (the per-chunk records it rebuilds from the forward's
// checkpoints, an error word, and fp32 dq/dk accumulators for grouped value heads). Some callers have no
// way to allocate it at call time: a host runtime that reaches this library over a plain C FFI with no
// device allocator of its own, or a plugin whose execute/enqueue hook is not allowed to allocate. This
// entry point takes the same arguments minus the workspace and uses a fixed scratch array that lives in
// this library's device image instead. It allocates nothing: no cudaMalloc, no cudaFree, no allocating
// library routine.
//
// Limits and sharing:
//  * the scratch holds GDN_NOALLOC_SCRATCH_BYTES (36 MiB) on every GPU that loads the library, until the
//    process exits; a problem whose gdn_chunk_bwd_workspace_size() exceeds it is rejected with
//    GDN_ERR_SCRATCH_LIMIT before anything is launched. The workspace is 256 bytes plus one record per
//    (64-token chunk, value head), so the array holds 418 chunk-heads of the chunked kernels: for example
//    T = 1,024 tokens with 16 heads (256 chunk-heads) or T = 4,096 with 6 heads (384) in one call;
//  * every call on a device uses the same array and leaves its contents behind; what must start at zero
//    (the error word, the dq/dk accumulators) is cleared by each call, on its stream;
//  * calls whose work overlaps on the GPU (different streams, or several host threads) race on the array:
//    order them on one stream or serialize them;
//  * the device-side error word of the bounded waits sits in the array, which the caller never sees: a
//    noalloc call cannot report a device-side timeout (GDN_ERR_TIMEOUT); use gdn_chunk_bwd with a workspace
//    and gdn_workspace_error where that report is needed;
//  * the first call on each device looks up the array's device address (cudaGetSymbolAddress, with that
//    device current) and keeps it for the life of the device's primary context; make that first call
//    before any stream capture begins.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = GDN_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// In host code this name is only a host-side stand-in for the device array; the kernels are given the
// address returned by cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

void* g_scratch_ptr[kMaxDevices];
std::once_flag g_scratch_once[kMaxDevices];
cudaError_t g_scratch_status[kMaxDevices];

}  // namespace

extern "C" int gdn_chunk_bwd_noalloc(const gdn_problem* p, const void* q, const void* k, const void* v,
                                     const void* g, const void* beta, const float* initial_state,
                                     const float* checkpoints, const void* dout, const float* dht, void* dq,
                                     void* dk, void* dv, float* dg, float* dbeta, float* dh0, gdn_stream_t stream) {
    const int st = gdn::problem_status(p);  // an invalid problem reports the same status as gdn_chunk_bwd
    if (st != GDN_OK) return st;
    const size_t need = gdn_chunk_bwd_workspace_size(p);
    if (need > kNoAllocScratchBytes) return GDN_ERR_SCRATCH_LIMIT;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_LAUNCH;
    std::call_once(g_scratch_once[dev], [dev] {
        g_scratch_status[dev] = cudaGetSymbolAddress(&g_scratch_ptr[dev], g_noalloc_scratch);
    });
    if (g_scratch_status[dev] != cudaSuccess || g_scratch_ptr[dev] == nullptr) return GDN_ERR_LAUNCH;
    return gdn_chunk_bwd(p, q, k, v, g, beta, initial_state, checkpoints, dout, dht, dq, dk, dv, dg, dbeta, dh0,
                         g_scratch_ptr[dev], kNoAllocScratchBytes, stream);
}
