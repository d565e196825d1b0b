// block_noalloc.cu -- the Mamba block forward with its scratch in a static
// device array, for callers that cannot allocate.
//
// sacc_mamba_block_forward keeps its intermediates (x_in, z, u, dt, B, C,
// delta, y and the RMSNorm row scales) in a workspace that the caller
// allocates.  Some callers cannot do that: a TensorRT-style plugin whose
// engine grants it no workspace (the scan plugins of this library report a
// workspace size of 0) may not allocate inside enqueue, and a per-frame
// tracking loop that runs under a fixed memory budget should not allocate on
// its critical path.  sacc_mamba_block_forward_noalloc serves them: the
// intermediates live in `g_block_scratch` below, a file-scope device array of
// SACC_NOALLOC_SCRATCH_BYTES (24 MiB, enough for 256 tracks x 32 frames at
// d_inner 256).  CUDA reserves it when it loads this module on a device; the
// entry point itself calls no cudaMalloc, cudaFree or allocating routine.
//
// Set-up: the first call on each device, with that device current, looks up
// the array's device address (cudaGetSymbolAddress) and caches it per device
// ordinal; later calls reuse it.  Make that first call before any stream
// capture.  A cudaDeviceReset drops the module and makes the cached address
// stale, so do not use this entry point across a device reset.
//
// Sharing: every call on a device uses the same array, and the array keeps
// the last call's contents.  Each intermediate is written in full before it
// is read; the one region that must start at zero, the chunk-parallel scan's
// hand-off flags, is cleared on the stream (cudaMemsetAsync, which allocates
// nothing) right before the scan launch that uses it, so flags left by an
// earlier call or graph replay never match.  Two calls whose work
// overlaps on the GPU (different streams without an event between them, or
// different host threads) race on the array; order them on one stream.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"

namespace sacc {
namespace {

__device__ __align__(256) unsigned char g_block_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_block_scratch on the current device, looked up once per
// device ordinal.
cudaError_t block_scratch(void** addr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaGetSymbolAddress(addr, g_block_scratch);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_block_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *addr = g_scratch_addr[dev];
    return cudaSuccess;
}

} // namespace

cudaError_t launch_mamba_block_noalloc(const SaccMambaBlockArgs& a, cudaStream_t stream) {
    if (mamba_block_workspace(a) > kNoAllocScratchBytes) return cudaErrorInvalidValue;
    void* scratch = nullptr;
    const cudaError_t e = block_scratch(&scratch);
    if (e != cudaSuccess) return e;
    return launch_mamba_block(a, scratch, stream);
}

} // namespace sacc
