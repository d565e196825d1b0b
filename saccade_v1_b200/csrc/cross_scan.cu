// cross_scan.cu -- Cross-Scan expand / merge around each level's Mamba block.
//
// Contract: reference cuda/selective_scan.cu:157-192 (kernels) and :402-434
// (host).  Direction k reads token t at the row-major position of the
// k-flipped map: 0 identity, 1 flip H and W, 2 flip W, 3 flip H; sequence row
// = direction * batch + image.  Merge averages ((y0 + y1) + y2) + y3 times
// 0.25, and falls back to summing the quarters when the sum overflows.
//
// B200 layout: x is (batch, C, H*W) and tokens are (4 batch, H*W, C), a
// transpose per direction.  Both kernels move 32x32 tiles through shared
// memory so that the global reads and writes are coalesced along their
// contiguous axis (positions for x/out, channels for tokens).
#include <cuda_runtime.h>

#include <cfloat>
#include <string>

#include "internal.h"

namespace sacc {
namespace {

constexpr int kTile = 32;
constexpr int kRows = 8; // 32 x 8 threads per tile

__device__ __forceinline__ bool finite32(float x) { return fabsf(x) <= FLT_MAX; }

// Source position (h * W + w) of token t in direction k (reference
// src/selective_scan.cpp:111-116; each flip is an involution, so this is also
// the token of position t in direction k).
__device__ __forceinline__ unsigned long long cross_source(unsigned k, unsigned long long t, unsigned long long H,
                                                           unsigned long long W) {
    const unsigned long long row = t / W, col = t % W;
    const bool flip_h = k == 1 || k == 3, flip_w = k == 1 || k == 2;
    return (flip_h ? H - 1 - row : row) * W + (flip_w ? W - 1 - col : col);
}

// grid: (ceil(L/32), ceil(C/32), 4 * batch).  Tile: 32 positions x 32 channels.
__global__ void __launch_bounds__(kTile* kRows) expand_kernel(CrossLaunch p, const float* __restrict__ x,
                                                              float* __restrict__ tokens) {
    __shared__ float tile[kTile][kTile + 1];
    const unsigned long long L = p.height * p.width, C = p.channels;
    const unsigned row = blockIdx.z; // direction * batch + image
    const unsigned k = static_cast<unsigned>(row / p.batch);
    const unsigned long long image = row % p.batch;
    const unsigned long long t_base = static_cast<unsigned long long>(blockIdx.x) * kTile;
    const unsigned long long c_base = static_cast<unsigned long long>(blockIdx.y) * kTile;
    // Read x[image, c, source(t)] for 32 tokens t: consecutive lanes take
    // consecutive tokens, whose sources are consecutive positions up to a flip.
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned long long c = c_base + r, t = t_base + threadIdx.x;
        if (c < C && t < L) tile[r][threadIdx.x] = x[(image * C + c) * L + cross_source(k, t, p.height, p.width)];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned long long t = t_base + r, c = c_base + threadIdx.x;
        if (c < C && t < L) tokens[(static_cast<unsigned long long>(row) * L + t) * C + c] = tile[threadIdx.x][r];
    }
}

// grid: (ceil(L/32), ceil(C/32), batch).  out[image, c, position].
__global__ void __launch_bounds__(kTile* kRows) merge_kernel(CrossLaunch p, const float* __restrict__ y,
                                                             float* __restrict__ out) {
    __shared__ float tile[kTile][kTile + 1];
    const unsigned long long L = p.height * p.width, C = p.channels, B = p.batch;
    const unsigned long long image = blockIdx.z;
    const unsigned long long pos_base = static_cast<unsigned long long>(blockIdx.x) * kTile;
    const unsigned long long c_base = static_cast<unsigned long long>(blockIdx.y) * kTile;
    // Lanes take consecutive channels of one position: coalesced token reads.
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned long long pos = pos_base + r, c = c_base + threadIdx.x;
        if (c < C && pos < L) {
            float v[4];
#pragma unroll
            for (unsigned k = 0; k < 4; ++k)
                v[k] = y[((k * B + image) * L + cross_source(k, pos, p.height, p.width)) * C + c];
            const float sum = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), v[2]), v[3]);
            float mean = __fmul_rn(sum, 0.25f);
            if (!finite32(sum))
                mean = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(v[0], 0.25f), __fmul_rn(v[1], 0.25f)), __fmul_rn(v[2], 0.25f)),
                                 __fmul_rn(v[3], 0.25f));
            tile[r][threadIdx.x] = mean;
        }
    }
    __syncthreads();
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned long long c = c_base + r, pos = pos_base + threadIdx.x;
        if (c < C && pos < L) out[(image * C + c) * L + pos] = tile[threadIdx.x][r];
    }
}

dim3 grid_for(const CrossLaunch& p, unsigned long long rows) {
    const unsigned long long L = p.height * p.width;
    return dim3(static_cast<unsigned>((L + kTile - 1) / kTile), static_cast<unsigned>((p.channels + kTile - 1) / kTile),
                static_cast<unsigned>(rows));
}

} // namespace

cudaError_t launch_cross_expand(const CrossLaunch& p, const float* x, float* tokens, int, cudaStream_t stream) {
    const unsigned long long L = p.height * p.width;
    if ((L + kTile - 1) / kTile > 0x7fffffffull || (p.channels + kTile - 1) / kTile > 65535ull || 4 * p.batch > 65535ull)
        return cudaErrorInvalidConfiguration;
    expand_kernel<<<grid_for(p, 4 * p.batch), dim3(kTile, kRows), 0, stream>>>(p, x, tokens);
    return cudaGetLastError();
}

cudaError_t launch_cross_merge(const CrossLaunch& p, const float* y, float* out, int, cudaStream_t stream) {
    const unsigned long long L = p.height * p.width;
    if ((L + kTile - 1) / kTile > 0x7fffffffull || (p.channels + kTile - 1) / kTile > 65535ull || p.batch > 65535ull)
        return cudaErrorInvalidConfiguration;
    merge_kernel<<<grid_for(p, p.batch), dim3(kTile, kRows), 0, stream>>>(p, y, out);
    return cudaGetLastError();
}

cudaError_t load_cross_kernels(std::string& report) {
    const std::pair<const char*, const void*> kernels[] = {{"cross_expand", reinterpret_cast<const void*>(expand_kernel)},
                                                           {"cross_merge", reinterpret_cast<const void*>(merge_kernel)}};
    for (const auto& k : kernels) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, k.second);
        if (e != cudaSuccess) return e;
        report += std::string("kernel=") + k.first + " registers=" + std::to_string(attr.numRegs) +
                  " local_bytes=" + std::to_string(attr.localSizeBytes) + " shared_bytes=" +
                  std::to_string(attr.sharedSizeBytes) + " max_threads=" + std::to_string(attr.maxThreadsPerBlock) + "\n";
    }
    return cudaSuccess;
}

} // namespace sacc
