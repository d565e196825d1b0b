// cross_block.cu -- the elementwise stages of one Cross-Scan head level with
// the expand and merge fused into the Mamba block (reference
// src/head_trt_network.cpp:200-232: CrossScanExpand, the block layers with the
// residual on the expanded tokens, CrossScanMerge; expand / merge kernels
// cuda/selective_scan.cu:157-192).
//
// The reference materialises tokens_k = expand_k(x), a (4 batch, L, C) FP32
// tensor, runs the block on it and averages the four directions back to the
// map.  in_proj and out_proj act on each token alone, so here
//   * x is transposed once to position-major rows (rows_from_maps) and in_proj
//     runs once per position; direction k's token t is row src(k, t);
//   * cross_conv reads the conv window of every direction through src and
//     writes u and the gate z of the 4 batch sequences the scan walks;
//   * cross_mean averages the four directions' gated scan outputs at each
//     position (the merge's order and overflow rule), one out_proj per
//     position follows (FP32 rows), and maps_from_rows writes them back to
//     the maps adding x as the residual: every direction's token at a
//     position is x there (each flip is an involution).
// src(k, t): direction 0 identity, 1 flip H and W, 2 flip W, 3 flip H.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <string>
#include <type_traits>

#include "internal.h"
#include "scan_common.cuh"

namespace sacc {
namespace {

constexpr int kTile = 32, kRows = 8;

// Position of direction k's token t (reference src/selective_scan.cpp:111-116).
__device__ __forceinline__ unsigned src_pos(unsigned k, unsigned t, unsigned H, unsigned W) {
    const unsigned row = t / W, col = t % W;
    const bool flip_h = k == 1 || k == 3, flip_w = k == 1 || k == 2;
    return (flip_h ? H - 1 - row : row) * W + (flip_w ? W - 1 - col : col);
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
    const std::uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        if constexpr (std::is_same_v<T, __half>) {
            const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[c]));
            f[2 * c] = p.x;
            f[2 * c + 1] = p.y;
        } else {
            f[2 * c] = __uint_as_float(w[c] << 16);
            f[2 * c + 1] = __uint_as_float(w[c] & 0xffff0000u);
        }
    }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    std::uint32_t o[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const T lo = from_f32<T>(f[2 * c]), hi = from_f32<T>(f[2 * c + 1]);
        std::uint32_t a, b;
        if constexpr (std::is_same_v<T, __half>) {
            a = __half_as_ushort(lo);
            b = __half_as_ushort(hi);
        } else {
            a = __bfloat16_as_ushort(lo);
            b = __bfloat16_as_ushort(hi);
        }
        o[c] = a | (b << 16);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// rows[b, p, c] = x[b, c, p] in T.  grid (ceil(L/32), ceil(C/32), batch);
// reads coalesced along positions, writes along channels.
template <typename T>
__global__ void __launch_bounds__(kTile* kRows) rows_from_maps_kernel(const float* __restrict__ x, unsigned L, unsigned C,
                                                                      T* __restrict__ rows) {
    pdl_wait();
    __shared__ float tile[kTile][kTile + 1];
    const unsigned b = blockIdx.z, p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned c = c0 + r, p = p0 + threadIdx.x;
        if (c < C && p < L) tile[r][threadIdx.x] = x[(static_cast<unsigned long long>(b) * C + c) * L + p];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned p = p0 + r, c = c0 + threadIdx.x;
        if (c < C && p < L) rows[(static_cast<unsigned long long>(b) * L + p) * C + c] = from_f32<T>(tile[threadIdx.x][r]);
    }
}

// out[b, c, p] = rows[b, p, c] (+ x[b, c, p]), FP32.  grid (ceil(L/32),
// ceil(C/32), batch); reads coalesced along channels, writes along positions.
__global__ void __launch_bounds__(kTile* kRows) maps_from_rows_kernel(const float* __restrict__ rows, const float* __restrict__ x,
                                                                      unsigned L, unsigned C, float* __restrict__ out) {
    pdl_wait();
    __shared__ float tile[kTile][kTile + 1];
    const unsigned b = blockIdx.z, p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned p = p0 + r, c = c0 + threadIdx.x;
        if (c < C && p < L) tile[r][threadIdx.x] = rows[(static_cast<unsigned long long>(b) * L + p) * C + c];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < kTile; r += kRows) {
        const unsigned c = c0 + r, p = p0 + threadIdx.x;
        if (c < C && p < L) {
            const unsigned long long i = (static_cast<unsigned long long>(b) * C + c) * L + p;
            out[i] = x ? tile[threadIdx.x][r] + x[i] : tile[threadIdx.x][r];
        }
    }
}

// One thread per (sequence s = k batch + b, token t, 8 channels): the 4-tap
// causal conv + SiLU of direction k over the x_in half of xz (position-major
// rows, pitch 2 D), rows t - 3 .. t read through src (zero before the
// sequence start), and the gate z of token t copied beside it.  Same
// operations in the same order as the block's conv kernels.
template <typename T>
__global__ void __launch_bounds__(256) cross_conv_kernel(const T* __restrict__ xz, const float* __restrict__ w,
                                                         const float* __restrict__ bias, unsigned batch, unsigned H, unsigned W,
                                                         unsigned D, T* __restrict__ u, T* __restrict__ z, ZeroSpan zero) {
    pdl_wait();
    if (zero.words != 0 && blockIdx.x == 0) // the fused scan's hand-off flags (internal.h, ZeroSpan)
        for (unsigned long long i = threadIdx.x; i < zero.words; i += blockDim.x) zero.ptr[i] = 0ull;
    constexpr int K = 4;
    const unsigned L = H * W, groups = D / 8;
    const unsigned long long gid = static_cast<unsigned long long>(blockIdx.x) * 256 + threadIdx.x;
    if (gid >= 4ull * batch * L * groups) return;
    const unsigned g = static_cast<unsigned>(gid % groups);
    const unsigned long long st = gid / groups;
    const unsigned t = static_cast<unsigned>(st % L), s = static_cast<unsigned>(st / L);
    const unsigned k = s / batch, b = s % batch, d0 = 8 * g;
    const unsigned long long base = static_cast<unsigned long long>(b) * L;
    float wk[8][K], acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + (d0 + c) * K));
        wk[c][0] = wv.x; wk[c][1] = wv.y; wk[c][2] = wv.z; wk[c][3] = wv.w;
        acc[c] = bias ? __ldg(bias + d0 + c) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
        float xr[8];
        const int tt = static_cast<int>(t) + j - (K - 1);
        if (tt >= 0) {
            const unsigned p = src_pos(k, static_cast<unsigned>(tt), H, W);
            unpack8<T>(*reinterpret_cast<const uint4*>(xz + (base + p) * 2ull * D + d0), xr);
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) xr[c] = 0.0f;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = fmaf(wk[c][j], xr[c], acc[c]);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = silu(acc[c]);
    const unsigned long long row = static_cast<unsigned long long>(s) * L + t;
    *reinterpret_cast<uint4*>(u + row * D + d0) = pack8<T>(acc);
    const unsigned p = src_pos(k, t, H, W);
    *reinterpret_cast<uint4*>(z + row * D + d0) = *reinterpret_cast<const uint4*>(xz + (base + p) * 2ull * D + D + d0);
}

// One thread per (image b, position p, 8 channels): the mean of the four
// directions' gated outputs at p, ((y0 + y1) + y2) + y3 times 0.25, the
// quarters summed instead when the sum overflows (the reference merge,
// cuda/selective_scan.cu:177-192), stored position-major in T.
template <typename T>
__global__ void __launch_bounds__(256) cross_mean_kernel(const T* __restrict__ y, unsigned batch, unsigned H, unsigned W,
                                                         unsigned D, T* __restrict__ mean) {
    pdl_wait();
    const unsigned L = H * W, groups = D / 8;
    const unsigned long long gid = static_cast<unsigned long long>(blockIdx.x) * 256 + threadIdx.x;
    if (gid >= static_cast<unsigned long long>(batch) * L * groups) return;
    const unsigned g = static_cast<unsigned>(gid % groups);
    const unsigned long long bp = gid / groups;
    const unsigned p = static_cast<unsigned>(bp % L), b = static_cast<unsigned>(bp / L), d0 = 8 * g;
    float v[4][8];
#pragma unroll
    for (unsigned k = 0; k < 4; ++k) {
        const unsigned long long row = (static_cast<unsigned long long>(k) * batch + b) * L + src_pos(k, p, H, W);
        unpack8<T>(*reinterpret_cast<const uint4*>(y + row * D + d0), v[k]);
    }
    float out[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float sum = __fadd_rn(__fadd_rn(__fadd_rn(v[0][c], v[1][c]), v[2][c]), v[3][c]);
        out[c] = __fmul_rn(sum, 0.25f);
        if (!(fabsf(sum) <= FLT_MAX))
            out[c] = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(v[0][c], 0.25f), __fmul_rn(v[1][c], 0.25f)), __fmul_rn(v[2][c], 0.25f)),
                               __fmul_rn(v[3][c], 0.25f));
    }
    *reinterpret_cast<uint4*>(mean + bp * D + d0) = pack8<T>(out);
}

} // namespace

cudaError_t launch_rows_from_maps(int dtype, const float* x, unsigned long long batch, unsigned long long L,
                                  unsigned long long C, void* rows, cudaStream_t stream) {
    if (batch > 65535 || (L + kTile - 1) / kTile > 0x7fffffffull || (C + kTile - 1) / kTile > 65535 || L * C > 0xffffffffull)
        return cudaErrorInvalidConfiguration;
    const dim3 grid(static_cast<unsigned>((L + kTile - 1) / kTile), static_cast<unsigned>((C + kTile - 1) / kTile),
                    static_cast<unsigned>(batch));
    const unsigned l = static_cast<unsigned>(L), c = static_cast<unsigned>(C);
    if (dtype == SACC_DTYPE_BF16)
        return launch_pdl_k(rows_from_maps_kernel<__nv_bfloat16>, grid, dim3(kTile, kRows), 0, stream, x, l, c,
                            static_cast<__nv_bfloat16*>(rows));
    return launch_pdl_k(rows_from_maps_kernel<__half>, grid, dim3(kTile, kRows), 0, stream, x, l, c, static_cast<__half*>(rows));
}

cudaError_t launch_maps_from_rows(const float* rows, const float* x, unsigned long long batch, unsigned long long L,
                                  unsigned long long C, float* out, cudaStream_t stream) {
    if (batch > 65535 || (L + kTile - 1) / kTile > 0x7fffffffull || (C + kTile - 1) / kTile > 65535 || L * C > 0xffffffffull)
        return cudaErrorInvalidConfiguration;
    const dim3 grid(static_cast<unsigned>((L + kTile - 1) / kTile), static_cast<unsigned>((C + kTile - 1) / kTile),
                    static_cast<unsigned>(batch));
    return launch_pdl_k(maps_from_rows_kernel, grid, dim3(kTile, kRows), 0, stream, rows, x, static_cast<unsigned>(L),
                        static_cast<unsigned>(C), out);
}

cudaError_t launch_cross_conv(int dtype, const void* xz, const float* w, const float* bias, unsigned long long batch,
                              unsigned long long H, unsigned long long W, unsigned long long D, void* u, void* z,
                              cudaStream_t stream, ZeroSpan zero) {
    const unsigned long long threads = 4 * batch * H * W * (D / 8), blocks = (threads + 255) / 256;
    if (D % 8 != 0 || H * W > 0xffffffffull || 4 * batch > 0xffffffffull || D > 0xffffffffull || blocks > 0x7fffffffull)
        return cudaErrorInvalidConfiguration;
    if (blocks == 0) return cudaSuccess;
    const unsigned b = static_cast<unsigned>(batch), h = static_cast<unsigned>(H), wd = static_cast<unsigned>(W),
                   d = static_cast<unsigned>(D);
    if (dtype == SACC_DTYPE_BF16)
        return launch_pdl_k(cross_conv_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                            static_cast<const __nv_bfloat16*>(xz), w, bias, b, h, wd, d, static_cast<__nv_bfloat16*>(u),
                            static_cast<__nv_bfloat16*>(z), zero);
    return launch_pdl_k(cross_conv_kernel<__half>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                        static_cast<const __half*>(xz), w, bias, b, h, wd, d, static_cast<__half*>(u), static_cast<__half*>(z),
                        zero);
}

cudaError_t launch_cross_mean(int dtype, const void* y, unsigned long long batch, unsigned long long H, unsigned long long W,
                              unsigned long long D, void* mean, cudaStream_t stream) {
    const unsigned long long threads = batch * H * W * (D / 8), blocks = (threads + 255) / 256;
    if (D % 8 != 0 || H * W > 0xffffffffull || 4 * batch > 0xffffffffull || D > 0xffffffffull || blocks > 0x7fffffffull)
        return cudaErrorInvalidConfiguration;
    if (blocks == 0) return cudaSuccess;
    const unsigned b = static_cast<unsigned>(batch), h = static_cast<unsigned>(H), wd = static_cast<unsigned>(W),
                   d = static_cast<unsigned>(D);
    if (dtype == SACC_DTYPE_BF16)
        return launch_pdl_k(cross_mean_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                            static_cast<const __nv_bfloat16*>(y), b, h, wd, d, static_cast<__nv_bfloat16*>(mean));
    return launch_pdl_k(cross_mean_kernel<__half>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                        static_cast<const __half*>(y), b, h, wd, d, static_cast<__half*>(mean));
}

cudaError_t load_cross_block_kernels(std::string& report) {
    const std::pair<const char*, const void*> ks[] = {
        {"rows_from_maps_bf16", reinterpret_cast<const void*>(rows_from_maps_kernel<__nv_bfloat16>)},
        {"rows_from_maps_f16", reinterpret_cast<const void*>(rows_from_maps_kernel<__half>)},
        {"cross_conv_bf16", reinterpret_cast<const void*>(cross_conv_kernel<__nv_bfloat16>)},
        {"cross_conv_f16", reinterpret_cast<const void*>(cross_conv_kernel<__half>)},
        {"cross_mean_bf16", reinterpret_cast<const void*>(cross_mean_kernel<__nv_bfloat16>)},
        {"cross_mean_f16", reinterpret_cast<const void*>(cross_mean_kernel<__half>)}};
    for (const auto& k : ks) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, k.second);
        if (e != cudaSuccess) return e;
        report += std::string("kernel=") + k.first + " registers=" + std::to_string(attr.numRegs) + "\n";
    }
    return cudaSuccess;
}

} // namespace sacc
