// block_kernels.cu -- the elementwise stages of the Mamba block around the scan
// (reference src/head_trt_network.cpp:192-230, binary64 twin
// src/head_reference.cpp:471-495), and the RMSNorm prologue of BASELINE
// configs 1 and 4 (not in the reference head).
//
// RMSNorm is folded into the in_proj GEMM: in_proj(rmsnorm(x)) =
// diag(r) x (W diag(w))^T with r = 1 / sqrt(mean(x^2) + eps) per token, so the
// prologue is one pass computing r (applied as a row scale in the GEMM
// epilogue) and a once-per-call scaling of the weight columns by w.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <type_traits>

#include "internal.h"
#include "scan_common.cuh"
#include "tma.cuh"

namespace sacc {

__device__ unsigned int g_block_fault; // set when a bounded wait of a block kernel ran out

namespace {

// RMSNorm folded into in_proj, in one launch: blocks [0, rms_blocks) give the
// per-token scales r[m] = 1 / sqrt(mean_k x[m,k]^2 + eps), one warp per token
// row; the blocks after them give W'[i, k] = W_in[i, k] * w[k] (the norm
// weight folded into W_in's columns, n rows).  Both parts are independent.
template <typename T>
__global__ void __launch_bounds__(256) rms_prep_kernel(const T* __restrict__ x, unsigned long long m, unsigned k, float eps,
                                                       float* __restrict__ r, unsigned rms_blocks, const T* __restrict__ w_in,
                                                       const float* __restrict__ w, unsigned long long n, T* __restrict__ out) {
    pdl_wait();
    if (blockIdx.x < rms_blocks) {
        const unsigned long long row = (static_cast<unsigned long long>(blockIdx.x) * 256 + threadIdx.x) / 32;
        const int lane = threadIdx.x % 32;
        if (row >= m) return;
        const T* xr = x + row * k;
        float acc = 0.0f;
        for (unsigned i = lane; i < k; i += 32) {
            const float v = to_f32(xr[i]);
            acc = fmaf(v, v, acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off /= 2) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) r[row] = rsqrtf(acc / static_cast<float>(k) + eps);
        return;
    }
    const unsigned long long i = static_cast<unsigned long long>(blockIdx.x - rms_blocks) * 256 + threadIdx.x;
    if (i >= n * k) return;
    out[i] = from_f32<T>(to_f32(w_in[i]) * w[i % k]);
}

// u[b, t, d] = silu(bias[d] + sum_j w[d, j] x[b, t + j - (K - 1), d]), zero
// outside the sequence (causal depthwise conv1d, reference
// src/head_reference.cpp:190-216); SiLU as x / (1 + 2^(-x log2 e)) with the
// special-function exp and a fast divide.  One thread per (sequence, channel)
// walks the tokens keeping the last K - 1 inputs in registers; consecutive
// threads take consecutive channels, so every load and store is coalesced.
// Block 0 of a launch clears `zero` (after griddepcontrol.wait: every earlier
// kernel of the stream, the previous user of these words included, is done).
__device__ __forceinline__ void clear_span(const ZeroSpan& zero) {
    if (zero.words != 0 && blockIdx.x == 0 && blockIdx.y == 0)
        for (unsigned long long i = threadIdx.x; i < zero.words; i += blockDim.x) zero.ptr[i] = 0ull;
}

template <typename T, int K>
__global__ void __launch_bounds__(256) conv_silu_kernel(const T* __restrict__ x, unsigned long long ldx,
                                                        const float* __restrict__ w, const float* __restrict__ bias,
                                                        unsigned long long batch, unsigned long long len,
                                                        unsigned long long dim, T* __restrict__ u, ZeroSpan zero) {
    pdl_wait();
    clear_span(zero);
    const unsigned long long lane = static_cast<unsigned long long>(blockIdx.x) * 256 + threadIdx.x;
    if (lane >= batch * dim) return;
    const unsigned long long b = lane / dim, d = lane % dim;
    float wk[K], hist[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        wk[j] = w[d * K + j];
        hist[j] = 0.0f;
    }
    const float bv = bias ? bias[d] : 0.0f;
    const T* xr = x + b * len * ldx + d;
    T* ur = u + b * len * dim + d;
    for (unsigned long long t = 0; t < len; ++t) {
#pragma unroll
        for (int j = 0; j < K - 1; ++j) hist[j] = hist[j + 1];
        hist[K - 1] = to_f32(xr[t * ldx]);
        float acc = bv;
#pragma unroll
        for (int j = 0; j < K; ++j) acc = fmaf(wk[j], hist[j], acc);
        ur[t * dim] = from_f32<T>(silu(acc));
    }
}

// Same conv + SiLU with one thread per (4 consecutive token rows of one
// sequence, 8 consecutive channels): rows t-3 .. t+3 are seven independent
// 16-byte loads (zero before the sequence start, none past its end), the
// weights and bias of the 8 channels load once for the 4 rows, and nothing
// walks a sequence; same arithmetic, in the same order, as the per-lane walk
// above.  Needs dim and ldx multiples of 8 and 16-byte aligned tensors.
template <typename T>
__global__ void __launch_bounds__(256) conv4_silu_rows_kernel(const T* __restrict__ x, unsigned long long ldx,
                                                              const float* __restrict__ w, const float* __restrict__ bias,
                                                              unsigned long long batch, unsigned long long len,
                                                              unsigned long long dim, T* __restrict__ u, ZeroSpan zero) {
    pdl_wait();
    clear_span(zero);
    constexpr int K = 4, R = 4; // taps, rows per thread
    // 32-bit index arithmetic (the launcher keeps the thread count below 2^32).
    const unsigned groups = static_cast<unsigned>(dim / 8), quads = static_cast<unsigned>((len + R - 1) / R);
    const unsigned gid = blockIdx.x * 256u + threadIdx.x;
    if (static_cast<unsigned long long>(gid) >= batch * quads * groups) return;
    const unsigned g = gid % groups, bq = gid / groups;
    const unsigned long long b = bq / quads, t0 = static_cast<unsigned long long>(bq % quads) * R, d0 = g * 8ull;
    float wk[8][K], bv[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w + (d0 + c) * K));
        wk[c][0] = wv.x; wk[c][1] = wv.y; wk[c][2] = wv.z; wk[c][3] = wv.w;
        bv[c] = bias ? __ldg(bias + d0 + c) : 0.0f;
    }
    // rows t0 - 3 .. t0 + 3 of sequence b (index i = row - t0 + 3)
    float xr[K - 1 + R][8];
#pragma unroll
    for (int i = 0; i < K - 1 + R; ++i) {
        const long long t = static_cast<long long>(t0) + i - (K - 1);
        if (t >= 0 && t < static_cast<long long>(len)) {
            const uint4 v = *reinterpret_cast<const uint4*>(x + (b * len + static_cast<unsigned long long>(t)) * ldx + d0);
            const std::uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                if constexpr (std::is_same_v<T, __half>) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[c]));
                    xr[i][2 * c] = f.x;
                    xr[i][2 * c + 1] = f.y;
                } else {
                    xr[i][2 * c] = __uint_as_float(wv[c] << 16);
                    xr[i][2 * c + 1] = __uint_as_float(wv[c] & 0xffff0000u);
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) xr[i][c] = 0.0f;
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (t0 + r >= len) break;
        std::uint32_t out[4];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float acc = bv[c];
#pragma unroll
            for (int j = 0; j < K; ++j) acc = fmaf(wk[c][j], xr[r + j][c], acc);
            const T v = from_f32<T>(silu(acc));
            std::uint32_t bits;
            if constexpr (std::is_same_v<T, __half>) bits = __half_as_ushort(v);
            else bits = __bfloat16_as_ushort(v);
            out[c / 2] = (c % 2 == 0) ? bits : (out[c / 2] | (bits << 16));
        }
        *reinterpret_cast<uint4*>(u + (b * len + t0 + r) * dim + d0) = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

// Same conv + SiLU over TMA tiles: a CTA takes 64 token rows x 128 channels
// of one sequence, loads rows t0 - 3 .. t0 + 63 in one 3D tile (channel, token,
// sequence) -- rows before the sequence start and past its end read as zeros,
// which is the causal padding -- and each thread slides the 4-tap window down
// its channel, so every input row is read once (plus a 3-row halo per tile).
// Same operations in the same order as the kernels above, so the same bits.
constexpr int kConvRows = 64, kConvCh = 128;

template <typename T>
__global__ void __launch_bounds__(kConvCh) conv4_silu_tile_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                                 const float* __restrict__ w, const float* __restrict__ bias,
                                                                 unsigned long long len, unsigned long long dim,
                                                                 unsigned tiles_per_seq, T* __restrict__ u, ZeroSpan zero) {
    pdl_wait();
    clear_span(zero);
    __shared__ alignas(128) T tile[(kConvRows + 3) * kConvCh];
    __shared__ alignas(8) std::uint64_t bar;
    const int tid = threadIdx.x;
    const unsigned long long b = blockIdx.x / tiles_per_seq;
    const int t0 = static_cast<int>(blockIdx.x % tiles_per_seq) * kConvRows;
    const unsigned d0 = blockIdx.y * kConvCh;
    if (tid == 0) {
        prefetch_tensor_map(&tm_x);
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(&bar, static_cast<std::uint32_t>(sizeof(tile)));
        tma_load_3d(tile, &tm_x, &bar, static_cast<int>(d0), t0 - 3, static_cast<int>(b));
    }
    const float4 wv = __ldg(reinterpret_cast<const float4*>(w + (d0 + tid) * 4ull));
    const float bv = bias ? __ldg(bias + d0 + tid) : 0.0f;
    const bool ok = mbar_wait_bounded(&bar, 0u);
    if (!__syncthreads_and(ok)) {
        if (tid == 0) atomicOr(&g_block_fault, 1u);
        return;
    }
    float x0 = to_f32(tile[tid]), x1 = to_f32(tile[kConvCh + tid]), x2 = to_f32(tile[2 * kConvCh + tid]);
    const unsigned long long left = len - static_cast<unsigned long long>(t0);
    const int rows = left < static_cast<unsigned long long>(kConvRows) ? static_cast<int>(left) : kConvRows;
    T* out = u + (b * len + static_cast<unsigned long long>(t0)) * dim + d0 + tid;
#pragma unroll 4
    for (int r = 0; r < rows; ++r) {
        const float x3 = to_f32(tile[(r + 3) * kConvCh + tid]);
        float acc = bv;
        acc = fmaf(wv.x, x0, acc);
        acc = fmaf(wv.y, x1, acc);
        acc = fmaf(wv.z, x2, acc);
        acc = fmaf(wv.w, x3, acc);
        out[static_cast<unsigned long long>(r) * dim] = from_f32<T>(silu(acc));
        x0 = x1;
        x1 = x2;
        x2 = x3;
    }
}

// dst = src (rows x cols, 16-bit) followed by copies - 1 more copies of its
// last row: the block's W_x for a rank-1 C.
__global__ void __launch_bounds__(256) repeat_last_row_kernel(const std::uint16_t* __restrict__ src, unsigned long long rows,
                                                              unsigned long long copies, unsigned long long cols,
                                                              std::uint16_t* __restrict__ dst) {
    pdl_wait();
    const unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * 256 + threadIdx.x;
    const unsigned long long out_rows = rows - 1 + copies;
    if (i >= out_rows * cols) return;
    const unsigned long long r = i / cols, c = i % cols;
    dst[i] = src[(r < rows ? r : rows - 1) * cols + c];
}

PFN_cuTensorMapEncodeTiled_v12000 conv_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

} // namespace

cudaError_t read_block_fault(unsigned* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_block_fault, sizeof(unsigned));
    if (e != cudaSuccess || !clear) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_block_fault, &zero, sizeof(unsigned));
}

cudaError_t launch_repeat_last_row(int dtype, const void* src, unsigned long long rows, unsigned long long copies,
                                   unsigned long long cols, void* dst, cudaStream_t stream) {
    (void)dtype; // a bit copy of 16-bit elements
    const unsigned long long blocks = ((rows - 1 + copies) * cols + 255) / 256;
    if (rows == 0 || copies == 0 || blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    return launch_pdl_k(repeat_last_row_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                        static_cast<const std::uint16_t*>(src), rows, copies, cols, static_cast<std::uint16_t*>(dst));
}

cudaError_t launch_rms_prep(int dtype, const void* x, unsigned long long m, unsigned k, float eps, float* r, const void* w_in,
                            const float* w, unsigned long long n, void* out, cudaStream_t stream) {
    const unsigned long long rms_blocks = (m * 32 + 255) / 256, col_blocks = (n * k + 255) / 256;
    if (rms_blocks + col_blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    const dim3 grid(static_cast<unsigned>(rms_blocks + col_blocks));
    const unsigned rb = static_cast<unsigned>(rms_blocks);
    if (dtype == SACC_DTYPE_BF16)
        return launch_pdl_k(rms_prep_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream, static_cast<const __nv_bfloat16*>(x), m, k,
                            eps, r, rb, static_cast<const __nv_bfloat16*>(w_in), w, n, static_cast<__nv_bfloat16*>(out));
    return launch_pdl_k(rms_prep_kernel<__half>, grid, dim3(256), 0, stream, static_cast<const __half*>(x), m, k, eps, r, rb,
                        static_cast<const __half*>(w_in), w, n, static_cast<__half*>(out));
}

cudaError_t launch_conv_silu(int dtype, int kwidth, const void* x, unsigned long long ldx, const float* w, const float* bias,
                             unsigned long long batch, unsigned long long len, unsigned long long dim, void* u,
                             cudaStream_t stream, ZeroSpan zero) {
    if (kwidth != 4) return cudaErrorInvalidConfiguration;
    const auto al16 = [](const void* ptr) { return reinterpret_cast<std::uintptr_t>(ptr) % 16 == 0; };
    // TMA tiles: channels in 128-wide blocks, 16-byte aligned rows.
    const unsigned long long tiles_per_seq = (len + kConvRows - 1) / kConvRows;
    auto enc = conv_encoder();
    if (enc && dim % kConvCh == 0 && ldx % 8 == 0 && al16(x) && al16(w) && len > 0 && batch * tiles_per_seq <= 0x7fffffffull &&
        dim / kConvCh <= 65535 && len < 0x7fffffffull && batch < 0x7fffffffull) {
        CUtensorMap tm{};
        const cuuint64_t dims[3] = {dim, len, batch};
        const cuuint64_t strides[2] = {ldx * 2, ldx * 2 * len};
        const cuuint32_t box[3] = {kConvCh, kConvRows + 3, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        const CUtensorMapDataType dt = dtype == SACC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        if (enc(&tm, dt, 3, const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
            const dim3 grid(static_cast<unsigned>(batch * tiles_per_seq), static_cast<unsigned>(dim / kConvCh));
            const unsigned tps = static_cast<unsigned>(tiles_per_seq);
            if (dtype == SACC_DTYPE_BF16)
                return launch_pdl_k(conv4_silu_tile_kernel<__nv_bfloat16>, grid, dim3(kConvCh), 0, stream, tm, w, bias, len, dim,
                                    tps, static_cast<__nv_bfloat16*>(u), zero);
            return launch_pdl_k(conv4_silu_tile_kernel<__half>, grid, dim3(kConvCh), 0, stream, tm, w, bias, len, dim, tps,
                                static_cast<__half*>(u), zero);
        }
    }
    const unsigned long long threads = batch * ((len + 3) / 4) * (dim / 8), row_blocks = (threads + 255) / 256;
    if (dim % 8 == 0 && ldx % 8 == 0 && al16(x) && al16(u) && al16(w) && row_blocks * 256 < 0xffffffffull && len > 0) {
        if (row_blocks == 0) return cudaSuccess;
        if (dtype == SACC_DTYPE_BF16)
            return launch_pdl_k(conv4_silu_rows_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(row_blocks)), dim3(256), 0,
                                stream, static_cast<const __nv_bfloat16*>(x), ldx, w, bias, batch, len, dim,
                                static_cast<__nv_bfloat16*>(u), zero);
        return launch_pdl_k(conv4_silu_rows_kernel<__half>, dim3(static_cast<unsigned>(row_blocks)), dim3(256), 0, stream,
                            static_cast<const __half*>(x), ldx, w, bias, batch, len, dim, static_cast<__half*>(u), zero);
    }
    const unsigned long long blocks = (batch * dim + 255) / 256;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    if (dtype == SACC_DTYPE_BF16)
        conv_silu_kernel<__nv_bfloat16, 4><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), ldx, w, bias, batch, len, dim, static_cast<__nv_bfloat16*>(u), zero);
    else
        conv_silu_kernel<__half, 4><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            static_cast<const __half*>(x), ldx, w, bias, batch, len, dim, static_cast<__half*>(u), zero);
    return cudaGetLastError();
}

cudaError_t load_block_kernels(std::string& report) {
    const void* ks[] = {reinterpret_cast<const void*>(rms_prep_kernel<__nv_bfloat16>),
                        reinterpret_cast<const void*>(rms_prep_kernel<__half>),
                        reinterpret_cast<const void*>(conv_silu_kernel<__nv_bfloat16, 4>),
                        reinterpret_cast<const void*>(conv_silu_kernel<__half, 4>),
                        reinterpret_cast<const void*>(conv4_silu_rows_kernel<__nv_bfloat16>),
                        reinterpret_cast<const void*>(conv4_silu_rows_kernel<__half>),
                        reinterpret_cast<const void*>(conv4_silu_tile_kernel<__nv_bfloat16>),
                        reinterpret_cast<const void*>(conv4_silu_tile_kernel<__half>),
                        reinterpret_cast<const void*>(repeat_last_row_kernel)};
    for (const void* k : ks) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, k);
        if (e != cudaSuccess) return e;
    }
    report += "kernels_loaded=block (rms_prep, conv_silu, repeat_last_row) x9\n";
    return cudaSuccess;
}

} // namespace sacc
