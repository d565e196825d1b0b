// gemm_tcgen05.cu -- C = A B^T (+ bias, + residual) on the sm_100a tensor cores.
//
// The dense projections around the scan (in_proj, x_proj, out_proj of the
// Mamba block, reference src/head_trt_network.cpp:192-230) are GEMMs of
// token rows A (M x K, K contiguous) with weight rows B (N x K, K contiguous).
//
// A persistent CTA (one per SM) walks 128 x BN tiles of C, accumulating each in
// one of two 128 x BN FP32 tensor-memory (TMEM) buffers so that the epilogue of
// a tile overlaps the MMAs of the next:
//   warp 0      TMA producer: 128 x 64 A and BN x 64 B bf16/fp16 tiles with
//               128-byte swizzle into a 4-stage ring (full / empty mbarriers);
//   warp 1      allocates TMEM, and one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = BN, K = 16)
//               four times per stage from shared-memory descriptors, then
//               tcgen05.commit to free the stage and, per tile, to signal
//               the epilogue;
//   warps 2..   epilogue (eight warps, four at BN = 64: two per TMEM lane
//               quarter, each half the columns): tcgen05.ld 32 lanes x 32 columns at a time, row
//               scale, bias, residual, conversion; 16-bit results go through
//               swizzled 32 x 32 shared tiles (sixteen per CTA, all but one per
//               warp in flight) and TMA stores (coalesced full lines), FP32 results straight to
//               global memory; then release the accumulator buffer.
// No multicast, no clusters.  Every mbarrier wait has an iteration limit and
// sets the library fault word when it runs out.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "internal.h"
#include "scan_common.cuh"
#include "tma.cuh"

namespace sacc {

__device__ unsigned int g_gemm_fault; // set when a bounded wait ran out; read by sacc_scan_fault()

namespace {

constexpr int kBM = 128, kBK = 64, kStages = 4;

// Epilogue warps E: four (one per TMEM lane quarter) or eight (two per
// quarter, each half of a tile's columns, so that each scheduler has two to
// interleave).  Eight pay off when a tile's MMAs are short: with one k-block
// (K = 64: config 4's dt_proj, 8.6 GB out) four warps stored at 2.0 TB/s, each
// warp's load - convert - stage - fence - store chain exposed, eight at 4.5
// TB/s; at K = 1024-2048 eight were up to 5 % slower (the MMA warp shares its
// scheduler with two of them).  BN = 64 keeps four: two CTAs share an SM.
template <int E>
__host__ __device__ constexpr int gemm_threads() {
    return 64 + 32 * E;
}
// 32 x 32 staging tiles per epilogue warp (sixteen in all): a warp keeps all
// but one of its TMA stores reading shared memory while it fills the next.
template <int E>
__host__ __device__ constexpr int stage_bufs() {
    return 16 / E;
}

// Ring depth: 4 stages, 3 at BN = 64 so that two CTAs fit on an SM.
template <int BN>
__host__ __device__ constexpr int stages_for() {
    return BN == 64 ? 3 : kStages;
}

template <int BN, int E>
struct GemmSmem {
    alignas(1024) std::uint16_t a[stages_for<BN>()][kBM * kBK];
    alignas(1024) std::uint16_t b[stages_for<BN>()][BN * kBK];
    alignas(8) std::uint64_t full[stages_for<BN>()];
    alignas(8) std::uint64_t empty[stages_for<BN>()];
    alignas(8) std::uint64_t acc_full[2];
    alignas(8) std::uint64_t acc_empty[2];
    // 16-bit epilogue staging: per epilogue warp stage_bufs 32 x 32 tiles (64-byte swizzle) for TMA stores
    // (at BN = 256 the whole struct is 231,424 bytes: with the 1 KB alignment slack exactly the opt-in limit).
    alignas(1024) std::uint16_t stage[E][stage_bufs<E>()][32 * 32];
    std::uint32_t tmem_base;
};

struct GemmParams {
    void* c;
    const void* residual;
    const float* bias;
    const float* row_scale;
    unsigned long long m, n, k, ldc, ldr;
    int out_dtype, in_dtype, kblocks, tiles_m, tiles_n, vec_store, tma_store, res_vec;
};

// Shared-memory matrix descriptor for a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row swizzle atoms 1024 bytes apart
// (stride byte offset), leading byte offset unused for swizzled K-major (1),
// descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ std::uint64_t sw128_desc(const void* tile) {
    const std::uint64_t addr = smem_addr(tile);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: FP32 accumulate, A/B format (0 = f16, 1 = bf16),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr std::uint32_t instr_desc(int ab_format, int m, int n) {
    return (1u << 4) | (static_cast<std::uint32_t>(ab_format) << 7) | (static_cast<std::uint32_t>(ab_format) << 10) |
           (static_cast<std::uint32_t>(n >> 3) << 17) | (static_cast<std::uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(std::uint32_t tmem_d, std::uint64_t adesc, std::uint64_t bdesc, std::uint32_t idesc,
                                        std::uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(std::uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 TMEM lanes (one per thread of the warp) x 32 consecutive 32-bit columns:
// tmem_ld32_issue starts the load, tmem_ld32_wait waits for every load of the
// thread and takes the destination registers as read-write operands, so that
// no use of them can be scheduled before the wait.
#define SACC_R32(r)                                                                                                  \
    "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),     \
        "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),      \
        "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),     \
        "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])

__device__ __forceinline__ void tmem_ld32_issue(std::uint32_t taddr, std::uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32_wait(std::uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : SACC_R32(r)::"memory");
}

__device__ __forceinline__ float load_elem(const void* p, unsigned long long i, int dtype) {
    if (dtype == SACC_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    if (dtype == SACC_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
    return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, unsigned long long i, int dtype, float v) {
    if (dtype == SACC_DTYPE_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else if (dtype == SACC_DTYPE_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
    else static_cast<float*>(p)[i] = v;
}

// Row scale, bias and residual on 32 consecutive columns of one row (the
// residual as 16-byte loads when its rows allow).  Every test is uniform
// across the warp and sits outside the element loops, which stay branch-free.
__device__ __forceinline__ void apply_chunk(const GemmParams& p, unsigned long long row, unsigned long long col0, float (&v)[32]) {
    const bool full = col0 + 32 <= p.n;
    if (p.row_scale) {
        const float rs = p.row_scale[row];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= rs;
    }
    if (p.bias) {
        if (full) {
            const float4* bq = reinterpret_cast<const float4*>(p.bias + col0);
            if ((reinterpret_cast<std::uintptr_t>(bq) & 15u) == 0) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 t = bq[q];
                    v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += p.bias[col0 + i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < p.n) v[i] += p.bias[col0 + i];
        }
    }
    if (p.residual) {
        if (full && p.res_vec && p.out_dtype == SACC_DTYPE_F32) {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.residual) + row * p.ldr + col0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 t = src[q];
                v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
            }
        } else if (full && p.res_vec) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const std::uint16_t*>(p.residual) + row * p.ldr + col0);
            const bool bf = p.out_dtype == SACC_DTYPE_BF16;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 w = src[q];
                const std::uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float lo, hi;
                    if (bf) {
                        lo = __uint_as_float(ws[j] << 16);
                        hi = __uint_as_float(ws[j] & 0xffff0000u);
                    } else {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ws[j]));
                        lo = f.x;
                        hi = f.y;
                    }
                    v[8 * q + 2 * j] += lo;
                    v[8 * q + 2 * j + 1] += hi;
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (full || col0 + i < p.n) v[i] += load_elem(p.residual, row * p.ldr + col0 + i, p.out_dtype);
        }
    }
}

// 32 results to 16-bit pairs, the output type chosen once.
__device__ __forceinline__ void pack16(const float (&v)[32], int dtype, std::uint32_t (&w)[16]) {
    if (dtype == SACC_DTYPE_BF16) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<const std::uint32_t*>(&t);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const __half2 t = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<const std::uint32_t*>(&t);
        }
    }
}

// Epilogue of 32 consecutive columns of one row straight to global memory
// (FP32 output, or a C the TMA cannot address): 16-byte stores when the row
// segment is aligned and complete.
__device__ __forceinline__ void store_chunk(const GemmParams& p, unsigned long long row, unsigned long long col0, float (&v)[32]) {
    apply_chunk(p, row, col0, v);
    const bool full = col0 + 32 <= p.n;
    if (full && p.vec_store) {
        if (p.out_dtype == SACC_DTYPE_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.c) + row * p.ldc + col0);
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<std::uint16_t*>(p.c) + row * p.ldc + col0);
            std::uint32_t w[16];
            pack16(v, p.out_dtype, w);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (col0 + i < p.n) store_elem(p.c, row * p.ldc + col0 + i, p.out_dtype, v[i]);
}

// Persistent: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...;
// two TMEM accumulators let the epilogue of one tile overlap the MMAs of the next.
template <int BN, int E>
__global__ void __launch_bounds__(gemm_threads<E>(), 1) gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                                                           const __grid_constant__ CUtensorMap tm_b,
                                                           const __grid_constant__ CUtensorMap tm_c, GemmParams p) {
    constexpr int S = stages_for<BN>();
    extern __shared__ unsigned char smem_raw[];
    auto& sm = shared_window<GemmSmem<BN, E>>(smem_raw);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int tiles = p.tiles_m * p.tiles_n;

    if (threadIdx.x == 0) {
        prefetch_tensor_map(&tm_a);
        prefetch_tensor_map(&tm_b);
        for (int s = 0; s < S; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm.acc_full[b], 1);
            mbar_init(&sm.acc_empty[b], E); // one arrival per epilogue warp
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                     "r"(2 * BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const std::uint32_t tmem = sm.tmem_base;
    // barriers and TMEM are set up; the previous kernel's results come next
    pdl_wait();

    bool fault = false;
    if (warp == 0) {
        if (lane == 0) {
            constexpr std::uint32_t bytes = (kBM + BN) * kBK * 2;
            unsigned g = 0; // k-blocks issued by this CTA
            for (int tile = blockIdx.x; tile < tiles && !fault; tile += gridDim.x) {
                const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * BN;
                for (int kb = 0; kb < p.kblocks; ++kb, ++g) {
                    const unsigned s = g % S;
                    if (g >= S && !mbar_wait_bounded(&sm.empty[s], ((g / S) - 1) & 1u)) {
                        fault = true;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.full[s], bytes);
                    tma_load_2d(sm.a[s], &tm_a, &sm.full[s], kb * kBK, m0);
                    tma_load_2d(sm.b[s], &tm_b, &sm.full[s], kb * kBK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const std::uint32_t idesc = instr_desc(p.in_dtype == SACC_DTYPE_BF16 ? 1 : 0, kBM, BN);
            unsigned g = 0, it = 0;
            for (int tile = blockIdx.x; tile < tiles && !fault; tile += gridDim.x, ++it) {
                const unsigned ab = it & 1u;
                if (it >= 2 && !mbar_wait_bounded(&sm.acc_empty[ab], ((it / 2) - 1) & 1u)) {
                    fault = true;
                    break;
                }
                tmem_fence_after();
                const std::uint32_t acc = tmem + ab * BN;
                for (int kb = 0; kb < p.kblocks; ++kb, ++g) {
                    const unsigned s = g % S;
                    if (!mbar_wait_bounded(&sm.full[s], (g / S) & 1u)) {
                        fault = true;
                        break;
                    }
                    tmem_fence_after();
                    const std::uint64_t ad = sw128_desc(sm.a[s]), bd = sw128_desc(sm.b[s]);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_f16(acc, ad + 2ull * kk, bd + 2ull * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
                    mma_commit(&sm.empty[s]);
                }
                if (fault) break;
                mma_commit(&sm.acc_full[ab]);
            }
        }
    } else {
        // Epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 = tile rows.
        // Warp 2 + e takes TMEM lanes of its quarter (a hardware rule: warp w
        // reaches lanes 32 (w % 4) .. + 31) and column half e / 4 of each tile.
        constexpr int kChunks = BN / 32 / (E / 4); // 32-column chunks per warp and tile
        const int quarter = warp % 4, e = warp - 2, c_first = (e / 4) * kChunks;
        unsigned it = 0, st = 0; // st: staging tiles used by this warp
        if (p.tma_store && lane == 0) prefetch_tensor_map(&tm_c);
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
            const unsigned ab = it & 1u;
            if (!mbar_wait_bounded(&sm.acc_full[ab], (it / 2) & 1u)) {
                fault = true;
                break;
            }
            tmem_fence_after();
            const int m0 = (tile / p.tiles_n) * kBM, n0 = (tile % p.tiles_n) * BN;
            const int r0 = m0 + quarter * 32; // first row of this warp
            const unsigned long long row = static_cast<unsigned long long>(r0 + lane);
            const std::uint32_t tbase =
                tmem + ab * BN + static_cast<std::uint32_t>(c_first * 32) + (static_cast<std::uint32_t>(quarter * 32) << 16);
            // Chunk c + 1 loads from TMEM while chunk c is finished and stored.
            std::uint32_t ra[32], rb[32];
            tmem_ld32_issue(tbase, ra);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                float v[32];
                if (c % 2 == 0) {
                    tmem_ld32_wait(ra);
                    if (c + 1 < kChunks) tmem_ld32_issue(tbase + static_cast<std::uint32_t>((c + 1) * 32), rb);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(ra[i]);
                } else {
                    tmem_ld32_wait(rb);
                    if (c + 1 < kChunks) tmem_ld32_issue(tbase + static_cast<std::uint32_t>((c + 1) * 32), ra);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rb[i]);
                }
                const unsigned long long col0 = static_cast<unsigned long long>(n0 + (c_first + c) * 32);
                if (!p.tma_store) {
                    if (row < p.m && col0 < p.n) store_chunk(p, row, col0, v);
                    continue;
                }
                if (static_cast<unsigned long long>(r0) >= p.m || col0 >= p.n) continue; // warp-uniform
                // Coalesced path: the warp's 32 x 32 block goes through a swizzled
                // shared tile and one TMA store (rows / columns past C are clipped).
                if (row < p.m) apply_chunk(p, row, col0, v);
                std::uint16_t* buf = sm.stage[e][st % stage_bufs<E>()];
                if (lane == 0) bulk_wait_read<stage_bufs<E>() - 1>(); // the store that last used this buffer has read it
                __syncwarp();
                std::uint32_t w[16];
                pack16(v, p.out_dtype, w);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<uint4*>(buf + lane * 32 + ((q ^ ((lane >> 1) & 3)) << 3)) =
                        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                fence_async_shared();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tm_c, buf, static_cast<int>(col0), r0);
                    bulk_commit();
                }
                ++st;
            }
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[ab]);
        }
    }
    if (fault) atomicOr(&g_gemm_fault, 1u);
    if (warp >= 2 && lane == 0 && p.tma_store) bulk_wait<0>(); // staged stores have left shared memory
    tmem_fence_before();
    __syncthreads();
    if (warp == 1) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode() {
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

// K-major 2D map (K innermost) with a (64, rows) box and 128-byte swizzle.
bool kmajor_map(CUtensorMap* map, int dtype, const void* base, unsigned long long k, unsigned long long rows,
                unsigned long long ld, unsigned box_rows) {
    auto fn = encode();
    if (!fn) return false;
    const cuuint64_t dims[2] = {k, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == SACC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

template <int BN, int E>
size_t gemm_smem() {
    return sizeof(GemmSmem<BN, E>) + 1024;
}

template <int BN, int E>
cudaError_t prepare_gemm() {
    static std::atomic<int> done[64];
    return once_per_device(done, [] {
        return cudaFuncSetAttribute(reinterpret_cast<const void*>(gemm_kernel<BN, E>), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(gemm_smem<BN, E>()));
    });
}

// C as a 2D map {n, m} with a 32 x 32 box and the 64-byte swizzle (16-bit
// output) for the epilogue's TMA stores.
bool c_map(CUtensorMap* map, int dtype, void* base, unsigned long long n, unsigned long long m, unsigned long long ld) {
    auto fn = encode();
    if (!fn) return false;
    const cuuint64_t dims[2] = {n, m};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = dtype == SACC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    return fn(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int E>
cudaError_t launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmParams p, int sm_count,
                      cudaStream_t stream) {
    const cudaError_t e = prepare_gemm<BN, E>();
    if (e != cudaSuccess) return e;
    p.tiles_m = static_cast<int>((p.m + kBM - 1) / kBM);
    p.tiles_n = static_cast<int>((p.n + BN - 1) / BN);
    const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
    // One CTA per SM; two at BN = 64 (2 x 97 KB of shared memory, 2 x 128 TMEM columns).
    const long long slots = static_cast<long long>(sm_count) * (BN == 64 ? 2 : 1);
    const unsigned grid = static_cast<unsigned>(tiles < slots ? tiles : slots);
    void* args[] = {const_cast<CUtensorMap*>(&ta), const_cast<CUtensorMap*>(&tb), const_cast<CUtensorMap*>(&tc), &p};
    return launch_pdl(reinterpret_cast<const void*>(gemm_kernel<BN, E>), dim3(grid), dim3(gemm_threads<E>()), gemm_smem<BN, E>(), stream,
                      args);
}

} // namespace

cudaError_t launch_gemm(const SaccGemmArgs& a, cudaStream_t stream) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // Widest tile that covers n, narrowed while the tile count leaves SMs idle
    // (the block's projections at config 1 have only 64 row tiles).
    unsigned bn = a.n <= 64 ? 64u : a.n <= 128 ? 128u : 256u;
    const unsigned long long mt = (a.m + kBM - 1) / kBM;
    while (bn > 64 && mt * ((a.n + bn - 1) / bn) < static_cast<unsigned long long>(sms)) bn /= 2;
    CUtensorMap ta{}, tb{};
    if (!kmajor_map(&ta, a.in_dtype, a.a, a.k, a.m, a.lda, kBM) || !kmajor_map(&tb, a.in_dtype, a.b, a.k, a.n, a.ldb, bn))
        return cudaErrorInvalidValue;
    GemmParams p{};
    p.c = a.c; p.residual = a.residual; p.bias = a.bias; p.row_scale = a.row_scale;
    p.m = a.m; p.n = a.n; p.k = a.k; p.ldc = a.ldc; p.ldr = a.residual ? a.ldr : 0;
    p.out_dtype = a.out_dtype; p.in_dtype = a.in_dtype;
    p.kblocks = static_cast<int>((a.k + kBK - 1) / kBK);
    const std::size_t eo = a.out_dtype == SACC_DTYPE_F32 ? 4 : 2;
    p.vec_store = (reinterpret_cast<std::uintptr_t>(a.c) % 16 == 0) && ((a.ldc * eo) % 16 == 0);
    p.res_vec = a.residual && (reinterpret_cast<std::uintptr_t>(a.residual) % 16 == 0) && ((a.ldr * eo) % 16 == 0);
    CUtensorMap tc{};
    p.tma_store = a.out_dtype != SACC_DTYPE_F32 && p.vec_store && c_map(&tc, a.out_dtype, a.c, a.n, a.m, a.ldc);
    const bool short_k = p.kblocks <= 8; // eight epilogue warps when a tile's MMAs are short (K <= 512)
    if (bn == 64) return launch_bn<64, 4>(ta, tb, tc, p, sms, stream);
    if (bn == 128) return short_k ? launch_bn<128, 8>(ta, tb, tc, p, sms, stream) : launch_bn<128, 4>(ta, tb, tc, p, sms, stream);
    return short_k ? launch_bn<256, 8>(ta, tb, tc, p, sms, stream) : launch_bn<256, 4>(ta, tb, tc, p, sms, stream);
}

cudaError_t load_gemm_kernels(std::string& report) {
    const std::pair<const char*, const void*> ks[] = {{"gemm_tcgen05_bn64", reinterpret_cast<const void*>(gemm_kernel<64, 4>)},
                                                      {"gemm_tcgen05_bn128", reinterpret_cast<const void*>(gemm_kernel<128, 4>)},
                                                      {"gemm_tcgen05_bn128_e8", reinterpret_cast<const void*>(gemm_kernel<128, 8>)},
                                                      {"gemm_tcgen05_bn256", reinterpret_cast<const void*>(gemm_kernel<256, 4>)},
                                                      {"gemm_tcgen05_bn256_e8", reinterpret_cast<const void*>(gemm_kernel<256, 8>)}};
    for (const auto& k : ks) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, k.second);
        if (e != cudaSuccess) return e;
        report += std::string("kernel=") + k.first + " registers=" + std::to_string(attr.numRegs) + "\n";
    }
    cudaError_t e = prepare_gemm<64, 4>();
    if (e == cudaSuccess) e = prepare_gemm<128, 4>();
    if (e == cudaSuccess) e = prepare_gemm<128, 8>();
    if (e == cudaSuccess) e = prepare_gemm<256, 4>();
    if (e == cudaSuccess) e = prepare_gemm<256, 8>();
    return e;
}

cudaError_t read_gemm_fault(unsigned* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_gemm_fault, sizeof(unsigned));
    if (e != cudaSuccess || !clear) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_gemm_fault, &zero, sizeof(unsigned));
}

} // namespace sacc
