// scan_bulk.cu -- high-throughput selective scan for 16-bit activations with
// FP32 state and N = 16 states, in Mamba's (B, D, L)
// layout or the reference's (B, L, D) layout.
//
// Work split: one thread owns one (batch, channel) lane and its 16 states in
// registers; a CTA of 128 threads owns 128 consecutive channels of one batch
// row and walks the sequence in chunks of 32 tokens.
//
// Data movement: per chunk, one thread issues TMA loads of the u / delta / z
// tiles and of the B / C tiles into a two-stage ring completed by mbarriers,
// and a TMA store of the y tile.  In (B, D, L) each thread's 32 tokens are one
// 64-byte row of a 64-byte-swizzled tile, read with conflict-free 16-byte
// shared loads; in (B, L, D) a warp reads 32 consecutive channels of one
// token.  B and C are converted once per chunk to an FP32 token-major table
// that all threads read with broadcast loads.  Every input byte crosses HBM
// once, every output byte once.
//
// Arithmetic: with N = 16 the scan is bound by the special-function unit, not
// by HBM: every state update needs one 2^x (MUFU ex2, 16 per SM per clock) and
// four FP32 operations (Delta*A, Delta*u*B, the state FMA and the C*h FMA),
// against 6 bytes of bf16 traffic per 16 updates.  softplus runs on the FMA
// pipe except for one ex2 (log1p(e) = e * P(e), a degree-7 fit with 3e-7
// relative error, gen_exp2_poly.py), so the special-function unit spends its
// cycles on the decays.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"
#include "scan_common.cuh"
#include "tma.cuh"

namespace sacc {

__device__ unsigned int g_bulk_fault; // set when a bounded wait ran out; read by sacc_scan_fault()

namespace {

constexpr int kLanes = 128; // threads (lanes) per CTA
constexpr int kT = 32;      // tokens per chunk
constexpr int kStages = 2;
constexpr int kN = 16;
constexpr int kMinBlocks = 4; // four CTAs per SM: 128 registers per thread

template <typename T, bool kHasZ>
struct Smem {
    alignas(1024) T u[kStages][kLanes * kT];
    alignas(1024) T dl[kStages][kLanes * kT];
    alignas(1024) T z[kHasZ ? kStages : 1][kHasZ ? kLanes * kT : 8];
    alignas(1024) T y[kLanes * kT];
    alignas(128) T braw[kStages][kN * kT];
    alignas(128) T craw[kStages][kN * kT];
    alignas(16) float bc[kT][2 * kN]; // per token: B[0..15], C[16..31] (C[16] only when rank 1)
    alignas(8) std::uint64_t full[kStages];
};

template <typename T, bool kHasZ>
constexpr size_t smem_bytes() {
    return sizeof(Smem<T, kHasZ>) + 1024; // + alignment slack for the 1024-byte swizzle atoms
}

struct BulkParams {
    const float *a, *d, *bias, *h0;
    float* h_final;
    const int32_t* cu; // packed varlen sequences ((B, L, D) with batch 1), else null
    void* y;           // plain stores of a varlen sequence's last, partial chunk
    unsigned long long length, channels, per_group;
    unsigned groups;
    int a_shared, c_full, has_d, softplus, nchunks;
};

template <typename T>
__device__ __forceinline__ float2 unpack2(std::uint32_t w);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(std::uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(std::uint32_t w) {
    __half2 h;
    std::memcpy(&h, &w, 4);
    return __half22float2(h);
}

template <typename T>
__device__ __forceinline__ std::uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ std::uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    std::uint32_t w;
    std::memcpy(&w, &v, 4);
    return w;
}
template <>
__device__ __forceinline__ std::uint32_t pack2<__half>(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    std::uint32_t w;
    std::memcpy(&w, &v, 4);
    return w;
}

// Eight tokens of one lane's u / raw delta / z.
struct Block8 {
    float u[8], x[8], z[8];
};

// (B, D, L): row `tid` of a 64-byte-swizzled [128][32] tile; chunk q of row r
// sits at q ^ ((r >> 1) & 3) (TMA 64-byte swizzle: address bits [4:5] ^= [7:8]).
template <typename T, bool kHasZ>
__device__ __forceinline__ void load_block_bdl(const T* u, const T* dl, const T* z, int tid, int q, Block8& blk) {
    const int off = tid * kT + ((q ^ ((tid >> 1) & 3)) << 3);
    const uint4 uq = *reinterpret_cast<const uint4*>(u + off);
    const uint4 xq = *reinterpret_cast<const uint4*>(dl + off);
    const std::uint32_t uw[4] = {uq.x, uq.y, uq.z, uq.w}, xw[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 a = unpack2<T>(uw[j]), b = unpack2<T>(xw[j]);
        blk.u[2 * j] = a.x; blk.u[2 * j + 1] = a.y;
        blk.x[2 * j] = b.x; blk.x[2 * j + 1] = b.y;
    }
    if constexpr (kHasZ) {
        const uint4 zq = *reinterpret_cast<const uint4*>(z + off);
        const std::uint32_t zw[4] = {zq.x, zq.y, zq.z, zq.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 c = unpack2<T>(zw[j]);
            blk.z[2 * j] = c.x; blk.z[2 * j + 1] = c.y;
        }
    }
}

template <typename T>
__device__ __forceinline__ void store_block_bdl(T* y, int tid, int q, const float (&out)[8]) {
    const int off = tid * kT + ((q ^ ((tid >> 1) & 3)) << 3);
    *reinterpret_cast<uint4*>(y + off) = make_uint4(pack2<T>(out[0], out[1]), pack2<T>(out[2], out[3]),
                                                    pack2<T>(out[4], out[5]), pack2<T>(out[6], out[7]));
}

// (B, L, D): token-major [32][128] tile; lane `tid` is column tid.
template <typename T, bool kHasZ>
__device__ __forceinline__ void load_block_bld(const T* u, const T* dl, const T* z, int tid, int q, Block8& blk) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int at = (q * 8 + j) * kLanes + tid;
        blk.u[j] = to_f32(u[at]);
        blk.x[j] = to_f32(dl[at]);
        if constexpr (kHasZ) blk.z[j] = to_f32(z[at]);
    }
}

template <typename T>
__device__ __forceinline__ void store_block_bld(T* y, int tid, int q, const float (&out)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) y[(q * 8 + j) * kLanes + tid] = from_f32<T>(out[j]);
}

// Loads of the chunk starting at token t0 into stage s.  (B, D, L): 2D maps,
// x = token, y = row (b * D + d).  (B, L, D): 3D maps (channel, token, batch),
// so that a chunk past the end of a sequence reads zeros instead of the next
// sequence; a packed varlen sequence reads whatever follows it, unused.
template <typename T, bool kBDL, bool kHasZ>
__device__ __forceinline__ void issue_chunk(Smem<T, kHasZ>& sm, int s, int t0, int row0, int brow0, int crow0, int bb,
                                            std::uint32_t c_bytes, const CUtensorMap* tu, const CUtensorMap* td,
                                            const CUtensorMap* tz, const CUtensorMap* tb, const CUtensorMap* tc) {
    constexpr std::uint32_t tile = kLanes * kT * sizeof(T), btile = kN * kT * sizeof(T);
    mbar_arrive_expect_tx(&sm.full[s], tile * (kHasZ ? 3u : 2u) + btile + c_bytes);
    if (kBDL) {
        tma_load_2d(sm.u[s], tu, &sm.full[s], t0, row0);
        tma_load_2d(sm.dl[s], td, &sm.full[s], t0, row0);
        if constexpr (kHasZ) tma_load_2d(sm.z[s], tz, &sm.full[s], t0, row0);
        tma_load_2d(sm.braw[s], tb, &sm.full[s], t0, brow0);
        tma_load_2d(sm.craw[s], tc, &sm.full[s], t0, crow0);
    } else {
        tma_load_3d(sm.u[s], tu, &sm.full[s], row0, t0, bb);
        tma_load_3d(sm.dl[s], td, &sm.full[s], row0, t0, bb);
        if constexpr (kHasZ) tma_load_3d(sm.z[s], tz, &sm.full[s], row0, t0, bb);
        tma_load_3d(sm.braw[s], tb, &sm.full[s], brow0, t0, bb);
        tma_load_3d(sm.craw[s], tc, &sm.full[s], crow0, t0, bb);
    }
}

// Eight tokens of one lane through the recurrence; with kGuard only the first
// `count` (fewer in a sequence's last, partial block; the others are left out
// of the state).
template <bool kFullC, bool kHasZ, bool kGuard>
__device__ __forceinline__ void scan_block8(const float (*bc)[2 * kN], int q, int count, const Block8& blk, const float (&a)[kN],
                                            float (&h)[kN], float bias, float dskip, int softplus, float (&out)[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        out[j] = 0.0f;
        if (kGuard && j >= count) continue;
        const int t = q * 8 + j;
        const float xv = blk.x[j] + bias;
        const float dt = softplus ? softplus_poly(xv) : xv;
        const float du = dt * blk.u[j];
        const float4* bcv = reinterpret_cast<const float4*>(bc[t]);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const float cr = kFullC ? 0.0f : bc[t][kN];
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
            const float4 bq = bcv[k4];
            const float bb[4] = {bq.x, bq.y, bq.z, bq.w};
            float cc[4] = {cr, cr, cr, cr};
            if constexpr (kFullC) {
                const float4 cq = bcv[4 + k4];
                cc[0] = cq.x; cc[1] = cq.y; cc[2] = cq.z; cc[3] = cq.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int n = 4 * k4 + i;
                const float decay = fast_exp2(dt * a[n]);
                h[n] = fmaf(decay, h[n], du * bb[i]);
                acc[i] = fmaf(cc[i], h[n], acc[i]);
            }
        }
        float y = fmaf(dskip, blk.u[j], (acc[0] + acc[1]) + (acc[2] + acc[3]));
        if constexpr (kHasZ) y *= silu(blk.z[j]);
        out[j] = y;
    }
}

template <typename T, bool kBDL, bool kHasZ, bool kFullC>
__global__ void __launch_bounds__(kLanes, kMinBlocks) bulk_kernel(const __grid_constant__ CUtensorMap tm_u,
                                                                  const __grid_constant__ CUtensorMap tm_d,
                                                                  const __grid_constant__ CUtensorMap tm_z,
                                                                  const __grid_constant__ CUtensorMap tm_b,
                                                                  const __grid_constant__ CUtensorMap tm_c,
                                                                  const __grid_constant__ CUtensorMap tm_y, BulkParams p) {
    extern __shared__ unsigned char smem_raw[];
    auto& sm = *reinterpret_cast<Smem<T, kHasZ>*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    const int tid = threadIdx.x;
    const unsigned long long D = p.channels, L = p.length;
    const unsigned long long tiles_per_row = D / kLanes;
    const unsigned long long b = blockIdx.x / tiles_per_row;
    const unsigned long long d0 = (blockIdx.x % tiles_per_row) * kLanes, d = d0 + tid;
    const unsigned long long lane = b * D + d;
    const unsigned long long g = d0 / p.per_group;
    const int cw = kFullC ? kN : 1;
    // Token range: the whole row, or packed sequence b ((B, L, D), batch 1),
    // its cu_seqlens entries clamped to [0, L] so no access leaves the tensors.
    unsigned long long tok0 = 0, len = L;
    if (!kBDL && p.cu) {
        const long long lo = p.cu[b], hi = p.cu[b + 1];
        tok0 = lo < 0 ? 0 : (static_cast<unsigned long long>(lo) > L ? L : static_cast<unsigned long long>(lo));
        const unsigned long long end = hi < 0 ? 0 : (static_cast<unsigned long long>(hi) > L ? L : static_cast<unsigned long long>(hi));
        len = end > tok0 ? end - tok0 : 0;
    }
    const int nchunks = (!kBDL && p.cu) ? static_cast<int>((len + kT - 1) / kT) : p.nchunks;
    // Tensor-map coordinates of this CTA.
    const int row0 = kBDL ? static_cast<int>(b * D + d0) : static_cast<int>(d0);
    const int bb = (!kBDL && p.cu) ? 0 : static_cast<int>(b);
    const int brow0 = kBDL ? static_cast<int>((b * p.groups + g) * kN) : static_cast<int>(g * kN);
    const int crow0 = kBDL ? static_cast<int>((b * p.groups + g) * cw) : static_cast<int>(g * cw);
    const std::uint32_t c_bytes = static_cast<std::uint32_t>(cw) * kT * sizeof(T);

    if (tid == 0) {
        prefetch_tensor_map(&tm_u);
        prefetch_tensor_map(&tm_d);
        prefetch_tensor_map(&tm_b);
        prefetch_tensor_map(&tm_c);
        prefetch_tensor_map(&tm_y);
        for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kStages && s < nchunks; ++s)
            issue_chunk<T, kBDL, kHasZ>(sm, s, static_cast<int>(tok0) + s * kT, row0, brow0, crow0, bb, c_bytes, &tm_u, &tm_d,
                                        &tm_z, &tm_b, &tm_c);

    // Per-lane constants: A * log2(e), D, dt bias, initial state.
    float a[kN], h[kN];
    const float* arow = p.a + (p.a_shared ? 0 : d * kN);
#pragma unroll
    for (int n = 0; n < kN; ++n) {
        a[n] = arow[n] * kLog2e;
        h[n] = p.h0 ? p.h0[lane * kN + n] : 0.0f;
    }
    const float dskip = p.has_d ? p.d[d] : 0.0f;
    const float bias = p.bias ? p.bias[d] : 0.0f;

    bool fault = false;
    for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int s = chunk % kStages;
        const bool ok = mbar_wait_bounded(&sm.full[s], static_cast<std::uint32_t>((chunk / kStages) & 1));
        if (tid == 0) bulk_wait_read<0>(); // the y tile is no longer read by the previous chunk's store
        if (!__syncthreads_and(ok)) {
            fault = true;
            break;
        }
        // B / C tiles to an FP32 token-major table.
        if (kBDL) {
            // raw [state][token]: a thread takes 8 tokens of one state (16 bytes).
            for (int i = tid; i < (kN + cw) * (kT / 8); i += kLanes) {
                const int rowi = i / (kT / 8), t0 = (i % (kT / 8)) * 8;
                const T* src = rowi < kN ? sm.braw[s] + rowi * kT + t0 : sm.craw[s] + (rowi - kN) * kT + t0;
                const uint4 v = *reinterpret_cast<const uint4*>(src);
                const std::uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = unpack2<T>(w[j]);
                    sm.bc[t0 + 2 * j][rowi] = f.x;
                    sm.bc[t0 + 2 * j + 1][rowi] = f.y;
                }
            }
        } else {
            // raw [token][state]: already token-major.
            for (int i = tid; i < kN * kT; i += kLanes) sm.bc[i / kN][i % kN] = to_f32(sm.braw[s][i]);
            for (int i = tid; i < cw * kT; i += kLanes) sm.bc[i / cw][kN + i % cw] = to_f32(sm.craw[s][i]);
        }
        __syncthreads();

        // Tokens past the end of the sequence (zero-filled by the TMA, or the
        // next packed sequence) are not run through the recurrence.
        const unsigned long long left = len - static_cast<unsigned long long>(chunk) * kT;
        const int valid = static_cast<int>(left < kT ? left : kT);
        const int blocks8 = (valid + 7) / 8;
#pragma unroll 1
        for (int q = 0; q < blocks8; ++q) {
            Block8 blk;
            if (kBDL) load_block_bdl<T, kHasZ>(sm.u[s], sm.dl[s], sm.z[kHasZ ? s : 0], tid, q, blk);
            else load_block_bld<T, kHasZ>(sm.u[s], sm.dl[s], sm.z[kHasZ ? s : 0], tid, q, blk);
            float out[8];
            scan_block8<kFullC, kHasZ, true>(sm.bc, q, valid - q * 8, blk, a, h, bias, dskip, p.softplus, out);
            if (kBDL) store_block_bdl<T>(sm.y, tid, q, out);
            else store_block_bld<T>(sm.y, tid, q, out);
        }
        fence_async_shared();
        __syncthreads();
        const int tc0 = static_cast<int>(tok0) + chunk * kT;
        const bool tail = !kBDL && p.cu && valid < kT;
        if (tail) {
            // A packed sequence's partial last chunk: a tile store would also
            // write the next sequence's rows, so store the valid rows only.
            T* yg = static_cast<T*>(p.y);
            for (int t = 0; t < valid; ++t) yg[(static_cast<unsigned long long>(tc0) + t) * D + d] = sm.y[t * kLanes + tid];
        }
        if (tid == 0) {
            if (!tail) {
                if (kBDL) tma_store_2d(&tm_y, sm.y, tc0, row0);
                else tma_store_3d(&tm_y, sm.y, row0, tc0, bb);
            }
            bulk_commit();
            if (chunk + kStages < nchunks)
                issue_chunk<T, kBDL, kHasZ>(sm, s, tc0 + kStages * kT, row0, brow0, crow0, bb, c_bytes, &tm_u, &tm_d, &tm_z,
                                            &tm_b, &tm_c);
        }
    }
    if (fault) {
        if (tid == 0) {
            atomicOr(&g_bulk_fault, 1u);
            // Give copies still in flight a bounded chance to land before the
            // CTA's shared memory is released.
            for (int s = 0; s < kStages; ++s) (void)mbar_wait_bounded(&sm.full[s], 0u, 1u << 16);
        }
        return;
    }
    if (tid == 0) bulk_wait<0>();
    if (p.h_final) {
#pragma unroll
        for (int n = 0; n < kN; ++n) p.h_final[lane * kN + n] = h[n];
    }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 3D map (inner, mid, outer) with a (box_inner, box_mid, 1) box, no swizzle;
// consecutive mid rows `row_stride` elements apart (0: dense, = inner).
bool make_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, unsigned long long inner,
                 unsigned long long mid, unsigned long long outer, unsigned box_inner, unsigned box_mid,
                 unsigned long long row_stride = 0) {
    auto fn = encode_fn();
    if (!fn) return false;
    const unsigned long long rs = row_stride ? row_stride : inner;
    const cuuint64_t dims[3] = {inner, mid, outer};
    const cuuint64_t strides[2] = {rs * 2, rs * mid * 2};
    const cuuint32_t box[3] = {box_inner, box_mid, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, unsigned long long inner,
                 unsigned long long rows, unsigned long long row_stride_bytes, unsigned box_inner, unsigned box_rows,
                 CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, bool kBDL, bool kHasZ, bool kFullC>
struct Variant {
    static const void* fn() { return reinterpret_cast<const void*>(bulk_kernel<T, kBDL, kHasZ, kFullC>); }
    static cudaError_t prepare() {
        static const cudaError_t status = cudaFuncSetAttribute(fn(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                               static_cast<int>(smem_bytes<T, kHasZ>()));
        return status;
    }
    static size_t smem() { return smem_bytes<T, kHasZ>(); }
};

struct Pick {
    const void* fn;
    size_t smem;
    cudaError_t (*prepare)();
};

template <typename T, bool kBDL, bool kHasZ, bool kFullC>
Pick make_pick() {
    using V = Variant<T, kBDL, kHasZ, kFullC>;
    return {V::fn(), V::smem(), &V::prepare};
}

template <typename T, bool kBDL>
Pick pick_z(bool z, bool full_c) {
    if (z) return full_c ? make_pick<T, kBDL, true, true>() : make_pick<T, kBDL, true, false>();
    return full_c ? make_pick<T, kBDL, false, true>() : make_pick<T, kBDL, false, false>();
}

Pick pick(int dtype, bool bdl, bool z, bool full_c) {
    if (dtype == SACC_DTYPE_BF16) return bdl ? pick_z<__nv_bfloat16, true>(z, full_c) : pick_z<__nv_bfloat16, false>(z, full_c);
    return bdl ? pick_z<__half, true>(z, full_c) : pick_z<__half, false>(z, full_c);
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

} // namespace

// The bulk kernel's domain: 16-bit activations, N = 16, no varlen, channels
// in 128-wide tiles inside one group, 16-byte aligned tensors and 16-byte row
// strides for the TMA ((B, D, L): L % 8 == 0; (B, L, D): a full-width C, whose
// rows are then 16 * groups * 2 bytes).  Other calls use the general kernel.
bool bulk_eligible(const SaccScanExArgs& a, const RowStrides* rs) {
    if (rs) {
        // Strided z / B / C rows (the block's fused projection outputs): dense
        // (B, L, D) rows only, 16-byte row pitches, rows at least as wide as the data.
        const unsigned long long cw = a.c_width;
        if (a.layout != SACC_LAYOUT_BLD || a.cu_seqlens != nullptr || (rs->z && (rs->z < a.channels || rs->z % 8)) ||
            (rs->b && (rs->b < a.groups * kN || rs->b % 8)) || (rs->c && (rs->c < a.groups * cw || rs->c % 8)))
            return false;
    }
    if ((a.dtype != SACC_DTYPE_BF16 && a.dtype != SACC_DTYPE_F16) || a.state != kN || a.length == 0 || a.groups == 0 ||
        a.channels % kLanes != 0 || (a.channels / a.groups) % kLanes != 0)
        return false;
    if (a.cu_seqlens != nullptr) {
        // Packed varlen: (B, L, D) with batch 1, any sequence lengths.
        if (a.layout != SACC_LAYOUT_BLD || a.batch != 1 || a.c_width != kN || a.channels % 8 != 0 || a.nseq <= 0 ||
            static_cast<unsigned long long>(a.nseq) * (a.channels / kLanes) > 0x7fffffffull)
            return false;
    } else if (a.layout == SACC_LAYOUT_BDL) {
        if (a.length % 8 != 0) return false;
    } else if (a.layout == SACC_LAYOUT_BLD) {
        if (a.c_width != kN || a.length % 8 != 0 || a.channels % 8 != 0) return false;
    } else {
        return false;
    }
    for (const void* ptr : {a.u, a.delta, a.b, a.c, a.z, static_cast<const void*>(a.y)})
        if (ptr && !aligned16(ptr)) return false;
    const unsigned long long rows = a.batch * a.channels, tokens = a.batch * a.length;
    return rows <= 0x7fffffffull && tokens <= 0x7fffffffull && a.batch * a.groups * kN <= 0x7fffffffull;
}

cudaError_t launch_scan_bulk(const SaccScanExArgs& a, cudaStream_t stream, const RowStrides* rs) {
    const RowStrides dense{0, 0, 0};
    if (!rs) rs = &dense;
    const bool bdl = a.layout == SACC_LAYOUT_BDL;
    const unsigned long long cw = a.c_width, B = a.batch, D = a.channels, L = a.length, G = a.groups;
    const CUtensorMapDataType dt = a.dtype == SACC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tu{}, td{}, tz{}, tb{}, tc{}, ty{};
    bool ok;
    if (bdl) {
        const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
        ok = make_map_2d(&tu, dt, a.u, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&td, dt, a.delta, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&tz, dt, a.z ? a.z : a.u, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&ty, dt, a.y, L, B * D, L * 2, kT, kLanes, sw) &&
             make_map_2d(&tb, dt, a.b, L, B * G * kN, L * 2, kT, kN, CU_TENSOR_MAP_SWIZZLE_NONE) &&
             make_map_2d(&tc, dt, a.c, L, B * G * cw, L * 2, kT, static_cast<unsigned>(cw), CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
        ok = make_map_3d(&tu, dt, a.u, D, L, B, kLanes, kT) && make_map_3d(&td, dt, a.delta, D, L, B, kLanes, kT) &&
             make_map_3d(&tz, dt, a.z ? a.z : a.u, D, L, B, kLanes, kT, a.z ? rs->z : 0) &&
             make_map_3d(&ty, dt, a.y, D, L, B, kLanes, kT) && make_map_3d(&tb, dt, a.b, G * kN, L, B, kN, kT, rs->b) &&
             make_map_3d(&tc, dt, a.c, G * cw, L, B, static_cast<unsigned>(cw), kT, rs->c);
    }
    if (!ok) return cudaErrorInvalidValue; // tensor-map encoding refused the (checked) layout
    BulkParams p{};
    p.a = a.a; p.d = a.d; p.bias = a.delta_bias; p.h0 = a.h0; p.h_final = a.h_final;
    p.length = L; p.channels = D; p.per_group = D / G; p.groups = static_cast<unsigned>(G);
    p.a_shared = a.a_rows == 1; p.c_full = cw != 1; p.has_d = a.d != nullptr; p.softplus = a.delta_softplus != 0;
    p.nchunks = static_cast<int>((L + kT - 1) / kT);
    p.cu = bdl ? nullptr : a.cu_seqlens;
    p.y = a.y;
    const unsigned long long rows = a.cu_seqlens ? static_cast<unsigned long long>(a.nseq) : B; // sequences
    const Pick k = pick(a.dtype, bdl, a.z != nullptr, cw != 1);
    const cudaError_t attr = k.prepare();
    if (attr != cudaSuccess) return attr;
    void* args[] = {&tu, &td, &tz, &tb, &tc, &ty, &p};
    return cudaLaunchKernel(k.fn, dim3(static_cast<unsigned>(rows * D / kLanes)), dim3(kLanes), args, k.smem, stream);
}

cudaError_t load_scan_bulk_kernels(std::string& report) {
    const char* names[2] = {"bld", "bdl"};
    for (int dtype : {SACC_DTYPE_BF16, SACC_DTYPE_F16})
        for (int bdl = 0; bdl < 2; ++bdl)
            for (int z = 0; z < 4; ++z) {
                if (!bdl && (z & 2) == 0) continue; // (B, L, D) always has a full-width C
                const Pick k = pick(dtype, bdl != 0, (z & 1) != 0, (z & 2) != 0);
                cudaFuncAttributes attr{};
                cudaError_t e = cudaFuncGetAttributes(&attr, k.fn);
                if (e != cudaSuccess) return e;
                e = k.prepare();
                if (e != cudaSuccess) return e;
                report += std::string("kernel=scan_bulk_") + names[bdl] + (dtype == SACC_DTYPE_BF16 ? "_bf16" : "_f16") +
                          ((z & 1) ? "_gate" : "") + ((z & 2) ? "" : "_rank1c") + " registers=" + std::to_string(attr.numRegs) +
                          " local_bytes=" + std::to_string(attr.localSizeBytes) +
                          " dynamic_shared_bytes=" + std::to_string(k.smem) + "\n";
            }
    return cudaSuccess;
}

cudaError_t read_bulk_fault(unsigned* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_bulk_fault, sizeof(unsigned));
    if (e != cudaSuccess || !clear) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_bulk_fault, &zero, sizeof(unsigned));
}

} // namespace sacc
