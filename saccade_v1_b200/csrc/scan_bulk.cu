// scan_bulk.cu -- high-throughput selective scan for 16-bit activations in
// Mamba's (B, D, L) layout, N = 16 states, FP32 state.
//
// Work split: one thread owns one (batch, channel) lane and its 16 states in
// registers; a CTA of 128 threads owns 128 consecutive channels of one batch
// row and walks the sequence in chunks of 32 tokens.
//
// Data movement: per chunk, one thread issues TMA loads of the u / delta / z
// tiles (128 rows x 64 bytes, 64-byte swizzle so that every thread reads its
// own row with conflict-free 16-byte shared loads) and of the B / C tiles
// (16 x 32 tokens) into a two-stage ring completed by mbarriers; the outputs
// are written into a swizzled shared tile and stored with a TMA store.  The
// chunk after next is in flight while one chunk is computed.  Inputs are read
// from HBM once; nothing is re-read.
//
// Arithmetic: the scan is bound by the FP32 and special-function pipes, not by
// HBM (16 state updates per 6 bytes of bf16 traffic: one exp, one multiply for
// Delta*A, one for Delta*u*B, one FMA for the state and one for C*h per
// update).  The 16 decays of a token are split between the MUFU ex2 unit and
// an FMA-pipe exp2 (Cody-Waite reduction 2^x = 2^j 2^f, degree-5 minimax
// polynomial for 2^f, coefficients from gen_exp2_poly.py, max relative error
// 2.4e-7), so both pipes work in parallel; state pairs use the packed
// fma/mul.rn.f32x2 instructions to halve the issue slots.
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
constexpr int kPairs = kN / 2;

template <typename T>
struct Smem {
    alignas(1024) T u[kStages][kLanes * kT];
    alignas(1024) T dl[kStages][kLanes * kT];
    alignas(1024) T z[kStages][kLanes * kT];
    alignas(1024) T y[2][kLanes * kT];
    alignas(128) T braw[kStages][kN * kT];
    alignas(128) T craw[kStages][kN * kT];
    alignas(16) float bc[kT][2 * kN]; // per token: B[0..15], C[16..31] (C[16] only when rank 1)
    alignas(8) std::uint64_t full[kStages];
};

struct BulkParams {
    const float *a, *d, *bias, *h0;
    float* h_final;
    unsigned long long length, channels, lanes, per_group;
    unsigned groups;
    int a_shared, c_full, has_d, softplus, has_z, nchunks;
};

__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(r);
}

// 2^x for a pair on the FMA pipe: j = rint(x) by the 1.5 * 2^23 addition,
// f = x - j in [-1/2, 1/2], p(f) ~ 2^f, exponent j added to p's bits.
// x is clamped to [-125, 126]; 2^-125 stands in for smaller decays.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
    x.x = fminf(fmaxf(x.x, -125.0f), 126.0f);
    x.y = fminf(fmaxf(x.y, -125.0f), 126.0f);
    const float2 magic = make_float2(12582912.0f, 12582912.0f);
    const float2 t = add2(x, magic);
    const float2 j = sub2(t, magic);
    const float2 f = sub2(x, j);
    float2 p = fma2(make_float2(1.3276472e-3f, 1.3276472e-3f), f, make_float2(9.675541e-3f, 9.675541e-3f));
    p = fma2(p, f, make_float2(5.550713e-2f, 5.550713e-2f));
    p = fma2(p, f, make_float2(2.4022120e-1f, 2.4022120e-1f));
    p = fma2(p, f, make_float2(6.9314694e-1f, 6.9314694e-1f));
    p = fma2(p, f, make_float2(1.0000001f, 1.0000001f));
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

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

template <typename T>
__device__ __forceinline__ float scalar16(T v) {
    return to_f32(v);
}

// One chunk's issue: u, delta (and z) tiles of this CTA's 128 rows, B and C tiles.
template <typename T>
__device__ __forceinline__ void issue_chunk(Smem<T>& sm, int s, int chunk, int row0, int brow0, int crow0, int cw,
                                            bool has_z, const CUtensorMap* tu, const CUtensorMap* td, const CUtensorMap* tz,
                                            const CUtensorMap* tb, const CUtensorMap* tc) {
    constexpr std::uint32_t tile = kLanes * kT * sizeof(T), btile = kN * kT * sizeof(T);
    const std::uint32_t bytes = tile * (has_z ? 3u : 2u) + btile + static_cast<std::uint32_t>(cw) * kT * sizeof(T);
    mbar_arrive_expect_tx(&sm.full[s], bytes);
    const int x = chunk * kT;
    tma_load_2d(sm.u[s], tu, &sm.full[s], x, row0);
    tma_load_2d(sm.dl[s], td, &sm.full[s], x, row0);
    if (has_z) tma_load_2d(sm.z[s], tz, &sm.full[s], x, row0);
    tma_load_2d(sm.braw[s], tb, &sm.full[s], x, brow0);
    tma_load_2d(sm.craw[s], tc, &sm.full[s], x, crow0);
}

template <typename T, int kPolyPairs>
__global__ void __launch_bounds__(kLanes) bulk_bdl_kernel(const __grid_constant__ CUtensorMap tm_u,
                                                          const __grid_constant__ CUtensorMap tm_d,
                                                          const __grid_constant__ CUtensorMap tm_z,
                                                          const __grid_constant__ CUtensorMap tm_b,
                                                          const __grid_constant__ CUtensorMap tm_c,
                                                          const __grid_constant__ CUtensorMap tm_y, BulkParams p) {
    extern __shared__ unsigned char smem_raw[];
    Smem<T>& sm = *reinterpret_cast<Smem<T>*>((reinterpret_cast<std::uintptr_t>(smem_raw) + 1023) & ~std::uintptr_t(1023));
    const int tid = threadIdx.x;
    const unsigned long long D = p.channels;
    const int row0 = blockIdx.x * kLanes; // first (batch * D + d) row of this CTA
    const unsigned long long lane = static_cast<unsigned long long>(row0) + tid;
    const unsigned long long b = static_cast<unsigned long long>(row0) / D, d = lane % D;
    const unsigned long long g = (static_cast<unsigned long long>(row0) % D) / p.per_group;
    const int cw = p.c_full ? kN : 1;
    const int brow0 = static_cast<int>((b * p.groups + g) * kN);
    const int crow0 = static_cast<int>((b * p.groups + g) * cw);
    const bool has_z = p.has_z != 0;

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
        for (int s = 0; s < kStages && s < p.nchunks; ++s)
            issue_chunk<T>(sm, s, s, row0, brow0, crow0, cw, has_z, &tm_u, &tm_d, &tm_z, &tm_b, &tm_c);

    // Per-lane constants: A * log2(e) per state pair, D, dt bias, initial state.
    float2 a2[kPairs], h[kPairs];
    const float* arow = p.a + (p.a_shared ? 0 : d * kN);
#pragma unroll
    for (int k = 0; k < kPairs; ++k) {
        a2[k] = make_float2(arow[2 * k] * kLog2e, arow[2 * k + 1] * kLog2e);
        h[k] = p.h0 ? make_float2(p.h0[lane * kN + 2 * k], p.h0[lane * kN + 2 * k + 1]) : make_float2(0.0f, 0.0f);
    }
    const float dskip = p.has_d ? p.d[d] : 0.0f;
    const float bias = p.bias ? p.bias[d] : 0.0f;
    const int sw = (tid >> 1) & 3; // 64-byte swizzle: 16-byte chunk q of row r sits at q ^ ((r >> 1) & 3)

    bool fault = false;
    for (int chunk = 0; chunk < p.nchunks; ++chunk) {
        const int s = chunk % kStages;
        const bool ok = mbar_wait_bounded(&sm.full[s], static_cast<std::uint32_t>((chunk / kStages) & 1));
        if (tid == 0) bulk_wait_read<1>(); // y tile (chunk & 1) no longer read by its previous store
        if (!__syncthreads_and(ok)) {
            fault = true;
            break;
        }
        // B / C tiles to FP32, token-major: 16 + (16 or 1) values per token.
        {
            const T* braw = sm.braw[s];
            for (int i = tid; i < kN * kT; i += kLanes) {
                const int n = i / kT, t = i % kT;
                sm.bc[t][n] = scalar16(braw[i]);
            }
            const T* craw = sm.craw[s];
            for (int i = tid; i < cw * kT; i += kLanes) {
                const int n = i / kT, t = i % kT;
                sm.bc[t][kN + n] = scalar16(craw[i]);
            }
        }
        __syncthreads();

        // Tokens past the end of the sequence (zero-filled by the TMA) are not
        // run through the recurrence; L is a multiple of 8.
        const int valid = static_cast<int>(p.length - static_cast<unsigned long long>(chunk) * kT);
        const int groups8 = (valid < kT ? valid : kT) / 8;
        const T* urow = sm.u[s] + tid * kT;
        const T* drow = sm.dl[s] + tid * kT;
        const T* zrow = sm.z[s] + tid * kT;
        T* yrow = sm.y[chunk & 1] + tid * kT;
#pragma unroll 1
        for (int q = 0; q < groups8; ++q) {
            const int off = (q ^ sw) * 8;
            const uint4 uq = *reinterpret_cast<const uint4*>(urow + off);
            const uint4 xq = *reinterpret_cast<const uint4*>(drow + off);
            uint4 zq = make_uint4(0, 0, 0, 0);
            if (has_z) zq = *reinterpret_cast<const uint4*>(zrow + off);
            const std::uint32_t uw[4] = {uq.x, uq.y, uq.z, uq.w}, xw[4] = {xq.x, xq.y, xq.z, xq.w},
                                zw[4] = {zq.x, zq.y, zq.z, zq.w};
            std::uint32_t yw[4];
#pragma unroll
            for (int j2 = 0; j2 < 4; ++j2) {
                const float2 u2 = unpack2<T>(uw[j2]), x2 = unpack2<T>(xw[j2]), z2 = unpack2<T>(zw[j2]);
                float yv[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int t = q * 8 + j2 * 2 + e;
                    const float uv = e ? u2.y : u2.x;
                    const float xv = __fadd_rn(e ? x2.y : x2.x, bias);
                    const float dt = p.softplus ? softplus_fast(xv) : xv;
                    const float du = __fmul_rn(dt, uv);
                    const float2 dt2 = make_float2(dt, dt), du2 = make_float2(du, du);
                    const float4* bcv = reinterpret_cast<const float4*>(sm.bc[t]);
                    float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
                    const float cr = sm.bc[t][kN];
#pragma unroll
                    for (int k = 0; k < kPairs; ++k) {
                        const float4 bq = bcv[k / 2];
                        const float2 b2 = (k & 1) ? make_float2(bq.z, bq.w) : make_float2(bq.x, bq.y);
                        float2 c2;
                        if (p.c_full) {
                            const float4 cq = bcv[4 + k / 2];
                            c2 = (k & 1) ? make_float2(cq.z, cq.w) : make_float2(cq.x, cq.y);
                        } else {
                            c2 = make_float2(cr, cr);
                        }
                        const float2 arg = mul2(dt2, a2[k]);
                        float2 dec;
                        if (k >= kPairs - kPolyPairs) {
                            dec = exp2_poly2(arg);
                        } else {
                            dec.x = fast_exp2(arg.x);
                            dec.y = fast_exp2(arg.y);
                        }
                        const float2 drv = mul2(du2, b2);
                        h[k] = fma2(dec, h[k], drv);
                        if (k & 1) acc1 = fma2(c2, h[k], acc1);
                        else acc0 = fma2(c2, h[k], acc0);
                    }
                    const float2 accs = add2(acc0, acc1);
                    float out = __fadd_rn(accs.x, accs.y);
                    if (p.has_d) out = __fmaf_rn(dskip, uv, out);
                    if (has_z) out = __fmul_rn(out, silu(e ? z2.y : z2.x));
                    yv[e] = out;
                }
                yw[j2] = pack2<T>(yv[0], yv[1]);
            }
            *reinterpret_cast<uint4*>(yrow + off) = make_uint4(yw[0], yw[1], yw[2], yw[3]);
        }
        fence_async_shared();
        __syncthreads();
        if (tid == 0) {
            tma_store_2d(&tm_y, sm.y[chunk & 1], chunk * kT, row0);
            bulk_commit();
            if (chunk + kStages < p.nchunks)
                issue_chunk<T>(sm, s, chunk + kStages, row0, brow0, crow0, cw, has_z, &tm_u, &tm_d, &tm_z, &tm_b, &tm_c);
        }
    }
    if (fault) {
        if (tid == 0) {
            atomicOr(&g_bulk_fault, 1u);
            // Give copies still in flight a bounded chance to land before the CTA's
            // shared memory is released.
            for (int s = 0; s < kStages; ++s) (void)mbar_wait_bounded(&sm.full[s], 0u, 1u << 16);
        }
        return;
    }
    if (tid == 0) bulk_wait<0>();
    if (p.h_final) {
#pragma unroll
        for (int k = 0; k < kPairs; ++k) {
            p.h_final[lane * kN + 2 * k] = h[k].x;
            p.h_final[lane * kN + 2 * k + 1] = h[k].y;
        }
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

constexpr int kPoly = 2; // state pairs on the FMA-pipe exp2 (of 8)

template <typename T>
const void* bulk_kernel_ptr() {
    return reinterpret_cast<const void*>(bulk_bdl_kernel<T, kPoly>);
}

template <typename T>
cudaError_t ensure_smem_attr() {
    static cudaError_t status = [] {
        return cudaFuncSetAttribute(bulk_kernel_ptr<T>(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(sizeof(Smem<T>) + 1024));
    }();
    return status;
}

bool aligned16(const void* p) { return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0; }

} // namespace

// The bulk kernel's domain: 16-bit (B, D, L) activations, N = 16, no varlen,
// L a multiple of 8 (16-byte TMA row strides), 128-channel tiles inside one
// group, 16-byte aligned tensors.  Other calls use the general kernel.
bool bulk_eligible(const SaccScanExArgs& a) {
    if (a.layout != SACC_LAYOUT_BDL || (a.dtype != SACC_DTYPE_BF16 && a.dtype != SACC_DTYPE_F16) || a.state != kN ||
        a.cu_seqlens != nullptr || a.length == 0 || a.length % 8 != 0 || a.channels % kLanes != 0 ||
        (a.channels / a.groups) % kLanes != 0)
        return false;
    for (const void* ptr : {a.u, a.delta, a.b, a.c, a.z, static_cast<const void*>(a.y)})
        if (ptr && !aligned16(ptr)) return false;
    const unsigned long long rows = a.batch * a.channels;
    return rows <= 0x7fffffffull && a.batch * a.groups * kN <= 0x7fffffffull && a.length <= 0x7fffffffull;
}

cudaError_t launch_scan_bulk(const SaccScanExArgs& a, cudaStream_t stream) {
    const unsigned long long rows = a.batch * a.channels;
    const unsigned long long cw = a.c_width;
    const CUtensorMapDataType dt = a.dtype == SACC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const unsigned long long stride = a.length * 2;
    CUtensorMap tu{}, td{}, tz{}, tb{}, tc{}, ty{};
    const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
    if (!make_map_2d(&tu, dt, a.u, a.length, rows, stride, kT, kLanes, sw) ||
        !make_map_2d(&td, dt, a.delta, a.length, rows, stride, kT, kLanes, sw) ||
        !make_map_2d(&tz, dt, a.z ? a.z : a.u, a.length, rows, stride, kT, kLanes, sw) ||
        !make_map_2d(&ty, dt, a.y, a.length, rows, stride, kT, kLanes, sw) ||
        !make_map_2d(&tb, dt, a.b, a.length, a.batch * a.groups * kN, stride, kT, kN, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&tc, dt, a.c, a.length, a.batch * a.groups * cw, stride, kT, static_cast<unsigned>(cw),
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue; // tensor-map encoding refused the (checked) layout
    BulkParams p{};
    p.a = a.a; p.d = a.d; p.bias = a.delta_bias; p.h0 = a.h0; p.h_final = a.h_final;
    p.length = a.length; p.channels = a.channels; p.lanes = rows; p.per_group = a.channels / a.groups;
    p.groups = static_cast<unsigned>(a.groups);
    p.a_shared = a.a_rows == 1; p.c_full = cw != 1; p.has_d = a.d != nullptr; p.softplus = a.delta_softplus != 0;
    p.has_z = a.z != nullptr;
    p.nchunks = static_cast<int>((a.length + kT - 1) / kT);
    const bool bf16 = a.dtype == SACC_DTYPE_BF16;
    const cudaError_t attr = bf16 ? ensure_smem_attr<__nv_bfloat16>() : ensure_smem_attr<__half>();
    if (attr != cudaSuccess) return attr;
    const size_t smem = (bf16 ? sizeof(Smem<__nv_bfloat16>) : sizeof(Smem<__half>)) + 1024;
    void* args[] = {&tu, &td, &tz, &tb, &tc, &ty, &p};
    return cudaLaunchKernel(bf16 ? bulk_kernel_ptr<__nv_bfloat16>() : bulk_kernel_ptr<__half>(),
                            dim3(static_cast<unsigned>(rows / kLanes)), dim3(kLanes), args, smem, stream);
}

cudaError_t load_scan_bulk_kernels(std::string& report) {
    for (const auto& k : {std::make_pair("scan_bulk_bdl_bf16", bulk_kernel_ptr<__nv_bfloat16>()),
                          std::make_pair("scan_bulk_bdl_f16", bulk_kernel_ptr<__half>())}) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, k.second);
        if (e != cudaSuccess) return e;
        report += std::string("kernel=") + k.first + " registers=" + std::to_string(attr.numRegs) +
                  " local_bytes=" + std::to_string(attr.localSizeBytes) +
                  " dynamic_shared_bytes=" + std::to_string(sizeof(Smem<__nv_bfloat16>) + 1024) + "\n";
    }
    cudaError_t e = ensure_smem_attr<__nv_bfloat16>();
    if (e != cudaSuccess) return e;
    return ensure_smem_attr<__half>();
}

cudaError_t read_bulk_fault(unsigned* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_bulk_fault, sizeof(unsigned));
    if (e != cudaSuccess || !clear) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_bulk_fault, &zero, sizeof(unsigned));
}

} // namespace sacc
