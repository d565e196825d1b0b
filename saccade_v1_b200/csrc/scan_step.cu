// scan_step.cu -- one L = 1 selective-scan update of carried per-track state
// (a tracker's per-frame step).  No counterpart in the
// reference, whose operator has no carried state (docs/SCAN_CONTRACT.md:60);
// the recurrence is the reference's (src/selective_scan.cpp:88-107) applied
// to one token starting from the stored state.
//
// HBM-bound: per (track, channel) lane the 16 FP32 states (64 bytes) are read
// and written once, against one exp and four FP32 operations per state.  Four
// threads share a lane, each owning four consecutive states, so that a warp's
// 16-byte state loads and stores cover eight lanes' 512 contiguous bytes; the
// C*h partial sums of a lane are combined with two shuffles.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <type_traits>

#include <cudaTypedefs.h>

#include <mutex>

#include "internal.h"
#include "scan_common.cuh"
#include "tma.cuh"

namespace sacc {

__device__ unsigned int g_step_fault; // set when a bounded wait of the pipelined step ran out

namespace {

constexpr int kThreads = 256;

struct StepParams {
    const void *u, *delta, *z, *b, *c;
    const float *a, *d, *bias;
    float* state;
    const int32_t* slot;
    void* y;
    unsigned long long nseq, channels, groups, per_group, slots;
    int a_shared, c_full, softplus;
};

template <int N>
struct StepShape {
    static constexpr int kPer = N >= 4 ? 4 : N;   // states per thread
    static constexpr int kSub = N / kPer;         // threads per lane (1, 2 or 4 ... 8 for N = 32)
};

template <typename T, int N, bool kPrecise>
__global__ void __launch_bounds__(kThreads) step_kernel(StepParams p) {
    pdl_wait();
    using S = StepShape<N>;
    const unsigned long long gid = static_cast<unsigned long long>(blockIdx.x) * kThreads + threadIdx.x;
    const unsigned long long lane = gid / S::kSub;
    const int sub = static_cast<int>(gid % S::kSub);
    const bool active = lane < p.nseq * p.channels;
    const unsigned long long seq = active ? lane / p.channels : 0, d = active ? lane % p.channels : 0;
    const long long slot = !active ? -1 : p.slot ? static_cast<long long>(p.slot[seq]) : static_cast<long long>(seq);
    const bool live = active && slot >= 0 && static_cast<unsigned long long>(slot) < p.slots;
    const T* u = static_cast<const T*>(p.u);
    const T* dl = static_cast<const T*>(p.delta);
    const T* bm = static_cast<const T*>(p.b);
    const T* cm = static_cast<const T*>(p.c);

    float partial = 0.0f, uv = 0.0f;
    if (live) {
        const unsigned long long g = d / p.per_group;
        const unsigned long long at = seq * p.channels + d;
        uv = to_f32(u[at]);
        const float x = __fadd_rn(to_f32(dl[at]), p.bias ? p.bias[d] : 0.0f);
        const float dt = p.softplus ? (kPrecise ? softplus_precise(x) : softplus_poly(x)) : x;
        const int n0 = sub * S::kPer;
        float* st = p.state + (static_cast<unsigned long long>(slot) * p.channels + d) * N + n0;
        float h[S::kPer];
        if constexpr (S::kPer == 4) {
            const float4 v = *reinterpret_cast<const float4*>(st);
            h[0] = v.x; h[1] = v.y; h[2] = v.z; h[3] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < S::kPer; ++i) h[i] = st[i];
        }
        const float* arow = p.a + (p.a_shared ? 0 : d * N) + n0;
        const unsigned long long bbase = (seq * p.groups + g) * N + n0;
        const unsigned long long cbase = (seq * p.groups + g) * (p.c_full ? N : 1) + (p.c_full ? n0 : 0);
        const float du = __fmul_rn(dt, uv);
#pragma unroll
        for (int i = 0; i < S::kPer; ++i) {
            const float decay = kPrecise ? expf(__fmul_rn(dt, arow[i])) : fast_exp2(__fmul_rn(dt, arow[i] * kLog2e));
            const float bv = to_f32(bm[bbase + i]);
            const float drive = kPrecise ? __fmul_rn(__fmul_rn(dt, bv), uv) : __fmul_rn(du, bv);
            h[i] = __fmaf_rn(decay, h[i], drive);
            partial = __fmaf_rn(to_f32(cm[cbase + (p.c_full ? i : 0)]), h[i], partial);
        }
        if constexpr (S::kPer == 4) {
            *reinterpret_cast<float4*>(st) = make_float4(h[0], h[1], h[2], h[3]);
        } else {
#pragma unroll
            for (int i = 0; i < S::kPer; ++i) st[i] = h[i];
        }
    }
    // Sum the lane's partial C*h over its kSub consecutive threads (aligned groups within the warp).
#pragma unroll
    for (int off = S::kSub / 2; off > 0; off /= 2) partial += __shfl_xor_sync(0xffffffffu, partial, off, S::kSub);
    if (active && sub == 0) {
        T* y = static_cast<T*>(p.y);
        const unsigned long long at = seq * p.channels + d;
        if (!live) {
            y[at] = from_f32<T>(0.0f);
            return;
        }
        float out = partial;
        if (p.d) out = __fmaf_rn(p.d[d], uv, out);
        if (p.z) out = __fmul_rn(out, kPrecise ? to_f32(static_cast<const T*>(p.z)[at]) /
                                                    (1.0f + expf(-to_f32(static_cast<const T*>(p.z)[at])))
                                              : silu(to_f32(static_cast<const T*>(p.z)[at])));
        y[at] = from_f32<T>(out);
    }
}

#ifndef SACC_STEP_LANES
#define SACC_STEP_LANES 128
#endif
constexpr int kLanes = SACC_STEP_LANES; // threads (= lanes) per CTA of the 16-bit N = 16 path

template <typename T>
__device__ __forceinline__ void unpack8(uint4 v, float* f) {
    const std::uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t;
        if constexpr (std::is_same_v<T, __half>) t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        else t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// 16-bit activations, N = 16 (the per-frame tracker step): one thread per
// (sequence, channel) lane holding all 16 states, so that the per-lane work
// (index math, softplus, u / delta / z loads, the gated output) is paid once
// per lane rather than once per four states; issue slots, not HBM, bound the
// four-threads-per-lane layout at this size.  The lane's 64-byte state row and
// A row load as four 16-byte vectors each (state with streaming, evict-first
// loads and stores: a step touches it once), the sequence's B and C rows as
// two 16-byte vectors each (the same address across the CTA).  The update is
// step_kernel<T, 16, false>'s, operation for operation: four partial C*h sums
// over states 0-3, 4-7, 8-11, 12-15, combined as (p0 + p2) + (p1 + p3) like
// that kernel's width-4 butterfly, so both kernels give identical bits.
// blockIdx.x is the sequence and blockIdx.y the channel block: no division.
template <typename T>
__global__ void __launch_bounds__(kLanes) step16_kernel(StepParams p) {
    pdl_wait();
    constexpr int N = 16;
    const unsigned d = blockIdx.y * kLanes + threadIdx.x;
    const unsigned long long seq = blockIdx.x;
    if (d >= p.channels) return;
    const unsigned long long at = seq * p.channels + d;
    T* y = static_cast<T*>(p.y);
    const long long slot = p.slot ? static_cast<long long>(p.slot[seq]) : static_cast<long long>(seq);
    if (slot < 0 || slot >= static_cast<long long>(p.slots)) {
        y[at] = from_f32<T>(0.0f);
        return;
    }
    const unsigned g = p.groups == 1 ? 0u : d / static_cast<unsigned>(p.per_group);
    const unsigned long long bg = seq * p.groups + g;
    float4* st = reinterpret_cast<float4*>(p.state + (static_cast<unsigned long long>(slot) * p.channels + d) * N);
    const float4* ar = reinterpret_cast<const float4*>(p.a + (p.a_shared ? 0u : d * N));
    float h[N], a[N], b[N], c[N];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 v = __ldcs(st + k);
        h[4 * k] = v.x; h[4 * k + 1] = v.y; h[4 * k + 2] = v.z; h[4 * k + 3] = v.w;
        const float4 w = __ldg(ar + k);
        a[4 * k] = w.x; a[4 * k + 1] = w.y; a[4 * k + 2] = w.z; a[4 * k + 3] = w.w;
    }
    const uint4* brow = reinterpret_cast<const uint4*>(static_cast<const T*>(p.b) + bg * N);
    unpack8<T>(__ldg(brow), b);
    unpack8<T>(__ldg(brow + 1), b + 8);
    if (p.c_full) {
        const uint4* crow = reinterpret_cast<const uint4*>(static_cast<const T*>(p.c) + bg * N);
        unpack8<T>(__ldg(crow), c);
        unpack8<T>(__ldg(crow + 1), c + 8);
    } else {
        const float c0 = to_f32(static_cast<const T*>(p.c)[bg]);
#pragma unroll
        for (int n = 0; n < N; ++n) c[n] = c0;
    }
    const float uv = to_f32(static_cast<const T*>(p.u)[at]);
    const float x = __fadd_rn(to_f32(static_cast<const T*>(p.delta)[at]), p.bias ? p.bias[d] : 0.0f);
    const float zv = p.z ? to_f32(static_cast<const T*>(p.z)[at]) : 0.0f;
    const float dv = p.d ? p.d[d] : 0.0f;

    const float dt = p.softplus ? softplus_poly(x) : x;
    const float du = __fmul_rn(dt, uv);
    float part[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        part[q] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = 4 * q + i;
            const float decay = fast_exp2(__fmul_rn(dt, a[n] * kLog2e));
            h[n] = __fmaf_rn(decay, h[n], __fmul_rn(du, b[n]));
            part[q] = __fmaf_rn(c[n], h[n], part[q]);
        }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) __stcs(st + k, make_float4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]));
    float out = __fadd_rn(__fadd_rn(part[0], part[2]), __fadd_rn(part[1], part[3]));
    if (p.d) out = __fmaf_rn(dv, uv, out);
    if (p.z) out = __fmul_rn(out, silu(zv));
    y[at] = from_f32<T>(out);
}

template <typename T, int N>
const void* pick_prec(bool precise) {
    return precise ? reinterpret_cast<const void*>(step_kernel<T, N, true>)
                   : reinterpret_cast<const void*>(step_kernel<T, N, false>);
}

template <typename T>
const void* pick_n(unsigned n, bool precise) {
    switch (n) {
    case 1: return pick_prec<T, 1>(precise);
    case 2: return pick_prec<T, 2>(precise);
    case 4: return pick_prec<T, 4>(precise);
    case 8: return pick_prec<T, 8>(precise);
    case 16: return pick_prec<T, 16>(precise);
    default: return pick_prec<T, 32>(precise);
    }
}

const void* pick_step(int dtype, unsigned n) {
    if (dtype == SACC_DTYPE_BF16) return pick_n<__nv_bfloat16>(n, false);
    if (dtype == SACC_DTYPE_F16) return pick_n<__half>(n, false);
    return pick_n<float>(n, true);
}

unsigned sub_threads(unsigned n) { return n >= 4 ? n / 4 : 1; }

// ------------------------------------------------ TMA-pipelined 16-bit N = 16

#ifndef SACC_STEP_STAGES
#define SACC_STEP_STAGES 4
#endif
constexpr int kPipeLanes = 256;                // channels per unit (one thread each)
constexpr int kPipeStages = SACC_STEP_STAGES;  // units in flight per CTA
constexpr int kPipeMaxGroups = 8;

// One unit = one sequence x 256 channels: the state tile (256 rows of 16 FP32,
// written by TMA with the 64-byte swizzle), u / delta / z, and the sequence's
// B and C rows for every group.
template <typename T>
struct alignas(1024) PipeStage {
    float state[kPipeLanes * 16];
    alignas(16) T u[kPipeLanes];
    alignas(16) T dl[kPipeLanes];
    alignas(16) T z[kPipeLanes];
    alignas(16) T b[kPipeMaxGroups * 16];
    alignas(16) T c[kPipeMaxGroups * 16];
};

template <typename T>
struct PipeSmem {
    PipeStage<T> stage[kPipeStages];
    alignas(8) std::uint64_t full[kPipeStages];
};

template <typename T>
constexpr size_t pipe_smem_bytes() {
    return sizeof(PipeSmem<T>) + 1024; // + alignment slack for the swizzle atoms
}

// 16-byte chunk k of row r of a tile written with the 64-byte swizzle (rows of
// 64 bytes): chunk bits 4-5 of the offset are XORed with bits 7-8.  Reading a
// row's four chunks this way is bank-conflict free across each quarter warp.
__device__ __forceinline__ float4* swizzled_chunk(float* tile, int r, int k) {
    return reinterpret_cast<float4*>(tile + r * 16 + ((k ^ ((r >> 1) & 3)) << 2));
}

template <typename T>
__device__ __forceinline__ void pipe_issue(PipeSmem<T>& sm, int s, const CUtensorMap* tm_state, const StepParams& p,
                                           unsigned long long seq, unsigned c0, unsigned nch) {
    std::uint64_t* bar = &sm.full[s];
    PipeStage<T>& st = sm.stage[s];
    const long long slot = p.slot ? static_cast<long long>(p.slot[seq]) : static_cast<long long>(seq);
    if (slot < 0 || slot >= static_cast<long long>(p.slots)) {
        mbar_arrive_plain(bar); // skipped sequence: nothing to load
        return;
    }
    const std::uint32_t act = nch * static_cast<std::uint32_t>(sizeof(T));
    const std::uint32_t bc = static_cast<std::uint32_t>(p.groups * 16 * sizeof(T));
    mbar_arrive_expect_tx(bar, static_cast<std::uint32_t>(sizeof(st.state)) + act * (p.z ? 3u : 2u) + 2u * bc);
    tma_load_3d(st.state, tm_state, bar, 0, static_cast<int>(c0), static_cast<int>(slot));
    const unsigned long long at = seq * p.channels + c0;
    bulk_load(st.u, static_cast<const T*>(p.u) + at, act, bar);
    bulk_load(st.dl, static_cast<const T*>(p.delta) + at, act, bar);
    if (p.z) bulk_load(st.z, static_cast<const T*>(p.z) + at, act, bar);
    bulk_load(st.b, static_cast<const T*>(p.b) + seq * p.groups * 16, bc, bar);
    bulk_load(st.c, static_cast<const T*>(p.c) + seq * p.groups * 16, bc, bar);
}

// The step16 update with its operands staged through shared memory: each
// persistent CTA owns one 256-channel block (blockIdx.y) and walks the
// sequences blockIdx.x, blockIdx.x + gridDim.x, ...; thread 0 keeps
// kPipeStages units in flight (TMA tile load of the state, bulk copies of the
// activations and B / C) and writes each updated state tile back with a TMA
// store, so HBM sees long streams of 16 KB tiles instead of one short burst
// per thread.  Per lane the arithmetic is step16_kernel's, operation for
// operation, so the two paths give identical bits.  Every wait is bounded: a
// wait that runs out sets g_step_fault and the CTA leaves.
template <typename T>
__global__ void __launch_bounds__(kPipeLanes) step16_pipe_kernel(const __grid_constant__ CUtensorMap tm_state, StepParams p) {
    pdl_wait();
    constexpr int N = 16;
    extern __shared__ unsigned char smem_raw[];
    auto& sm = shared_window<PipeSmem<T>>(smem_raw);
    const int tid = threadIdx.x;
    const unsigned c0 = blockIdx.y * kPipeLanes;
    const unsigned nch = static_cast<unsigned>(p.channels - c0 < kPipeLanes ? p.channels - c0 : kPipeLanes);
    const unsigned d = c0 + tid;
    const bool lane_ok = tid < static_cast<int>(nch);
    const unsigned long long first = blockIdx.x, step = gridDim.x;

    if (tid == 0) {
        prefetch_tensor_map(&tm_state);
        for (int s = 0; s < kPipeStages; ++s) mbar_init(&sm.full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < kPipeStages; ++s)
            if (first + s * step < p.nseq) pipe_issue<T>(sm, s, &tm_state, p, first + s * step, c0, nch);

    float a[N];
    const float* arow = p.a + (p.a_shared ? 0u : (lane_ok ? d : 0u) * N);
#pragma unroll
    for (int n = 0; n < N; ++n) a[n] = arow[n] * kLog2e;
    const float bias = lane_ok && p.bias ? p.bias[d] : 0.0f;
    const float dv = lane_ok && p.d ? p.d[d] : 0.0f;
    const unsigned g = p.groups == 1 ? 0u : (lane_ok ? d : 0u) / static_cast<unsigned>(p.per_group);
    T* y = static_cast<T*>(p.y);

    bool fault = false;
    int i = 0;
    for (unsigned long long seq = first; seq < p.nseq; seq += step, ++i) {
        const int s = i % kPipeStages;
        const bool ok = mbar_wait_bounded(&sm.full[s], static_cast<std::uint32_t>((i / kPipeStages) & 1));
        if (!__syncthreads_and(ok)) {
            fault = true;
            break;
        }
        const long long slot = p.slot ? static_cast<long long>(p.slot[seq]) : static_cast<long long>(seq);
        const bool live = slot >= 0 && slot < static_cast<long long>(p.slots);
        PipeStage<T>& st = sm.stage[s];
        if (lane_ok) {
            const unsigned long long at = seq * p.channels + d;
            if (!live) {
                y[at] = from_f32<T>(0.0f);
            } else {
                float h[N], b[N], c[N];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 v = *swizzled_chunk(st.state, tid, k);
                    h[4 * k] = v.x; h[4 * k + 1] = v.y; h[4 * k + 2] = v.z; h[4 * k + 3] = v.w;
                }
                const uint4* bq = reinterpret_cast<const uint4*>(st.b + g * N);
                const uint4* cq = reinterpret_cast<const uint4*>(st.c + g * N);
                unpack8<T>(bq[0], b);
                unpack8<T>(bq[1], b + 8);
                unpack8<T>(cq[0], c);
                unpack8<T>(cq[1], c + 8);
                const float uv = to_f32(st.u[tid]);
                const float x = __fadd_rn(to_f32(st.dl[tid]), bias);
                const float dt = p.softplus ? softplus_poly(x) : x;
                const float du = __fmul_rn(dt, uv);
                float part[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    part[q] = 0.0f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int n = 4 * q + j;
                        const float decay = fast_exp2(__fmul_rn(dt, a[n]));
                        h[n] = __fmaf_rn(decay, h[n], __fmul_rn(du, b[n]));
                        part[q] = __fmaf_rn(c[n], h[n], part[q]);
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    *swizzled_chunk(st.state, tid, k) = make_float4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]);
                float out = __fadd_rn(__fadd_rn(part[0], part[2]), __fadd_rn(part[1], part[3]));
                if (p.d) out = __fmaf_rn(dv, uv, out);
                if (p.z) out = __fmul_rn(out, silu(to_f32(st.z[tid])));
                y[at] = from_f32<T>(out);
            }
        }
        fence_async_shared();
        __syncthreads();
        if (tid == 0) {
            if (live) tma_store_3d(&tm_state, st.state, 0, static_cast<int>(c0), static_cast<int>(slot));
            bulk_commit();
            // The previous unit's store has finished reading its stage: refill
            // that stage with the unit kPipeStages - 1 ahead of the next one.
            bulk_wait_read<1>();
            if (i >= 1) {
                const unsigned long long next = seq + (kPipeStages - 1) * step;
                if (next < p.nseq) pipe_issue<T>(sm, (i - 1) % kPipeStages, &tm_state, p, next, c0, nch);
            }
        }
    }
    if (tid == 0) {
        if (fault) {
            atomicOr(&g_step_fault, 1u);
            // Give loads still in flight a bounded chance to land before the
            // CTA's shared memory is released.
            for (int s = 0; s < kPipeStages; ++s) (void)mbar_wait_bounded(&sm.full[s], 0u, 1u << 16);
        }
        bulk_wait<0>();
    }
}

PFN_cuTensorMapEncodeTiled_v12000 step_encoder() {
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

// State table (slots, channels, 16) FP32 as a 3D map {16, channels, slots}
// with a {16, 256, 1} box and the 64-byte swizzle: rows past `channels` are
// zero-filled on load and skipped on store.
bool state_map(CUtensorMap* map, float* state, unsigned long long channels, unsigned long long slots) {
    auto fn = step_encoder();
    if (!fn) return false;
    const cuuint64_t dims[3] = {16, channels, slots};
    const cuuint64_t strides[2] = {16 * sizeof(float), channels * 16 * sizeof(float)};
    const cuuint32_t box[3] = {16, kPipeLanes, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, state, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
cudaError_t prepare_pipe() {
    static std::atomic<int> done[64];
    return once_per_device(done, [] {
        const void* fn = reinterpret_cast<const void*>(step16_pipe_kernel<T>);
        const cudaError_t e =
            cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pipe_smem_bytes<T>()));
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    });
}

// The pipelined path: 16-bit, N = 16, full-width C, at most 8 groups,
// channels a multiple of 8 (16-byte bulk copies), 16-byte aligned u / delta /
// z / B / C / state, and enough sequences to fill the machine.
bool pipe_eligible(const SaccScanStepArgs& a) {
    auto al = [](const void* ptr) { return reinterpret_cast<std::uintptr_t>(ptr) % 16 == 0; };
    return (a.dtype == SACC_DTYPE_BF16 || a.dtype == SACC_DTYPE_F16) && a.state == 16 && a.c_width == 16 &&
           a.groups <= kPipeMaxGroups && a.channels % 8 == 0 && a.channels / kPipeLanes < 65535 && a.nseq >= 256 &&
           a.slots < 0x7fffffffull && a.channels < 0x7fffffffull && al(a.u) && al(a.delta) && (a.z == nullptr || al(a.z)) &&
           al(a.b) && al(a.c) && al(a.state_io);
}

// The 16-bit N = 16 path needs 16-byte aligned A, B and (full) C rows (the
// state rows are 16-byte aligned on every path) and channel blocks within
// gridDim.y; the sequence index rides on gridDim.x.
bool step16_eligible(const SaccScanStepArgs& a) {
    auto al = [](const void* ptr, std::uintptr_t n) { return reinterpret_cast<std::uintptr_t>(ptr) % n == 0; };
    return (a.dtype == SACC_DTYPE_BF16 || a.dtype == SACC_DTYPE_F16) && a.state == 16 && al(a.b, 16) &&
           (a.c_width == 1 || al(a.c, 16)) && al(a.a, 16) && (a.channels + kLanes - 1) / kLanes <= 65535ull &&
           a.nseq <= 0x7fffffffull;
}

} // namespace

cudaError_t launch_scan_step(const SaccScanStepArgs& a, cudaStream_t stream) {
    StepParams p{};
    p.u = a.u; p.delta = a.delta; p.z = a.z; p.b = a.b; p.c = a.c;
    p.a = a.a; p.d = a.d; p.bias = a.delta_bias; p.state = a.state_io; p.slot = a.slot; p.y = a.y;
    p.nseq = a.nseq; p.channels = a.channels; p.groups = a.groups; p.per_group = a.channels / a.groups;
    p.slots = a.slot ? a.slots : a.nseq;
    p.a_shared = a.a_rows == 1; p.c_full = a.c_width != 1; p.softplus = a.delta_softplus != 0;
    const unsigned long long threads = a.nseq * a.channels * sub_threads(static_cast<unsigned>(a.state));
    void* args[] = {&p};
    if (pipe_eligible(a)) {
        CUtensorMap tm;
        if (!state_map(&tm, a.state_io, a.channels, p.slots)) return cudaErrorInvalidValue;
        const bool bf = a.dtype == SACC_DTYPE_BF16;
        const cudaError_t e = bf ? prepare_pipe<__nv_bfloat16>() : prepare_pipe<__half>();
        if (e != cudaSuccess) return e;
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const unsigned cblocks = static_cast<unsigned>((a.channels + kPipeLanes - 1) / kPipeLanes);
        unsigned long long gx = (2ull * sms + cblocks - 1) / cblocks; // two CTAs per SM
        if (gx > a.nseq) gx = a.nseq;
        void* pargs[] = {&tm, &p};
        const void* fn = bf ? reinterpret_cast<const void*>(step16_pipe_kernel<__nv_bfloat16>)
                            : reinterpret_cast<const void*>(step16_pipe_kernel<__half>);
        return launch_pdl(fn, dim3(static_cast<unsigned>(gx), cblocks), dim3(kPipeLanes),
                          bf ? pipe_smem_bytes<__nv_bfloat16>() : pipe_smem_bytes<__half>(), stream, pargs);
    }
    if (step16_eligible(a)) {
        if (threads == 0) return cudaSuccess;
        const dim3 grid(static_cast<unsigned>(a.nseq), static_cast<unsigned>((a.channels + kLanes - 1) / kLanes));
        const void* fn = a.dtype == SACC_DTYPE_BF16 ? reinterpret_cast<const void*>(step16_kernel<__nv_bfloat16>)
                                                    : reinterpret_cast<const void*>(step16_kernel<__half>);
        return launch_pdl(fn, grid, dim3(kLanes), 0, stream, args);
    }
    const unsigned long long blocks = (threads + kThreads - 1) / kThreads;
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    return launch_pdl(pick_step(a.dtype, static_cast<unsigned>(a.state)), dim3(static_cast<unsigned>(blocks)), dim3(kThreads), 0,
                      stream, args);
}

cudaError_t read_step_fault(unsigned* out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_step_fault, sizeof(unsigned));
    if (e != cudaSuccess || !clear) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_step_fault, &zero, sizeof(unsigned));
}

cudaError_t load_scan_step_kernels(std::string& report) {
    if (cudaError_t e = prepare_pipe<__half>(); e != cudaSuccess) return e;
    if (cudaError_t e = prepare_pipe<__nv_bfloat16>(); e != cudaSuccess) return e;
    int count = 0;
    for (int dtype : {SACC_DTYPE_F32, SACC_DTYPE_BF16, SACC_DTYPE_F16})
        for (unsigned n : {1u, 2u, 4u, 8u, 16u, 32u}) {
            cudaFuncAttributes attr{};
            const cudaError_t e = cudaFuncGetAttributes(&attr, pick_step(dtype, n));
            if (e != cudaSuccess) return e;
            ++count;
            if (n == 16 && dtype == SACC_DTYPE_F16)
                report += "kernel=scan_step_n16_f16 registers=" + std::to_string(attr.numRegs) + "\n";
        }
    for (const void* fn : {reinterpret_cast<const void*>(step16_kernel<__nv_bfloat16>),
                           reinterpret_cast<const void*>(step16_kernel<__half>),
                           reinterpret_cast<const void*>(step16_pipe_kernel<__nv_bfloat16>),
                           reinterpret_cast<const void*>(step16_pipe_kernel<__half>)}) {
        cudaFuncAttributes attr{};
        const cudaError_t e = cudaFuncGetAttributes(&attr, fn);
        if (e != cudaSuccess) return e;
        ++count;
    }
    report += "kernels_loaded=scan_step x" + std::to_string(count) + "\n";
    return cudaSuccess;
}

} // namespace sacc
