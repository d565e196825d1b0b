// scan_step.cu -- one L = 1 selective-scan update of carried per-track state
// (a tracker's per-frame step).  No counterpart in the
// reference, whose operator has no carried state (docs/SCAN_CONTRACT.md:60);
// the recurrence is the reference's (src/selective_scan.cpp:152-170) applied
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

#include "internal.h"
#include "scan_common.cuh"

namespace sacc {
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
        const float dt = p.softplus ? (kPrecise ? softplus_precise(x) : softplus_fast(x)) : x;
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

} // namespace

cudaError_t launch_scan_step(const SaccScanStepArgs& a, cudaStream_t stream) {
    StepParams p{};
    p.u = a.u; p.delta = a.delta; p.z = a.z; p.b = a.b; p.c = a.c;
    p.a = a.a; p.d = a.d; p.bias = a.delta_bias; p.state = a.state_io; p.slot = a.slot; p.y = a.y;
    p.nseq = a.nseq; p.channels = a.channels; p.groups = a.groups; p.per_group = a.channels / a.groups;
    p.slots = a.slot ? a.slots : a.nseq;
    p.a_shared = a.a_rows == 1; p.c_full = a.c_width != 1; p.softplus = a.delta_softplus != 0;
    const unsigned long long threads = a.nseq * a.channels * sub_threads(static_cast<unsigned>(a.state));
    const unsigned long long blocks = (threads + kThreads - 1) / kThreads;
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    void* args[] = {&p};
    return cudaLaunchKernel(pick_step(a.dtype, static_cast<unsigned>(a.state)), dim3(static_cast<unsigned>(blocks)),
                            dim3(kThreads), args, 0, stream);
}

cudaError_t load_scan_step_kernels(std::string& report) {
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
    report += "kernels_loaded=scan_step x" + std::to_string(count) + "\n";
    return cudaSuccess;
}

} // namespace sacc
