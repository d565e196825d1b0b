// scan_ex.cu -- extended selective scan: bf16/fp16/fp32 activations, FP32
// state, (B,L,D) or (B,D,L) layouts, fused dt bias + softplus, D skip and
// SiLU(z) gate, optional initial / final state and packed varlen sequences.
//
// This translation unit holds the general kernel: one thread per
// (sequence, channel) lane with the N states in registers, tokens walked in
// order.  It covers every argument combination; the bulk kernel in
// scan_bulk.cu takes over the high-throughput configurations.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "internal.h"
#include "scan_common.cuh"

namespace sacc {
namespace {

constexpr int kThreads = 128;

struct ExParams {
    const void *u, *delta, *b, *c, *z;
    const float *a, *d, *bias, *h0;
    float* h_final;
    const int32_t* cu;
    void* y;
    unsigned long long batch, length, channels, groups, per_group, lanes, nseq;
    int a_shared, c_full, softplus;
};

template <typename T, int N, bool kBDL, bool kPrecise>
__global__ void __launch_bounds__(kThreads) scan_ex_kernel(ExParams p) {
    const unsigned long long lane = static_cast<unsigned long long>(blockIdx.x) * kThreads + threadIdx.x;
    if (lane >= p.lanes) return;
    const unsigned long long D = p.channels, L = p.length, G = p.groups;
    const unsigned long long seq = lane / D, d = lane % D, g = d / p.per_group;
    const unsigned long long bb = p.cu ? 0 : seq;
    // cu_seqlens entries clamped to [0, L] (and t1 >= t0) so no access leaves the tensors.
    auto clamp_tok = [L](long long v) { return v < 0 ? 0ull : (static_cast<unsigned long long>(v) > L ? L : static_cast<unsigned long long>(v)); };
    const unsigned long long t0 = p.cu ? clamp_tok(p.cu[seq]) : 0;
    const unsigned long long t1r = p.cu ? clamp_tok(p.cu[seq + 1]) : L;
    const unsigned long long t1 = t1r < t0 ? t0 : t1r;
    const T* u = static_cast<const T*>(p.u);
    const T* dl = static_cast<const T*>(p.delta);
    const T* z = static_cast<const T*>(p.z);
    const T* bm = static_cast<const T*>(p.b);
    const T* cm = static_cast<const T*>(p.c);
    T* y = static_cast<T*>(p.y);

    float a[N], h[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const float av = p.a[(p.a_shared ? 0 : d * N) + n];
        a[n] = kPrecise ? av : av * kLog2e;
        h[n] = p.h0 ? p.h0[lane * N + n] : 0.0f;
    }
    const float dskip = p.d ? p.d[d] : 0.0f;
    const float bias = p.bias ? p.bias[d] : 0.0f;
    const unsigned long long cw = p.c_full ? N : 1;
    for (unsigned long long t = t0; t < t1; ++t) {
        unsigned long long at, b0, bs, c0, cs;
        if (kBDL) {
            at = (bb * D + d) * L + t;
            b0 = (bb * G + g) * N * L + t;
            bs = L;
            c0 = (bb * G + g) * cw * L + t;
            cs = L;
        } else {
            at = (bb * L + t) * D + d;
            b0 = ((bb * L + t) * G + g) * N;
            bs = 1;
            c0 = ((bb * L + t) * G + g) * cw;
            cs = 1;
        }
        const float uv = to_f32(u[at]);
        float x = __fadd_rn(to_f32(dl[at]), bias);
        const float dt = p.softplus ? (kPrecise ? softplus_precise(x) : softplus_fast(x)) : x;
        const float du = __fmul_rn(dt, uv);
        float acc = 0.0f;
#pragma unroll
        for (int n = 0; n < N; ++n) {
            const float decay = kPrecise ? expf(__fmul_rn(dt, a[n])) : fast_exp2(__fmul_rn(dt, a[n]));
            const float bv = to_f32(bm[b0 + n * bs]);
            const float drive = kPrecise ? __fmul_rn(__fmul_rn(dt, bv), uv) : __fmul_rn(du, bv);
            h[n] = __fmaf_rn(decay, h[n], drive);
            const float cv = to_f32(cm[c0 + (p.c_full ? n : 0) * cs]);
            acc = __fmaf_rn(cv, h[n], acc);
        }
        if (p.d) acc = __fmaf_rn(dskip, uv, acc);
        if (p.z) acc = __fmul_rn(acc, silu(to_f32(z[at])));
        y[at] = from_f32<T>(acc);
    }
    if (p.h_final) {
#pragma unroll
        for (int n = 0; n < N; ++n) p.h_final[lane * N + n] = h[n];
    }
}

template <typename T, int N>
const void* pick_layout(int layout, bool precise) {
    if (layout == SACC_LAYOUT_BDL)
        return precise ? reinterpret_cast<const void*>(scan_ex_kernel<T, N, true, true>)
                       : reinterpret_cast<const void*>(scan_ex_kernel<T, N, true, false>);
    return precise ? reinterpret_cast<const void*>(scan_ex_kernel<T, N, false, true>)
                   : reinterpret_cast<const void*>(scan_ex_kernel<T, N, false, false>);
}

template <typename T>
const void* pick_state(unsigned state, int layout, bool precise) {
    switch (state) {
    case 1: return pick_layout<T, 1>(layout, precise);
    case 2: return pick_layout<T, 2>(layout, precise);
    case 4: return pick_layout<T, 4>(layout, precise);
    case 8: return pick_layout<T, 8>(layout, precise);
    case 16: return pick_layout<T, 16>(layout, precise);
    default: return pick_layout<T, 32>(layout, precise);
    }
}

const void* pick_general(const SaccScanExArgs& a) {
    const bool precise = a.dtype == SACC_DTYPE_F32;
    const unsigned n = static_cast<unsigned>(a.state);
    if (a.dtype == SACC_DTYPE_BF16) return pick_state<__nv_bfloat16>(n, a.layout, precise);
    if (a.dtype == SACC_DTYPE_F16) return pick_state<__half>(n, a.layout, precise);
    return pick_state<float>(n, a.layout, precise);
}

} // namespace

cudaError_t launch_scan_general(const SaccScanExArgs& a, cudaStream_t stream) {
    ExParams p{};
    p.u = a.u; p.delta = a.delta; p.b = a.b; p.c = a.c; p.z = a.z;
    p.a = a.a; p.d = a.d; p.bias = a.delta_bias; p.h0 = a.h0; p.h_final = a.h_final; p.cu = a.cu_seqlens; p.y = a.y;
    p.batch = a.batch; p.length = a.length; p.channels = a.channels; p.groups = a.groups;
    p.per_group = a.channels / a.groups;
    p.nseq = a.cu_seqlens ? static_cast<unsigned long long>(a.nseq) : a.batch;
    p.lanes = p.nseq * a.channels;
    p.a_shared = a.a_rows == 1;
    p.c_full = a.c_width != 1;
    p.softplus = a.delta_softplus != 0;
    const unsigned long long blocks = (p.lanes + kThreads - 1) / kThreads;
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    void* args[] = {&p};
    return cudaLaunchKernel(pick_general(a), dim3(static_cast<unsigned>(blocks)), dim3(kThreads), args, 0, stream);
}

cudaError_t load_scan_general_kernels(std::string& report) {
    int count = 0;
    for (int dtype : {SACC_DTYPE_F32, SACC_DTYPE_BF16, SACC_DTYPE_F16})
        for (int layout : {SACC_LAYOUT_BLD, SACC_LAYOUT_BDL})
            for (unsigned n : {1u, 2u, 4u, 8u, 16u, 32u}) {
                SaccScanExArgs a{};
                a.dtype = dtype; a.layout = layout; a.state = n;
                cudaFuncAttributes attr{};
                const cudaError_t e = cudaFuncGetAttributes(&attr, pick_general(a));
                if (e != cudaSuccess) return e;
                ++count;
                if (n == 16 && layout == SACC_LAYOUT_BDL)
                    report += "kernel=scan_ex_general_n16_bdl_dtype" + std::to_string(dtype) + " registers=" +
                              std::to_string(attr.numRegs) + " local_bytes=" + std::to_string(attr.localSizeBytes) + "\n";
            }
    report += "kernels_loaded=scan_ex_general x" + std::to_string(count) + "\n";
    return cudaSuccess;
}

} // namespace sacc

namespace sacc {

cudaError_t launch_scan_ex(const SaccScanExArgs& a, int sm_count, cudaStream_t stream) {
    (void)sm_count;
    if (bulk_eligible(a)) return launch_scan_bulk(a, stream);
    return launch_scan_general(a, stream);
}

cudaError_t load_scan_ex_kernels(std::string& report) {
    const cudaError_t e = load_scan_general_kernels(report);
    if (e != cudaSuccess) return e;
    return load_scan_bulk_kernels(report);
}

} // namespace sacc
