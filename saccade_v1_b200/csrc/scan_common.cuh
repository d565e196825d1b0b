// scan_common.cuh -- device helpers shared by the extended scan kernels.
#pragma once

#include <cstddef>
#include <utility>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace sacc {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel of the stream still runs.
// pdl_launch_dependents lets the next kernel start its own set-up once every
// block of this grid has called it (or exited); pdl_wait returns when the
// previous grid has completed and its writes are visible.  Every kernel calls
// both before it reads anything another kernel wrote.  Without the launch
// attribute both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Typed form of launch_pdl (internal.h) for kernels launched with their
// arguments: programmatic stream serialization on this launch.
template <typename... P, typename... A>
inline cudaError_t launch_pdl_k(void (*kernel)(P...), dim3 grid, dim3 block, std::size_t smem, cudaStream_t stream,
                                A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float fast_exp2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// softplus with the reference's threshold (x > 20 passes through,
// src/selective_scan.cpp:59), FP32 library functions.
__device__ __forceinline__ float softplus_precise(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// Same threshold; e^x from the special-function unit, log1p from the library
// (log1p keeps full relative precision where 1 + e^x rounds to 1).
__device__ __forceinline__ float softplus_fast(float x) {
    return x > 20.0f ? x : log1pf(fast_exp2(__fmul_rn(x, kLog2e)));
}

// softplus(x) = max(x, 0) + log1p(e^-|x|) with log1p(e) = e * P(e) on
// e in (0, 1]: P of degree 5, the minimax fit of the relative error
// (gen_softplus_poly.py in this directory: Remez exchange in binary64,
// coefficients rounded to FP32; the FP32 Horner evaluation is within 8.5e-6
// relative of log1p(e), a thousandth of the 16-bit paths' 1e-2 tolerance;
// degree 7 reaches 3.3e-7 for two more FMAs, 1.7 % of config 2's time): one
// special-function exp and six FMAs, no library call.  x > 20 passes through
// as in the reference (src/selective_scan.cpp:59).
__device__ __forceinline__ float softplus_poly(float x) {
    const float e = fast_exp2(-fabsf(x) * kLog2e);
    float q = fmaf(-2.38691512e-02f, e, 1.01222284e-01f);
    q = fmaf(q, e, -2.10048690e-01f);
    q = fmaf(q, e, 3.25206667e-01f);
    q = fmaf(q, e, -4.99361366e-01f);
    q = fmaf(q, e, 9.99991596e-01f);
    const float r = fmaf(e, q, fmaxf(x, 0.0f));
    return x > 20.0f ? x : r;
}

// x * sigmoid(x) = x / (1 + e^-x); __fdividef returns 0 when e^-x overflows.
__device__ __forceinline__ float silu(float x) { return __fdividef(x, __fadd_rn(1.0f, fast_exp2(__fmul_rn(-x, kLog2e)))); }

} // namespace sacc
