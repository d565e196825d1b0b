// scan_f32.cu -- reference-ABI FP32 selective scan for sm_100a.
//
// Contract: reference cuda/selective_scan.cu:270-311 (selective_scan_cuda),
// arithmetic: cuda/selective_scan.cu:41-132.  Layouts (B,L,Dc) row-major FP32.
//
// B200 design (differs from the reference's one-thread-per-(b,d,n) kernel):
//  * one thread owns a (batch, channel) lane and keeps all N states of that
//    lane in registers, so per-token work (softplus, u/delta loads, D skip,
//    output store) is done once per lane instead of N times and the state sum
//    needs no shuffles; for N >= 8, four threads share a lane, N / 4 states
//    each (scan_f32_quad_kernel), for four times the warps per SM;
//  * the length axis is split into K chunks (K a power of two) when there are
//    too few lanes to fill 148 SMs.  Chunk k of a lane first runs the
//    recurrence from zero over its tokens (pass 1) and publishes
//    (product of decays, local state) per state in shared memory; every chunk
//    then folds its predecessors' carries into its true starting state and
//    reruns its tokens with outputs (pass 2).  All chunks of a lane live in one
//    CTA: no workspace, one kernel;
//  * one call is the reference's memset + check + scan + finalize (the
//    graph a captured call holds), with the scan overlapping the check: the
//    check kernel releases the scan at once (programmatic dependent launch),
//    the scan waits for the check grid only at its end, and finalize waits for
//    the scan, so it sees both grids' status bits.
//
// The same kernels serve FP16 activations (plugin SelectiveScan v3): u,
// delta, B and C are widened to FP32 as they are loaded and y is rounded to
// nearest FP16 as it is stored, so the outputs are the FP32 path's outputs on
// the widened inputs, rounded; an output at or beyond 65520 (which rounds to
// infinity in FP16) is reported as an output range failure.
//
// Per-token arithmetic keeps the reference's FP32 algorithm, so its running
// error bound (docs/SCAN_CUDA.md section 5 of the reference) applies: the plain
// FP32 products are used whenever they provably equal the reference's
// mantissa/exponent-scaled products (Delta, Delta*B and Delta*B*u normal), and
// the scaled form is evaluated otherwise.  With K = 1 the outputs are the
// reference algorithm's bits (same operations, same summation tree).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cfloat>
#include <climits>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <type_traits>

#include "internal.h"
#include "scan_common.cuh"

namespace sacc {
namespace {

constexpr int kThreads = 256;
constexpr unsigned kDecay = SACC_SCAN_DECAY_RANGE, kDrive = SACC_SCAN_DRIVE_RANGE, kState = SACC_SCAN_STATE_RANGE,
                   kTerm = SACC_SCAN_TERM_RANGE, kSkip = SACC_SCAN_SKIP_RANGE, kOutput = SACC_SCAN_OUTPUT_RANGE;

__device__ __forceinline__ bool finite32(float x) { return fabsf(x) <= FLT_MAX; } // false for NaN and +-inf

// Smallest magnitude that rounds to infinity in FP16 (the midpoint between
// 65504 and 2^16 rounds to the even 2^16).
constexpr float kHalfOverflow = 65520.0f;

template <typename T>
__device__ __forceinline__ float load_act(const T* p) {
    if constexpr (std::is_same_v<T, __half>) return __half2float(__ldg(p));
    else return __ldg(p);
}

template <typename T>
__device__ __forceinline__ void store_act(T* p, float v) {
    if constexpr (std::is_same_v<T, __half>) *p = __float2half_rn(v);
    else *p = v;
}

// value = m * 2^e with m in [0.5, 1) or m == 0 (frexpf / ldexpf are exact).
struct Scaled {
    float m;
    int e;
};
__device__ __forceinline__ Scaled split(float x) {
    int e = 0;
    const float m = frexpf(x, &e);
    return {m, e};
}

// softplus(x) with the reference's threshold (x > 20 passes through), kept as
// (m, e) so that a Delta below the FP32 normal range keeps full precision
// (reference cuda/selective_scan.cu:49-61).  For -1024 <= x < -80 the result is
// e^x (log1p(e^x) = e^x to 1e-35 relative there), formed as e^r * 2^k with the
// Cody-Waite reduction k = rint(x / ln2), r = (x - k ln2_hi) - k ln2_lo
// (ln2_hi = 0x3f317200 has 16 significant bits, so k * ln2_hi is exact).
__device__ Scaled softplus_scaled(float x) {
    if (x > 20.0f) return split(x);
    if (x >= -80.0f) return split(log1pf(expf(x)));
    if (x < -1024.0f) return {0.0f, 0};
    const float ln2_hi = __int_as_float(0x3f317200), ln2_lo = 1.42860677e-6f;
    const float k = rintf(__fmul_rn(x, 1.44269504f));
    const float r = __fmaf_rn(-k, ln2_lo, __fmaf_rn(-k, ln2_hi, x));
    Scaled s = split(expf(r));
    s.e += static_cast<int>(k);
    return s;
}

// Sum of N values with the association of an xor butterfly over N lanes
// (offset N/2 first), i.e. the reference's group_sum order; destroys v.
template <int N>
__device__ __forceinline__ float tree_sum(float (&v)[N]) {
#pragma unroll
    for (int w = N / 2; w > 0; w /= 2)
#pragma unroll
        for (int i = 0; i < w; ++i) v[i] = __fadd_rn(v[i], v[i + w]);
    return v[0];
}

struct Params {
    const void *u, *delta, *b, *c; // FP32 or FP16 (the kernel's T)
    const float *a, *d;
    void* y;
    unsigned long long length, channels, lanes;
    int a_shared, c_full, has_d, vec_b, vec_c;
    int chunks, lanes_per_cta;
    unsigned scan_blocks;
};

// N values of a row; `vec`: the row starts 16-byte (FP32) or 8-byte (FP16)
// aligned, four values per load.
template <typename T, int N>
__device__ __forceinline__ void load_row(const T* p, float (&out)[N], bool vec) {
    if constexpr (N % 4 == 0) {
        if (vec) {
#pragma unroll
            for (int i = 0; i < N; i += 4) {
                if constexpr (std::is_same_v<T, __half>) {
                    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p) + i / 4);
                    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
                    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
                    out[i] = lo.x; out[i + 1] = lo.y; out[i + 2] = hi.x; out[i + 3] = hi.y;
                } else {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i / 4);
                    out[i] = v.x; out[i + 1] = v.y; out[i + 2] = v.z; out[i + 3] = v.w;
                }
            }
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = load_act(p + i);
}

// Operands of one token of one lane.
// One token of a lane: u, raw delta, the B row and the C row (CW = N values,
// or one value broadcast over the states when C has width 1).
template <int N, int CW>
struct Token {
    float u, x;
    float b[N];
    float c[CW];
};

template <typename T, int N, int CW>
__device__ __forceinline__ void load_token(const Params& p, unsigned long long token, unsigned long long d, Token<N, CW>& k) {
    const unsigned long long at = token * p.channels + d;
    k.u = load_act(static_cast<const T*>(p.u) + at);
    k.x = load_act(static_cast<const T*>(p.delta) + at);
    load_row<T, N>(static_cast<const T*>(p.b) + token * N, k.b, p.vec_b);
    if constexpr (CW > 1) load_row<T, N>(static_cast<const T*>(p.c) + token * N, k.c, p.vec_c);
    else k.c[0] = load_act(static_cast<const T*>(p.c) + token);
}

// New states of one token; returns false when the plain FP32 products may
// differ from the reference's scaled ones (then the caller uses the scaled form).
// softplus as the plain FP32 path forms it (x > 20 passes through).
__device__ __forceinline__ float softplus_plain(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// states_fast with Delta = softplus_plain(k.x) already formed (dv).
template <int N, int CW>
__device__ __forceinline__ bool states_fast_dv(const float (&h)[N], const float (&a)[N], const Token<N, CW>& k, float dv,
                                               float (&hn)[N], float (&decay)[N], float (&drive)[N]) {
    if (!(k.x >= -80.0f)) return false;
    bool fast = true;
#pragma unroll
    for (int n = 0; n < N; ++n) {
        decay[n] = expf(__fmul_rn(dv, a[n]));
        const float db = __fmul_rn(dv, k.b[n]);
        drive[n] = __fmul_rn(db, k.u);
        fast = fast & (fabsf(db) >= 0x1p-126f) & (fabsf(drive[n]) >= 0x1p-126f) & (fabsf(drive[n]) <= FLT_MAX);
        hn[n] = __fmaf_rn(decay[n], h[n], drive[n]);
    }
    return fast;
}

template <int N, int CW>
__device__ __forceinline__ bool states_fast(const float (&h)[N], const float (&a)[N], const Token<N, CW>& k, float (&hn)[N],
                                            float (&decay)[N], float (&drive)[N]) {
    if (!(k.x >= -80.0f)) return false;
    const float dv = softplus_plain(k.x);
    bool fast = true;
#pragma unroll
    for (int n = 0; n < N; ++n) {
        decay[n] = expf(__fmul_rn(dv, a[n]));
        const float db = __fmul_rn(dv, k.b[n]);
        drive[n] = __fmul_rn(db, k.u);
        fast = fast & (fabsf(db) >= 0x1p-126f) & (fabsf(drive[n]) >= 0x1p-126f) & (fabsf(drive[n]) <= FLT_MAX);
        hn[n] = __fmaf_rn(decay[n], h[n], drive[n]);
    }
    return fast;
}

// The reference's scaled per-token state update (cuda/selective_scan.cu:100-103).
template <int N, int CW>
__device__ __forceinline__ void states_scaled(const float (&h)[N], const float (&a)[N], const Token<N, CW>& k, float (&hn)[N],
                                           float (&decay)[N], float (&drive)[N]) {
    const Scaled dl = softplus_scaled(k.x), su = split(k.u);
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const Scaled sb = split(k.b[n]);
        decay[n] = expf(ldexpf(__fmul_rn(dl.m, a[n]), dl.e));
        drive[n] = ldexpf(__fmul_rn(__fmul_rn(dl.m, sb.m), su.m), dl.e + sb.e + su.e);
        hn[n] = __fmaf_rn(decay[n], h[n], drive[n]);
    }
}

// Pass 1: state update without outputs, accumulating the decay product.
template <int N, int CW>
__device__ __forceinline__ void step_carry(float (&h)[N], float (&prod)[N], const float (&a)[N], const Token<N, CW>& k) {
    float hn[N], decay[N], drive[N];
    if (!states_fast<N, CW>(h, a, k, hn, decay, drive)) states_scaled<N, CW>(h, a, k, hn, decay, drive);
#pragma unroll
    for (int n = 0; n < N; ++n) {
        h[n] = hn[n];
        prod[n] = __fmul_rn(prod[n], decay[n]);
    }
}

// Pass 2: one token with output and the reference's failure order
// (cuda/selective_scan.cu:104-129).  Returns the failure bits (0 = ok).  With
// kHalfOut an output that FP16 cannot hold is an output range failure.
template <int N, int CW, bool kHalfOut>
__device__ __forceinline__ unsigned step_out(float (&h)[N], const float (&a)[N], const Token<N, CW>& k, bool has_d, float skip_d,
                                             float& y) {
    float hn[N], decay[N], drive[N];
    if (!states_fast<N, CW>(h, a, k, hn, decay, drive)) states_scaled<N, CW>(h, a, k, hn, decay, drive);
    unsigned fail = 0;
    float term[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        term[n] = __fmul_rn(k.c[CW > 1 ? n : 0], hn[n]);
        fail |= !finite32(decay[n]) ? kDecay : !finite32(drive[n]) ? kDrive : !finite32(hn[n]) ? kState
              : !finite32(term[n]) ? kTerm : 0u;
        h[n] = hn[n];
    }
    if (fail) return fail;
    float s[N];
#pragma unroll
    for (int n = 0; n < N; ++n) s[n] = term[n];
    const float sum = tree_sum<N>(s);
    const float skip = __fmul_rn(skip_d, k.u);
    if (has_d && !finite32(skip)) return kSkip;
    float out = has_d ? __fadd_rn(sum, skip) : sum;
    if (!finite32(out)) {
        // Every term is finite but a partial sum left the FP32 range: repeat
        // with exact power-of-two scaling (reference cuda/selective_scan.cu:116-122).
#pragma unroll
        for (int n = 0; n < N; ++n) s[n] = __fmul_rn(term[n], 0x1p-8f);
        const float scaled = tree_sum<N>(s);
        out = has_d ? __fadd_rn(scaled, __fmul_rn(skip, 0x1p-8f)) : scaled;
        if (fabsf(out) <= FLT_MAX * 0x1p-8f) out = __fmul_rn(out, 0x1p8f);
        else return kOutput;
    }
    if (kHalfOut && !(fabsf(out) < kHalfOverflow)) return kOutput;
    y = out;
    return 0;
}

// Exact NaN/Inf test over the listed tensors (reference cuda/selective_scan.cu:137-147).
__device__ void check_tensors(const CheckList& list, unsigned long long first, unsigned long long stride,
                              SaccScanStatus* status) {
    std::uint32_t found = 0;
    for (unsigned t = 0; t < list.size; ++t) {
        const CheckedTensor ct = list.tensor[t];
        if (ct.half) {
            // FP16: NaN or infinity iff the five exponent bits are all ones.
            const unsigned short* data = static_cast<const unsigned short*>(ct.data);
            unsigned long long i0 = 0;
            bool bad = false;
            if ((reinterpret_cast<std::uintptr_t>(data) & 15u) == 0) {
                const unsigned long long octs = ct.count / 8;
                const uint4* q = reinterpret_cast<const uint4*>(data);
                for (unsigned long long i = first; i < octs; i += stride) {
                    const uint4 v = __ldg(q + i);
                    const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        bad |= ((w[j] & 0x7C00u) == 0x7C00u) | ((w[j] & 0x7C000000u) == 0x7C000000u);
                }
                i0 = octs * 8;
            }
            for (unsigned long long i = i0 + first; i < ct.count; i += stride) bad |= (__ldg(data + i) & 0x7C00u) == 0x7C00u;
            if (bad) found |= ct.bit;
            continue;
        }
        const float* data = static_cast<const float*>(ct.data);
        unsigned long long i0 = 0;
        const bool aligned = (reinterpret_cast<std::uintptr_t>(data) & 15u) == 0;
        if (aligned) {
            const unsigned long long quads = ct.count / 4;
            const float4* q = reinterpret_cast<const float4*>(data);
            bool bad = false;
            for (unsigned long long i = first; i < quads; i += stride) {
                const float4 v = __ldg(q + i);
                bad |= !(finite32(v.x) & finite32(v.y) & finite32(v.z) & finite32(v.w));
            }
            if (bad) found |= ct.bit;
            i0 = quads * 4;
        }
        bool bad = false;
        for (unsigned long long i = i0 + first; i < ct.count; i += stride) bad |= !finite32(__ldg(data + i));
        if (bad) found |= ct.bit;
    }
    if (found) atomicOr(&status->flags, found);
}

template <typename T, int N, int CW>
__global__ void __launch_bounds__(kThreads) scan_f32_kernel(Params p, SaccScanStatus* status) {
    extern __shared__ float2 carry[]; // [chunk][lane in CTA][state]: (decay product, local state)
    __shared__ int chunk_failed[kThreads];
    const int K = p.chunks, LPC = p.lanes_per_cta;
    const int tid = threadIdx.x, li = tid % LPC, k = tid / LPC;
    const unsigned long long lane = static_cast<unsigned long long>(blockIdx.x) * LPC + li;
    const bool active = lane < p.lanes;
    const unsigned long long L = p.length, Dc = p.channels;
    const unsigned long long bb = active ? lane / Dc : 0, d = active ? lane % Dc : 0;
    const unsigned long long t0 = L * k / K, t1 = L * (k + 1) / K;

    float a[N];
#pragma unroll
    for (int n = 0; n < N; ++n) a[n] = active ? __ldg(p.a + (p.a_shared ? 0 : d * N) + n) : 0.0f;
    const float skip_d = (active && p.has_d) ? __ldg(p.d + d) : 0.0f;
    float h[N];
#pragma unroll
    for (int n = 0; n < N; ++n) h[n] = 0.0f;

    if (K > 1) {
        float prod[N];
#pragma unroll
        for (int n = 0; n < N; ++n) prod[n] = 1.0f;
        if (active && k < K - 1) {
            Token<N, CW> cur;
            if (t0 < t1) load_token<T, N, CW>(p, bb * L + t0, d, cur);
            for (unsigned long long t = t0; t < t1; ++t) {
                Token<N, CW> nxt;
                if (t + 1 < t1) load_token<T, N, CW>(p, bb * L + t + 1, d, nxt);
                step_carry<N, CW>(h, prod, a, cur);
                cur = nxt;
            }
        }
        float2* mine = carry + (static_cast<size_t>(k) * LPC + li) * N;
#pragma unroll
        for (int n = 0; n < N; ++n) mine[n] = make_float2(prod[n], h[n]);
        __syncthreads();
        // Fold the carries of chunks 0..k-1: H = prod_j * H + local_j.
#pragma unroll
        for (int n = 0; n < N; ++n) h[n] = 0.0f;
        for (int j = 0; j < k; ++j) {
            const float2* cj = carry + (static_cast<size_t>(j) * LPC + li) * N;
#pragma unroll
            for (int n = 0; n < N; ++n) {
                const float2 v = cj[n];
                h[n] = h[n] == 0.0f ? v.y : __fmaf_rn(v.x, h[n], v.y);
            }
        }
    }

    unsigned fail = 0;
    if (active && t0 < t1) {
        Token<N, CW> cur;
        load_token<T, N, CW>(p, bb * L + t0, d, cur);
        for (unsigned long long t = t0; t < t1; ++t) {
            Token<N, CW> nxt;
            if (t + 1 < t1) load_token<T, N, CW>(p, bb * L + t + 1, d, nxt);
            float y = 0.0f;
            fail = step_out<N, CW, std::is_same_v<T, __half>>(h, a, cur, p.has_d != 0, skip_d, y);
            if (fail) break;
            store_act(static_cast<T*>(p.y) + (bb * L + t) * Dc + d, y);
            cur = nxt;
        }
    }
    if (K > 1) {
        // A lane reports the failure of its earliest failing chunk only, as the
        // sequential recurrence stops at its first failure.
        chunk_failed[tid] = fail ? 1 : 0;
        __syncthreads();
        if (fail) {
            bool earlier = false;
            for (int j = 0; j < k; ++j) earlier |= chunk_failed[j * LPC + li] != 0;
            if (!earlier) atomicOr(&status->flags, fail);
        }
    } else if (fail) {
        atomicOr(&status->flags, fail);
    }
    // The check grid released this grid before it finished: one thread waits
    // for it here, so this grid completes only after the check has (finalize
    // waits for this grid and then reads both grids' status bits).
    if (blockIdx.x == 0 && threadIdx.x == 0) pdl_wait();
}

// N >= 8 with four threads per lane (scan_f32_quad_kernel): thread q of a
// lane owns states q, q + 4, ..., q + N - 4, so the reference's butterfly sum
// (offset N/2 first) runs its levels of offset 4 and more inside each thread
// (offset w pairs the thread's values j and j + w/4: tree_sum over them) and
// its last two as xor shuffles over the four threads (offsets 2, then 1): the
// same association, so the same bits.  A thread holds a quarter of the states
// and a CTA four times the warps.
constexpr int kQuad = 4;

template <typename T, int N, int CW>
__device__ __forceinline__ void load_token_quad(const Params& p, unsigned long long token, unsigned long long d, int q,
                                                Token<N / kQuad, (CW > 1 ? N / kQuad : 1)>& k) {
    constexpr int S = N / kQuad;
    const unsigned long long at = token * p.channels + d;
    k.u = load_act(static_cast<const T*>(p.u) + at);
    k.x = load_act(static_cast<const T*>(p.delta) + at);
    const T* b = static_cast<const T*>(p.b) + token * N + q;
#pragma unroll
    for (int j = 0; j < S; ++j) k.b[j] = load_act(b + 4 * j);
    if constexpr (CW > 1) {
        const T* c = static_cast<const T*>(p.c) + token * N + q;
#pragma unroll
        for (int j = 0; j < S; ++j) k.c[j] = load_act(c + 4 * j);
    } else {
        k.c[0] = load_act(static_cast<const T*>(p.c) + token);
    }
}

// The four lanes of the calling thread's group: the groups of a warp walk
// different chunks and lanes, so every shuffle names its own group only.
__device__ __forceinline__ unsigned quad_mask() { return 0xfu << (threadIdx.x & 28u); }

// The sum over all N states of one token in the reference's association:
// the in-thread levels (for N = 16: (q + (q + 8)) + ((q + 4) + (q + 12))),
// then the partner at xor 2 and at xor 1.  Every thread of the four gets the
// same bits (IEEE addition is commutative).
template <int S>
__device__ __forceinline__ float quad_sum(const float (&t)[S]) {
    const unsigned m = quad_mask();
    float w[S];
#pragma unroll
    for (int j = 0; j < S; ++j) w[j] = t[j];
    float v = tree_sum<S>(w);
    v = __fadd_rn(v, __shfl_xor_sync(m, v, 2));
    return __fadd_rn(v, __shfl_xor_sync(m, v, 1));
}

// step_out for a quarter of the states: the four threads' failure bits are
// combined (each state's first failure in the reference's order, OR-ed over
// the states as the reference's group does), so all four return together.
template <int N, int CW, bool kHalfOut>
__device__ __forceinline__ unsigned step_out_quad(float (&h)[N / kQuad], const float (&a)[N / kQuad],
                                                  const Token<N / kQuad, (CW > 1 ? N / kQuad : 1)>& k, float dv, bool has_d,
                                                  float skip_d, float& y) {
    constexpr int S = N / kQuad, CQ = CW > 1 ? S : 1;
    float hn[S], decay[S], drive[S];
    if (!states_fast_dv<S, CQ>(h, a, k, dv, hn, decay, drive)) states_scaled<S, CQ>(h, a, k, hn, decay, drive);
    unsigned fail = 0;
    float term[S];
#pragma unroll
    for (int j = 0; j < S; ++j) {
        term[j] = __fmul_rn(k.c[CQ > 1 ? j : 0], hn[j]);
        fail |= !finite32(decay[j]) ? kDecay : !finite32(drive[j]) ? kDrive : !finite32(hn[j]) ? kState
              : !finite32(term[j]) ? kTerm : 0u;
        h[j] = hn[j];
    }
    fail |= __shfl_xor_sync(quad_mask(), fail, 1);
    fail |= __shfl_xor_sync(quad_mask(), fail, 2);
    if (fail) return fail;
    const float sum = quad_sum<S>(term);
    const float skip = __fmul_rn(skip_d, k.u);
    if (has_d && !finite32(skip)) return kSkip;
    float out = has_d ? __fadd_rn(sum, skip) : sum;
    if (!finite32(out)) {
        // Every term is finite but a partial sum left the FP32 range: repeat
        // with exact power-of-two scaling (reference cuda/selective_scan.cu:116-122).
        float sc[S];
#pragma unroll
        for (int j = 0; j < S; ++j) sc[j] = __fmul_rn(term[j], 0x1p-8f);
        const float scaled = quad_sum<S>(sc);
        out = has_d ? __fadd_rn(scaled, __fmul_rn(skip, 0x1p-8f)) : scaled;
        if (fabsf(out) <= FLT_MAX * 0x1p-8f) out = __fmul_rn(out, 0x1p8f);
        else return kOutput;
    }
    if (kHalfOut && !(fabsf(out) < kHalfOverflow)) return kOutput;
    y = out;
    return 0;
}

// Pass 1 step for a quarter of the states, Delta given.
template <int S, int CQ>
__device__ __forceinline__ void step_carry_quad(float (&h)[S], float (&prod)[S], const float (&a)[S], const Token<S, CQ>& k, float dv) {
    float hn[S], decay[S], drive[S];
    if (!states_fast_dv<S, CQ>(h, a, k, dv, hn, decay, drive)) states_scaled<S, CQ>(h, a, k, hn, decay, drive);
#pragma unroll
    for (int j = 0; j < S; ++j) {
        h[j] = hn[j];
        prod[j] = __fmul_rn(prod[j], decay[j]);
    }
}

// Delta of token t of a walk from t0: every fourth token, thread q of the
// lane forms softplus_plain of token t + q from the raw delta it loaded a
// group earlier (`next`; past t1: unused) and loads the one of token
// t + 4 + q; token t's Delta comes from thread (t - t0) % 4 of the group.
struct QuadDelta {
    float mine, next;
};
template <typename T>
__device__ __forceinline__ float quad_delta_load(const Params& p, unsigned long long row0, unsigned long long t,
                                                 unsigned long long t1, unsigned long long d) {
    return t < t1 ? load_act(static_cast<const T*>(p.delta) + (row0 + t) * p.channels + d) : 0.0f;
}
template <typename T>
__device__ __forceinline__ float quad_delta(const Params& p, unsigned long long row0, unsigned long long t, unsigned long long t0,
                                            unsigned long long t1, unsigned long long d, int q, QuadDelta& qd) {
    const int j = static_cast<int>((t - t0) & 3u);
    if (j == 0) {
        qd.mine = softplus_plain(qd.next);
        qd.next = quad_delta_load<T>(p, row0, t + 4 + static_cast<unsigned long long>(q), t1, d);
    }
    return __shfl_sync(quad_mask(), qd.mine, static_cast<int>(threadIdx.x & 28u) | j);
}

// scan_f32_kernel for N >= 8 at four threads per lane: the same chunks, carry
// fold and failure rules, each (lane, chunk) a group of four consecutive
// threads.  With the same chunk count its outputs are scan_f32_kernel's bits.
template <typename T, int N, int CW>
__global__ void __launch_bounds__(kThreads) scan_f32_quad_kernel(Params p, SaccScanStatus* status) {
    constexpr int S = N / kQuad, CQ = CW > 1 ? S : 1;
    extern __shared__ float2 carry[]; // [chunk][lane in CTA][state]: (decay product, local state)
    __shared__ int chunk_failed[kThreads / kQuad];
    const int K = p.chunks, LPC = p.lanes_per_cta;
    const int tid = threadIdx.x, q = tid % kQuad, g = tid / kQuad, li = g % LPC, k = g / LPC;
    const unsigned long long lane = static_cast<unsigned long long>(blockIdx.x) * LPC + li;
    const bool active = lane < p.lanes; // uniform over a lane's four threads
    const unsigned long long L = p.length, Dc = p.channels;
    const unsigned long long bb = active ? lane / Dc : 0, d = active ? lane % Dc : 0;
    const unsigned long long t0 = L * k / K, t1 = L * (k + 1) / K;

    float a[S];
#pragma unroll
    for (int j = 0; j < S; ++j) a[j] = active ? __ldg(p.a + (p.a_shared ? 0 : d * N) + q + 4 * j) : 0.0f;
    const float skip_d = (active && p.has_d) ? __ldg(p.d + d) : 0.0f;
    float h[S];
#pragma unroll
    for (int j = 0; j < S; ++j) h[j] = 0.0f;

    if (K > 1) {
        float prod[S];
#pragma unroll
        for (int j = 0; j < S; ++j) prod[j] = 1.0f;
        if (active && k < K - 1) {
            Token<S, CQ> cur;
            QuadDelta sp{0.0f, quad_delta_load<T>(p, bb * L, t0 + static_cast<unsigned long long>(q), t1, d)};
            if (t0 < t1) load_token_quad<T, N, CW>(p, bb * L + t0, d, q, cur);
            for (unsigned long long t = t0; t < t1; ++t) {
                const float dv = quad_delta<T>(p, bb * L, t, t0, t1, d, q, sp);
                Token<S, CQ> nxt;
                if (t + 1 < t1) load_token_quad<T, N, CW>(p, bb * L + t + 1, d, q, nxt);
                step_carry_quad<S, CQ>(h, prod, a, cur, dv);
                cur = nxt;
            }
        }
        float2* mine = carry + (static_cast<size_t>(k) * LPC + li) * N;
#pragma unroll
        for (int j = 0; j < S; ++j) mine[q + 4 * j] = make_float2(prod[j], h[j]);
        __syncthreads();
        // Fold the carries of chunks 0..k-1: H = prod_j * H + local_j.
#pragma unroll
        for (int j = 0; j < S; ++j) h[j] = 0.0f;
        for (int c = 0; c < k; ++c) {
            const float2* cj = carry + (static_cast<size_t>(c) * LPC + li) * N;
#pragma unroll
            for (int j = 0; j < S; ++j) {
                const float2 v = cj[q + 4 * j];
                h[j] = h[j] == 0.0f ? v.y : __fmaf_rn(v.x, h[j], v.y);
            }
        }
    }

    unsigned fail = 0;
    if (active && t0 < t1) {
        Token<S, CQ> cur;
        QuadDelta sp{0.0f, quad_delta_load<T>(p, bb * L, t0 + static_cast<unsigned long long>(q), t1, d)};
        load_token_quad<T, N, CW>(p, bb * L + t0, d, q, cur);
        for (unsigned long long t = t0; t < t1; ++t) {
            const float dv = quad_delta<T>(p, bb * L, t, t0, t1, d, q, sp);
            Token<S, CQ> nxt;
            if (t + 1 < t1) load_token_quad<T, N, CW>(p, bb * L + t + 1, d, q, nxt);
            float y = 0.0f;
            fail = step_out_quad<N, CW, std::is_same_v<T, __half>>(h, a, cur, dv, p.has_d != 0, skip_d, y);
            if (fail) break;
            if (q == 0) store_act(static_cast<T*>(p.y) + (bb * L + t) * Dc + d, y);
            cur = nxt;
        }
    }
    if (K > 1) {
        // A lane reports the failure of its earliest failing chunk only, as the
        // sequential recurrence stops at its first failure.
        if (q == 0) chunk_failed[g] = fail ? 1 : 0;
        __syncthreads();
        if (fail && q == 0) {
            bool earlier = false;
            for (int c = 0; c < k; ++c) earlier |= chunk_failed[c * LPC + li] != 0;
            if (!earlier) atomicOr(&status->flags, fail);
        }
    } else if (fail && q == 0) {
        atomicOr(&status->flags, fail);
    }
    // The check grid released this grid before it finished: one thread waits
    // for it here, so this grid completes only after the check has.
    if (blockIdx.x == 0 && threadIdx.x == 0) pdl_wait();
}

// Exact NaN / Inf bits of the inputs.  Releases the next kernel of the stream
// at once when that one is launched with programmatic stream serialization
// (the scan, which does not read what the check writes).
__global__ void __launch_bounds__(kThreads) check_kernel(CheckList list, SaccScanStatus* status) {
    pdl_launch_dependents();
    check_tensors(list, static_cast<unsigned long long>(blockIdx.x) * kThreads + threadIdx.x,
                  static_cast<unsigned long long>(gridDim.x) * kThreads, status);
}

// Last kernel of every call: poison every output on failure (the FP32 quiet
// NaN 0x7fc00000, or the FP16 one 0x7e00), then write done (reference
// cuda/selective_scan.cu:149-155).
template <typename W, unsigned kPoison>
__global__ void __launch_bounds__(kThreads) finalize_kernel(W* out, unsigned long long count, SaccScanStatus* status) {
    pdl_wait(); // launched with programmatic stream serialization: the previous grid's status bits first
    const unsigned long long first = static_cast<unsigned long long>(blockIdx.x) * kThreads + threadIdx.x;
    const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * kThreads;
    if (status->flags)
        for (unsigned long long i = first; i < count; i += stride) out[i] = static_cast<W>(kPoison);
    if (first == 0) status->done = SACC_SCAN_DONE;
}

// CW: the C row's width, N (full) or 1 (one C per token).
template <typename T, int N, int CW = N>
const void* scan_kernel_ptr() {
    return reinterpret_cast<const void*>(scan_f32_kernel<T, N, CW>);
}

template <typename T>
const void* pick_kernel_t(unsigned state, bool c_full) {
    switch (state) {
    case 1: return scan_kernel_ptr<T, 1>();
    case 2: return c_full ? scan_kernel_ptr<T, 2>() : scan_kernel_ptr<T, 2, 1>();
    case 4: return c_full ? scan_kernel_ptr<T, 4>() : scan_kernel_ptr<T, 4, 1>();
    case 8: return c_full ? scan_kernel_ptr<T, 8>() : scan_kernel_ptr<T, 8, 1>();
    case 16: return c_full ? scan_kernel_ptr<T, 16>() : scan_kernel_ptr<T, 16, 1>();
    default: return c_full ? scan_kernel_ptr<T, 32>() : scan_kernel_ptr<T, 32, 1>();
    }
}

template <typename T>
const void* pick_quad_t(unsigned state, bool c_full) {
    switch (state) {
    case 8: return c_full ? reinterpret_cast<const void*>(scan_f32_quad_kernel<T, 8, 8>)
                          : reinterpret_cast<const void*>(scan_f32_quad_kernel<T, 8, 1>);
    case 16: return c_full ? reinterpret_cast<const void*>(scan_f32_quad_kernel<T, 16, 16>)
                           : reinterpret_cast<const void*>(scan_f32_quad_kernel<T, 16, 1>);
    default: return c_full ? reinterpret_cast<const void*>(scan_f32_quad_kernel<T, 32, 32>)
                           : reinterpret_cast<const void*>(scan_f32_quad_kernel<T, 32, 1>);
    }
}

// Threads per lane: four for N >= 8 (scan_f32_quad_kernel), one otherwise.
// SACC_F32_KERNEL=one_thread keeps every N on scan_f32_kernel, the kernel the
// four-thread one reproduces bit for bit when both split a lane into the same
// chunks (tests compare the two).
int threads_per_lane(unsigned state) {
    if (state < 8) return 1;
    const char* v = std::getenv("SACC_F32_KERNEL");
    return (v && std::strcmp(v, "one_thread") == 0) ? 1 : kQuad;
}

const void* pick_kernel(unsigned state, bool half, bool c_full) {
    if (threads_per_lane(state) == kQuad) {
        if (half) return pick_quad_t<__half>(state, c_full);
        return pick_quad_t<float>(state, c_full);
    }
    return half ? pick_kernel_t<__half>(state, c_full) : pick_kernel_t<float>(state, c_full);
}

// CTAs of the FP32 scan kernel for (`state`, C width) that one SM holds at
// once, queried once per kernel and device (the kernel loader fills the
// figures).  The FP16-activation launch uses the FP32 kernel's figure too, so
// both split a lane into the same chunks and the FP16 outputs stay the FP32
// outputs rounded.
int resident_per_sm(unsigned state, bool c_full) {
    static std::atomic<int> cache[64][24] = {};
    int idx = 0;
    while ((1u << idx) < state && idx < 5) ++idx;
    const int tpl = threads_per_lane(state);
    idx = (tpl == kQuad ? 12 : 0) + 2 * idx + (c_full ? 1 : 0);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    int v = cache[dev][idx].load(std::memory_order_relaxed);
    if (v > 0) return v;
    const void* fn = pick_kernel(state, false, c_full);
    const size_t smem = static_cast<size_t>(kThreads / tpl) * state * sizeof(float2);
    int n = 0;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        n = 1;
    else if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem) != cudaSuccess || n < 1)
        n = 1;
    cache[dev][idx].store(n, std::memory_order_relaxed);
    return n;
}

unsigned long long total_checked(const CheckList& l) {
    unsigned long long n = 0;
    for (unsigned i = 0; i < l.size; ++i) n += l.tensor[i].count;
    return n;
}

unsigned check_blocks(unsigned long long elements, int sm_count) {
    const unsigned long long want = (elements + kThreads * 16ull - 1) / (kThreads * 16ull);
    const unsigned long long cap = 2ull * static_cast<unsigned long long>(sm_count);
    return static_cast<unsigned>(want < 1 ? 1 : want > cap ? cap : want);
}

} // namespace

cudaError_t launch_scan_f32(const ScanF32Launch& s, SaccScanStatus* status, int sm_count, cudaStream_t stream) {
    Params p{};
    p.u = s.u; p.delta = s.delta; p.a = s.a; p.b = s.b; p.c = s.c; p.d = s.d; p.y = s.y;
    p.length = s.length; p.channels = s.channels; p.lanes = s.lanes;
    p.a_shared = s.a_shared; p.c_full = s.c_full; p.has_d = s.has_d;
    const std::uintptr_t vec_align = s.half ? 7u : 15u; // four values per load
    p.vec_b = (reinterpret_cast<std::uintptr_t>(s.b) & vec_align) == 0;
    p.vec_c = (reinterpret_cast<std::uintptr_t>(s.c) & vec_align) == 0;
    // Chunks: as many (lane, chunk) threads as the SMs hold at once (one wave:
    // a chunk's work grows with L / K and its fold with K, and a second wave
    // doubles the time), at least 2 tokens per chunk, at most 64 chunks; one
    // chunk when the lanes alone fill the SMs.  At 165 registers an SM holds
    // one 256-thread CTA of the N = 16 kernel, so the HR deploy level of 1,024
    // lanes x 960 tokens runs 32 chunks in 128 CTAs.
    const unsigned long long target =
        static_cast<unsigned long long>(sm_count) * static_cast<unsigned long long>(resident_per_sm(s.state, s.c_full)) * kThreads;
    const int tpl = threads_per_lane(s.state);
    int K = 1;
    while (K < 64 && s.lanes * static_cast<unsigned long long>(K * tpl) * 2ull <= target &&
           s.length >= static_cast<unsigned long long>(K) * 2ull * 2ull)
        K *= 2;
    p.chunks = K;
    p.lanes_per_cta = kThreads / tpl / K;
    const unsigned long long blocks = (s.lanes + p.lanes_per_cta - 1) / p.lanes_per_cta;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidValue;
    p.scan_blocks = static_cast<unsigned>(blocks);
    const size_t smem = K > 1 ? static_cast<size_t>(kThreads / tpl) * s.state * sizeof(float2) : 0;
    void* args[] = {&p, &status};
    const void* fn = pick_kernel(s.state, s.half, s.c_full);
    if (smem > 48 * 1024) {
        // Also set by the kernel loader; repeated here so that a call before
        // sacc_scan_load_kernels still launches.
        const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    // After the check kernel, which releases this launch at its start.
    return launch_pdl(fn, dim3(p.scan_blocks), dim3(kThreads), smem, stream, args);
}

cudaError_t launch_check(const CheckList& list, SaccScanStatus* status, int sm_count, cudaStream_t stream) {
    check_kernel<<<check_blocks(total_checked(list), sm_count), kThreads, 0, stream>>>(list, status);
    return cudaGetLastError();
}

cudaError_t launch_finalize(void* out, unsigned long long count, SaccScanStatus* status, int sm_count, cudaStream_t stream,
                            bool half) {
    const unsigned long long want = (count + kThreads * 8ull - 1) / (kThreads * 8ull);
    const unsigned long long cap = 4ull * static_cast<unsigned long long>(sm_count);
    const unsigned blocks = static_cast<unsigned>(want < 1 ? 1 : want > cap ? cap : want);
    if (half)
        return launch_pdl_k(finalize_kernel<unsigned short, 0x7e00u>, dim3(blocks), dim3(kThreads), 0, stream,
                            static_cast<unsigned short*>(out), count, status);
    return launch_pdl_k(finalize_kernel<unsigned, 0x7fc00000u>, dim3(blocks), dim3(kThreads), 0, stream,
                        static_cast<unsigned*>(out), count, status);
}

cudaError_t load_scan_f32_kernels(std::string& report) {
    struct Entry { const char* name; const void* fn; size_t smem; };
    const Entry kernels[] = {
        {"scan_f32_n1", scan_kernel_ptr<float, 1>(), kThreads * 1 * sizeof(float2)},
        {"scan_f32_n2", scan_kernel_ptr<float, 2>(), kThreads * 2 * sizeof(float2)},
        {"scan_f32_n4", scan_kernel_ptr<float, 4>(), kThreads * 4 * sizeof(float2)},
        {"scan_f32_n8", scan_kernel_ptr<float, 8>(), kThreads * 8 * sizeof(float2)},
        {"scan_f32_n16", scan_kernel_ptr<float, 16>(), kThreads * 16 * sizeof(float2)},
        {"scan_f32_n32", scan_kernel_ptr<float, 32>(), kThreads * 32 * sizeof(float2)},
        {"scan_f16io_n1", scan_kernel_ptr<__half, 1>(), kThreads * 1 * sizeof(float2)},
        {"scan_f16io_n2", scan_kernel_ptr<__half, 2>(), kThreads * 2 * sizeof(float2)},
        {"scan_f16io_n4", scan_kernel_ptr<__half, 4>(), kThreads * 4 * sizeof(float2)},
        {"scan_f16io_n8", scan_kernel_ptr<__half, 8>(), kThreads * 8 * sizeof(float2)},
        {"scan_f16io_n16", scan_kernel_ptr<__half, 16>(), kThreads * 16 * sizeof(float2)},
        {"scan_f16io_n32", scan_kernel_ptr<__half, 32>(), kThreads * 32 * sizeof(float2)},
        {"scan_f32_c1_n2", scan_kernel_ptr<float, 2, 1>(), kThreads * 2 * sizeof(float2)},
        {"scan_f32_c1_n4", scan_kernel_ptr<float, 4, 1>(), kThreads * 4 * sizeof(float2)},
        {"scan_f32_c1_n8", scan_kernel_ptr<float, 8, 1>(), kThreads * 8 * sizeof(float2)},
        {"scan_f32_c1_n16", scan_kernel_ptr<float, 16, 1>(), kThreads * 16 * sizeof(float2)},
        {"scan_f32_c1_n32", scan_kernel_ptr<float, 32, 1>(), kThreads * 32 * sizeof(float2)},
        {"scan_f16io_c1_n2", scan_kernel_ptr<__half, 2, 1>(), kThreads * 2 * sizeof(float2)},
        {"scan_f16io_c1_n4", scan_kernel_ptr<__half, 4, 1>(), kThreads * 4 * sizeof(float2)},
        {"scan_f16io_c1_n8", scan_kernel_ptr<__half, 8, 1>(), kThreads * 8 * sizeof(float2)},
        {"scan_f16io_c1_n16", scan_kernel_ptr<__half, 16, 1>(), kThreads * 16 * sizeof(float2)},
        {"scan_f16io_c1_n32", scan_kernel_ptr<__half, 32, 1>(), kThreads * 32 * sizeof(float2)},
        {"scan_f32_quad_n8", reinterpret_cast<const void*>(scan_f32_quad_kernel<float, 8, 8>), 0},
        {"scan_f32_quad_n16", reinterpret_cast<const void*>(scan_f32_quad_kernel<float, 16, 16>), 0},
        {"scan_f32_quad_n32", reinterpret_cast<const void*>(scan_f32_quad_kernel<float, 32, 32>), 0},
        {"scan_f32_quad_c1_n8", reinterpret_cast<const void*>(scan_f32_quad_kernel<float, 8, 1>), 0},
        {"scan_f32_quad_c1_n16", reinterpret_cast<const void*>(scan_f32_quad_kernel<float, 16, 1>), 0},
        {"scan_f32_quad_c1_n32", reinterpret_cast<const void*>(scan_f32_quad_kernel<float, 32, 1>), 0},
        {"scan_f16io_quad_n8", reinterpret_cast<const void*>(scan_f32_quad_kernel<__half, 8, 8>), 0},
        {"scan_f16io_quad_n16", reinterpret_cast<const void*>(scan_f32_quad_kernel<__half, 16, 16>), 0},
        {"scan_f16io_quad_n32", reinterpret_cast<const void*>(scan_f32_quad_kernel<__half, 32, 32>), 0},
        {"scan_f16io_quad_c1_n8", reinterpret_cast<const void*>(scan_f32_quad_kernel<__half, 8, 1>), 0},
        {"scan_f16io_quad_c1_n16", reinterpret_cast<const void*>(scan_f32_quad_kernel<__half, 16, 1>), 0},
        {"scan_f16io_quad_c1_n32", reinterpret_cast<const void*>(scan_f32_quad_kernel<__half, 32, 1>), 0},
        {"check", reinterpret_cast<const void*>(check_kernel), 0},
        {"finalize", reinterpret_cast<const void*>(finalize_kernel<unsigned, 0x7fc00000u>), 0},
        {"finalize_f16", reinterpret_cast<const void*>(finalize_kernel<unsigned short, 0x7e00u>), 0},
    };
    for (const auto& k : kernels) {
        cudaFuncAttributes attr{};
        cudaError_t e = cudaFuncGetAttributes(&attr, k.fn);
        if (e != cudaSuccess) return e;
        if (k.smem > 48 * 1024) {
            e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(k.smem));
            if (e != cudaSuccess) return e;
        }
        report += std::string("kernel=") + k.name + " registers=" + std::to_string(attr.numRegs) +
                  " local_bytes=" + std::to_string(attr.localSizeBytes) + " shared_bytes=" +
                  std::to_string(attr.sharedSizeBytes) + " max_threads=" + std::to_string(attr.maxThreadsPerBlock) + "\n";
    }
    // The chunk split's residency figures, so that no call queries them later.
    for (unsigned state = 1; state <= 32; state *= 2) report += "scan_f32_resident_ctas_per_sm_n" + std::to_string(state) + "=" +
                                                               std::to_string(resident_per_sm(state, true)) + "\n";
    for (unsigned state = 2; state <= 32; state *= 2) report += "scan_f32_c1_resident_ctas_per_sm_n" + std::to_string(state) + "=" +
                                                               std::to_string(resident_per_sm(state, false)) + "\n";
    return cudaSuccess;
}

} // namespace sacc
